"""Persisted index files (host side, no GPU): format round trip, row-range reads, checksums and the errors a reader
must raise on damaged files. The device loader (vk_index_load) is covered in test_parity_gpu.py."""
import os

import numpy as np
import pytest

from veckern_b200 import data


def make(n, m, dsub, seed=0):
    rng = np.random.default_rng(seed)
    return rng.normal(size=(m, 256, dsub)).astype(np.float32), rng.integers(0, 256, size=(n, m), dtype=np.uint8)


def test_crc32c_known_answer_and_paths():
    # CRC-32C check value of "123456789" (RFC 3720, appendix B.4)
    assert data.crc32c(b"123456789") == 0xE3069283
    assert data.crc32c(b"123456789", hardware=False) == 0xE3069283
    assert data.crc32c(b"") == 0
    rng = np.random.default_rng(1)
    for size in [1, 7, 8, 9, 63, 4096, 100_003]:
        buf = rng.integers(0, 256, size=size, dtype=np.uint8)
        assert data.crc32c(buf) == data.crc32c(buf, hardware=False)


def test_round_trip_and_ranges(tmp_path):
    cent, codes = make(5003, 16, 8)
    p = tmp_path / "a.vkpq"
    data.write_index(p, cent, codes)
    assert data.index_info(p) == {"n": 5003, "d": 128, "m": 16, "dsub": 8}
    c2, k2 = data.read_index(p)
    assert np.array_equal(c2, cent) and np.array_equal(k2, codes)
    for lo, hi in [(0, 1), (1000, 1777), (4999, 5003), (5003, 5003)]:
        _, part = data.read_index(p, rows=(lo, hi))
        assert np.array_equal(part, codes[lo:hi])
    with pytest.raises(ValueError):
        data.read_index(p, rows=(5000, 5004))
    with open(p, "rb") as f:
        head = f.read(128)
    assert head[:8] == b"VKPQIDX1"
    assert os.path.getsize(p) % 4 == 0


def test_multi_block_ranges_and_shards(tmp_path):
    """Files span several checksum blocks (2^20 rows); any range, verified or not, reads the same bytes, and the
    shards of shard_of() read separately concatenate to the whole."""
    from veckern_b200.shard import shard_of
    n = (1 << 20) * 2 + 12_345
    cent, codes = make(n, 4, 2, seed=2)
    p = tmp_path / "big.vkpq"
    data.write_index(p, cent, codes)
    for lo, hi in [(0, n), ((1 << 20) - 5, (1 << 20) + 5), (2 << 20, n), (123, 124)]:
        for verify in (True, False):
            _, part = data.read_index(p, rows=(lo, hi), verify=verify)
            assert np.array_equal(part, codes[lo:hi]), (lo, hi, verify)
    parts = []
    for r in range(3):
        sh = shard_of(n, 3, r)
        parts.append(data.read_index(p, rows=(sh.lo, sh.hi))[1])
    assert np.array_equal(np.concatenate(parts), codes)


def corrupt(path, offset, xor=0x40):
    with open(path, "r+b") as f:
        f.seek(offset)
        b = f.read(1)
        f.seek(offset)
        f.write(bytes([b[0] ^ xor]))


def test_damage_is_detected(tmp_path):
    cent, codes = make(3000, 16, 8, seed=3)
    good = tmp_path / "good.vkpq"
    data.write_index(good, cent, codes)
    raw = good.read_bytes()
    codes_off = int.from_bytes(raw[48:56], "little")
    cent_off = int.from_bytes(raw[40:48], "little")

    def variant(name, mutate):
        p = tmp_path / name
        p.write_bytes(raw)
        mutate(p)
        return p

    p = variant("code.vkpq", lambda p: corrupt(p, codes_off + 1234))
    with pytest.raises(data.IndexFileError, match="checksum"):
        data.read_index(p)
    data.read_index(p, verify=False)  # unverified reads do not look at the code checksums
    p = variant("cent.vkpq", lambda p: corrupt(p, cent_off + 17))
    with pytest.raises(data.IndexFileError, match="centroid checksum"):
        data.read_index(p)
    p = variant("head.vkpq", lambda p: corrupt(p, 20))
    with pytest.raises(data.IndexFileError, match="header checksum"):
        data.index_info(p)
    p = variant("magic.vkpq", lambda p: corrupt(p, 0))
    with pytest.raises(data.IndexFileError, match="magic"):
        data.index_info(p)
    p = variant("short.vkpq", lambda p: p.write_bytes(raw[: len(raw) - 100]))
    with pytest.raises(data.IndexFileError, match="truncated"):
        data.index_info(p)
    with pytest.raises(data.IndexFileError, match="cannot open"):
        data.index_info(tmp_path / "missing.vkpq")


def test_crafted_headers_with_valid_checksums_are_rejected(tmp_path):
    """Headers whose own CRC-32C is right but whose sizes would wrap 64-bit offset arithmetic (or ask for absurd
    shapes) are refused before any buffer is sized from them."""
    cent, codes = make(1000, 16, 8, seed=4)
    good = tmp_path / "good.vkpq"
    data.write_index(good, cent, codes)
    raw = bytearray(good.read_bytes())

    def forged(name, **fields):
        b = bytearray(raw)
        layout = {"n": (16, 8), "d": (24, 4), "m": (28, 4), "dsub": (32, 4), "codes_off": (48, 8),
                  "block_rows": (56, 8), "crc_off": (64, 8)}
        for k, v in fields.items():
            off, size = layout[k]
            b[off:off + size] = int(v).to_bytes(size, "little")
        b[76:80] = data.crc32c(bytes(b[:76])).to_bytes(4, "little")  # re-sign the header
        p = tmp_path / name
        p.write_bytes(bytes(b))
        return p

    bad = [
        forged("wrap_n.vkpq", n=(1 << 64) // 16 + 1),                          # n * m wraps to a small number
        forged("huge_m.vkpq", m=1 << 30, dsub=4, d=0),                          # m * dsub = 2^32 wraps to 0 in 32 bits
        forged("huge_blocks.vkpq", block_rows=1),                               # fine shape, crc section past the end
        forged("wrap_off.vkpq", codes_off=(1 << 64) - 4096),                   # offset + size wraps
        forged("wrap_crc.vkpq", crc_off=(1 << 64) - 8),
    ]
    for p in bad:
        with pytest.raises(data.IndexFileError):
            data.index_info(p)
    assert data.index_info(forged("resigned.vkpq")) == {"n": 1000, "d": 128, "m": 16, "dsub": 8}
