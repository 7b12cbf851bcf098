"""CPU: the native libraries load and export every declared entry point; host-side logic (tuning validation,
PQ training/encoding, generators) matches the reference's behaviour. No GPU compute calls here."""
import ctypes as C
import re
import subprocess
import textwrap
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import REPO, bits, load_golden
from veckern_b200 import _native as N
from veckern_b200 import data


def _declared(header: Path) -> set[str]:
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(vk_\w+)\s*\(", text))


def test_abi_exports_every_declared_symbol():
    lib = C.CDLL(str(N.LIB_PATH))
    declared = _declared(REPO / "include" / "vk_abi.h")
    assert declared, "no declarations parsed"
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    assert declared == set(N.ABI), "Python bindings and header disagree"


def test_host_exports_every_declared_symbol():
    lib = C.CDLL(str(N.HOST_LIB_PATH))
    declared = _declared(REPO / "include" / "vk_host.h")
    assert declared and all(hasattr(lib, s) for s in declared)
    assert declared == set(N.HOST_ABI)


def test_cxx_api_symbols_exported():
    """The drop-in C++ API (include/veckern/gpu.hpp) is implemented by libveckern_b200.so."""
    out = subprocess.run(["nm", "-DC", "--defined-only", str(N.LIB_PATH)], capture_output=True, text=True).stdout
    for sym in ["veckern::gpu::PQSearcher::PQSearcher(veckern::ProductQuantizer const&, unsigned char const*, "
                "unsigned long)", "veckern::gpu::PQSearcher::search(", "veckern::gpu::PQSearcher::distances(",
                "veckern::gpu::PQSearcher::set_tuning(", "veckern::gpu::PQSearcher::last_launch() const",
                "veckern::gpu::device_info(int)", "veckern::gpu::variant_name(", "veckern::gpu::is_fused("]:
        assert sym in out, sym


def test_c_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text(textwrap.dedent("""
        #include "vk_abi.h"
        #include "vk_host.h"
        int main(void) { vk_tuning_t t; vk_tuning_default(&t); return vk_tuning_validate(&t); }
    """))
    exe = tmp_path / "t"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{REPO / 'include'}", str(src), "-o", str(exe),
                    f"-L{N.NATIVE}", "-lveckern_b200", f"-Wl,-rpath,{N.NATIVE}"], check=True)
    assert subprocess.run([str(exe)]).returncode == 0


def test_tuning_defaults_and_rejections():
    """Same defaults and rejects as the reference (include/veckern/gpu.hpp:29-34, tests/test_gpu.cpp:176-189)."""
    lib = N.lib()
    t = N.Tuning()
    lib.vk_tuning_default(C.byref(t))
    assert (t.scan_threads, t.blocks_per_query, t.queries_per_block, t.vectors_per_step, t.early_abandon) == \
        (256, 0, 2, 4, 1)
    assert lib.vk_tuning_validate(C.byref(t)) == 0
    for bad in [(100, 0, 2, 1, 1), (256, -1, 2, 1, 1), (256, 0, 3, 1, 1), (256, 0, 2, 3, 1), (0, 0, 2, 1, 1),
                (1056, 0, 2, 1, 1), (256, 0, 2, 1, 2)]:
        assert lib.vk_tuning_validate(C.byref(N.Tuning(*bad))) == N.VK_ERR_INVALID
        assert N.last_error()


def test_null_arguments_rejected_without_gpu():
    lib = N.lib()
    h = C.c_void_p()
    assert lib.vk_index_create(0, None, 16, 8, None, 10, 0, C.byref(h)) == N.VK_ERR_INVALID
    assert lib.vk_search(None, None, 1, 10, 8, None, None, None, None) == N.VK_ERR_INVALID
    assert lib.vk_merge_topk_device(0, None, 1, 1, 1, 1, 1, 0, None, None) == N.VK_ERR_INVALID  # k = 0


def test_pq_train_encode_match_reference_fixture():
    g = load_golden("cpu_fixture")
    base = data.synthetic_clustered(4000, 32, 20, 7)
    q = data.synthetic_clustered(12, 32, 20, 8)
    assert np.array_equal(bits(q), bits(g["queries"]))
    cent = data.pq_train(base, 8, 10, 1)
    assert np.array_equal(bits(cent), bits(g["centroids"]))
    assert np.array_equal(data.pq_encode(cent, base), g["codes"])


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built here")
@pytest.mark.parametrize("iters,seed", [(0, 1), (3, 7)])
def test_pq_matches_reference_on_mixture(iters, seed):
    R = oracle.ref()
    x = data.gen_mixture(0, 0, 3000, 64, ncomp=50)
    pq = R.pq(64, 16)
    pq.train(x, 3000, iters, seed)
    cent = data.pq_train(x, 16, iters, seed)
    assert np.array_equal(bits(cent), bits(pq.centroids))
    assert np.array_equal(data.pq_encode(cent, x), pq.encode(x))
    assert np.array_equal(bits(data.pq_decode(cent, pq.encode(x))), bits(pq.decode(pq.encode(x))))


def test_generators_are_range_independent():
    a = data.gen_normal(5, 100, 16)
    b = data.gen_normal(5, 40, 16, row0=60)
    assert np.array_equal(bits(a[60:]), bits(b))
    m1 = data.gen_mixture(0, 3, 50)
    m2 = data.gen_mixture(0, 3, 20, row0=30)
    assert np.array_equal(m1[30:], m2) and m1.min() >= 0 and m1.max() <= 255 and (m1 == np.round(m1)).all()
    cdf = data.gen_cdf(4, 8, 16, 0.3)
    assert (np.diff(cdf.astype(np.int64), axis=2) >= 0).all() and (cdf[:, :, 255] == 0xFFFFFFFF).all()
    c1 = data.gen_codes(4, cdf, 0, 3000)
    c2 = data.gen_codes(4, cdf, 1000, 2000)
    assert np.array_equal(c1[1000:], c2)


def test_generated_codes_follow_their_cluster_distributions():
    """Dirichlet(0.3) categoricals are concentrated: few codes carry most of each cluster's mass."""
    cdf = data.gen_cdf(4, 1, 2, 0.3)
    codes = data.gen_codes(4, cdf, 0, 200_000)  # one cluster: every row uses cdf[0]
    w = np.diff(np.concatenate([[0], cdf[0, 0].astype(np.float64)])) / 2.0**32
    w[255] = 1 - cdf[0, 0, 254] / 2.0**32
    freq = np.bincount(codes[:, 0], minlength=256) / codes.shape[0]
    assert np.abs(freq - w).max() < 0.01
    assert np.sort(w)[::-1][:26].sum() > 0.5  # top 10% of codes carry most of the mass


def test_pq4_trainer_and_encoder():
    """4-bit trainer: with no Lloyd iteration its 16 centroids per sub-space are the first 16 rows the reference's
    draws pick (the 8-bit trainer, pinned to the reference, picks 256 with the same shuffles); one iteration replaces
    each non-empty cluster's centroid by the float32 mean of its rows, summed in row order. The encoder equals the
    oracle's restatement."""
    import oracle

    x = data.gen_mixture(0, 0, 400, 32, ncomp=20)
    c8 = data.pq_train(x, 8, 0, 5)
    c4 = data.pq4_train(x, 8, 0, 5)
    assert c4.shape == (8, 16, 4) and np.array_equal(bits(c4), bits(c8[:, :16]))
    c41 = data.pq4_train(x, 8, 1, 5)
    for s in range(8):
        xs = x[:, s * 4:(s + 1) * 4]
        dist = np.zeros((400, 16), np.float32)
        for c in range(16):
            acc = np.zeros(400, np.float32)
            for j in range(4):
                diff = xs[:, j] - c4[s, c, j]
                acc = acc + diff * diff
            dist[:, c] = acc
        assign = np.argmin(dist, 1)
        for c in range(16):
            rows = np.nonzero(assign == c)[0]
            if rows.size == 0:
                continue  # reseeded from an rng draw
            acc = np.zeros(4, np.float32)
            for r in rows:
                acc = acc + xs[r]
            assert np.array_equal(bits(c41[s, c]), bits(acc / np.float32(rows.size)))
    codes = data.pq4_encode(c41, x)
    assert codes.shape == (400, 4)
    assert np.array_equal(codes, oracle.port().pq4_encode(c41, x))
