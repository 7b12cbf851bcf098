"""Input side of the search path on the host: product quantizer and synthetic data (include/vk_host.h).

These produce the database, codebooks and queries the GPU path searches; they are deterministic (counter-based
or the reference's own std:: engines) so every machine regenerates identical inputs.
"""
from __future__ import annotations

import numpy as np

from ._native import host, ptr


def _ok(rc: int, what: str) -> None:
    if rc != 0:
        raise ValueError(f"{what}: bad arguments")


def pq_train(x: np.ndarray, m: int, iters: int, seed: int = 1) -> np.ndarray:
    """The reference's ProductQuantizer::train (src/cpu/pq.cpp:31-69) on all rows of x -> [m, 256, d/m]."""
    x = np.ascontiguousarray(x, np.float32)
    n, d = x.shape
    cent = np.empty((m, 256, d // m), np.float32)
    _ok(host().vk_host_pq_train(ptr(x), n, d, m, iters, seed, ptr(cent)), "pq_train")
    return cent


def pq_encode(centroids: np.ndarray, x: np.ndarray) -> np.ndarray:
    """Nearest centroid per sub-space (src/cpu/pq.cpp:71-76) -> [n, m] uint8."""
    centroids = np.ascontiguousarray(centroids, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    m, _, dsub = centroids.shape
    codes = np.empty((x.shape[0], m), np.uint8)
    _ok(host().vk_host_pq_encode(ptr(centroids), m * dsub, m, ptr(x), x.shape[0], ptr(codes)), "pq_encode")
    return codes


def pq4_train(x: np.ndarray, m: int, iters: int, seed: int = 1) -> np.ndarray:
    """4-bit PQ codebooks: the same trainer with 16 centroids per sub-space -> [m, 16, d/m]."""
    x = np.ascontiguousarray(x, np.float32)
    n, d = x.shape
    cent = np.empty((m, 16, d // m), np.float32)
    _ok(host().vk_host_pq4_train(ptr(x), n, d, m, iters, seed, ptr(cent)), "pq4_train")
    return cent


def pq4_encode(centroids: np.ndarray, x: np.ndarray) -> np.ndarray:
    """First nearest of the 16 centroids per sub-space, packed two per byte (sub-code s in nibble s % 2, low
    first, of byte s / 2) -> [n, ceil(m / 2)] uint8."""
    centroids = np.ascontiguousarray(centroids, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    m, _, dsub = centroids.shape
    codes = np.empty((x.shape[0], (m + 1) // 2), np.uint8)
    _ok(host().vk_host_pq4_encode(ptr(centroids), m * dsub, m, ptr(x), x.shape[0], ptr(codes)), "pq4_encode")
    return codes


def pq_decode(centroids: np.ndarray, codes: np.ndarray) -> np.ndarray:
    centroids = np.ascontiguousarray(centroids, np.float32)
    codes = np.ascontiguousarray(codes, np.uint8)
    m, _, dsub = centroids.shape
    x = np.empty((codes.shape[0], m * dsub), np.float32)
    _ok(host().vk_host_pq_decode(ptr(centroids), m * dsub, m, ptr(codes), codes.shape[0], ptr(x)), "pq_decode")
    return x


def synthetic_clustered(n: int, d: int, clusters: int, seed: int) -> np.ndarray:
    """The reference's Gaussian blobs (src/cpu/io.cpp:54-69), as its test fixtures use them."""
    out = np.empty((n, d), np.float32)
    _ok(host().vk_host_synthetic_clustered(n, d, clusters, seed, ptr(out)), "synthetic_clustered")
    return out


def gen_normal(seed: int, rows: int, d: int, row0: int = 0) -> np.ndarray:
    out = np.empty((rows, d), np.float32)
    _ok(host().vk_host_gen_normal(seed, row0, rows, d, ptr(out)), "gen_normal")
    return out


def gen_mixture(mix_seed: int, sample_seed: int, rows: int, d: int = 128, ncomp: int = 1000, sigma: float = 12.0,
                row0: int = 0) -> np.ndarray:
    out = np.empty((rows, d), np.float32)
    _ok(host().vk_host_gen_mixture(mix_seed, ncomp, sigma, sample_seed, row0, rows, d, ptr(out)), "gen_mixture")
    return out


def gen_cdf(seed: int, clusters: int, m: int, alpha: float) -> np.ndarray:
    out = np.empty((clusters, m, 256), np.uint32)
    _ok(host().vk_host_gen_cdf(seed, clusters, m, alpha, ptr(out)), "gen_cdf")
    return out


def gen_codes(seed: int, cdf: np.ndarray, row0: int, n: int) -> np.ndarray:
    cdf = np.ascontiguousarray(cdf, np.uint32)
    clusters, m, _ = cdf.shape
    out = np.empty((n, m), np.uint8)
    _ok(host().vk_host_gen_codes(seed, ptr(cdf), clusters, m, row0, n, ptr(out)), "gen_codes")
    return out


def gen_codes_rows(seed: int, cdf: np.ndarray, rows) -> np.ndarray:
    """The listed rows of the generated code database (any order; negative rows give zeros)."""
    cdf = np.ascontiguousarray(cdf, np.uint32)
    rows = np.ascontiguousarray(rows, np.int64).ravel()
    clusters, m, _ = cdf.shape
    out = np.empty((rows.shape[0], m), np.uint8)
    _ok(host().vk_host_gen_codes_rows(seed, ptr(cdf), clusters, m, ptr(rows), rows.shape[0], ptr(out)),
        "gen_codes_rows")
    return out


def pq_train_gpu(x, m: int, iters: int, seed: int = 1, device: int | None = None) -> np.ndarray:
    """ProductQuantizer::train on the GPU (vk_pq_train_device): bit-identical centroids [m, 256, d/m]."""
    import torch

    from ._native import check, lib
    dev = torch.cuda.current_device() if device is None else device
    with torch.cuda.device(dev):
        xs = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x, np.float32))
        xs = xs.to(device=f"cuda:{dev}", dtype=torch.float32).contiguous()
        n, d = xs.shape
        cent = np.empty((m, 256, d // m), np.float32)
        check(lib().vk_pq_train_device(dev, ptr(xs), n, d, m, iters, seed, ptr(cent),
                                       torch.cuda.current_stream().cuda_stream), "pq_train")
    return cent


def gpu_trainer(device: int | None = None):
    """train(x, m, iters, seed) -> centroids on the GPU (same result as pq_train)."""
    return lambda x, m, iters, seed: pq_train_gpu(x, m, iters, seed, device)


def gpu_encoder(device: int | None = None):
    """encode(centroids, x) -> codes on the GPU (vk_encode_device: bit-exact nearest centroid), 1M rows at a time."""
    def enc(cent, x):
        import torch

        from ._native import check, lib
        cent = np.ascontiguousarray(cent, np.float32)
        m, _, dsub = cent.shape
        dev = torch.cuda.current_device() if device is None else device
        out = np.empty((x.shape[0], m), np.uint8)
        step = 1 << 20
        with torch.cuda.device(dev):
            for a in range(0, x.shape[0], step):
                xs = torch.from_numpy(np.ascontiguousarray(x[a:a + step])).cuda()
                cs = torch.empty((xs.shape[0], m), dtype=torch.uint8, device="cuda")
                check(lib().vk_encode_device(dev, ptr(cent), m, dsub, ptr(xs), xs.shape[0], ptr(cs),
                                             torch.cuda.current_stream().cuda_stream), "encode")
                out[a:a + xs.shape[0]] = cs.cpu().numpy()
        return out
    return enc


# ---------------------------------------------------------------------------------------------- index files
class IndexFileError(IOError):
    pass


def _host_check(rc: int, what: str) -> None:
    if rc != 0:
        import ctypes as C
        buf = C.create_string_buffer(1024)
        host().vk_host_last_error(buf, len(buf))
        msg = buf.value.decode(errors="replace")
        if rc == -1:
            raise ValueError(f"{what}: {msg}")
        raise IndexFileError(f"{what}: {msg}")


def crc32c(data, hardware: bool = True) -> int:
    a = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray)) else data)
    return int(host().vk_host_crc32c(ptr(a), a.nbytes, int(hardware)))


def write_index(path, centroids: np.ndarray, codes: np.ndarray) -> None:
    """Persisted index file: centroids [m, 256, dsub] fp32 + codes [n, m] uint8 (format in include/vk_host.h)."""
    centroids = np.ascontiguousarray(centroids, np.float32)
    codes = np.ascontiguousarray(codes, np.uint8)
    m, _, dsub = centroids.shape
    if codes.ndim != 2 or codes.shape[1] != m:
        raise ValueError("codes must be [n, m] uint8")
    _host_check(host().vk_host_index_write(str(path).encode(), ptr(centroids), m, dsub, ptr(codes), codes.shape[0]),
                "write_index")


def index_info(path) -> dict:
    import ctypes as C
    n, d, m, dsub = C.c_int64(), C.c_int(), C.c_int(), C.c_int()
    _host_check(host().vk_host_index_info(str(path).encode(), C.byref(n), C.byref(d), C.byref(m), C.byref(dsub)),
                "index_info")
    return {"n": n.value, "d": d.value, "m": m.value, "dsub": dsub.value}


def read_index(path, rows: tuple[int, int] | None = None, verify: bool = True):
    """(centroids [m, 256, dsub], codes of rows [lo, hi)) of a persisted index file; only that range is read."""
    info = index_info(path)
    lo, hi = rows if rows is not None else (0, info["n"])
    cent = np.empty((info["m"], 256, info["dsub"]), np.float32)
    codes = np.empty((max(0, hi - lo), info["m"]), np.uint8)
    _host_check(host().vk_host_index_read(str(path).encode(), ptr(cent), lo, hi - lo, ptr(codes), int(verify)),
                "read_index")
    return cent, codes
