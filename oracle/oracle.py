"""ctypes wrappers for the CPU checkers — TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Port: the plain-C restatement of the reference CPU path (oracle/vk_oracle.c, built to oracle/_build/).
Ref:  the reference's own CPU sources + oracle/ref_shim.cpp (built to oracle/_ref/ by oracle/Makefile).
All arrays are numpy, C-contiguous; results come back as (dists float32 [nq, k], ids int32 [nq, k]).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_SO = HERE / "_build" / "libvk_oracle.so"
REF_SO = HERE / "_ref" / "libveckern_ref.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i64 = C.c_int64


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


class Port:
    """The plain-C restatement (kind "port")."""

    def __init__(self, path: Path = PORT_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle oracle` (or __graft_entry__.build())")
        L = self.lib = C.CDLL(str(path))
        L.vko_compute_lut.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _i64, _f32p]
        L.vko_adc_scan.argtypes = [_f32p, _i64, _u8p, _i64, C.c_int, _f32p]
        L.vko_select_topk.argtypes = [_f32p, _i64, _i64, C.c_int, _f32p, _i32p]
        L.vko_adc_search.argtypes = [_f32p, C.c_int, C.c_int, _u8p, _i64, _f32p, _i64, C.c_int, _f32p, _i32p,
                                     C.c_int]
        L.vko_topk_push_all.argtypes = [_f32p, _i32p, _i64, C.c_int, _f32p, _i32p]
        L.vko_merge_topk.argtypes = [_f32p, _i32p, C.c_int, C.c_int, _i64, C.c_int, _f32p, _i32p]
        L.vko_rerank_exact.argtypes = [_f32p, C.c_int, _f32p, _i64, _i32p, C.c_int, C.c_int, _f32p, _i32p]
        L.vko_recall_at_k.argtypes = [_i32p, _i64, _i32p, _i64, _i64, C.c_int]
        L.vko_recall_at_k.restype = C.c_double
        L.vko_compute_lut_h16.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _i64, _f32p,
                                          np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")]
        L.vko_adc_search_h16.argtypes = [_f32p, C.c_int, C.c_int, _u8p, _i64, _f32p, _i64, C.c_int, _f32p, _i32p,
                                         C.c_int]
        L.vko_ivf_search.argtypes = [_f32p, C.c_int, C.c_int, _u8p, _i32p, _i64, _f32p, C.c_int, _f32p, _i64,
                                     C.c_int, C.c_int, _f32p, _i32p, _i32p, C.c_int]
        L.vko_pq4_encode.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _i64, _u8p]
        L.vko_compute_lut_pq4.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _i64, _f32p]
        L.vko_adc_search_pq4.argtypes = [_f32p, C.c_int, C.c_int, _u8p, _i64, _f32p, _i64, C.c_int, _f32p, _i32p,
                                         C.c_int]
        L.vko_stream_create.argtypes = [_f32p, _i64, C.c_int, C.c_int]
        L.vko_stream_create.restype = C.c_void_p
        L.vko_stream_feed.argtypes = [C.c_void_p, _u8p, _i64, _i64, C.c_int]
        L.vko_stream_finish.argtypes = [C.c_void_p, _f32p, _i32p]
        L.vko_stream_destroy.argtypes = [C.c_void_p]

    def compute_lut(self, centroids, queries):
        centroids = _f32(centroids)
        m, ksub, dsub = centroids.shape
        queries = _f32(queries).reshape(-1, m * dsub)
        lut = np.empty((queries.shape[0], m, 256), np.float32)
        self.lib.vko_compute_lut(centroids, m, dsub, queries, queries.shape[0], lut)
        return lut

    def adc_scan(self, lut, codes):
        lut = _f32(lut)
        codes = _u8(codes)
        nq, m = lut.shape[0], lut.shape[1]
        n = codes.shape[0]
        out = np.empty((nq, n), np.float32)
        self.lib.vko_adc_scan(lut, nq, codes, n, m, out)
        return out

    def select_topk(self, dists, k):
        dists = _f32(dists)
        nq, n = dists.shape
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        self.lib.vko_select_topk(dists, nq, n, k, d, i)
        return d, i

    def adc_search(self, centroids, codes, queries, k, threads=0):
        centroids = _f32(centroids)
        m, _, dsub = centroids.shape
        codes = _u8(codes)
        queries = _f32(queries).reshape(-1, m * dsub)
        nq = queries.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        self.lib.vko_adc_search(centroids, m, dsub, codes, codes.shape[0], queries, nq, k, d, i, threads)
        return d, i

    def compute_lut_h16(self, centroids, queries):
        """(tables [nq, m, 256]: the half-rounded, scaled entries as float32, exponents [nq] int32) of the
        half-precision LUT search."""
        centroids = _f32(centroids)
        m, ksub, dsub = centroids.shape
        queries = _f32(queries).reshape(-1, m * dsub)
        lut = np.empty((queries.shape[0], m, 256), np.float32)
        exps = np.empty(queries.shape[0], np.int32)
        self.lib.vko_compute_lut_h16(centroids, m, dsub, queries, queries.shape[0], lut, exps)
        return lut, exps

    def adc_search_h16(self, centroids, codes, queries, k, threads=0):
        """The half-precision LUT search (VK_LUT_F16 definition) -> (dists [nq, k], ids [nq, k])."""
        centroids = _f32(centroids)
        m, _, dsub = centroids.shape
        codes = _u8(codes)
        queries = _f32(queries).reshape(-1, m * dsub)
        nq = queries.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        self.lib.vko_adc_search_h16(centroids, m, dsub, codes, codes.shape[0], queries, nq, k, d, i, threads)
        return d, i

    def ivf_search(self, centroids, codes, list_of, coarse, queries, nprobe, k, threads=0):
        """IVF search (flat search over the rows of each query's nprobe nearest lists) -> (dists, ids, probes)."""
        centroids = _f32(centroids)
        m, _, dsub = centroids.shape
        codes = _u8(codes)
        list_of = np.ascontiguousarray(list_of, np.int32)
        coarse = _f32(coarse)
        queries = _f32(queries).reshape(-1, m * dsub)
        nq = queries.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        probes = np.empty((nq, nprobe), np.int32)
        self.lib.vko_ivf_search(centroids, m, dsub, codes, list_of, codes.shape[0], coarse, coarse.shape[0], queries,
                                nq, nprobe, k, d, i, probes, threads)
        return d, i, probes

    def pq4_encode(self, centroids, x):
        """4-bit codes [n, ceil(m / 2)] (first nearest of 16 centroids, sub-code s in nibble s % 2 of byte s / 2)."""
        centroids = _f32(centroids)
        m, _, dsub = centroids.shape
        x = _f32(x).reshape(-1, m * dsub)
        codes = np.empty((x.shape[0], (m + 1) // 2), np.uint8)
        self.lib.vko_pq4_encode(centroids, m, dsub, x, x.shape[0], codes)
        return codes

    def compute_lut_pq4(self, centroids, queries):
        centroids = _f32(centroids)
        m, _, dsub = centroids.shape
        queries = _f32(queries).reshape(-1, m * dsub)
        lut = np.empty((queries.shape[0], m, 16), np.float32)
        self.lib.vko_compute_lut_pq4(centroids, m, dsub, queries, queries.shape[0], lut)
        return lut

    def adc_search_pq4(self, centroids, codes, queries, k, threads=0):
        """The 4-bit PQ search (centroids [m, 16, dsub], packed codes) -> (dists [nq, k], ids [nq, k])."""
        centroids = _f32(centroids)
        m, _, dsub = centroids.shape
        codes = _u8(codes)
        queries = _f32(queries).reshape(-1, m * dsub)
        nq = queries.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        self.lib.vko_adc_search_pq4(centroids, m, dsub, codes, codes.shape[0], queries, nq, k, d, i, threads)
        return d, i

    def topk_push_all(self, dists, ids, k):
        dists = _f32(dists)
        ids = np.ascontiguousarray(ids, np.int32)
        d = np.empty(k, np.float32)
        i = np.empty(k, np.int32)
        self.lib.vko_topk_push_all(dists, ids, dists.shape[0], k, d, i)
        return d, i

    def merge_topk(self, d, ids, k):
        """d, ids: [nq, lists, k_in] -> the k best of the union per query."""
        d = _f32(d)
        ids = np.ascontiguousarray(ids, np.int32)
        nq, lists, k_in = d.shape
        od = np.empty((nq, k), np.float32)
        oi = np.empty((nq, k), np.int32)
        self.lib.vko_merge_topk(d, ids, lists, k_in, nq, k, od, oi)
        return od, oi

    def rerank_exact(self, base, queries, cand_ids, k):
        base = _f32(base)
        queries = _f32(queries)
        cand_ids = np.ascontiguousarray(cand_ids, np.int32)
        nq, r = cand_ids.shape
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        self.lib.vko_rerank_exact(base, base.shape[1], queries, nq, cand_ids, r, k, d, i)
        return d, i

    def recall_at_k(self, found, truth, k):
        found = np.ascontiguousarray(found, np.int32)
        truth = np.ascontiguousarray(truth, np.int32)
        return self.lib.vko_recall_at_k(found, found.shape[1], truth, truth.shape[1], found.shape[0], k)

    def stream_search(self, lut, code_blocks, k, threads=0):
        """code_blocks: iterable of (codes [count, m] uint8, id_base). Returns the top-k over all blocks."""
        lut = _f32(lut)
        nq, m = lut.shape[0], lut.shape[1]
        s = self.lib.vko_stream_create(lut, nq, m, k)
        try:
            for codes, base in code_blocks:
                codes = _u8(codes)
                self.lib.vko_stream_feed(s, codes, codes.shape[0], base, threads)
            d = np.empty((nq, k), np.float32)
            i = np.empty((nq, k), np.int32)
            self.lib.vko_stream_finish(s, d, i)
            return d, i
        finally:
            self.lib.vko_stream_destroy(s)


class Ref:
    """The reference's own CPU library (kind "reference"); present only where it was built."""

    def __init__(self, path: Path = REF_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: built by `make -C oracle ref` where the reference exists")
        L = self.lib = C.CDLL(str(path))
        L.ref_pq_create.argtypes = [_i64, _i64]
        L.ref_pq_create.restype = C.c_void_p
        L.ref_pq_destroy.argtypes = [C.c_void_p]
        L.ref_pq_train.argtypes = [C.c_void_p, _f32p, _i64, _i64, C.c_uint64]
        L.ref_pq_encode.argtypes = [C.c_void_p, _f32p, _i64, _u8p]
        L.ref_pq_decode.argtypes = [C.c_void_p, _u8p, _i64, _f32p]
        L.ref_pq_get_centroids.argtypes = [C.c_void_p, _f32p]
        L.ref_pq_set_centroids.argtypes = [C.c_void_p, _f32p]
        L.ref_compute_lut.argtypes = [C.c_void_p, _f32p, _i64, _f32p]
        L.ref_adc_scan.argtypes = [_f32p, _i64, _u8p, _i64, _i64, _f32p]
        L.ref_select_topk.argtypes = [_f32p, _i64, _i64, _i64, _f32p, _i32p]
        L.ref_adc_search.argtypes = [C.c_void_p, _u8p, _i64, _f32p, _i64, _i64, _f32p, _i32p]
        L.ref_exact_knn.argtypes = [_f32p, _i64, _f32p, _i64, _i64, _i64, _f32p, _i32p]
        L.ref_topk_push_all.argtypes = [_f32p, _i32p, _i64, _i64, _f32p, _i32p]
        L.ref_rerank_exact.argtypes = [_f32p, _i64, _f32p, _i64, _i32p, _i64, _i64, _f32p, _i32p]
        L.ref_synthetic_clustered.argtypes = [_i64, _i64, _i64, C.c_uint64, _f32p]
        L.ref_set_threads.argtypes = [C.c_int]
        L.ref_get_threads.restype = C.c_int

    def set_threads(self, n: int) -> int:
        """OpenMP threads of the reference's parallel loops (overrides an inherited OMP_NUM_THREADS); returns the
        count now in effect."""
        self.lib.ref_set_threads(int(n))
        return int(self.lib.ref_get_threads())

    class PQ:
        def __init__(self, lib, d, m):
            self.lib, self.d, self.m, self.dsub = lib, d, m, d // m
            self.h = lib.ref_pq_create(d, m)

        def __del__(self):
            if getattr(self, "h", None):
                self.lib.ref_pq_destroy(self.h)
                self.h = None

        def train(self, x, n, iters, seed=1):
            self.lib.ref_pq_train(self.h, _f32(x), n, iters, seed)

        def encode(self, x):
            x = _f32(x).reshape(-1, self.d)
            codes = np.empty((x.shape[0], self.m), np.uint8)
            self.lib.ref_pq_encode(self.h, x, x.shape[0], codes)
            return codes

        def decode(self, codes):
            codes = _u8(codes)
            x = np.empty((codes.shape[0], self.d), np.float32)
            self.lib.ref_pq_decode(self.h, codes, codes.shape[0], x)
            return x

        @property
        def centroids(self):
            c = np.empty((self.m, 256, self.dsub), np.float32)
            self.lib.ref_pq_get_centroids(self.h, c)
            return c

        @centroids.setter
        def centroids(self, c):
            self.lib.ref_pq_set_centroids(self.h, _f32(c))

    def pq(self, d, m):
        return Ref.PQ(self.lib, d, m)

    def compute_lut(self, pq, queries):
        queries = _f32(queries).reshape(-1, pq.d)
        lut = np.empty((queries.shape[0], pq.m, 256), np.float32)
        self.lib.ref_compute_lut(pq.h, queries, queries.shape[0], lut)
        return lut

    def adc_scan(self, lut, codes):
        lut = _f32(lut)
        codes = _u8(codes)
        out = np.empty((lut.shape[0], codes.shape[0]), np.float32)
        self.lib.ref_adc_scan(lut, lut.shape[0], codes, codes.shape[0], lut.shape[1], out)
        return out

    def select_topk(self, dists, k):
        dists = _f32(dists)
        d = np.empty((dists.shape[0], k), np.float32)
        i = np.empty((dists.shape[0], k), np.int32)
        self.lib.ref_select_topk(dists, dists.shape[0], dists.shape[1], k, d, i)
        return d, i

    def adc_search(self, pq, codes, queries, k):
        codes = _u8(codes)
        queries = _f32(queries).reshape(-1, pq.d)
        nq = queries.shape[0]
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        self.lib.ref_adc_search(pq.h, codes, codes.shape[0], queries, nq, k, d, i)
        return d, i

    def exact_knn(self, base, queries, k):
        base = _f32(base)
        queries = _f32(queries)
        nq, dim = queries.shape
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        self.lib.ref_exact_knn(base, base.shape[0], queries, nq, dim, k, d, i)
        return d, i

    def topk_push_all(self, dists, ids, k):
        d = np.empty(k, np.float32)
        i = np.empty(k, np.int32)
        self.lib.ref_topk_push_all(_f32(dists), np.ascontiguousarray(ids, np.int32), len(dists), k, d, i)
        return d, i

    def rerank_exact(self, base, queries, cand_ids, k):
        base = _f32(base)
        queries = _f32(queries)
        cand_ids = np.ascontiguousarray(cand_ids, np.int32)
        nq, r = cand_ids.shape
        d = np.empty((nq, k), np.float32)
        i = np.empty((nq, k), np.int32)
        self.lib.ref_rerank_exact(base, base.shape[1], queries, nq, cand_ids, r, k, d, i)
        return d, i

    def synthetic_clustered(self, n, d, clusters, seed):
        out = np.empty((n, d), np.float32)
        self.lib.ref_synthetic_clustered(n, d, clusters, seed, out)
        return out


_port = None
_ref = None


def port() -> Port:
    global _port
    if _port is None:
        _port = Port()
    return _port


def ref_available() -> bool:
    return REF_SO.exists()


def ref() -> Ref:
    global _ref
    if _ref is None:
        _ref = Ref()
    return _ref


def set_threads(n: int) -> None:
    os.environ["OMP_NUM_THREADS"] = str(n)


REFGPU_SO = HERE / "_ref" / "libveckern_refgpu.so"


def refgpu_available() -> bool:
    return REFGPU_SO.exists()


def refgpu_sweep(centroids, codes, queries, k, points, reps=5):
    """The reference's own v8 kernel (FusedWarp through its veckern::gpu::PQSearcher, compiled for sm_100a) on
    these inputs: for each (queries_per_block, ilp) in `points`, median stage times of `reps` searches after one
    warm-up. Returns (rows: list of dicts, (dists, ids) of the first point)."""
    L = C.CDLL(str(REFGPU_SO))
    L.refgpu_sweep.argtypes = [_f32p, _i64, _i64, _u8p, _i64, _f32p, _i64, _i64, _i32p, _i32p, C.c_int, C.c_int,
                               np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS"), _f32p, _i32p]
    L.refgpu_last_error.restype = C.c_char_p
    centroids = _f32(centroids)
    m, _, dsub = centroids.shape
    codes = _u8(codes)
    queries = _f32(queries).reshape(-1, m * dsub)
    nq = queries.shape[0]
    qs = np.array([p[0] for p in points], np.int32)
    ilps = np.array([p[1] for p in points], np.int32)
    out = np.zeros((len(points), 10), np.float64)
    d = np.empty((nq, k), np.float32)
    i = np.empty((nq, k), np.int32)
    if L.refgpu_sweep(centroids, m * dsub, m, codes, codes.shape[0], queries, nq, k, qs, ilps, len(points), reps,
                      out, d, i) != 0:
        raise RuntimeError("reference GPU search failed: " + L.refgpu_last_error().decode(errors="replace"))
    keys = ("total_ms", "transfer_ms", "lut_ms", "scan_ms", "select_ms", "threads", "blocks_x", "grid_y",
            "queries_per_block", "vectors_per_step")
    return [dict(zip(keys, (float(x) for x in row))) for row in out], (d, i)
