"""Python mirror of the reference's GPU search API (include/veckern/gpu.hpp of shivdeshpande/VecKern) over the
C ABI: same names, argument meaning and errors (VkError, a RuntimeError, where the reference throws
std::runtime_error).

    searcher = PQSearcher(centroids, codes)                   # centroids [m, 256, dsub] f32, codes [n, m] u8
    searcher = PQSearcher(centroids4, codes4)                 # 4-bit PQ: [m, 16, dsub] f32, codes [n, m / 2] u8
    timings = searcher.search(queries, k, ScanVariant.FusedWarp, out)   # out: [nq, k] NEIGHBOR_DTYPE
    dist, ids = neighbors_split(out)
"""
from __future__ import annotations

import ctypes as C
import enum
from dataclasses import dataclass

import numpy as np

from . import _native as N
from ._native import NEIGHBOR_DTYPE, VkError, check, lib, ptr


class ScanVariant(enum.IntEnum):
    """include/veckern/gpu.hpp:13-23 of the reference; here only validation rules differ between them."""
    GlobalLut = 0
    SharedLut = 1
    SharedLutVec = 2
    Interleaved = 3
    Fused = 4
    FusedReg = 5
    FusedVec = 6
    FusedVecMQ = 7
    FusedWarp = 8


_VARIANT_NAMES = ["v0_global_lut", "v1_shared_lut", "v2_shared_lut_vec", "v3_interleaved", "v4_fused",
                  "v5_fused_reg", "v6_fused_vec", "v7_fused_vec_mq", "v8_fused_warp"]


def variant_name(v: ScanVariant) -> str:
    return _VARIANT_NAMES[int(v)]


def is_fused(v: ScanVariant) -> bool:
    return ScanVariant.Fused <= v <= ScanVariant.FusedWarp


@dataclass
class Tuning:
    """include/veckern/gpu.hpp:29-34 of the reference (same defaults and accepted values)."""
    scan_threads: int = 256
    blocks_per_query: int = 0
    queries_per_block: int = 2
    vectors_per_step: int = 4
    early_abandon: bool = True  # exact pruning by partial sums (results identical); False = full scan
    lut_f16: bool = False       # half-precision LUTs (vk_abi.h VK_LUT_F16: an approximate search, exactly defined)

    def c(self) -> N.Tuning:
        return N.Tuning(self.scan_threads, self.blocks_per_query, self.queries_per_block, self.vectors_per_step,
                        int(self.early_abandon), N.VK_LUT_F16 if self.lut_f16 else N.VK_LUT_F32)


@dataclass
class Timings:
    transfer_ms: float = 0.0
    lut_ms: float = 0.0
    scan_ms: float = 0.0
    select_ms: float = 0.0

    def kernel_ms(self) -> float:
        return self.lut_ms + self.scan_ms + self.select_ms

    def total_ms(self) -> float:
        return self.transfer_ms + self.kernel_ms()


@dataclass
class LaunchShape:
    threads: int = 0
    blocks_x: int = 0
    grid_y: int = 0
    queries_per_block: int = 1
    vectors_per_step: int = 1
    blocks_per_sm: int = 0
    waves: float = 0.0


@dataclass
class DeviceInfo:
    name: str
    sm_count: int
    peak_bandwidth_gbs: float
    max_smem_per_block: int
    clock_mhz: int


def device_info(device: int = 0) -> DeviceInfo:
    d = N.DeviceInfo()
    check(lib().vk_device_info(device, C.byref(d)), "vk_device_info")
    return DeviceInfo(d.name.decode(), d.sm_count, d.peak_bandwidth_gbs, d.max_smem_per_block, d.clock_mhz)


def neighbors_split(out: np.ndarray):
    """(dist float32 [..., k], ids int32 [..., k]) views of a NEIGHBOR_DTYPE array."""
    return out["dist"], out["id"]


def empty_neighbors(nq: int, k: int) -> np.ndarray:
    return np.empty((nq, k), NEIGHBOR_DTYPE)


class PQSearcher:
    """One PQ code database resident on one GPU (include/veckern/gpu.hpp:53-78 of the reference)."""

    def __init__(self, centroids, codes=None, *, device: int = 0, id_base: int = 0, _handle=None):
        self._h = C.c_void_p()
        self.tuning = Tuning()
        self.last = LaunchShape()
        if _handle is not None:
            self._h = _handle
        else:
            centroids = np.ascontiguousarray(centroids, np.float32)
            if centroids.ndim != 3 or centroids.shape[1] not in (16, 256):
                raise ValueError("centroids must be [m, 256, dsub] (8-bit codes) or [m, 16, dsub] (4-bit codes) float32")
            m, ksub, dsub = centroids.shape
            if ksub == 16:  # 4-bit PQ: codes [n, m / 2], sub-code s in nibble s % 2 (low first) of byte s / 2
                codes = np.ascontiguousarray(codes, np.uint8)
                if codes.ndim != 2 or codes.shape[1] != (m + 1) // 2:
                    raise ValueError("4-bit codes must be [n, ceil(m / 2)] uint8 (two sub-codes per byte)")
                check(lib().vk_index_create_pq4(device, ptr(centroids), m, dsub, ptr(codes), codes.shape[0], id_base,
                                                C.byref(self._h)), "vk_index_create_pq4")
            elif hasattr(codes, "data_ptr"):  # torch tensor already on the device
                n = codes.shape[0]
                check(lib().vk_index_create_from_device(device, ptr(centroids), m, dsub, ptr(codes), n, id_base,
                                                        C.byref(self._h)), "vk_index_create_from_device")
            else:
                codes = np.ascontiguousarray(codes, np.uint8)
                if codes.ndim != 2 or codes.shape[1] != m:
                    raise ValueError("codes must be [n, m] uint8")
                check(lib().vk_index_create(device, ptr(centroids), m, dsub, ptr(codes), codes.shape[0], id_base,
                                            C.byref(self._h)), "vk_index_create")
        n, m, dsub, base, dev = C.c_int64(), C.c_int(), C.c_int(), C.c_int64(), C.c_int()
        check(lib().vk_index_info(self._h, C.byref(n), C.byref(m), C.byref(dsub), C.byref(base), C.byref(dev)))
        self.n, self.m, self.dsub, self.id_base, self.device = n.value, m.value, dsub.value, base.value, dev.value
        self.d = self.m * self.dsub
        bits = C.c_int()
        check(lib().vk_index_bits(self._h, C.byref(bits)))
        self.nbits = bits.value  # 8, or 4 for 4-bit PQ

    @classmethod
    def generated(cls, centroids, seed: int, cdf: np.ndarray, row_first: int, n: int, *, device: int = 0,
                  id_base: int = 0) -> "PQSearcher":
        """Codes generated on the device (rows [row_first, row_first + n) of the config-3/4 generator)."""
        centroids = np.ascontiguousarray(centroids, np.float32)
        cdf = np.ascontiguousarray(cdf, np.uint32)
        m, _, dsub = centroids.shape
        h = C.c_void_p()
        check(lib().vk_index_create_generated(device, ptr(centroids), m, dsub, seed, ptr(cdf), cdf.shape[0],
                                              row_first, n, id_base, C.byref(h)), "vk_index_create_generated")
        return cls(None, _handle=h)

    @classmethod
    def load(cls, path: str, *, rows: tuple[int, int] | None = None, id_base: int | None = None, device: int = 0,
             verify: bool = True) -> "PQSearcher":
        """An index built from rows [lo, hi) (default: all) of a persisted index file (vk_index_load); ids default
        to the file's row numbers. Reads only that range: each shard of a multi-GPU search loads its own rows."""
        lo, hi = rows if rows is not None else (0, -1)
        h = C.c_void_p()
        count = -1 if hi < 0 else hi - lo
        check(lib().vk_index_load(device, str(path).encode(), lo, count, -1 if id_base is None else id_base,
                                  int(verify), C.byref(h)), "vk_index_load")
        return cls(None, _handle=h)

    def save(self, path: str) -> None:
        """Writes the centroids and the codes (row order) to a persisted index file (vk_index_save)."""
        check(lib().vk_index_save(self._h, str(path).encode()), "vk_index_save")

    def close(self) -> None:
        if self._h:
            lib().vk_index_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_tuning(self, tuning: Tuning) -> None:
        t = tuning.c()
        check(lib().vk_tuning_validate(C.byref(t)), "set_tuning")
        self.tuning = tuning

    def last_launch(self) -> LaunchShape:
        return self.last

    def search(self, queries, k: int, variant: ScanVariant = ScanVariant.FusedWarp, out: np.ndarray | None = None):
        """HOST queries [nq, d] -> HOST results [nq, k] (NEIGHBOR_DTYPE). Returns (out, Timings)."""
        queries = np.ascontiguousarray(queries, np.float32).reshape(-1, self.d)
        nq = queries.shape[0]
        if out is None:
            out = empty_neighbors(nq, k)
        if out.dtype != NEIGHBOR_DTYPE or out.size != nq * k or not out.flags.c_contiguous:
            raise ValueError("out must be a C-contiguous [nq, k] NEIGHBOR_DTYPE array")
        t, s, tun = N.Timings(), N.LaunchShape(), self.tuning.c()
        check(lib().vk_search(self._h, ptr(queries), nq, k, int(variant), C.byref(tun), ptr(out), C.byref(t),
                              C.byref(s)), "search")
        if nq:
            self.last = LaunchShape(s.threads, s.blocks_x, s.grid_y, s.queries_per_block, s.vectors_per_step,
                                    s.blocks_per_sm, s.waves)
        return out, Timings(t.transfer_ms, t.lut_ms, t.scan_ms, t.select_ms)

    def distances(self, queries, variant: ScanVariant = ScanVariant.SharedLut, out: np.ndarray | None = None):
        """HOST queries -> HOST [nq, n] float32 ADC distances (unfused variants only)."""
        queries = np.ascontiguousarray(queries, np.float32).reshape(-1, self.d)
        nq = queries.shape[0]
        if out is None:
            out = np.empty((nq, self.n), np.float32)
        t, tun = N.Timings(), self.tuning.c()
        check(lib().vk_distances(self._h, ptr(queries), nq, int(variant), C.byref(tun), ptr(out), C.byref(t)),
              "distances")
        return out, Timings(t.transfer_ms, t.lut_ms, t.scan_ms, t.select_ms)

    # ---- device-resident path (torch tensors on this index's device)
    def search_device(self, d_queries, k: int, d_out, stream=None, tuning: Tuning | None = None) -> None:
        """DEVICE queries (torch float32 [nq, d]) -> DEVICE results (torch int64 [nq, k] holding (dist, id)
        pairs; see device_result_split). Asynchronous on `stream` (a torch.cuda.Stream; default: current)."""
        nq = d_queries.shape[0]
        tun = (tuning or self.tuning).c()
        s = _stream_handle(stream)
        check(lib().vk_search_device(self._h, ptr(d_queries), nq, k, C.byref(tun), ptr(d_out), s), "search_device")

    def search_device_coop(self, coop: "CoopSearch", epoch: int, d_queries, k: int, d_out, stream=None,
                           tuning: Tuning | None = None) -> None:
        """search_device as one shard of a cooperative sharded search (vk_search_device_coop): the lists are exact
        only once merged with the other shards' lists of the same epoch."""
        nq = d_queries.shape[0]
        tun = (tuning or self.tuning).c()
        check(lib().vk_search_device_coop(self._h, coop._h, epoch, ptr(d_queries), nq, k, C.byref(tun), ptr(d_out),
                                          _stream_handle(stream)), "search_device_coop")

    def sync(self, stream=None) -> None:
        check(lib().vk_index_sync(self._h, _stream_handle(stream)), "sync")

    def compute_lut_device(self, d_queries, d_lut, stream=None) -> None:
        check(lib().vk_compute_lut_device(self._h, ptr(d_queries), d_queries.shape[0], ptr(d_lut),
                                          _stream_handle(stream)), "compute_lut")

    def get_codes(self, first: int = 0, count: int | None = None) -> np.ndarray:
        count = self.n - first if count is None else count
        out = np.empty((count, self.m), np.uint8)
        check(lib().vk_index_get_codes(self._h, first, count, ptr(out)), "get_codes")
        return out

    def get_placement(self, count: int | None = None) -> np.ndarray:
        """uint8 per position of the device layout (the first `count`, default all n_pad): the row, within its
        64-position window, stored there."""
        n_pad = (self.n + 127) // 128 * 128
        count = n_pad if count is None else min(n_pad, count)
        out = np.empty(count, np.uint8)
        check(lib().vk_index_get_placement(self._h, 0, count, ptr(out)), "get_placement")
        return out


class IVFSearcher:
    """IVF (inverted-file) PQ search on one GPU (vk_ivf_*, include/vk_abi.h): the flat search restricted to the rows
    of each query's nprobe nearest lists. list_of: the list of each row (e.g. assign_lists)."""

    def __init__(self, centroids, codes, coarse, list_of, *, device: int = 0):
        centroids = np.ascontiguousarray(centroids, np.float32)
        codes = np.ascontiguousarray(codes, np.uint8)
        coarse = np.ascontiguousarray(coarse, np.float32)
        list_of = np.ascontiguousarray(list_of, np.int32)
        m, _, dsub = centroids.shape
        if codes.ndim != 2 or codes.shape[1] != m or list_of.shape != (codes.shape[0],):
            raise ValueError("codes must be [n, m] uint8 and list_of [n] int32")
        if coarse.ndim != 2 or coarse.shape[1] != m * dsub:
            raise ValueError("coarse must be [nlist, d] float32")
        self._h = C.c_void_p()
        check(lib().vk_ivf_create(device, ptr(centroids), m, dsub, ptr(codes), codes.shape[0], ptr(coarse),
                                  coarse.shape[0], ptr(list_of), C.byref(self._h)), "vk_ivf_create")
        self.d, self.device, self.nlist, self.n = m * dsub, device, coarse.shape[0], codes.shape[0]
        self.tuning = Tuning(queries_per_block=8, vectors_per_step=2)

    def set_tuning(self, tuning: Tuning) -> None:
        t = tuning.c()
        check(lib().vk_tuning_validate(C.byref(t)), "set_tuning")
        self.tuning = tuning

    def search(self, queries, k: int, nprobe: int, out: np.ndarray | None = None):
        """HOST queries [nq, d] -> HOST results [nq, k] (NEIGHBOR_DTYPE). Returns (out, Timings)."""
        queries = np.ascontiguousarray(queries, np.float32).reshape(-1, self.d)
        nq = queries.shape[0]
        if out is None:
            out = empty_neighbors(nq, k)
        t, tun = N.Timings(), self.tuning.c()
        check(lib().vk_ivf_search(self._h, ptr(queries), nq, k, nprobe, C.byref(tun), ptr(out), C.byref(t)),
              "ivf_search")
        return out, Timings(t.transfer_ms, t.lut_ms, t.scan_ms, t.select_ms)

    def search_device(self, d_queries, k: int, nprobe: int, d_out, stream=None) -> None:
        tun = self.tuning.c()
        check(lib().vk_ivf_search_device(self._h, ptr(d_queries), d_queries.shape[0], k, nprobe, C.byref(tun),
                                         ptr(d_out), _stream_handle(stream)), "ivf_search_device")

    def sync(self, stream=None) -> None:
        check(lib().vk_ivf_sync(self._h, _stream_handle(stream)), "ivf_sync")

    def close(self) -> None:
        if self._h:
            lib().vk_ivf_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def assign_lists(x, coarse, device: int = 0) -> np.ndarray:
    """The nearest coarse centroid of each row of x (vk_ivf_assign_device: exact l2sq, first minimum wins)."""
    import torch

    coarse = np.ascontiguousarray(coarse, np.float32)
    with torch.cuda.device(device):
        dc = torch.from_numpy(coarse).cuda()
        out = np.empty(x.shape[0], np.int32)
        step = 1 << 20
        for a in range(0, x.shape[0], step):
            xs = torch.from_numpy(np.ascontiguousarray(x[a:a + step], np.float32)).cuda()
            o = torch.empty(xs.shape[0], dtype=torch.int32, device="cuda")
            check(lib().vk_ivf_assign_device(device, ptr(xs), xs.shape[0], xs.shape[1], ptr(dc), coarse.shape[0],
                                             ptr(o), torch.cuda.current_stream().cuda_stream), "ivf_assign")
            out[a:a + xs.shape[0]] = o.cpu().numpy()
    return out


class CoopSearch:
    """The pruning-bound exchange of one shard of a cooperative sharded search (vk_coop_*, include/vk_abi.h)."""

    def __init__(self, device: int, nq_max: int):
        self._h = C.c_void_p()
        check(lib().vk_coop_create(device, nq_max, C.byref(self._h)), "vk_coop_create")

    def ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(N.COOP_HANDLE_BYTES)
        check(lib().vk_coop_ipc_handle(self._h, buf), "vk_coop_ipc_handle")
        return buf.raw

    def attach_ipc(self, handles) -> None:
        """Maps the other shards' exchange arrays from their handles (all shards' handles, this one's included)."""
        blob = b"".join(handles)
        check(lib().vk_coop_attach_ipc(self._h, len(handles), C.c_char_p(blob)), "vk_coop_attach_ipc")

    def attach(self, coops) -> None:
        """The same for shards in this process."""
        arr = (C.c_void_p * len(coops))(*[c._h for c in coops])
        check(lib().vk_coop_attach(self._h, len(coops), arr), "vk_coop_attach")

    def close(self) -> None:
        if self._h:
            lib().vk_coop_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MultiPQSearcher:
    """One database split into contiguous row shards over several GPUs of this process (vk_multi_*): every shard
    searches on its own device and stream, the per-shard lists are gathered and merged on devices[0]. Results are
    identical to one PQSearcher over all rows."""

    def __init__(self, centroids, codes=None, *, devices=(0,), _handle=None):
        self._h = C.c_void_p()
        self.tuning = Tuning()
        if _handle is not None:
            self._h = _handle
        else:
            centroids = np.ascontiguousarray(centroids, np.float32)
            codes = np.ascontiguousarray(codes, np.uint8)
            m, _, dsub = centroids.shape
            if codes.ndim != 2 or codes.shape[1] != m:
                raise ValueError("codes must be [n, m] uint8")
            devs = np.ascontiguousarray(devices, np.int32)
            check(lib().vk_multi_create(len(devs), ptr(devs), ptr(centroids), m, dsub, ptr(codes), codes.shape[0],
                                        C.byref(self._h)), "vk_multi_create")
        n, shards = C.c_int64(), C.c_int()
        check(lib().vk_multi_info(self._h, C.byref(n), C.byref(shards)))
        self.n, self.shards = n.value, shards.value

    @classmethod
    def load(cls, path: str, *, devices=(0,), verify: bool = True) -> "MultiPQSearcher":
        devs = np.ascontiguousarray(devices, np.int32)
        h = C.c_void_p()
        check(lib().vk_multi_load(len(devs), ptr(devs), str(path).encode(), int(verify), C.byref(h)), "vk_multi_load")
        return cls(None, _handle=h)

    def set_tuning(self, tuning: Tuning) -> None:
        t = tuning.c()
        check(lib().vk_tuning_validate(C.byref(t)), "set_tuning")
        self.tuning = tuning

    def search(self, queries, k: int, out: np.ndarray | None = None):
        """HOST queries [nq, d] -> HOST results [nq, k] (NEIGHBOR_DTYPE), Timings."""
        queries = np.ascontiguousarray(queries, np.float32)
        queries = queries.reshape(-1, queries.shape[-1]) if queries.ndim > 1 else queries.reshape(1, -1)
        nq = queries.shape[0]
        if out is None:
            out = empty_neighbors(nq, k)
        t, tun = N.Timings(), self.tuning.c()
        check(lib().vk_multi_search(self._h, ptr(queries), nq, k, C.byref(tun), ptr(out), C.byref(t)), "multi search")
        return out, Timings(t.transfer_ms, t.lut_ms, t.scan_ms, t.select_ms)

    def close(self) -> None:
        if self._h:
            lib().vk_multi_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _stream_handle(stream):
    """cudaStream_t of a torch.cuda.Stream / raw handle; None -> torch's current stream (0 = default stream)."""
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return C.c_void_p(getattr(stream, "cuda_stream", stream))


def device_result_split(d_out):
    """(dist float32, ids int32) views of a torch int64 [nq, k] device result."""
    import torch
    v = d_out.view(torch.int32).view(*d_out.shape, 2)
    return v[..., 0].view(torch.float32), v[..., 1]


def merge_topk_device(device: int, d_in, nq: int, lists: int, k_in: int, query_stride: int, list_stride: int,
                      k: int, d_out, stream=None) -> None:
    """k best of `lists` sorted candidate lists per query, all in device memory ((dist, id) int64 pairs)."""
    check(lib().vk_merge_topk_device(device, ptr(d_in), nq, lists, k_in, query_stride, list_stride, k, ptr(d_out),
                                     _stream_handle(stream)), "merge_topk")


def rerank_device(device: int, d_base, d_queries, d_candidates, k: int, d_out, stream=None) -> None:
    """Exact re-rank on the GPU (the reference's rerank_exact): torch tensors d_base [n, d] f32, d_queries [nq, d]
    f32, d_candidates [nq, r] int64 (dist, id) pairs (ids < 0 skipped), d_out [nq, k] int64 pairs."""
    nq, r = d_candidates.shape
    check(lib().vk_rerank_device(device, ptr(d_base), d_base.shape[0], d_base.shape[1], ptr(d_queries), nq,
                                 ptr(d_candidates), r, k, ptr(d_out), _stream_handle(stream)), "rerank")


__all__ = ["rerank_device", "ScanVariant", "Tuning", "Timings", "LaunchShape", "DeviceInfo", "PQSearcher", "VkError",
           "NEIGHBOR_DTYPE", "device_info", "variant_name", "is_fused", "neighbors_split", "empty_neighbors",
           "device_result_split", "merge_topk_device"]
