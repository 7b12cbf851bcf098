"""ctypes bindings for the in-tree native libraries (include/vk_abi.h, include/vk_host.h).

The CUDA library must exist: there is no Python or CPU fallback for the search path. Importing this module on a
machine without the built library raises immediately with the build command to run.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

NATIVE = Path(__file__).resolve().parent / "_native"
LIB_PATH = NATIVE / "libveckern_b200.so"
HOST_LIB_PATH = NATIVE / "libveckern_b200_host.so"

VK_OK = 0
VK_ERR_INVALID = -1
VK_ERR_CUDA = -2
VK_ERR_NOMEM = -3
VK_ERR_DEVICE = -4
VK_ERR_UNSUPPORTED = -5


class VkError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{msg} (status {code})")
        self.code = code


class DeviceInfo(C.Structure):
    _fields_ = [("name", C.c_char * 256), ("sm_count", C.c_int), ("peak_bandwidth_gbs", C.c_double),
                ("max_smem_per_block", C.c_size_t), ("clock_mhz", C.c_int)]


class Tuning(C.Structure):
    _fields_ = [("scan_threads", C.c_int), ("blocks_per_query", C.c_int), ("queries_per_block", C.c_int),
                ("vectors_per_step", C.c_int), ("early_abandon", C.c_int), ("lut_precision", C.c_int)]


VK_LUT_F32 = 0
VK_LUT_F16 = 1


class Timings(C.Structure):
    _fields_ = [("transfer_ms", C.c_double), ("lut_ms", C.c_double), ("scan_ms", C.c_double),
                ("select_ms", C.c_double)]


class LaunchShape(C.Structure):
    _fields_ = [("threads", C.c_int), ("blocks_x", C.c_int), ("grid_y", C.c_int), ("queries_per_block", C.c_int),
                ("vectors_per_step", C.c_int), ("blocks_per_sm", C.c_int), ("waves", C.c_double)]


# (dist, id) pairs: the reference's Neighbor layout
NEIGHBOR_DTYPE = np.dtype([("dist", "<f4"), ("id", "<i4")])

_vp = C.c_void_p
_i64 = C.c_int64
_u64 = C.c_uint64

# name -> (restype, argtypes); every function declared in include/vk_abi.h
ABI = {
    "vk_device_info": (C.c_int, [C.c_int, C.POINTER(DeviceInfo)]),
    "vk_last_error": (C.c_size_t, [C.c_char_p, C.c_size_t]),
    "vk_tuning_default": (None, [C.POINTER(Tuning)]),
    "vk_tuning_validate": (C.c_int, [C.POINTER(Tuning)]),
    "vk_index_create": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _vp, _i64, _i64, C.POINTER(_vp)]),
    "vk_index_create_pq4": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _vp, _i64, _i64, C.POINTER(_vp)]),
    "vk_index_bits": (C.c_int, [_vp, C.POINTER(C.c_int)]),
    "vk_index_create_from_device": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _vp, _i64, _i64, C.POINTER(_vp)]),
    "vk_index_create_generated": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _u64, _vp, C.c_int, _i64, _i64, _i64,
                                            C.POINTER(_vp)]),
    "vk_index_destroy": (C.c_int, [_vp]),
    "vk_index_info": (C.c_int, [_vp, C.POINTER(_i64), C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(_i64),
                                C.POINTER(C.c_int)]),
    "vk_index_get_codes": (C.c_int, [_vp, _i64, _i64, _vp]),
    "vk_index_get_placement": (C.c_int, [_vp, _i64, _i64, _vp]),
    "vk_index_save": (C.c_int, [_vp, C.c_char_p]),
    "vk_multi_create": (C.c_int, [C.c_int, _vp, _vp, C.c_int, C.c_int, _vp, _i64, C.POINTER(_vp)]),
    "vk_multi_load": (C.c_int, [C.c_int, _vp, C.c_char_p, C.c_int, C.POINTER(_vp)]),
    "vk_multi_search": (C.c_int, [_vp, _vp, _i64, C.c_int, C.POINTER(Tuning), _vp, C.POINTER(Timings)]),
    "vk_multi_info": (C.c_int, [_vp, C.POINTER(_i64), C.POINTER(C.c_int)]),
    "vk_multi_destroy": (C.c_int, [_vp]),
    "vk_index_load": (C.c_int, [C.c_int, C.c_char_p, _i64, _i64, _i64, C.c_int, C.POINTER(_vp)]),
    "vk_search": (C.c_int, [_vp, _vp, _i64, C.c_int, C.c_int, C.POINTER(Tuning), _vp, C.POINTER(Timings),
                            C.POINTER(LaunchShape)]),
    "vk_search_device": (C.c_int, [_vp, _vp, _i64, C.c_int, C.POINTER(Tuning), _vp, _vp]),
    "vk_index_sync": (C.c_int, [_vp, _vp]),
    "vk_distances": (C.c_int, [_vp, _vp, _i64, C.c_int, C.POINTER(Tuning), _vp, C.POINTER(Timings)]),
    "vk_compute_lut_device": (C.c_int, [_vp, _vp, _i64, _vp, _vp]),
    "vk_merge_topk_device": (C.c_int, [C.c_int, _vp, _i64, C.c_int, C.c_int, _i64, _i64, C.c_int, _vp, _vp]),
    "vk_rerank_device": (C.c_int, [C.c_int, _vp, _i64, C.c_int, _vp, _i64, _vp, C.c_int, C.c_int, _vp, _vp]),
    "vk_encode_device": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _vp, _i64, _vp, _vp]),
    "vk_pq_train_device": (C.c_int, [C.c_int, _vp, _i64, C.c_int, C.c_int, _i64, _u64, _vp, _vp]),
    "vk_gen_codes_device": (C.c_int, [C.c_int, _u64, _vp, C.c_int, C.c_int, _i64, _i64, _vp, _vp]),
    "vk_search_noalloc": (C.c_int, [_vp, _vp, _i64, C.c_int, C.POINTER(Tuning), _vp, _vp]),
    "vk_coop_create": (C.c_int, [C.c_int, _i64, C.POINTER(_vp)]),
    "vk_coop_ipc_handle": (C.c_int, [_vp, _vp]),
    "vk_coop_attach_ipc": (C.c_int, [_vp, C.c_int, _vp]),
    "vk_coop_attach": (C.c_int, [_vp, C.c_int, _vp]),
    "vk_coop_destroy": (C.c_int, [_vp]),
    "vk_search_device_coop": (C.c_int, [_vp, _vp, C.c_uint32, _vp, _i64, C.c_int, C.POINTER(Tuning), _vp, _vp]),
    "vk_ivf_create": (C.c_int, [C.c_int, _vp, C.c_int, C.c_int, _vp, _i64, _vp, C.c_int, _vp, C.POINTER(_vp)]),
    "vk_ivf_destroy": (C.c_int, [_vp]),
    "vk_ivf_info": (C.c_int, [_vp, C.POINTER(_i64), C.POINTER(C.c_int), C.POINTER(_i64)]),
    "vk_ivf_search": (C.c_int, [_vp, _vp, _i64, C.c_int, C.c_int, C.POINTER(Tuning), _vp, C.POINTER(Timings)]),
    "vk_ivf_search_device": (C.c_int, [_vp, _vp, _i64, C.c_int, C.c_int, C.POINTER(Tuning), _vp, _vp]),
    "vk_ivf_sync": (C.c_int, [_vp, _vp]),
    "vk_ivf_assign_device": (C.c_int, [C.c_int, _vp, _i64, C.c_int, _vp, C.c_int, _vp, _vp]),
}
COOP_HANDLE_BYTES = 80  # VK_COOP_HANDLE_BYTES
NOALLOC_SCRATCH_BYTES = 32 << 20  # VK_NOALLOC_SCRATCH_BYTES

HOST_ABI = {
    "vk_host_pq_train": (C.c_int, [_vp, _i64, C.c_int, C.c_int, _i64, _u64, _vp]),
    "vk_host_pq_encode": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _i64, _vp]),
    "vk_host_pq_decode": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _i64, _vp]),
    "vk_host_pq4_train": (C.c_int, [_vp, _i64, C.c_int, C.c_int, _i64, _u64, _vp]),
    "vk_host_pq4_encode": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _i64, _vp]),
    "vk_host_synthetic_clustered": (C.c_int, [_i64, C.c_int, _i64, _u64, _vp]),
    "vk_host_gen_normal": (C.c_int, [_u64, _i64, _i64, C.c_int, _vp]),
    "vk_host_gen_mixture": (C.c_int, [_u64, C.c_int, C.c_float, _u64, _i64, _i64, C.c_int, _vp]),
    "vk_host_gen_cdf": (C.c_int, [_u64, C.c_int, C.c_int, C.c_double, _vp]),
    "vk_host_gen_codes": (C.c_int, [_u64, _vp, C.c_int, C.c_int, _i64, _i64, _vp]),
    "vk_host_gen_codes_rows": (C.c_int, [_u64, _vp, C.c_int, C.c_int, _vp, _i64, _vp]),
    "vk_host_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "vk_host_crc32c": (C.c_uint32, [_vp, C.c_size_t, C.c_int]),
    "vk_host_index_write": (C.c_int, [C.c_char_p, _vp, C.c_int, C.c_int, _vp, _i64]),
    "vk_host_index_info": (C.c_int, [C.c_char_p, C.POINTER(_i64), C.POINTER(C.c_int), C.POINTER(C.c_int),
                                     C.POINTER(C.c_int)]),
    "vk_host_index_read": (C.c_int, [C.c_char_p, _vp, _i64, _i64, _vp, C.c_int]),
}

_lib = None
_host = None


def _bind(lib, table):
    for name, (res, args) in table.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


def lib():
    """The CUDA library (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m veckern_b200.build`")
        _lib = _bind(C.CDLL(str(LIB_PATH)), ABI)
    return _lib


def host():
    global _host
    if _host is None:
        if not HOST_LIB_PATH.exists():
            raise RuntimeError(f"{HOST_LIB_PATH} is missing: run `python -m veckern_b200.build`")
        _host = _bind(C.CDLL(str(HOST_LIB_PATH)), HOST_ABI)
    return _host


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    lib().vk_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(code: int, what: str = "") -> None:
    if code != VK_OK:
        raise VkError(code, f"{what}: {last_error()}" if what else last_error())


def ptr(a) -> C.c_void_p:
    """Address of a numpy array or a torch tensor."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return C.c_void_p(a.ctypes.data)
