"""GPU: vk_search_noalloc, the search entry point that allocates nothing.

It is for callers that must not call cudaMalloc/cudaFree during a search (an allocation can synchronise the
device and stall other streams, or the process has handed its memory to its own allocator): its working memory is
one fixed array inside the library. Called through the C ABI, its results must equal the allocating device-path
entry point's exactly (the same bit-exact contract), on two calls in a row, because the array keeps the previous
call's contents; the second call must leave the device's free memory unchanged. This file is collected last on
purpose.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_same_topk
from veckern_b200 import PQSearcher, Tuning, device_result_split
from veckern_b200 import _native as N

pytestmark = pytest.mark.gpu


def _noalloc(s, d_q, k, tuning, d_out):
    t = tuning.c()
    return N.lib().vk_search_noalloc(s._h, N.ptr(d_q), d_q.shape[0], k, C.byref(t), N.ptr(d_out), None)


def test_noalloc_matches_allocating_entry_point_twice(golden):
    import torch

    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        d_q = torch.from_numpy(g["queries"]).cuda()
        # two different calls in a row: the second must not see the first call's leftovers
        for k, tuning in ((100, Tuning(queries_per_block=8)), (10, Tuning(queries_per_block=4)),
                          (10, Tuning(queries_per_block=4, early_abandon=False))):
            ref = torch.empty((d_q.shape[0], k), dtype=torch.int64, device="cuda")
            s.search_device(d_q, k, ref, None, tuning=tuning)
            s.sync(None)
            rd, ri = (x.cpu().numpy() for x in device_result_split(ref))
            outs = [torch.full((d_q.shape[0], k), -1, dtype=torch.int64, device="cuda") for _ in range(2)]
            torch.cuda.synchronize()
            for call in range(2):
                free_before = torch.cuda.mem_get_info()[0]
                assert _noalloc(s, d_q, k, tuning, outs[call]) == N.VK_OK, N.last_error()
                if call == 1:  # after the first call (kernel code loaded), a call takes no device memory
                    assert torch.cuda.mem_get_info()[0] == free_before, "vk_search_noalloc changed free memory"
                od, oi = (x.cpu().numpy() for x in device_result_split(outs[call]))
                assert_same_topk(od, oi, rd, ri, f"no-alloc call {call} k={k}")
            assert_same_topk(od, oi, g[f"d_k{k}"], g[f"i_k{k}"], "no-alloc vs reference fixture")


def test_noalloc_single_query_wide_merge(golden):
    """One query over many chunk lists: the few-query merge (one block per query), as on the allocating path."""
    import torch

    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        d_q = torch.from_numpy(g["queries"][:1].copy()).cuda()
        for k in (100, 10):
            ref = torch.empty((1, k), dtype=torch.int64, device="cuda")
            s.search_device(d_q, k, ref, None, tuning=Tuning())
            s.sync(None)
            rd, ri = (x.cpu().numpy() for x in device_result_split(ref))
            for call in range(2):
                out = torch.full((1, k), -1, dtype=torch.int64, device="cuda")
                assert _noalloc(s, d_q, k, Tuning(), out) == N.VK_OK, N.last_error()
                od, oi = (x.cpu().numpy() for x in device_result_split(out))
                assert_same_topk(od, oi, rd, ri, f"no-alloc nq=1 call {call} k={k}")


def test_noalloc_rejects_work_beyond_its_array(golden):
    import torch

    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        nq = 4096  # 4096 queries x 16 KiB of LUTs = 64 MiB > the 32 MiB array
        d_q = torch.from_numpy(np.resize(g["queries"], (nq, g["queries"].shape[1]))).cuda()
        out = torch.empty((nq, 10), dtype=torch.int64, device="cuda")
        assert _noalloc(s, d_q, 10, Tuning(queries_per_block=4), out) == N.VK_ERR_INVALID
        assert "working memory" in N.last_error()
