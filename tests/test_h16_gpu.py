"""GPU: half-precision lookup tables (VK_LUT_F16), the fp16 LUT the reference lists as a next step
(README.md:219). It is an approximate search with an exact definition (include/vk_abi.h, lut_precision): per
query the fp32 entries are scaled by 2^e so that the largest lies in [2^14, 2^15), rounded to half, summed in fp32
in sub-space order and scaled back by 2^-e. The CUDA path must equal the CPU restatement of that definition
(oracle vko_adc_search_h16) bit for bit, for every Q / ILP / k template, pruning on and off, through the host,
device and no-allocation entry points, and at config 1's full size.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_same_topk
from veckern_b200 import PQSearcher, Tuning, VkError, configs, data, device_result_split
from veckern_b200 import _native as N

pytestmark = pytest.mark.gpu


def random_db(seed, n, m, dsub, nq, scale=1.0):
    rng = np.random.default_rng(seed)
    cent = (rng.normal(size=(m, 256, dsub)) * scale).astype(np.float32)
    codes = rng.integers(0, 256, size=(n, m)).astype(np.uint8)
    q = (rng.normal(size=(nq, m * dsub)) * scale).astype(np.float32)
    return cent, codes, q


def h16(**kw):
    return Tuning(lut_f16=True, **kw)


@pytest.mark.parametrize("k", [1, 10, 33, 100, 128])
@pytest.mark.parametrize("qpb", [4, 8])
@pytest.mark.parametrize("prune", [True, False])
def test_h16_fixture_every_k(golden, port, k, qpb, prune):
    g = golden("gpu_fixture")
    ed, ei = port.adc_search_h16(g["centroids"], g["codes"], g["queries"], k)
    with PQSearcher(g["centroids"], g["codes"]) as s:
        for ilp in (1, 2):
            s.set_tuning(h16(queries_per_block=qpb, vectors_per_step=ilp, early_abandon=prune))
            out, _ = s.search(g["queries"], k)
            assert_same_topk(out["dist"], out["id"], ed, ei, f"h16 k={k} Q={qpb} ilp={ilp} prune={prune}")


@pytest.mark.parametrize("m,dsub,n,nq", [(16, 8, 50_003, 37), (32, 4, 20_011, 9), (64, 2, 10_007, 5),
                                         (16, 8, 129, 1), (32, 4, 33, 2)])
def test_h16_shapes(port, m, dsub, n, nq):
    # values spread over several binades so that the per-query scales differ
    cent, codes, q = random_db(m + n, n, m, dsub, nq, scale=40.0)
    k = min(10, n)
    ed, ei = port.adc_search_h16(cent, codes, q, k)
    with PQSearcher(cent, codes) as s:
        for prune in (True, False):
            s.set_tuning(h16(queries_per_block=8, vectors_per_step=2, early_abandon=prune))
            out, _ = s.search(q, k)
            assert_same_topk(out["dist"], out["id"], ed, ei, f"h16 m={m} n={n} prune={prune}")


def test_h16_ids_offset_and_device_paths(golden, port):
    """Device-resident entry points (with an id offset) and the no-allocation entry point give the same lists."""
    import torch

    g = golden("gpu_fixture")
    k = 10
    ed, ei = port.adc_search_h16(g["centroids"], g["codes"], g["queries"], k)
    with PQSearcher(g["centroids"], g["codes"], id_base=1000) as s:
        d_q = torch.from_numpy(g["queries"]).cuda()
        t = h16(queries_per_block=8, vectors_per_step=2)
        out = torch.empty((d_q.shape[0], k), dtype=torch.int64, device="cuda")
        s.search_device(d_q, k, out, None, tuning=t)
        s.sync(None)
        od, oi = (x.cpu().numpy() for x in device_result_split(out))
        assert_same_topk(od, oi - 1000, ed, ei, "h16 device path")
        for call in range(2):
            out2 = torch.full((d_q.shape[0], k), -1, dtype=torch.int64, device="cuda")
            tc = t.c()
            assert N.lib().vk_search_noalloc(s._h, N.ptr(d_q), d_q.shape[0], k, C.byref(tc), N.ptr(out2),
                                             None) == N.VK_OK, N.last_error()
            assert torch.equal(out2, out), f"no-alloc call {call}"


def test_h16_rejects_generic_m(port):
    cent, codes, q = random_db(3, 1000, 12, 4, 3)
    with PQSearcher(cent, codes) as s:
        s.set_tuning(h16())
        with pytest.raises(VkError):
            s.search(q, 5)


def test_h16_c1_full(port):
    """Config 1 at full size (m = 16): all 1,000 queries against the CPU restatement; recall against fp32."""
    w = configs.make("c1", encode=data.gpu_encoder())
    ed, ei = port.adc_search_h16(w.centroids, w.codes, w.queries, w.k)
    with PQSearcher(w.centroids, w.codes) as s:
        s.set_tuning(h16(queries_per_block=8, vectors_per_step=2))
        out, _ = s.search(w.queries, w.k)
        s.set_tuning(Tuning(queries_per_block=8, vectors_per_step=2))
        exact, _ = s.search(w.queries, w.k)
    assert_same_topk(out["dist"], out["id"], ed, ei, "h16 c1")
    recall = np.mean([len(set(a) & set(b)) / w.k for a, b in zip(out["id"], exact["id"])])
    assert recall > 0.9, recall
