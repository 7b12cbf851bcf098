"""GPU: 4-bit PQ (16 centroids per sub-space, two sub-codes per byte), the 4-bit codes the reference lists as a
next step (README.md:219). Its definition (include/vk_abi.h, vk_index_create_pq4; restated on the CPU by oracle
vko_adc_search_pq4): LUT entries l2sq(query sub-vector, centroid) with the 8-bit path's fp32 arithmetic, summed in
sub-space order, the k smallest (distance, id) pairs. The CUDA path must equal that restatement bit for bit: every
k template, Q = 4 / 8, ILP 1 / 2, pruning on and off, m = 16 / 32 / 64, ragged n, exact ties, id offsets, the device
and no-allocation entry points, and config 1's rows at full size.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_same_topk
from veckern_b200 import PQSearcher, Tuning, VkError, configs, data, device_result_split
from veckern_b200 import _native as N

pytestmark = pytest.mark.gpu


def random_db4(seed, n, m, dsub, nq, scale=1.0):
    rng = np.random.default_rng(seed)
    cent = (rng.normal(size=(m, 16, dsub)) * scale).astype(np.float32)
    codes = rng.integers(0, 256, size=(n, (m + 1) // 2)).astype(np.uint8)
    q = (rng.normal(size=(nq, m * dsub)) * scale).astype(np.float32)
    return cent, codes, q


@pytest.mark.parametrize("k", [1, 10, 33, 100, 128])
@pytest.mark.parametrize("qpb", [4, 8])
@pytest.mark.parametrize("prune", [True, False])
def test_pq4_every_k(port, k, qpb, prune):
    cent, codes, q = random_db4(k + qpb, 20_011, 32, 4, 37)
    ed, ei = port.adc_search_pq4(cent, codes, q, k)
    with PQSearcher(cent, codes) as s:
        assert s.nbits == 4
        for ilp in (1, 2):
            s.set_tuning(Tuning(queries_per_block=qpb, vectors_per_step=ilp, early_abandon=prune))
            out, _ = s.search(q, k)
            assert_same_topk(out["dist"], out["id"], ed, ei, f"pq4 k={k} Q={qpb} ilp={ilp} prune={prune}")
            assert s.last_launch().queries_per_block == qpb


@pytest.mark.parametrize("m,dsub,n,nq", [(16, 8, 50_003, 13), (32, 4, 20_011, 9), (64, 2, 10_007, 5),
                                         (16, 8, 129, 1), (32, 4, 33, 2), (64, 2, 1, 3), (32, 4, 128, 8)])
def test_pq4_shapes(port, m, dsub, n, nq):
    cent, codes, q = random_db4(m + n, n, m, dsub, nq, scale=3.0)
    k = min(10, n)
    ed, ei = port.adc_search_pq4(cent, codes, q, k)
    with PQSearcher(cent, codes) as s:
        for prune in (True, False):
            for qpb in (4, 8):
                s.set_tuning(Tuning(queries_per_block=qpb, vectors_per_step=2, early_abandon=prune))
                out, _ = s.search(q, k)
                assert_same_topk(out["dist"], out["id"], ed, ei, f"pq4 m={m} n={n} Q={qpb} prune={prune}")


@pytest.mark.parametrize("m", [16, 32, 64])
def test_pq4_trained_clustered(port, m):
    """Codebooks and codes from the 4-bit trainer and encoder on clustered rows (pruning bites early)."""
    x = data.synthetic_clustered(60_000, 128, 64, 11)
    cent = data.pq4_train(x[:20_000], m, 4, 1)
    codes = data.pq4_encode(cent, x)
    assert np.array_equal(codes, port.pq4_encode(cent, x))
    q = x[::997][:31] + np.float32(0.01)
    ed, ei = port.adc_search_pq4(cent, codes, q, 10)
    with PQSearcher(cent, codes) as s:
        for prune in (True, False):
            s.set_tuning(Tuning(queries_per_block=8, vectors_per_step=2, early_abandon=prune))
            out, _ = s.search(q, 10)
            assert_same_topk(out["dist"], out["id"], ed, ei, f"pq4 clustered m={m} prune={prune}")


def test_pq4_ties(port):
    """Few distinct codes: long runs of equal distances, resolved by the lower id."""
    rng = np.random.default_rng(5)
    m, dsub, n = 32, 4, 30_000
    cent = rng.integers(0, 3, size=(m, 16, dsub)).astype(np.float32)
    codes = (rng.integers(0, 2, size=(n, m // 2)) * 0x11).astype(np.uint8)
    q = rng.integers(0, 3, size=(11, m * dsub)).astype(np.float32)
    for k in (10, 100):
        ed, ei = port.adc_search_pq4(cent, codes, q, k)
        with PQSearcher(cent, codes) as s:
            for prune in (True, False):
                s.set_tuning(Tuning(queries_per_block=8, vectors_per_step=2, early_abandon=prune))
                out, _ = s.search(q, k)
                assert_same_topk(out["dist"], out["id"], ed, ei, f"pq4 ties k={k} prune={prune}")


def test_pq4_codes_roundtrip():
    cent, codes, _ = random_db4(2, 5_003, 32, 4, 1)
    with PQSearcher(cent, codes) as s:
        got = np.empty_like(codes)
        N.check(N.lib().vk_index_get_codes(s._h, 0, codes.shape[0], N.ptr(got)))
        assert np.array_equal(got, codes)
        place = np.empty(5_120, np.uint8)
        N.check(N.lib().vk_index_get_placement(s._h, 0, place.size, N.ptr(place)))
        assert np.array_equal(place, np.arange(place.size) % 64)  # rows stay in id order


def test_pq4_device_paths_and_noalloc(port):
    """Device-resident search with an id offset, and two no-allocation calls in a row, equal the restatement."""
    import torch

    cent, codes, q = random_db4(9, 40_009, 32, 4, 29)
    k = 10
    ed, ei = port.adc_search_pq4(cent, codes, q, k)
    with PQSearcher(cent, codes, id_base=500) as s:
        d_q = torch.from_numpy(q).cuda()
        t = Tuning(queries_per_block=8, vectors_per_step=2)
        out = torch.empty((d_q.shape[0], k), dtype=torch.int64, device="cuda")
        s.search_device(d_q, k, out, None, tuning=t)
        s.sync(None)
        od, oi = (x.cpu().numpy() for x in device_result_split(out))
        assert_same_topk(od, oi - 500, ed, ei, "pq4 device path")
        for call in range(2):
            out2 = torch.full((d_q.shape[0], k), -1, dtype=torch.int64, device="cuda")
            tc = t.c()
            assert N.lib().vk_search_noalloc(s._h, N.ptr(d_q), d_q.shape[0], k, C.byref(tc), N.ptr(out2),
                                             None) == N.VK_OK, N.last_error()
            assert torch.equal(out2, out), f"no-alloc call {call}"


def test_pq4_rejections():
    cent, codes, q = random_db4(3, 1000, 24, 4, 3)
    with pytest.raises(VkError):  # m = 24: not built
        PQSearcher(cent, codes)
    cent, codes, q = random_db4(3, 1000, 32, 4, 3)
    with PQSearcher(cent, codes) as s:
        s.set_tuning(Tuning(lut_f16=True))
        with pytest.raises(VkError):
            s.search(q, 5)
        with pytest.raises(VkError):
            s.distances(q)
    with pytest.raises(ValueError):  # 8-bit-shaped codes for a 4-bit codebook
        PQSearcher(cent, np.zeros((10, 32), np.uint8))


def test_pq4_c1_full(port):
    """Config 1's rows and queries with 4-bit codes at m = 32 (16 bytes per row, as the 8-bit m = 16 index): all
    1,000 queries against the CPU restatement, pruned and full scans."""
    w = configs.make_pq4("c1", m=32)
    ed, ei = port.adc_search_pq4(w.centroids, w.codes, w.queries, w.k)
    with PQSearcher(w.centroids, w.codes) as s:
        for prune in (True, False):
            s.set_tuning(Tuning(queries_per_block=8, vectors_per_step=2, early_abandon=prune))
            out, _ = s.search(w.queries, w.k)
            assert_same_topk(out["dist"], out["id"], ed, ei, f"pq4 c1 prune={prune}")
