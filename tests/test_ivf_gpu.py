"""GPU: IVF (inverted-file) PQ search, the IVF partitioning the reference lists as a next step (README.md:219).
Definition (include/vk_abi.h, restated on the CPU by the oracle's vko_ivf_search): each query probes the nprobe
lists with the smallest exact l2sq to their coarse centroids (ties to the lower list) and gets the k smallest
(distance, id) pairs among those lists' rows, distances being the flat search's. The CUDA path must equal it bit for
bit: host and device entry points, k and nprobe templates, pruning on and off, Q = 4 / 8, m = 16 / 32, tiny and
empty lists, nprobe = nlist (the flat search), and config 1 at full size with a 256-list coarse quantizer trained by
the device PQ trainer.
"""
import numpy as np
import pytest

from conftest import assert_same_topk
from veckern_b200 import IVFSearcher, PQSearcher, Tuning, assign_lists, configs, data, device_result_split

pytestmark = pytest.mark.gpu


def l2sq_rows(x, c):
    """[n, nlist] exact l2sq in float32, dimensions added in order (the reference's l2sq, no FMA)."""
    acc = np.zeros((x.shape[0], c.shape[0]), np.float32)
    for j in range(x.shape[1]):
        diff = (x[:, None, j] - c[None, :, j]).astype(np.float32)
        acc = (acc + (diff * diff).astype(np.float32)).astype(np.float32)
    return acc


def ivf_db(seed, n, m, dsub, nlist, nq, empty_lists=0):
    rng = np.random.default_rng(seed)
    d = m * dsub
    x = rng.normal(size=(n, d)).astype(np.float32)
    cent = rng.normal(size=(m, 256, dsub)).astype(np.float32)
    codes = data.pq_encode(cent, x)
    coarse = x[rng.choice(n, nlist, replace=False)].copy()
    if empty_lists:  # coarse centroids far away from every row: lists nobody belongs to
        coarse[:empty_lists] += 1000.0
    lists = np.argmin(l2sq_rows(x, coarse), axis=1).astype(np.int32)
    q = rng.normal(size=(nq, d)).astype(np.float32)
    return cent, codes, coarse, lists, q, x


def test_assign_lists_matches_exact_l2sq():
    rng = np.random.default_rng(5)
    x = rng.normal(size=(3000, 128)).astype(np.float32)
    coarse = rng.normal(size=(77, 128)).astype(np.float32)
    coarse[5] = coarse[9]  # a tie: the lower list wins
    got = assign_lists(x, coarse)
    assert np.array_equal(got, np.argmin(l2sq_rows(x, coarse), axis=1))


@pytest.mark.parametrize("m,dsub", [(16, 8), (32, 4)])
@pytest.mark.parametrize("k", [1, 10, 100])
def test_ivf_matches_oracle(port, m, dsub, k):
    cent, codes, coarse, lists, q, _ = ivf_db(m * 7 + k, 40_000, m, dsub, 64, 37, empty_lists=3)
    with IVFSearcher(cent, codes, coarse, lists) as s:
        for nprobe in (1, 5, 16):
            ed, ei, _ = port.ivf_search(cent, codes, lists, coarse, q, nprobe, k)
            for t in (Tuning(queries_per_block=8, vectors_per_step=2), Tuning(queries_per_block=4, vectors_per_step=1),
                      Tuning(queries_per_block=8, vectors_per_step=2, early_abandon=False)):
                s.set_tuning(t)
                out, _ = s.search(q, k, nprobe)
                assert_same_topk(out["dist"], out["id"], ed, ei, f"ivf m={m} k={k} nprobe={nprobe} {t}")


def test_ivf_all_lists_is_the_flat_search(port):
    cent, codes, coarse, lists, q, _ = ivf_db(3, 20_011, 16, 8, 40, 9)
    with IVFSearcher(cent, codes, coarse, lists) as s:
        out, _ = s.search(q, 10, 40)
    ed, ei = port.adc_search(cent, codes, q, 10)
    assert_same_topk(out["dist"], out["id"], ed, ei, "ivf nprobe = nlist vs flat")


def test_ivf_device_path_and_small_lists(port):
    """Device entry point; a list smaller than k (padding {+inf, -1}); one query."""
    import torch

    cent, codes, coarse, lists, q, _ = ivf_db(11, 5_000, 16, 8, 1000, 13)
    with IVFSearcher(cent, codes, coarse, lists) as s:
        for nq in (13, 1):
            d_q = torch.from_numpy(q[:nq].copy()).cuda()
            out = torch.empty((nq, 100), dtype=torch.int64, device="cuda")
            s.search_device(d_q, 100, 1, out)
            s.sync()
            od, oi = (x.cpu().numpy() for x in device_result_split(out))
            ed, ei, _ = port.ivf_search(cent, codes, lists, coarse, q[:nq], 1, 100)
            assert_same_topk(od, oi, ed, ei, f"ivf device nq={nq}")
            assert (oi == -1).any(), "lists of ~5 rows cannot fill k = 100"


def test_ivf_c1_full(port):
    """Config 1 (1M rows, m = 16) with 256 lists: coarse centroids from the device PQ trainer with m = 1 (the
    reference's Lloyd iterations over whole vectors), rows assigned on the GPU; all 1,000 queries at nprobe = 16."""
    w = configs.make("c1", encode=data.gpu_encoder(), keep_base=True)
    sample = w.base[:100_000]
    coarse = data.pq_train_gpu(sample, 1, 10, 1).reshape(256, 128)
    lists = assign_lists(w.base, coarse)
    ed, ei, _ = port.ivf_search(w.centroids, w.codes, lists, coarse, w.queries, 16, w.k)
    with IVFSearcher(w.centroids, w.codes, coarse, lists) as s:
        out, _ = s.search(w.queries, w.k, 16)
    assert_same_topk(out["dist"], out["id"], ed, ei, "ivf c1 nprobe 16")
