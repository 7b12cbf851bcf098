"""GPU: cooperative sharded search (vk_search_device_coop). Shards of one database share each query's pruning
bound while they scan (posted atomics into the other shards' exchange arrays); each shard's lists are exact only
once merged. Here the shards live on one GPU in one process (vk_coop_attach), searched one after another (later
shards prune with the earlier shards' bounds) and concurrently on separate streams; the merged lists must equal
one index over all rows, bit for bit, for several k, epochs and query sets.
"""
import numpy as np
import pytest

from conftest import assert_same_topk
from veckern_b200 import CoopSearch, PQSearcher, Tuning, configs, data, device_result_split, merge_topk_device

pytestmark = pytest.mark.gpu


def sharded_coop(cent, codes, queries_sets, k, shards, tuning, concurrent=False):
    """[(dist, ids)] per query set: the shards' cooperative searches (epoch = set index + 1), merged on the GPU."""
    import torch

    n = codes.shape[0]
    bounds = np.linspace(0, n, shards + 1).astype(np.int64)
    idx = [PQSearcher(cent, codes[a:b], id_base=int(a)) for a, b in zip(bounds[:-1], bounds[1:])]
    nq_max = max(q.shape[0] for q in queries_sets)
    coops = [CoopSearch(0, nq_max) for _ in idx]
    for c in coops:
        c.attach(coops)
    streams = [torch.cuda.Stream() for _ in idx] if concurrent else [None] * shards
    out = []
    try:
        for epoch, q in enumerate(queries_sets, start=1):
            d_q = torch.from_numpy(q).cuda()
            nq = q.shape[0]
            lists = torch.empty((shards, nq, k), dtype=torch.int64, device="cuda")
            torch.cuda.synchronize()
            for j, s in enumerate(idx):
                s.search_device_coop(coops[j], epoch, d_q, k, lists[j], streams[j], tuning=tuning)
            torch.cuda.synchronize()
            for s in idx:
                s.sync(None)
            merged = torch.empty((nq, k), dtype=torch.int64, device="cuda")
            merge_topk_device(0, lists, nq, shards, k, k, nq * k, k, merged)
            torch.cuda.synchronize()
            d, i = (x.cpu().numpy() for x in device_result_split(merged))
            out.append((d, i))
    finally:
        torch.cuda.synchronize()
        for s in idx:
            s.close()
        for c in coops:
            c.close()
    return out


@pytest.mark.parametrize("k", [1, 10, 100])
@pytest.mark.parametrize("concurrent", [False, True])
def test_coop_fixture(golden, k, concurrent):
    g = golden("gpu_fixture")
    q2 = g["queries"][::-1].copy()  # a second search (epoch 2) with other queries
    res = sharded_coop(g["centroids"], g["codes"], [g["queries"], q2], k, 4,
                       Tuning(queries_per_block=8, vectors_per_step=2), concurrent)
    assert_same_topk(*res[0], g[f"d_k{k}"], g[f"i_k{k}"], f"coop k={k} epoch 1")
    assert_same_topk(*res[1], g[f"d_k{k}"][::-1], g[f"i_k{k}"][::-1], f"coop k={k} epoch 2")


def test_coop_c1_eight_shards(port):
    """Config 1 split into 8 shards (125k rows each, as on 8 GPUs), cooperative, all 1,000 queries against the
    oracle; also with half-precision LUTs against their CPU restatement."""
    w = configs.make("c1", encode=data.gpu_encoder())
    ed, ei = port.adc_search(w.centroids, w.codes, w.queries, w.k)
    (d, i), = sharded_coop(w.centroids, w.codes, [w.queries], w.k, 8, Tuning(queries_per_block=8, vectors_per_step=2),
                           concurrent=True)
    assert_same_topk(d, i, ed, ei, "coop c1 8 shards")
    hd, hi = port.adc_search_h16(w.centroids, w.codes, w.queries, w.k)
    (d, i), = sharded_coop(w.centroids, w.codes, [w.queries], w.k, 8,
                           Tuning(queries_per_block=8, vectors_per_step=2, lut_f16=True), concurrent=True)
    assert_same_topk(d, i, hd, hi, "coop c1 8 shards, half LUTs")
