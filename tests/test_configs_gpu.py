"""GPU: the five BASELINE.json configurations at full size, bit-exact against the CPU oracle.

c0: every query against the oracle. c1 (m = 16, 32, 64) and c2 (k = 100): all queries searched on the GPU, a
fixed sample of them against the oracle. c3 (100M rows) and c4 (1B rows), generated on the GPU: every returned
distance is recomputed on the host from independently regenerated codes (exact ADC sum), results are ascending,
a split of the database into id-offset shards merged on the GPU gives the same result, and sampled queries are
checked against the oracle streaming the host-regenerated database.
"""
import numpy as np
import pytest

from conftest import assert_same_topk, bits
from veckern_b200 import PQSearcher, Tuning, configs, data, merge_topk_device

pytestmark = pytest.mark.gpu


def gpu_topk(cent, codes, q, k, qpb=4):
    with PQSearcher(cent, codes) as s:
        s.set_tuning(Tuning(queries_per_block=qpb))
        out, _ = s.search(q, k)
    return out["dist"].copy(), out["id"].copy()


def exact_adc(port, cent, q, codes_of_ids):
    """distances of (query, row) pairs: codes_of_ids [nq, k, m] -> [nq, k], summed in sub-space order in fp32."""
    lut = port.compute_lut(cent, q)  # [nq, m, 256]
    nq, k, m = codes_of_ids.shape
    acc = np.zeros((nq, k), np.float32)
    qi = np.arange(nq)[:, None]
    for s in range(m):
        acc = acc + lut[qi, s, codes_of_ids[:, :, s]]
    return acc


def test_c0_full(port):
    w = configs.make("c0")
    d, i = gpu_topk(w.centroids, w.codes, w.queries, w.k)
    ed, ei = port.adc_search(w.centroids, w.codes, w.queries, w.k)
    assert_same_topk(d, i, ed, ei, "c0")


@pytest.mark.parametrize("m", [16, 32, 64])
def test_c1_full(port, m):
    w = configs.make("c1", m=m, encode=data.gpu_encoder())
    d, i = gpu_topk(w.centroids, w.codes, w.queries, w.k, qpb=4 if m <= 32 else 2)
    sample = np.arange(0, w.queries.shape[0], 16)
    ed, ei = port.adc_search(w.centroids, w.codes, w.queries[sample], w.k)
    assert_same_topk(d[sample], i[sample], ed, ei, f"c1 m={m}")


def test_c2_full(port):
    w = configs.make("c2", encode=data.gpu_encoder())
    d, i = gpu_topk(w.centroids, w.codes, w.queries, 100)
    sample = np.arange(0, w.queries.shape[0], 100)
    ed, ei = port.adc_search(w.centroids, w.codes, w.queries[sample], 100)
    assert_same_topk(d[sample], i[sample], ed, ei, "c2 k=100")
    d1, i1 = gpu_topk(w.centroids, w.codes, w.queries[:1], 10)  # the single-query latency case
    assert_same_topk(d1, i1, ed[:1, :10], ei[:1, :10], "c2 nq=1 k=10")


def _generated_checks(port, name, nq, ks, oracle_queries, split):
    w = configs.make(name, nq=nq)
    s = w.spec
    n = s["n"]
    with PQSearcher.generated(w.centroids, s["code_seed"], w.cdf, 0, n) as idx:
        idx.set_tuning(Tuning(queries_per_block=4))
        results = {k: idx.search(w.queries, k)[0].copy() for k in ks}
    for k, out in results.items():
        d, i = out["dist"], out["id"]
        assert (i >= 0).all() and (i < n).all()
        assert (np.diff(d, axis=1) >= 0).all(), "not ascending"
        # every returned distance, recomputed from host-regenerated codes of the returned rows
        codes = data.gen_codes_rows(s["code_seed"], w.cdf, i.ravel()).reshape(nq, k, s["m"])
        assert np.array_equal(bits(exact_adc(port, w.centroids, w.queries, codes)), bits(d)), f"{name} k={k}"
    # id-offset shards merged on the GPU == one index
    import torch
    k = ks[0]
    bounds = np.linspace(0, n, split + 1).astype(np.int64)
    parts = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        with PQSearcher.generated(w.centroids, s["code_seed"], w.cdf, int(a), int(b - a), id_base=int(a)) as sh:
            sh.set_tuning(Tuning(queries_per_block=4))
            parts.append(sh.search(w.queries, k)[0].view(np.int64).copy())
    gathered = torch.from_numpy(np.stack(parts)).cuda()  # [shard][q][k]
    merged = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    merge_topk_device(0, gathered, nq, split, k, k, nq * k, k, merged)  # [shard][q][k]: query stride k
    torch.cuda.synchronize()
    assert np.array_equal(merged.cpu().numpy(), results[k].view(np.int64)), f"{name}: {split} merged shards differ"
    # sampled queries against the oracle over the host-regenerated database
    for k in ks:
        sample = np.array(oracle_queries)
        lut = port.compute_lut(w.centroids, w.queries[sample])
        block = 1 << 23

        def blocks():
            for a in range(0, n, block):
                yield data.gen_codes(s["code_seed"], w.cdf, a, min(block, n - a)), a

        ed, ei = port.stream_search(lut, blocks(), k)
        out = results[k]
        assert_same_topk(out["dist"][sample], out["id"][sample], ed, ei, f"{name} oracle k={k}")


def test_c3_full(port):
    _generated_checks(port, "c3", nq=10_000, ks=[10], oracle_queries=[0, 4_999, 9_999], split=4)


def test_c4_full(port):
    _generated_checks(port, "c4", nq=256, ks=[10, 100], oracle_queries=[0], split=2)
