"""GPU: the five BASELINE.json configurations at full size, bit-exact against the CPU oracle.

c0, c1 (m = 16, 32, 64) and c2 (k = 100, and the nq = 1 latency case): every query of the configuration against
the oracle, under the planner's default tuning and under the benchmark's (Q = 8, ILP = 2). c3 (100M rows, all
10,000 queries) and c4 (1B rows, 1,000 queries, k = 10 and 100), generated on the GPU: every returned distance is
recomputed on the host from independently regenerated codes (exact ADC sum), results are ascending, a split of the
database into id-offset shards merged on the GPU gives the same result, and sampled queries are checked against
the oracle streaming the host-regenerated database (one pass at the largest k; a top-k list's first entries are
the top-k' list for k' < k).
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


def gpu_topk_tunings(cent, codes, q, k, tunings):
    """[(dist, ids)] of one index searched under each tuning."""
    res = []
    with PQSearcher(cent, codes) as s:
        for t in tunings:
            s.set_tuning(t)
            out, _ = s.search(q, k)
            res.append((out["dist"].copy(), out["id"].copy()))
    return res


BENCH_TUNING = Tuning(queries_per_block=8, vectors_per_step=2)


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
    """All 1,000 queries of config 1 at each m, bit-exact against the oracle."""
    w = configs.make("c1", m=m, encode=data.gpu_encoder())
    assert w.queries.shape[0] == 1000
    ed, ei = port.adc_search(w.centroids, w.codes, w.queries, w.k)
    tunings = [Tuning(queries_per_block=4 if m <= 32 else 2), BENCH_TUNING,
               Tuning(queries_per_block=8, vectors_per_step=2, early_abandon=False)]
    for t, (d, i) in zip(tunings, gpu_topk_tunings(w.centroids, w.codes, w.queries, w.k, tunings)):
        assert_same_topk(d, i, ed, ei, f"c1 m={m} {t}")


def test_c2_full(port):
    """All 1,000 queries of config 2 at k = 100, and the single-query latency case, against the oracle."""
    w = configs.make("c2", encode=data.gpu_encoder())
    assert w.queries.shape[0] == 1000
    ed, ei = port.adc_search(w.centroids, w.codes, w.queries, 100)
    tunings = [Tuning(queries_per_block=4), BENCH_TUNING]
    for t, (d, i) in zip(tunings, gpu_topk_tunings(w.centroids, w.codes, w.queries, 100, tunings)):
        assert_same_topk(d, i, ed, ei, f"c2 k=100 {t}")
    for t, (d1, i1) in zip(tunings, gpu_topk_tunings(w.centroids, w.codes, w.queries[:1], 10, tunings)):
        assert_same_topk(d1, i1, ed[:1, :10], ei[:1, :10], f"c2 nq=1 k=10 {t}")


def _generated_checks(port, name, nq, ks, oracle_queries, split):
    w = configs.make(name, nq=nq)
    s = w.spec
    n = s["n"]
    with PQSearcher.generated(w.centroids, s["code_seed"], w.cdf, 0, n) as idx:
        idx.set_tuning(Tuning(queries_per_block=4))
        results = {k: idx.search(w.queries, k)[0].copy() for k in ks}
        idx.set_tuning(BENCH_TUNING)  # the benchmark's plan gives the same lists
        for k in ks:
            assert np.array_equal(idx.search(w.queries, k)[0].view(np.int64), results[k].view(np.int64)), k
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
    # sampled queries against the oracle over the host-regenerated database: one pass at the largest k
    sample = np.array(oracle_queries)
    lut = port.compute_lut(w.centroids, w.queries[sample])
    block = 1 << 23
    kmax = max(ks)

    def blocks():
        for a in range(0, n, block):
            yield data.gen_codes(s["code_seed"], w.cdf, a, min(block, n - a)), a

    ed, ei = port.stream_search(lut, blocks(), kmax)
    for k in ks:
        out = results[k]
        assert_same_topk(out["dist"][sample], out["id"][sample], ed[:, :k], ei[:, :k], f"{name} oracle k={k}")


def test_c3_full(port):
    _generated_checks(port, "c3", nq=10_000, ks=[10], oracle_queries=[0, 1, 2_500, 4_999, 7_777, 9_999], split=4)


def test_c4_full(port):
    _generated_checks(port, "c4", nq=1_000, ks=[10, 100], oracle_queries=[0, 1, 333, 500, 998, 999], split=2)
