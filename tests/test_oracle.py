"""CPU: the oracle (plain-C restatement of the reference CPU path) against the reference's own outputs.

The golden fixtures were produced by running the reference's CPU library (tests/golden/make_golden.py); where that
library is built here (oracle/_ref), the oracle is also compared with it directly on fresh random inputs.
"""
import numpy as np
import pytest

import oracle
from conftest import assert_same_topk, bits


def test_topk_known_answer(port, golden):
    g = golden("topk_kat")
    d, i = port.topk_push_all(g["kat_values"], np.arange(5, dtype=np.int32), 3)
    assert list(i) == [1, 3, 4]  # tie on 1.0 broken by the lower id (reference tests/test_cpu.cpp:33-41)
    assert np.array_equal(bits(d), bits(g["kat_d"])) and np.array_equal(i, g["kat_i"])
    d, i = port.topk_push_all(np.array([2.0], np.float32), np.array([9], np.int32), 4)
    assert list(i) == [9, -1, -1, -1] and np.isinf(d[1:]).all()  # padding (tests/test_cpu.cpp:42-45)
    for r, k in enumerate(g["seq_k"]):
        d, i = port.topk_push_all(g["seq_v"][r], g["seq_i"][r], int(k))
        assert np.array_equal(i, g["seq_out_i"][r, :k]) and np.array_equal(bits(d), bits(g["seq_out_d"][r, :k]))


def test_cpu_fixture_lut_scan_search(port, golden):
    g = golden("cpu_fixture")
    lut = port.compute_lut(g["centroids"], g["queries"])
    assert np.array_equal(bits(lut), bits(g["lut"]))
    dists = port.adc_scan(lut, g["codes"])
    assert np.array_equal(bits(dists), bits(g["dists"]))
    d, i = port.adc_search(g["centroids"], g["codes"], g["queries"], 10)
    assert_same_topk(d, i, g["top_d"], g["top_i"], "cpu fixture")


def test_staged_equals_fused(port, golden):
    """The reference's only exact-equality CPU test (tests/test_cpu.cpp:84-94): LUT+scan+select == adc_search."""
    g = golden("cpu_fixture")
    lut = port.compute_lut(g["centroids"], g["queries"])
    sd, si = port.select_topk(port.adc_scan(lut, g["codes"]), 10)
    fd, fi = port.adc_search(g["centroids"], g["codes"], g["queries"], 10)
    assert_same_topk(sd, si, fd, fi, "staged vs fused")


@pytest.mark.parametrize("k", [1, 8, 10, 16, 32, 33, 64, 100, 128])
def test_gpu_fixture_all_k(port, golden, k):
    g = golden("gpu_fixture")
    d, i = port.adc_search(g["centroids"], g["codes"], g["queries"], k)
    assert_same_topk(d, i, g[f"d_k{k}"], g[f"i_k{k}"], f"k={k}")


def test_c0_pipeline_small(port, golden):
    """Config 0's pipeline (N(0,1) rows, PQ from 256 rows picked with seed 1, encode) reproduces the reference's
    codebook, codes and results."""
    from veckern_b200 import data

    g = golden("c0_small")
    x = data.gen_normal(0, 20_000, 128)
    q = data.gen_normal(2, 100, 128)
    assert np.array_equal(bits(q), bits(g["queries"]))
    cent = data.pq_train(x, 16, 0, 1)
    assert np.array_equal(bits(cent), bits(g["centroids"]))
    assert np.array_equal(data.pq_encode(cent, x), g["codes"])
    d, i = port.adc_search(cent, g["codes"], q, 10)
    assert_same_topk(d, i, g["top_d"], g["top_i"], "c0 small")


@pytest.mark.parametrize("k", [10, 100])
def test_exact_ties(port, golden, k):
    g = golden("ties")
    d, i = port.adc_search(g["centroids"], g["codes"], g["queries"], k)
    assert_same_topk(d, i, g[f"d_k{k}"], g[f"i_k{k}"], f"ties k={k}")
    # the fixture really has ties, broken by id
    assert (np.diff(g[f"d_k{k}"], axis=1) == 0).sum() > 0


def test_merge_of_shards_equals_unsharded(port, golden):
    g = golden("gpu_fixture")
    n = g["codes"].shape[0]
    k = 33
    bounds = [0, 5000, 5001, 12_345, n]
    parts_d, parts_i = [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        d, i = port.adc_search(g["centroids"], g["codes"][a:b], g["queries"], k)
        parts_d.append(d)
        parts_i.append(np.where(i >= 0, i + a, -1).astype(np.int32))
    d = np.stack(parts_d, axis=1)
    i = np.stack(parts_i, axis=1)
    md, mi = port.merge_topk(d, i, k)
    assert_same_topk(md, mi, g[f"d_k{k}"], g[f"i_k{k}"], "merged shards")


def test_stream_search_equals_search(port, golden):
    g = golden("gpu_fixture")
    lut = port.compute_lut(g["centroids"], g["queries"])
    codes = g["codes"]
    blocks = [(codes[a:a + 4096], a) for a in range(0, codes.shape[0], 4096)]
    d, i = port.stream_search(lut, blocks, 100)
    assert_same_topk(d, i, g["d_k100"], g["i_k100"], "stream")


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built here")
@pytest.mark.parametrize("seed,n,m,dsub,nq,k", [(1, 3001, 4, 8, 5, 7), (2, 999, 16, 2, 3, 128), (3, 257, 3, 5, 4, 1)])
def test_port_matches_reference_random(port, seed, n, m, dsub, nq, k):
    R = oracle.ref()
    rng = np.random.default_rng(seed)
    pq = R.pq(m * dsub, m)
    pq.centroids = rng.normal(size=(m, 256, dsub)).astype(np.float32)
    codes = rng.integers(0, 256, size=(n, m)).astype(np.uint8)
    q = rng.normal(size=(nq, m * dsub)).astype(np.float32)
    assert np.array_equal(bits(R.compute_lut(pq, q)), bits(port.compute_lut(pq.centroids, q)))
    rd, ri = R.adc_search(pq, codes, q, k)
    pd, pi = port.adc_search(pq.centroids, codes, q, k)
    assert_same_topk(pd, pi, rd, ri, "port vs reference")


def test_rerank_matches_reference_fixture(port, golden):
    """Exact re-rank of 100 PQ candidates (one padding entry) to 10, as the reference computes it."""
    from veckern_b200 import data

    g = golden("cpu_fixture")
    base = data.synthetic_clustered(4000, 32, 20, 7)
    d, i = port.rerank_exact(base, g["queries"], g["cand_i"], 10)
    assert_same_topk(d, i, g["rr_d"], g["rr_i"], "rerank")


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built here")
def test_rerank_port_matches_reference_with_duplicates():
    R = oracle.ref()
    rng = np.random.default_rng(8)
    base = rng.integers(-2, 3, size=(500, 16)).astype(np.float32)  # small integers: many exact ties
    q = rng.integers(-2, 3, size=(7, 16)).astype(np.float32)
    cand = rng.integers(-1, 500, size=(7, 90)).astype(np.int32)  # duplicates and padding on purpose
    for k in (1, 10, 64, 128):
        rd, ri = R.rerank_exact(base, q, cand, k)
        pd, pi = oracle.port().rerank_exact(base, q, cand, k)
        assert_same_topk(pd, pi, rd, ri, f"rerank k={k}")


def test_reference_arm_inputs_match_the_package():
    """bench.py's reference arm builds its workload without this repository's libraries (numpy generators + the
    reference's own ProductQuantizer); it must be the very workload the package's arm searches."""
    from oracle import inputs
    from veckern_b200 import configs, data

    for seed, row0 in ((0, 0), (3, 0), (0, 777_777)):
        a = inputs.gen_mixture(0, seed, 3_000, 128, row0=row0)
        assert np.array_equal(bits(a), bits(data.gen_mixture(0, seed, 3_000, 128, row0=row0)))
    assert np.array_equal(bits(inputs.gen_normal(2, 500, 128, row0=5)), bits(data.gen_normal(2, 500, 128, row0=5)))
    if not oracle.ref_available():
        pytest.skip("reference library not built")
    for name, n in (("c0", 30_000), ("c1", 30_000)):
        spec = configs.spec(name, n=n, nq=50)
        pq, codes, q = inputs.reference_workload(spec, oracle.ref())
        w = configs.make(name, n=n, nq=50)
        assert np.array_equal(bits(pq.centroids), bits(w.centroids)), name
        assert np.array_equal(codes, w.codes), name
        assert np.array_equal(bits(q), bits(w.queries)), name


def test_h16_definition_restated_in_numpy(port):
    """The oracle's half-precision LUT search against an independent numpy statement of the same definition
    (numpy float16 conversion rounds to nearest even; sums in float32 in sub-space order)."""
    rng = np.random.default_rng(11)
    m, dsub, n, nq, k = 16, 8, 3_000, 7, 10
    cent = (rng.normal(size=(m, 256, dsub)) * 30).astype(np.float32)
    codes = rng.integers(0, 256, size=(n, m)).astype(np.uint8)
    q = (rng.normal(size=(nq, m * dsub)) * 30).astype(np.float32)
    raw = port.compute_lut(cent, q)
    tab, exps = port.compute_lut_h16(cent, q)
    for j in range(nq):
        mx = raw[j].max()
        _, E = np.frexp(np.float32(mx))
        assert exps[j] == int(np.clip(15 - E, -64, 64))
        scaled = (raw[j].astype(np.float64) * 2.0 ** exps[j]).astype(np.float32)
        assert scaled.max() >= 2 ** 14 and scaled.max() < 2 ** 15
        ref = scaled.astype(np.float16).astype(np.float32)
        assert np.array_equal(bits(tab[j]), bits(ref))
    d, i = port.adc_search_h16(cent, codes, q, k)
    for j in range(nq):
        acc = np.zeros(n, np.float32)
        for s in range(m):
            acc = acc + tab[j, s, codes[:, s]]
        dist = (acc.astype(np.float64) * 2.0 ** -int(exps[j])).astype(np.float32)
        order = np.lexsort((np.arange(n), dist))[:k]
        assert np.array_equal(i[j], order) and np.array_equal(bits(d[j]), bits(dist[order]))


def _l2sq_rows(x, c):
    """The reference's l2sq (common.hpp:27-34) for every row of x against one vector c, float32, j in order."""
    acc = np.zeros(x.shape[0], np.float32)
    for j in range(x.shape[1]):
        diff = x[:, j] - c[j]
        acc = acc + diff * diff
    return acc


def test_pq4_definition_restated_in_numpy(port):
    """The oracle's 4-bit PQ (encode, LUT, search) against an independent numpy statement of the definition."""
    rng = np.random.default_rng(12)
    m, dsub, n, nq, k = 32, 4, 2_000, 6, 10
    cent = rng.normal(size=(m, 16, dsub)).astype(np.float32)
    x = rng.normal(size=(n, m * dsub)).astype(np.float32)
    q = rng.normal(size=(nq, m * dsub)).astype(np.float32)
    codes = port.pq4_encode(cent, x)
    assert codes.shape == (n, m // 2)
    sub = np.zeros((n, m), np.uint8)
    for s in range(m):
        dist = np.stack([_l2sq_rows(x[:, s * dsub:(s + 1) * dsub], cent[s, c]) for c in range(16)], 1)
        sub[:, s] = np.argmin(dist, 1)  # first minimum
    assert np.array_equal(codes, (sub[:, 0::2] | (sub[:, 1::2] << 4)).astype(np.uint8))
    lut = port.compute_lut_pq4(cent, q)
    for j in range(nq):
        for s in range(m):
            ref = np.array([_l2sq_rows(q[j:j + 1, s * dsub:(s + 1) * dsub], cent[s, c])[0] for c in range(16)],
                           np.float32)
            assert np.array_equal(bits(lut[j, s]), bits(ref))
    d, i = port.adc_search_pq4(cent, codes, q, k)
    for j in range(nq):
        acc = np.zeros(n, np.float32)
        for s in range(m):
            acc = acc + lut[j, s, sub[:, s]]
        order = np.lexsort((np.arange(n), acc))[:k]
        assert np.array_equal(i[j], order) and np.array_equal(bits(d[j]), bits(acc[order]))
