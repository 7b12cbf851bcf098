"""GPU parity: the sm_100a search path, called through the C ABI, against the CPU oracle and the reference's
golden outputs. The bar is bit-exact distances and identical ids (ties to the lower id).

Mirrors the reference's GPU suite (tests/test_gpu.cpp) with its tolerances tightened to equality, plus edge cases
(ragged n, n < 32, k = n, nq = 0/1/prime, m not a multiple of 16, exact ties, every Q / ILP / S template).
"""
import numpy as np
import pytest

from conftest import assert_same_topk, bits
from veckern_b200 import PQSearcher, ScanVariant, Tuning, VkError, device_info

pytestmark = pytest.mark.gpu

FUSED = [ScanVariant.Fused, ScanVariant.FusedReg, ScanVariant.FusedVec, ScanVariant.FusedVecMQ,
         ScanVariant.FusedWarp]
SCANS = [ScanVariant.GlobalLut, ScanVariant.SharedLut, ScanVariant.SharedLutVec, ScanVariant.Interleaved]


def random_db(seed, n, m, dsub, nq, dup_rows=0):
    rng = np.random.default_rng(seed)
    cent = rng.normal(size=(m, 256, dsub)).astype(np.float32)
    codes = rng.integers(0, 256, size=(n, m)).astype(np.uint8)
    if dup_rows:
        codes = codes[rng.integers(0, dup_rows, size=n)]
    q = rng.normal(size=(nq, m * dsub)).astype(np.float32)
    return cent, codes, q


def gpu_search(cent, codes, q, k, variant=ScanVariant.FusedWarp, tuning=None):
    with PQSearcher(cent, codes) as s:
        if tuning:
            s.set_tuning(tuning)
        out, _ = s.search(q, k, variant)
        return out["dist"].copy(), out["id"].copy(), s.last_launch()


def test_device_info():
    info = device_info(0)
    assert info.sm_count > 0 and info.peak_bandwidth_gbs > 0 and info.max_smem_per_block >= 200 * 1024
    print(f"{info.name}: {info.sm_count} SMs, {info.peak_bandwidth_gbs:.0f} GB/s, {info.clock_mhz} MHz")


@pytest.mark.parametrize("k", [1, 8, 10, 16, 32, 33, 64, 100, 128])
def test_golden_gpu_fixture(golden, k):
    g = golden("gpu_fixture")
    d, i, _ = gpu_search(g["centroids"], g["codes"], g["queries"], k)
    assert_same_topk(d, i, g[f"d_k{k}"], g[f"i_k{k}"], f"k={k}")


def test_golden_cpu_fixture_m8(golden):
    """m = 8: the fused (non word-interleaved) variants accept it; results match the reference exactly."""
    g = golden("cpu_fixture")
    for v in [ScanVariant.GlobalLut, ScanVariant.SharedLut, ScanVariant.Interleaved, ScanVariant.Fused,
              ScanVariant.FusedReg]:
        d, i, _ = gpu_search(g["centroids"], g["codes"], g["queries"], 10, v)
        assert_same_topk(d, i, g["top_d"], g["top_i"], str(v))


def test_golden_c0_small(golden):
    g = golden("c0_small")
    d, i, _ = gpu_search(g["centroids"], g["codes"], g["queries"], 10)
    assert_same_topk(d, i, g["top_d"], g["top_i"], "c0 small")


@pytest.mark.parametrize("k", [10, 100])
@pytest.mark.parametrize("q", [1, 2, 4, 8])
def test_golden_ties(golden, k, q):
    g = golden("ties")
    d, i, _ = gpu_search(g["centroids"], g["codes"], g["queries"], k, tuning=Tuning(queries_per_block=q))
    assert_same_topk(d, i, g[f"d_k{k}"], g[f"i_k{k}"], f"ties k={k} Q={q}")


def test_distances_every_scan_variant(golden, port):
    """Reference tests/test_gpu.cpp:69-79, bit-exact: the materialising scan equals the CPU ADC matrix."""
    g = golden("gpu_fixture")
    lut = port.compute_lut(g["centroids"], g["queries"])
    expected = port.adc_scan(lut, g["codes"])
    with PQSearcher(g["centroids"], g["codes"]) as s:
        for v in SCANS:
            got, _ = s.distances(g["queries"], v)
            assert np.array_equal(bits(got), bits(expected)), v
        for threads in (64, 128, 512):
            s.set_tuning(Tuning(scan_threads=threads))
            got, _ = s.distances(g["queries"], ScanVariant.SharedLut)
            assert np.array_equal(bits(got), bits(expected))
        with pytest.raises(VkError):
            s.distances(g["queries"], ScanVariant.FusedWarp)


def test_distances_cpu_fixture_m8(golden):
    g = golden("cpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        got, _ = s.distances(g["queries"], ScanVariant.Interleaved)
    assert np.array_equal(bits(got), bits(g["dists"]))


@pytest.mark.parametrize("variant", SCANS + FUSED)
def test_all_variants_k10(golden, variant):
    g = golden("gpu_fixture")
    d, i, _ = gpu_search(g["centroids"], g["codes"], g["queries"], 10, variant)
    assert_same_topk(d, i, g["d_k10"], g["i_k10"], str(variant))


@pytest.mark.parametrize("prune", [True, False], ids=["early_abandon", "full_scan"])
@pytest.mark.parametrize("q", [1, 2, 4, 8])
@pytest.mark.parametrize("ilp", [1, 2, 4])
@pytest.mark.parametrize("k", [1, 10, 33, 64, 128])
def test_every_q_ilp_k(golden, q, ilp, k, prune):
    """nq = 37 is prime, so every Q > 1 leaves a partial last group (reference tests/test_gpu.cpp:93-101).
    Both the exact early-abandoning scan and the full scan must give the reference's results."""
    g = golden("gpu_fixture")
    d, i, shape = gpu_search(g["centroids"], g["codes"], g["queries"], k,
                             tuning=Tuning(queries_per_block=q, vectors_per_step=ilp, early_abandon=prune))
    assert_same_topk(d, i, g[f"d_k{k}"], g[f"i_k{k}"], f"Q={q} ILP={ilp} k={k} prune={prune}")
    assert shape.queries_per_block == q and shape.grid_y == -(-37 // q)


@pytest.mark.parametrize("m,dsub", [(16, 8), (32, 4), (64, 2)])
@pytest.mark.parametrize("k", [1, 10, 100])
def test_early_abandon_on_clustered_data(port, m, dsub, k):
    """Clustered data (where most pairs are abandoned early) with many queries per group: pruned == full ==
    oracle, bit for bit."""
    from veckern_b200 import data

    x = data.gen_mixture(0, 0, 30_011, m * dsub, ncomp=100)
    q = data.gen_mixture(0, 3, 29, m * dsub, ncomp=100)
    cent = data.pq_train(x[:5000], m, 3, 1)
    codes = data.pq_encode(cent, x)
    ed, ei = port.adc_search(cent, codes, q, k)
    for qpb in (2, 4, 8):
        for prune in (True, False):
            d, i, _ = gpu_search(cent, codes, q, k, tuning=Tuning(queries_per_block=qpb, early_abandon=prune))
            assert_same_topk(d, i, ed, ei, f"m={m} k={k} Q={qpb} prune={prune}")


@pytest.mark.parametrize("bpq", [1, 3, 7, 16])
def test_blocks_per_query_overrides(golden, bpq):
    g = golden("gpu_fixture")
    for ilp in (1, 4):
        d, i, shape = gpu_search(g["centroids"], g["codes"], g["queries"], 33,
                                 tuning=Tuning(blocks_per_query=bpq, vectors_per_step=ilp))
        assert_same_topk(d, i, g["d_k33"], g["i_k33"], f"bpq={bpq}")
        assert shape.blocks_x <= bpq


def test_launch_shape_reporting(golden):
    """Reference tests/test_gpu.cpp:131-150: default Q = 2 gives grid_y = ceil(37 / 2) = 19, and one query is
    spread over at least min(wave, ceil(n / (threads * 16))) blocks."""
    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        s.search(g["queries"], 10, ScanVariant.FusedVecMQ)
        shape = s.last_launch()
        assert shape.queries_per_block == 2 and shape.grid_y == 19
        assert shape.blocks_per_sm > 0 and shape.waves > 0
        s.search(g["queries"][:1], 10, ScanVariant.FusedWarp)
        one = s.last_launch()
        wave = one.blocks_x / one.waves
        assert one.blocks_x >= min(wave, np.ceil(s.n / (one.threads * 16.0))) - 0.5


@pytest.mark.parametrize("n,m,dsub,nq,k", [
    (1, 16, 8, 3, 1), (31, 16, 4, 2, 31), (32, 16, 4, 5, 32), (33, 32, 2, 4, 33), (129, 64, 2, 3, 128),
    (1000, 12, 3, 7, 10), (5003, 4, 16, 9, 100), (2047, 20, 1, 6, 17), (4099, 48, 2, 5, 64), (777, 1, 8, 3, 5),
])
def test_random_shapes_against_oracle(port, n, m, dsub, nq, k):
    cent, codes, q = random_db(n * 7 + m, n, m, dsub, nq)
    ed, ei = port.adc_search(cent, codes, q, k)
    for variant in (ScanVariant.FusedReg, ScanVariant.SharedLut):
        for tq in (1, 4, 8):
            d, i, _ = gpu_search(cent, codes, q, k, variant, Tuning(queries_per_block=tq))
            assert_same_topk(d, i, ed, ei, f"n={n} m={m} Q={tq}")


@pytest.mark.parametrize("prune", [True, False])
def test_windowed_item_order_many_query_groups(port, prune):
    """Many query groups (1,400 queries of m = 64: 700 groups x 128 KB of LUTs, more than the L2 share for one
    window) run window by window of groups; results stay those of the oracle."""
    cent, codes, q = random_db(41, 200_003, 64, 2, 1_400)
    ed, ei = port.adc_search(cent, codes, q, 10)
    d, i, shape = gpu_search(cent, codes, q, 10, tuning=Tuning(queries_per_block=2, vectors_per_step=2,
                                                              early_abandon=prune))
    assert shape.grid_y == 700
    assert_same_topk(d, i, ed, ei, f"windowed order prune={prune}")


def test_rejections(golden):
    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        for k in (0, 129):
            with pytest.raises(VkError):
                s.search(g["queries"][:1], k, ScanVariant.Fused)
        with pytest.raises(VkError):
            s.set_tuning(Tuning(queries_per_block=3))
    cg = golden("cpu_fixture")  # m = 8
    with PQSearcher(cg["centroids"], cg["codes"]) as s:
        for v in (ScanVariant.SharedLutVec, ScanVariant.FusedVec, ScanVariant.FusedVecMQ, ScanVariant.FusedWarp):
            with pytest.raises(VkError):
                s.search(cg["queries"], 10, v)
    cent, codes, q = random_db(5, 20, 16, 2, 2)
    with PQSearcher(cent, codes) as s:
        with pytest.raises(VkError):
            s.search(q, 21, ScanVariant.FusedWarp)  # k > n
        out, _ = s.search(q, 20, ScanVariant.FusedWarp)  # k == n is fine
        assert sorted(out["id"][0]) == list(range(20))


def test_empty_query_batch(golden):
    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        out, t = s.search(g["queries"][:0], 10)
        assert out.shape == (0, 10) and t.total_ms() == 0


def test_id_base_offsets_ids(port):
    cent, codes, q = random_db(11, 3000, 16, 4, 4)
    ed, ei = port.adc_search(cent, codes, q, 25)
    with PQSearcher(cent, codes, id_base=1_000_000) as s:
        out, _ = s.search(q, 25)
    assert_same_topk(out["dist"], out["id"] - 1_000_000, ed, ei, "id_base")


def test_repeated_searches_are_identical(golden):
    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        s.set_tuning(Tuning(queries_per_block=4))
        a, _ = s.search(g["queries"], 100)
        for _ in range(3):
            b, _ = s.search(g["queries"], 100)
            assert np.array_equal(a.view(np.int64), b.view(np.int64))


def test_device_path_matches_host_path(golden):
    """vk_search_device (queries and results in HBM, caller's stream) == vk_search (host buffers)."""
    import torch

    from veckern_b200 import device_result_split

    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        s.set_tuning(Tuning(queries_per_block=8, vectors_per_step=4))
        host, _ = s.search(g["queries"], 64)
        d_q = torch.from_numpy(g["queries"]).cuda()
        for stream in (None, torch.cuda.Stream()):
            d_out = torch.empty((d_q.shape[0], 64), dtype=torch.int64, device="cuda")
            s.search_device(d_q, 64, d_out, stream)
            s.sync(stream)
            dd, di = device_result_split(d_out)
            assert_same_topk(dd.cpu().numpy(), di.cpu().numpy(), host["dist"], host["id"], f"stream {stream}")


def test_merge_kernel_matches_oracle(port):
    import torch

    from veckern_b200 import merge_topk_device

    rng = np.random.default_rng(3)
    nq, lists, k_in, k = 23, 7, 40, 37
    d = np.sort(rng.integers(0, 50, size=(nq, lists, k_in)).astype(np.float32), axis=2)  # many ties
    ids = rng.permutation(nq * lists * k_in).astype(np.int32).reshape(nq, lists, k_in) % 997
    ids[:, 3, 30:] = -1  # padding entries are skipped
    # lists must be sorted by (dist, id) for the merge's contract
    order = np.lexsort((ids, d), axis=2)
    d = np.take_along_axis(d, order, 2)
    ids = np.take_along_axis(ids, order, 2)
    pairs = np.stack([d.view(np.int32), ids], axis=-1).astype(np.int32)
    d_in = torch.from_numpy(pairs.copy()).cuda().view(torch.int64).reshape(nq, lists, k_in)
    d_out = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    merge_topk_device(0, d_in, nq, lists, k_in, lists * k_in, k_in, k, d_out)
    torch.cuda.synchronize()
    out = d_out.cpu().numpy().view(np.int32).reshape(nq, k, 2)
    ed, ei = port.merge_topk(d, ids, k)
    assert_same_topk(out[..., 0].view(np.float32), out[..., 1], ed, ei, "merge")


def test_encode_kernel_matches_host():
    import torch

    from veckern_b200 import _native as N
    from veckern_b200 import data

    x = data.gen_mixture(0, 5, 20_000, 128, ncomp=100)
    cent = data.pq_train(x[:5000], 32, 2, 1)
    expected = data.pq_encode(cent, x)
    d_x = torch.from_numpy(x).cuda()
    d_c = torch.empty((x.shape[0], 32), dtype=torch.uint8, device="cuda")
    N.check(N.lib().vk_encode_device(0, N.ptr(cent), 32, 4, N.ptr(d_x), x.shape[0], N.ptr(d_c), None), "encode")
    torch.cuda.synchronize()
    assert np.array_equal(d_c.cpu().numpy(), expected)


def test_generated_database_matches_host_generator(port):
    """Codes generated on the device == the host generator, and search over them == the oracle."""
    import torch

    from veckern_b200 import _native as N
    from veckern_b200 import data

    cdf = data.gen_cdf(4, 64, 16, 0.3)
    rows0, n = 123_457, 40_009
    d_c = torch.empty((n, 16), dtype=torch.uint8, device="cuda")
    N.check(N.lib().vk_gen_codes_device(0, 4, N.ptr(cdf), 64, 16, rows0, n, N.ptr(d_c), None), "gen")
    torch.cuda.synchronize()
    host = data.gen_codes(4, cdf, rows0, n)
    assert np.array_equal(d_c.cpu().numpy(), host)
    cent = data.gen_normal(6, 16 * 256, 8).reshape(16, 256, 8)
    q = data.gen_normal(7, 11, 128)
    with PQSearcher.generated(cent, 4, cdf, rows0, n, id_base=5) as s:
        assert np.array_equal(s.get_codes(), host)
        s.set_tuning(Tuning(queries_per_block=4))
        out, _ = s.search(q, 10)
    ed, ei = port.adc_search(cent, host, q, 10)
    assert_same_topk(out["dist"], out["id"] - 5, ed, ei, "generated")


def test_index_codes_roundtrip(golden):
    g = golden("gpu_fixture")
    with PQSearcher(g["centroids"], g["codes"]) as s:
        assert np.array_equal(s.get_codes(), g["codes"])
        assert np.array_equal(s.get_codes(20_000, 11), g["codes"][20_000:])


def quarter_warp_wavefronts(codes, lanes=8):
    """Mean shared-memory wavefronts of one 16-byte LUT fetch per 32 positions (phases of `lanes` lanes, entry c of a
    table in bank group c % lanes; equal codes in a phase are one access)."""
    n, m = codes.shape
    c = codes[: n // 32 * 32].reshape(-1, 32 // lanes, lanes, m).astype(np.int64)
    total = 0
    for g in c.reshape(-1, lanes, m):
        for s in range(m):
            u = np.unique(g[:, s])
            total += np.bincount(u % lanes, minlength=lanes).max()
    return total / (len(c) * m)


@pytest.mark.parametrize("m,dsub", [(16, 8), (32, 4), (64, 2), (20, 4)])
def test_lane_placement(m, dsub):
    """Rows of every whole 64-row window are permuted (ids unaffected), partial windows keep the identity, codes
    read back in row order, and the placement lowers the bank-group load of 16-byte LUT fetches."""
    rng = np.random.default_rng(m)
    n = 50_003
    cent = rng.normal(size=(m, 256, dsub)).astype(np.float32)
    codes = (rng.normal(128, 40, size=(n, m)).clip(0, 255)).astype(np.uint8)  # skewed, like trained codes
    with PQSearcher(cent, codes) as s:
        perm = s.get_placement()
        assert np.array_equal(s.get_codes(), codes)
        assert np.array_equal(s.get_codes(12_345, 777), codes[12_345:12_345 + 777])
    full = n // 64 * 64
    windows = perm[:full].reshape(-1, 64)
    assert (np.sort(windows, axis=1) == np.arange(64)).all()
    assert (windows != np.arange(64)).any(axis=1).mean() > 0.9
    assert np.array_equal(perm[full:], np.tile(np.arange(64, dtype=np.uint8), (len(perm) - full) // 64))
    placed = codes[(np.arange(full) & ~63) + perm[:full]]
    if m <= 32:  # 16-byte entries; the placement weighs the pruned scan's phase-A sub-spaces most
        ss = {16: 8, 32: 12}.get(m, m)
        before = quarter_warp_wavefronts(codes[:8192, :ss])
        after = quarter_warp_wavefronts(placed[:8192, :ss])
        assert after < 0.9 * before, (before, after)


@pytest.mark.parametrize("m,iters", [(16, 5), (32, 3), (64, 2), (4, 2), (1, 1), (16, 0)])
def test_pq_train_device_matches_host(m, iters):
    """vk_pq_train_device == ProductQuantizer::train's steps on the host (itself pinned to the reference by
    test_host.py): same draws, same arithmetic, bit-identical centroids."""
    from veckern_b200 import data
    x = data.gen_mixture(0, 0, 12_000, 128)
    host = data.pq_train(x, m, iters, 7)
    dev = data.pq_train_gpu(x, m, iters, 7)
    assert np.array_equal(bits(host), bits(dev))


def test_pq_train_device_reseeds_empty_clusters():
    """Few distinct points: duplicate initial centroids leave clusters empty, which are re-seeded with rng() % n
    draws in cluster order (pq.cpp:60-63)."""
    from veckern_b200 import data
    rng = np.random.default_rng(3)
    pts = rng.normal(size=(40, 32)).astype(np.float32)
    x = pts[rng.integers(0, 40, size=700)]
    host = data.pq_train(x, 4, 4, 11)
    dev = data.pq_train_gpu(x, 4, 4, 11)
    assert np.array_equal(bits(host), bits(dev))


def test_index_file_load_and_save(golden, tmp_path):
    """vk_index_load (whole file, row ranges with file-row ids, verified) searches exactly like an index built from
    the same arrays; vk_index_save writes the codes back in row order; damaged files are refused."""
    from veckern_b200 import data
    g = golden("gpu_fixture")
    cent, codes, q = g["centroids"], g["codes"], g["queries"]
    p = tmp_path / "fixture.vkpq"
    data.write_index(p, cent, codes)
    with PQSearcher(cent, codes) as ref, PQSearcher.load(p) as ld:
        assert (ld.n, ld.m, ld.id_base) == (len(codes), codes.shape[1], 0)
        assert np.array_equal(ld.get_codes(), codes)
        a, _ = ref.search(q, 10)
        b, _ = ld.search(q, 10)
        assert np.array_equal(a.view(np.int64), b.view(np.int64))
    lo, hi = 7_001, 19_999
    with PQSearcher(cent, codes[lo:hi], id_base=lo) as ref, PQSearcher.load(p, rows=(lo, hi)) as ld:
        assert ld.id_base == lo
        a, _ = ref.search(q, 33)
        b, _ = ld.search(q, 33)
        assert np.array_equal(a.view(np.int64), b.view(np.int64))
    p2 = tmp_path / "saved.vkpq"
    with PQSearcher(cent, codes) as s:
        s.save(p2)
    c2, k2 = data.read_index(p2)
    assert np.array_equal(c2, cent) and np.array_equal(k2, codes)
    raw = bytearray(p.read_bytes())
    raw[int.from_bytes(raw[48:56], "little") + 99] ^= 1
    bad = tmp_path / "bad.vkpq"
    bad.write_bytes(bytes(raw))
    with pytest.raises(VkError, match="checksum"):
        PQSearcher.load(bad)
    with pytest.raises(VkError):
        PQSearcher.load(p, rows=(0, len(codes) + 1))


@pytest.mark.parametrize("devices,k", [([0, 0, 0], 10), ([0, 0], 128), ([0] * 5, 33)])
def test_multi_gpu_searcher_matches_one_index(golden, devices, k):
    """vk_multi_* (shards listed on the one device here; each shard on its own stream, lists gathered with
    cudaMemcpyPeerAsync and merged) == one index over all rows."""
    from veckern_b200 import MultiPQSearcher
    g = golden("gpu_fixture")
    cent, codes, q = g["centroids"], g["codes"], g["queries"]
    with PQSearcher(cent, codes) as one, MultiPQSearcher(cent, codes, devices=devices) as mx:
        assert (mx.n, mx.shards) == (len(codes), len(devices))
        a, _ = one.search(q, k)
        b, t = mx.search(q, k)
        assert np.array_equal(a.view(np.int64), b.view(np.int64))
        assert t.scan_ms > 0


def test_multi_gpu_searcher_pads_small_shards_and_loads(tmp_path):
    """Shards with fewer than k rows (their lists padded for the merge), and shards loaded from one index file."""
    from veckern_b200 import MultiPQSearcher, data
    cent, codes, q = random_db(21, 301, 16, 8, 9, dup_rows=40)
    with PQSearcher(cent, codes) as one:
        a, _ = one.search(q, 100)
    with MultiPQSearcher(cent, codes, devices=[0, 0, 0, 0]) as mx:
        b, _ = mx.search(q, 100)
    assert np.array_equal(a.view(np.int64), b.view(np.int64))
    p = tmp_path / "db.vkpq"
    data.write_index(p, cent, codes)
    with MultiPQSearcher.load(p, devices=[0, 0, 0]) as mx:
        c, _ = mx.search(q, 100)
    assert np.array_equal(a.view(np.int64), c.view(np.int64))
    with pytest.raises(VkError):
        MultiPQSearcher(cent, codes[:3], devices=[0] * 4)


def test_rerank_kernel_matches_reference(golden, port):
    """GPU exact re-rank == the reference's rerank_exact (fixture) and the oracle (duplicates, padding, ties)."""
    import torch

    from veckern_b200 import data, rerank_device

    g = golden("cpu_fixture")
    base = data.synthetic_clustered(4000, 32, 20, 7)

    def gpu(base, q, cand_ids, k):
        pairs = np.stack([np.zeros_like(cand_ids), cand_ids], axis=-1).astype(np.int32)
        d_c = torch.from_numpy(np.ascontiguousarray(pairs)).cuda().view(torch.int64).reshape(cand_ids.shape)
        d_out = torch.empty((q.shape[0], k), dtype=torch.int64, device="cuda")
        rerank_device(0, torch.from_numpy(base).cuda(), torch.from_numpy(q).cuda(), d_c, k, d_out)
        torch.cuda.synchronize()
        o = d_out.cpu().numpy().view(np.int32).reshape(q.shape[0], k, 2)
        return o[..., 0].view(np.float32), o[..., 1]

    d, i = gpu(base, g["queries"], g["cand_i"], 10)
    assert_same_topk(d, i, g["rr_d"], g["rr_i"], "rerank fixture")
    rng = np.random.default_rng(8)
    base = rng.integers(-2, 3, size=(500, 16)).astype(np.float32)
    q = rng.integers(-2, 3, size=(37, 16)).astype(np.float32)
    cand = rng.integers(-1, 500, size=(37, 90)).astype(np.int32)
    for k in (1, 10, 64, 128):
        ed, ei = port.rerank_exact(base, q, cand, k)
        d, i = gpu(base, q, cand, k)
        assert_same_topk(d, i, ed, ei, f"rerank k={k}")
