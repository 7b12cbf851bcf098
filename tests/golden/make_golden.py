"""Generates the golden fixtures in this directory by running the reference's own CPU library.

The reference (shivdeshpande/VecKern) ships no golden data files; its tests generate fixtures from seeds. This
script runs the reference's code itself (oracle/_ref/libveckern_ref.so, built from the reference's unmodified
src/cpu/*.cpp by oracle/Makefile) on small seeded inputs and stores inputs and outputs, so that tests on machines
without the reference can pin the CPU oracle and the GPU path to the reference's results.

    make -C oracle ref && python tests/golden/make_golden.py

Fixtures (npz):
  topk_kat.npz       TopK known-answer test of the reference (tests/test_cpu.cpp:33-46) plus tie-heavy sequences
  cpu_fixture.npz    the reference CPU test fixture (tests/test_cpu.cpp:14-24): n=4000 d=32 m=8 nq=12,
                     LUT, full ADC matrix, top-10
  gpu_fixture.npz    the reference GPU test fixture's shapes (tests/test_gpu.cpp:15-31) with n reduced to 20,011:
                     d=64 m=16 nq=37; adc_search for k in {1, 8, 10, 16, 32, 33, 64, 100, 128}
  c0_small.npz       config 0's pipeline at n=20,000: N(0,1) rows, PQ from 256 rows picked with seed 1
                     (train with 0 iterations), N(0,1) queries, k=10
  ties.npz           a database with many duplicate codes (exact distance ties), k in {10, 100}
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import oracle  # noqa: E402
from veckern_b200 import data  # noqa: E402


def main() -> None:
    R = oracle.ref()

    # ---- TopK KAT + tie-heavy sequences
    vals = np.array([5, 1, 4, 1, 3], np.float32)
    kat_d, kat_i = R.topk_push_all(vals, np.arange(5, dtype=np.int32), 3)
    pad_d, pad_i = R.topk_push_all(np.array([2.0], np.float32), np.array([9], np.int32), 4)
    rng = np.random.default_rng(1234)
    seq_v = rng.integers(0, 8, size=(6, 500)).astype(np.float32)
    seq_i = np.stack([rng.permutation(500).astype(np.int32) for _ in range(6)])
    seq_k = np.array([1, 3, 10, 32, 33, 128], np.int32)
    seq_out_d = np.full((6, 128), np.nan, np.float32)
    seq_out_i = np.full((6, 128), -2, np.int32)
    for r in range(6):
        d, i = R.topk_push_all(seq_v[r], seq_i[r], int(seq_k[r]))
        seq_out_d[r, : seq_k[r]] = d
        seq_out_i[r, : seq_k[r]] = i
    np.savez_compressed(HERE / "topk_kat.npz", kat_values=vals, kat_d=kat_d, kat_i=kat_i, pad_d=pad_d,
                        pad_i=pad_i, seq_v=seq_v, seq_i=seq_i, seq_k=seq_k, seq_out_d=seq_out_d,
                        seq_out_i=seq_out_i)

    # ---- reference CPU test fixture
    n, d, m, nq = 4000, 32, 8, 12
    base = R.synthetic_clustered(n, d, 20, 7)
    queries = R.synthetic_clustered(nq, d, 20, 8)
    pq = R.pq(d, m)
    pq.train(base, n, 10, 1)
    codes = pq.encode(base)
    lut = R.compute_lut(pq, queries)
    dists = R.adc_scan(lut, codes)
    top_d, top_i = R.adc_search(pq, codes, queries, 10)
    np.savez_compressed(HERE / "cpu_fixture.npz", queries=queries, centroids=pq.centroids, codes=codes,
                        lut=lut, dists=dists, top_d=top_d, top_i=top_i)

    # ---- reference GPU test fixture shapes (n reduced)
    n, d, m, nq = 20_011, 64, 16, 37
    base = R.synthetic_clustered(n, d, 50, 11)
    queries = R.synthetic_clustered(nq, d, 50, 12)
    pq = R.pq(d, m)
    pq.train(base, 8_000, 8, 1)
    codes = pq.encode(base)
    out = {}
    for k in (1, 8, 10, 16, 32, 33, 64, 100, 128):
        out[f"d_k{k}"], out[f"i_k{k}"] = R.adc_search(pq, codes, queries, k)
    np.savez_compressed(HERE / "gpu_fixture.npz", queries=queries, centroids=pq.centroids, codes=codes, **out)

    # ---- config 0 pipeline at reduced n
    n, nq = 20_000, 100
    x = data.gen_normal(0, n, 128)
    q = data.gen_normal(2, nq, 128)
    pq = R.pq(128, 16)
    pq.train(x, n, 0, 1)
    codes = pq.encode(x)
    top_d, top_i = R.adc_search(pq, codes, q, 10)
    np.savez_compressed(HERE / "c0_small.npz", queries=q, centroids=pq.centroids, codes=codes, top_d=top_d,
                        top_i=top_i)

    # ---- exact ties: few distinct code rows, repeated
    n, m, nq = 6_007, 16, 9
    rng = np.random.default_rng(99)
    cent = rng.integers(-3, 4, size=(m, 256, 4)).astype(np.float32)  # small integers: many equal LUT values
    uniq = rng.integers(0, 256, size=(23, m)).astype(np.uint8)
    codes = uniq[rng.integers(0, 23, size=n)]
    q = rng.integers(-3, 4, size=(nq, m * 4)).astype(np.float32)
    pq = R.pq(m * 4, m)
    pq.centroids = cent
    out = {}
    for k in (10, 100):
        out[f"d_k{k}"], out[f"i_k{k}"] = R.adc_search(pq, codes, q, k)
    np.savez_compressed(HERE / "ties.npz", queries=q, centroids=cent, codes=codes, **out)
    for p in sorted(HERE.glob("*.npz")):
        print(f"{p.name}: {p.stat().st_size / 1024:.0f} KB")


if __name__ == "__main__":
    main()
