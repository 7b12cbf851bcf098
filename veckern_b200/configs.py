"""The five benchmark configurations (c0..c4), generated deterministically from their seeds.

c0  n=100,000 d=128 N(0,1) rows (seed 0); PQ m=16 from 256 rows picked with seed 1 (train with 0 Lloyd
    iterations); queries nq=100 N(0,1) (seed 2); k=10.
c1  n=1,000,000 d=128 rows of a 1,000-component mixture (means U[0,64]^128 from seed 0, sigma 12, rounded and
    clipped to [0,255]); PQ m in {16,32,64}, 10 Lloyd iterations on a 100,000-row sample (the first 100,000 rows:
    rows are i.i.d. draws), train seed 1; queries nq=1,000 from the same mixture (sample seed 3); k=10.
c2  the first 10,000,000 rows of c1's mixture; m=32 trained as c1; nq=1,000 k=100, and nq=1 k=10.
c3  n=100,000,000 codes generated directly: per row a cluster of 4,096, per sub-space a code drawn from that
    cluster's Dirichlet(0.3) categorical (code seed 4); m=16, centroids N(0,1) dsub=8 (seed 6); queries
    nq=10,000 N(0,1) (seed 7); k=10, Q=4; sharded by id over 1/2/4/8 GPUs.
c4  as c3 with n=1,000,000,000 and code seed 5; k in {10, 100}.
Config 1 stands in for SIFT1M's shapes and value range; no SIFT data is used.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import data

SLICE_ROWS = 2_000_000  # rows generated and encoded at a time for large databases

SPECS = {
    "c0": dict(kind="normal", n=100_000, d=128, m=16, nq=100, k=10, data_seed=0, pq_seed=1, pq_iters=0,
               query_seed=2),
    "c1": dict(kind="mixture", n=1_000_000, d=128, m=16, nq=1000, k=10, mix_seed=0, query_seed=3, pq_seed=1,
               pq_iters=10, train_rows=100_000),
    "c2": dict(kind="mixture", n=10_000_000, d=128, m=32, nq=1000, k=100, mix_seed=0, query_seed=3, pq_seed=1,
               pq_iters=10, train_rows=100_000),
    "c3": dict(kind="generated", n=100_000_000, d=128, m=16, nq=10_000, k=10, code_seed=4, clusters=4096,
               alpha=0.3, centroid_seed=6, query_seed=7, queries_per_block=4),
    "c4": dict(kind="generated", n=1_000_000_000, d=128, m=16, nq=10_000, k=10, code_seed=5, clusters=4096,
               alpha=0.3, centroid_seed=6, query_seed=7, queries_per_block=4),
}


@dataclass
class Workload:
    name: str
    spec: dict
    centroids: np.ndarray            # [m, 256, dsub]
    queries: np.ndarray              # [nq, d]
    codes: np.ndarray | None = None  # [n, m] (None for generated configs: see cdf / code_seed)
    cdf: np.ndarray | None = None    # [clusters, m, 256] for generated configs
    base: np.ndarray | None = None   # fp32 database rows (kept only when asked)
    extra: dict = field(default_factory=dict)

    @property
    def n(self) -> int:
        return self.spec["n"]

    @property
    def k(self) -> int:
        return self.spec["k"]


def spec(name: str, **overrides) -> dict:
    s = dict(SPECS[name])
    s.update({k: v for k, v in overrides.items() if v is not None})
    return s


def make_pq4(name: str, *, m: int = 32, n: int | None = None, nq: int | None = None, k: int | None = None,
             keep_base: bool = False, rows: tuple[int, int] | None = None) -> Workload:
    """4-bit PQ variant of a trained configuration (c0, c1, c2): the same database rows, queries and training sample,
    with 16 centroids per sub-space trained by the same steps (data.pq4_train) and codes packed two per byte
    (data.pq4_encode). m = 32 keeps config 1's 16 code bytes per row."""
    w = make(name, n=n, m=m, nq=nq, k=k, keep_base=keep_base, rows=rows, train=data.pq4_train,
             encode=data.pq4_encode)
    w.extra["nbits"] = 4
    return w


def make(name: str, *, n: int | None = None, m: int | None = None, nq: int | None = None, k: int | None = None,
         keep_base: bool = False, encode=None, train=None, rows: tuple[int, int] | None = None) -> Workload:
    """Generates config `name` (optionally resized). encode(centroids, x) -> codes and train(x, m, iters, seed) ->
    centroids may be given to run on the GPU (same results); the defaults run on the host. rows=(lo, hi): only that
    shard of the database is generated and encoded (codes[i] is row lo + i); the codebooks are the same as for the
    whole database."""
    s = spec(name, n=n, m=m, nq=nq, k=k)
    train_fn = train
    d = s["d"]
    lo, hi = rows if rows is not None else (0, s["n"])
    if s["kind"] == "generated":
        cent = data.gen_normal(s["centroid_seed"], s["m"] * 256, d // s["m"]).reshape(s["m"], 256, d // s["m"])
        q = data.gen_normal(s["query_seed"], s["nq"], d)
        cdf = data.gen_cdf(s["code_seed"], s["clusters"], s["m"], s["alpha"])
        return Workload(name, s, cent, q, cdf=cdf)
    if s["kind"] == "normal":
        x = data.gen_normal(s["data_seed"], s["n"], d)  # training draws from all rows
        q = data.gen_normal(s["query_seed"], s["nq"], d)
        train_x = x
        x = x[lo:hi]
    else:
        q = data.gen_mixture(s["mix_seed"], s["query_seed"], s["nq"], d)
        t = min(s["train_rows"], s["n"])
        train_x = data.gen_mixture(s["mix_seed"], s["mix_seed"], t, d)  # rows [0, t): the database's first rows
        cent = (train_fn or data.pq_train)(train_x, s["m"], s["pq_iters"], s["pq_seed"])
        enc = encode or data.pq_encode
        if keep_base or hi - lo <= SLICE_ROWS:
            x = data.gen_mixture(s["mix_seed"], s["mix_seed"], hi - lo, d, row0=lo)
            codes = enc(cent, x)
        else:  # large databases: generate and encode slice by slice, keeping only the codes
            x = None
            codes = None
            for a in range(lo, hi, SLICE_ROWS):
                b = min(hi, a + SLICE_ROWS)
                part = enc(cent, data.gen_mixture(s["mix_seed"], s["mix_seed"], b - a, d, row0=a))
                if codes is None:  # code bytes per row: m, or m / 2 for 4-bit codes
                    codes = np.empty((hi - lo, part.shape[1]), np.uint8)
                codes[a - lo:b - lo] = part
        w = Workload(name, s, cent, q, codes=codes, base=x if keep_base else None)
        w.extra["row0"] = lo
        return w
    cent = (train_fn or data.pq_train)(train_x, s["m"], s["pq_iters"], s["pq_seed"])
    codes = (encode or data.pq_encode)(cent, x)
    w = Workload(name, s, cent, q, codes=codes, base=x if keep_base else None)
    w.extra["row0"] = lo
    return w
