"""Inputs of the benchmark configurations in plain numpy — TEST INFRASTRUCTURE ONLY.

bench.py's reference arm builds its workload with these functions and the reference's own ProductQuantizer
(oracle.ref()), so that the timed reference process maps no library of this repository. They restate the
counter-based generators of the package's host library (veckern_b200/csrc/host/host_lib.cpp, vk_host_gen_normal /
vk_host_gen_mixture, and vk_gen.h's mix64) operation for operation in uint64 / float64 numpy arithmetic; the CPU
tests check them element for element against the host library.

    mix64(x)         SplitMix64 finaliser (uint64 arithmetic wraps mod 2^64, as in C)
    normal_at(k, i)  Box-Muller from the two draws mix64(k + 2i) (open (0, 1)) and mix64(k + 2i + 1) ([0, 1))
    gen_normal       value (row, j) = float(normal_at(key, row * d + j))
    gen_mixture      row's component = hi32(mix64(kpick + row)) * ncomp >> 32; value = clip(rint(mu + sigma *
                     normal_at(knoise, row * d + j)), 0, 255) with means 64 * U[0, 1) from mix64(kmean + e)
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_U = np.uint64
_GOLDEN = _U(0x9E3779B97F4A7C15)
_M1 = _U(0xBF58476D1CE4E5B9)
_M2 = _U(0x94D049BB133111EB)
_TWO_M53 = 1.0 / 9007199254740992.0
_TWO_PI = 6.283185307179586


def mix64(x):
    x = np.asarray(x, dtype=np.uint64) + _GOLDEN
    x = (x ^ (x >> _U(30))) * _M1
    x = (x ^ (x >> _U(27))) * _M2
    return x ^ (x >> _U(31))


def _mix_scalar(x: int) -> np.uint64:
    return mix64(np.array([x], np.uint64))[0]


def _normal_at(key: np.uint64, idx: np.ndarray) -> np.ndarray:
    two = idx * _U(2)
    u1 = ((mix64(key + two) >> _U(11)).astype(np.float64) + 0.5) * _TWO_M53
    u2 = (mix64(key + two + _U(1)) >> _U(11)).astype(np.float64) * _TWO_M53
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(_TWO_PI * u2)


def _blocks(rows: int, block: int, fill) -> None:
    """fill(a, b) for row blocks [a, b), on a thread pool (numpy's ufuncs release the GIL)."""
    starts = range(0, rows, block)
    with ThreadPoolExecutor(max_workers=max(1, min(len(starts), len(os.sched_getaffinity(0))))) as ex:
        list(ex.map(lambda a: fill(a, min(rows, a + block)), starts))


def gen_normal(seed: int, rows: int, d: int, row0: int = 0, block: int = 1 << 13) -> np.ndarray:
    key = _mix_scalar(int(seed) ^ 0x4E4F524D414C5321)
    out = np.empty((rows, d), np.float32)
    j = np.arange(d, dtype=np.uint64)

    def fill(a, b):
        r = np.arange(row0 + a, row0 + b, dtype=np.uint64)
        out[a:b] = _normal_at(key, r[:, None] * _U(d) + j[None, :]).astype(np.float32)
    _blocks(rows, block, fill)
    return out


def gen_mixture(mix_seed: int, sample_seed: int, rows: int, d: int = 128, ncomp: int = 1000, sigma: float = 12.0,
                row0: int = 0, block: int = 1 << 13) -> np.ndarray:
    kmean = _mix_scalar(int(mix_seed) ^ 0x4D49585F4D45414E)
    kpick = _mix_scalar(int(sample_seed) ^ 0x4D49585F5049434B)
    knoise = _mix_scalar(int(sample_seed) ^ 0x4D49585F4E4F4953)
    e = np.arange(ncomp * d, dtype=np.uint64)
    means = (64.0 * ((mix64(kmean + e) >> _U(11)).astype(np.float64) * _TWO_M53)).astype(np.float32).reshape(ncomp, d)
    sig = float(np.float32(sigma))
    out = np.empty((rows, d), np.float32)
    j = np.arange(d, dtype=np.uint64)

    def fill(a, b):
        r = np.arange(row0 + a, row0 + b, dtype=np.uint64)
        comp = (((mix64(kpick + r) >> _U(32)) * _U(ncomp)) >> _U(32)).astype(np.int64)
        v = means[comp].astype(np.float64) + sig * _normal_at(knoise, r[:, None] * _U(d) + j[None, :])
        # + 0.0 turns the -0.0 of rint(-0.3) into +0.0, as std::max(0.0, v) returns its first argument on a tie
        out[a:b] = (np.clip(np.rint(v), 0.0, 255.0) + 0.0).astype(np.float32)
    _blocks(rows, block, fill)
    return out


def reference_workload(spec: dict, ref):
    """(centroids [m, 256, dsub], codes [n, m], queries [nq, d]) of a mixture or normal configuration, with the
    codebook trained and the database encoded by the reference's own ProductQuantizer (`ref` = oracle.ref()),
    following the configuration's definition (veckern_b200/configs.py)."""
    d, m, n = spec["d"], spec["m"], spec["n"]
    if spec["kind"] == "normal":
        x = gen_normal(spec["data_seed"], n, d)
        q = gen_normal(spec["query_seed"], spec["nq"], d)
        train_x = x
    elif spec["kind"] == "mixture":
        q = gen_mixture(spec["mix_seed"], spec["query_seed"], spec["nq"], d)
        x = None
        train_x = gen_mixture(spec["mix_seed"], spec["mix_seed"], min(spec["train_rows"], n), d)
    else:
        raise ValueError(f"no numpy generator for {spec['kind']} configurations")
    pq = ref.pq(d, m)
    pq.train(train_x, train_x.shape[0], spec["pq_iters"], spec["pq_seed"])
    if x is not None:
        codes = pq.encode(x)
    else:
        codes = np.empty((n, m), np.uint8)
        step = 1 << 20
        for a in range(0, n, step):
            b = min(n, a + step)
            codes[a:b] = pq.encode(gen_mixture(spec["mix_seed"], spec["mix_seed"], b - a, d, row0=a))
    return pq, codes, q
