"""Shared test fixtures. GPU tests are marked `gpu` (run with -m gpu on a B200); everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size configuration checks")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden():
    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = load_golden(name)
        return cache[name]

    return get


@pytest.fixture(scope="session")
def port():
    import oracle

    return oracle.port()


def bits(a: np.ndarray) -> np.ndarray:
    """float32 array as its uint32 bit patterns (bit-exact comparisons)."""
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_same_topk(got_d, got_i, exp_d, exp_i, what=""):
    got_d = np.asarray(got_d, np.float32)
    exp_d = np.asarray(exp_d, np.float32)
    got_i = np.asarray(got_i, np.int32)
    exp_i = np.asarray(exp_i, np.int32)
    assert got_i.shape == exp_i.shape, f"{what}: shape {got_i.shape} vs {exp_i.shape}"
    bad = np.argwhere((got_i != exp_i) | (bits(got_d) != bits(exp_d)))
    if bad.size:
        q, j = bad[0]
        raise AssertionError(f"{what}: {len(bad)} mismatches; first at query {q} rank {j}: got ({got_d[q, j]!r}, "
                             f"{got_i[q, j]}) expected ({exp_d[q, j]!r}, {exp_i[q, j]})")
