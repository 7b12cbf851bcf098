"""GPU: the drop-in C++ boundary. The reference's callers link veckern::gpu::PQSearcher (include/veckern/gpu.hpp);
these tests run that class, not the Python mirror:

* the reference's own GPU test suite (its tests/test_gpu.cpp, compiled unchanged against this repository's
  libveckern_b200.so by `oracle/Makefile dropin` where the reference sources exist) must report 0 failures;
* a C++ driver of PQSearcher (tests/cpp/searcher_check.cpp, built here with g++ against include/) must return
  results bit-identical to the golden outputs of the reference's CPU path, under the reference's default Tuning and
  under the benchmark's.
"""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import REPO, assert_same_topk

pytestmark = pytest.mark.gpu

NATIVE = REPO / "veckern_b200" / "_native"


def test_reference_gpu_suite_against_dropin():
    exe = REPO / "oracle" / "_ref" / "test_gpu"
    if not exe.exists():
        pytest.skip("oracle/_ref/test_gpu is built only where the reference sources exist (make -C oracle dropin)")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert " 0 failed" in out, out[-4000:]


def _build_checker(tmp_path: Path) -> Path:
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path / "searcher_check"
    cmd = [gxx, "-O2", "-std=c++17", f"-I{REPO / 'include'}", str(REPO / "tests" / "cpp" / "searcher_check.cpp"),
           f"-L{NATIVE}", "-lveckern_b200", "-lveckern_b200_host", f"-Wl,-rpath,{NATIVE}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


@pytest.mark.parametrize("k", [10, 100])
def test_cpp_pqsearcher_bit_exact(tmp_path, golden, k):
    g = golden("gpu_fixture")
    cent, codes, q = g["centroids"], g["codes"], g["queries"]
    m, _, dsub = cent.shape
    n, nq = codes.shape[0], q.shape[0]
    (tmp_path / "meta.txt").write_text(f"{n} {m} {dsub} {nq} {k}\n")
    np.ascontiguousarray(cent, np.float32).tofile(tmp_path / "centroids.f32")
    np.ascontiguousarray(codes, np.uint8).tofile(tmp_path / "codes.u8")
    np.ascontiguousarray(q, np.float32).tofile(tmp_path / "queries.f32")
    exe = _build_checker(tmp_path)
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    dt = np.dtype([("dist", "<f4"), ("id", "<i4")])
    for name in ("out_default.bin", "out_q8.bin"):
        out = np.fromfile(tmp_path / name, dt).reshape(nq, k)
        assert_same_topk(out["dist"], out["id"], g[f"d_k{k}"], g[f"i_k{k}"], f"C++ PQSearcher {name}")
    threads, blocks_x, grid_y, qpb, ilp = map(int, (tmp_path / "shape.txt").read_text().split())
    assert qpb == 2 and grid_y == (nq + 1) // 2, "the reference's default Tuning asks for 2 queries per block"
