"""Builds the native libraries in-tree (sm_100a only).

    veckern_b200/_native/libveckern_b200.so       CUDA kernels + C ABI (include/vk_abi.h) + veckern::gpu::PQSearcher
    veckern_b200/_native/libveckern_b200_host.so  PQ training/encoding + data generators (include/vk_host.h)

Run `python -m veckern_b200.build` (or __graft_entry__.build()). Rebuilds only what is out of date.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
OBJ = PKG / "_build"
NATIVE = PKG / "_native"
LIB = NATIVE / "libveckern_b200.so"
HOST_LIB = NATIVE / "libveckern_b200_host.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _tool(name: str) -> str:
    path = shutil.which(name, path="/usr/bin:" + os.environ.get("PATH", ""))
    if not path:
        raise RuntimeError(f"{name} not found")
    return path


def _nvcc() -> str:
    p = CUDA_HOME / "bin" / "nvcc"
    return str(p) if p.exists() else _tool("nvcc")


def _headers() -> list[Path]:
    return (sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((CSRC / "host").glob("*.h"))
            + sorted(INCLUDE.rglob("*.h*")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build(verbose: bool = False, jobs: int | None = None) -> None:
    OBJ.mkdir(exist_ok=True)
    NATIVE.mkdir(exist_ok=True)
    gxx = _tool("g++")
    nvcc = _nvcc()
    headers = _headers()
    cu_srcs = [CSRC / "vk_abi.cu"] + sorted(CSRC.glob("scan_*.cu"))
    jobs_list = []
    objs = []
    for src in cu_srcs:
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src] + headers):
            jobs_list.append([nvcc, *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                              "-ccbin", gxx, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)])
    searcher = CSRC / "host" / "searcher.cpp"
    sobj = OBJ / "searcher.o"
    objs.append(sobj)
    if _stale(sobj, [searcher] + headers):
        jobs_list.append([gxx, "-O2", "-std=c++17", "-fPIC", f"-I{INCLUDE}", f"-I{CUDA_HOME / 'include'}",
                          "-c", str(searcher), "-o", str(sobj)])
    host_src = CSRC / "host" / "host_lib.cpp"
    host_job = None
    if _stale(HOST_LIB, [host_src] + headers):
        host_job = [gxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
                    f"-I{INCLUDE}", f"-I{CSRC}", str(host_src), "-o", str(HOST_LIB)]
        jobs_list.append(host_job)
    if jobs_list:
        with ThreadPoolExecutor(max_workers=jobs or max(1, min(len(jobs_list), os.cpu_count() or 4))) as ex:
            for cmd in jobs_list:
                if verbose:
                    print(" ".join(cmd), flush=True)
            list(ex.map(_run, jobs_list))
    if _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-ccbin", gxx, "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        _run(cmd)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(f"built {LIB} and {HOST_LIB}")
