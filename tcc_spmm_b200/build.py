"""Build recipe of the native libraries, in-tree (the built .so files travel with the repo).

    python -m tcc_spmm_b200.build            # libtcc_spmm_b200.so + libtcc_workloads.so

Device code is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``);
nvcc cross-compiles without a GPU. Host code is C++17, ``-O3``, no fast-math.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "_lib"
BUILD = ROOT / "_build"
INCLUDE = ROOT / "include"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
CUDA_INCLUDE = Path(NVCC).resolve().parent.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB_SOURCES = ["format.cpp", "capi_host.cpp", "cxx_api.cpp", "upload.cpp", "features.cu", "spmm.cu", "format_gpu.cu",
               "matrix_market.cpp"]


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose_ptxas: bool = False) -> Path:
    """Compile libtcc_spmm_b200.so (C ABI + C++ drop-in API + sm_100a kernels)."""
    LIBDIR.mkdir(exist_ok=True)
    obj_dir = BUILD / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    headers = sorted(p for d in (CSRC, INCLUDE) for ext in ("*.h", "*.hpp", "*.cuh") for p in d.rglob(ext))
    objs = []
    for name in LIB_SOURCES:
        src = CSRC / name
        obj = obj_dir / (name + ".o")
        objs.append(obj)
        if not force and not _stale(obj, [src, *headers]):
            continue
        common = ["-I", str(INCLUDE), "-I", str(CSRC), "-O3", "-std=c++17"]
        if name.endswith(".cu"):
            cmd = [NVCC, *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", *common, "-c", str(src),
                   "-o", str(obj)]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
        else:
            cmd = [CXX, "-fPIC", "-pthread", "-Wall", "-Wextra", "-I", str(CUDA_INCLUDE), *common, "-c", str(src),
                   "-o", str(obj)]
        _run(cmd)
    lib = LIBDIR / "libtcc_spmm_b200.so"
    if force or _stale(lib, objs):
        # Link with nvcc so the CUDA runtime is statically linked (no dependency on a
        # particular libcudart soname); C ABI and C++ API symbols are exported explicitly.
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-Xlinker", f"--version-script={CSRC / 'exports.map'}",
              *map(str, objs), "-o", str(lib), "-lpthread"])
    return lib


def build_workloads(force: bool = False) -> Path:
    """Compile libtcc_workloads.so (seeded synthetic matrices: host generators, and the R-MAT
    generator for sm_100a devices)."""
    LIBDIR.mkdir(exist_ok=True)
    obj_dir = BUILD / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    deps = [CSRC / "workloads.h"]
    host_src, gpu_src = CSRC / "workloads.cpp", CSRC / "workloads_gpu.cu"
    host_obj, gpu_obj = obj_dir / "workloads.cpp.o", obj_dir / "workloads_gpu.cu.o"
    if force or _stale(host_obj, [host_src, *deps]):
        _run([CXX, "-O3", "-std=c++17", "-fPIC", "-pthread", "-I", str(CSRC), "-c", str(host_src), "-o", str(host_obj)])
    if force or _stale(gpu_obj, [gpu_src, *deps]):
        _run([NVCC, *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-O3", "-std=c++17", "-I", str(CSRC), "-c", str(gpu_src),
              "-o", str(gpu_obj)])
    lib = LIBDIR / "libtcc_workloads.so"
    if force or _stale(lib, [host_obj, gpu_obj]):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", str(host_obj), str(gpu_obj), "-o", str(lib), "-lpthread"])
    return lib


def build_all(force: bool = False) -> None:
    build_library(force)
    build_workloads(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
