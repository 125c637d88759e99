"""ORACLE build recipe - test infrastructure, not product code.

    python oracle/build.py

1. oracle/_lib/libtcc_oracle.so: the C restatement (tcc_oracle.c), gcc, OpenMP, IEEE
   arithmetic (no fast-math, no FP contraction).
2. When the reference tree is present, the reference compiled from its own sources where they
   lie, outputs only under oracle/_ref/. The tree is located by the REFERENCE_DIR environment
   variable, else by the "reference_path" entry of the repository's BASELINE.json:
     libtcc_ref_host.so        src/format/{sw32,csr,matrix_market}.cpp + ref_host_shim.cpp
     libtcc_ref_cuda_sm80.so   src/kernel/spmm.cu + src/format/{int8_quantize,pack_int8}.cu
                               + ref_cuda_shim.cu as compute_80 PTX (JIT on the B200)
     libtcc_ref_cuda_sm100a.so the same sources compiled for sm_100a
   The reference's own build system (CMake) is not used; its sources need nothing but the
   CUDA runtime and libstdc++. The reference's symbols are hidden inside these libraries.
   On the GPU box the reference tree is absent and the prebuilt files are used as they are.
"""
from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "_lib"
REF_OUT = HERE / "_ref"


def _reference_dir() -> Path | None:
    """The reference source tree: $REFERENCE_DIR, else BASELINE.json's "reference_path"."""
    env = os.environ.get("REFERENCE_DIR")
    if env:
        return Path(env)
    try:
        path = json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
    except (OSError, ValueError):
        return None
    return Path(path) if path else None


REFERENCE = _reference_dir()
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")


def _run(cmd):
    print("+", " ".join(map(str, cmd)), flush=True)
    subprocess.run(list(map(str, cmd)), check=True)


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build_oracle(force: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    out = LIB / "libtcc_oracle.so"
    src = HERE / "tcc_oracle.c"
    if force or _stale(out, [src]):
        _run(["gcc", "-O3", "-march=x86-64-v3", "-fno-fast-math", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
              "-fvisibility=hidden", src, "-o", out, "-lm"])
    return out


def reference_present() -> bool:
    return REFERENCE is not None and (REFERENCE / "src" / "format" / "sw32.cpp").exists()


def build_reference(force: bool = False) -> bool:
    """Compile the reference into oracle/_ref (only where the reference tree exists)."""
    if not reference_present():
        return False
    REF_OUT.mkdir(exist_ok=True)
    inc = REFERENCE / "include"
    host_srcs = [REFERENCE / "src/format/sw32.cpp", REFERENCE / "src/format/csr.cpp",
                 REFERENCE / "src/format/matrix_market.cpp", HERE / "ref_host_shim.cpp"]
    host = REF_OUT / "libtcc_ref_host.so"
    if force or _stale(host, host_srcs):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden", "-I", inc, *host_srcs, "-o", host])
    cuda_srcs = [REFERENCE / "src/kernel/spmm.cu", REFERENCE / "src/format/int8_quantize.cu",
                 REFERENCE / "src/format/pack_int8.cu", HERE / "ref_cuda_shim.cu"]
    for tag, gencode in (("sm80", "arch=compute_80,code=compute_80"), ("sm100a", "arch=compute_100a,code=sm_100a")):
        lib = REF_OUT / f"libtcc_ref_cuda_{tag}.so"
        if force or _stale(lib, cuda_srcs):
            _run([NVCC, "-O3", "-lineinfo", "-std=c++17", "-gencode", gencode, "-shared", "-Xcompiler",
                  "-fPIC,-fvisibility=hidden", "-I", inc, "-I", REFERENCE / "src/kernel", *cuda_srcs, "-o", lib])
    return True


def build_dropin(force: bool = False) -> bool:
    """The reference's own CLI driver (src/main.cu + src/device_matrix.cuh, unmodified) built
    twice into oracle/_ref:
      tcc_spmm_run_ref     against the reference library (all reference sources, sm_100a)
      tcc_spmm_run_dropin  against this repository's headers (include/) and
                           libtcc_spmm_b200.so - the drop-in check: the reference's caller
                           compiles and links unchanged against the new library."""
    if not reference_present():
        return False
    repo = HERE.parent
    lib = repo / "tcc_spmm_b200" / "_lib" / "libtcc_spmm_b200.so"
    if not lib.exists():
        return False
    REF_OUT.mkdir(exist_ok=True)
    main = REFERENCE / "src/main.cu"
    ref_bin = REF_OUT / "tcc_spmm_run_ref"
    srcs = [main, REFERENCE / "src/format/sw32.cpp", REFERENCE / "src/format/csr.cpp",
            REFERENCE / "src/format/matrix_market.cpp", REFERENCE / "src/format/int8_quantize.cu",
            REFERENCE / "src/format/pack_int8.cu", REFERENCE / "src/kernel/spmm.cu"]
    if force or _stale(ref_bin, srcs):
        _run([NVCC, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I", REFERENCE / "include",
              "-I", REFERENCE / "src", "-I", REFERENCE / "src/kernel", "-x", "cu", *srcs, "-o", ref_bin])
    dropin = REF_OUT / "tcc_spmm_run_dropin"
    if force or _stale(dropin, [main, lib, *sorted((repo / "include").rglob("*.h*"))]):
        # Only the repository's include/ precedes the reference's src/ (which holds nothing but
        # main.cu and device_matrix.cuh), so every library header comes from this repository.
        _run([NVCC, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I", repo / "include", "-I",
              REFERENCE / "src", main, "-L", lib.parent, "-ltcc_spmm_b200", "-Xlinker",
              "-rpath=$ORIGIN/../../tcc_spmm_b200/_lib", "-o", dropin])
    return True


if __name__ == "__main__":
    force = "--force" in sys.argv
    build_oracle(force)
    print("reference built" if build_reference(force) else "reference tree absent: using prebuilt oracle/_ref")
