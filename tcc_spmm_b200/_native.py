"""ctypes bindings of the two in-tree native libraries.

``lib()`` loads ``_lib/libtcc_spmm_b200.so`` (the C ABI of include/tcc_spmm_b200.h) and
``workloads()`` loads ``_lib/libtcc_workloads.so``. A missing library raises ImportError:
there is no Python fallback for any operator.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIBDIR = Path(__file__).resolve().parent / "_lib"
_lib = None
_wl = None

u8p = C.POINTER(C.c_uint8)
i8p = C.POINTER(C.c_int8)
u32p = C.POINTER(C.c_uint32)
u64p = C.POINTER(C.c_uint64)
f32p = C.POINTER(C.c_float)


class Sw32Task(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("sw", "begin", "end", "partial", "mask", "chunks", "reduceFirst")]


class Sw32ReduceRange(C.Structure):
    _fields_ = [("begin", C.c_uint32), ("end", C.c_uint32)]


class Sw32DeviceView(C.Structure):
    """Byte-compatible with Sw32DeviceView / tcc_sw32_device_view (nine pointers + u32)."""

    _fields_ = [
        ("windowOffsets", C.c_void_p),
        ("sourceIds", C.c_void_p),
        ("rowGroupMasks", C.c_void_p),
        ("sourceMetadata", C.c_void_p),
        ("values", C.c_void_p),
        ("bucketOffsets", C.c_void_p),
        ("tasks", C.c_void_p),
        ("reductions", C.c_void_p),
        ("partialIds", C.c_void_p),
        ("taskCount", C.c_uint32),
    ]


class Sw32Sizes(C.Structure):
    _fields_ = [
        ("rows", C.c_uint32),
        ("cols", C.c_uint32),
        ("partialCount", C.c_uint32),
        ("bucketed", C.c_uint32),
        ("windowOffsets", C.c_uint64),
        ("sourceIds", C.c_uint64),
        ("rowGroupMasks", C.c_uint64),
        ("values", C.c_uint64),
        ("bucketOffsets", C.c_uint64),
        ("tasks", C.c_uint64),
        ("reductions", C.c_uint64),
        ("partialIds", C.c_uint64),
    ]


class Sw32Arrays(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("windowOffsets", "sourceIds", "rowGroupMasks", "sourceMetadata", "values",
                                          "bucketOffsets", "tasks", "reductions", "partialIds")]


class WlCsr(C.Structure):
    _fields_ = [
        ("rows", C.c_uint32),
        ("cols", C.c_uint32),
        ("nnz", C.c_uint64),
        ("rowOffsets", u32p),
        ("sourceIds", u32p),
        ("values", f32p),
    ]


# Exported C ABI: name -> (restype, argtypes). Kept in sync with include/tcc_spmm_b200.h;
# tests check that every declaration of the header is exported.
SIGNATURES = {
    "tcc_last_error": (C.c_char_p, []),
    "tcc_version": (C.c_char_p, []),
    "tcc_launch_spmm_int8": (C.c_int, [C.POINTER(Sw32DeviceView), C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
                                       C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "tcc_launch_spmm_int8_variant": (C.c_int, [C.POINTER(Sw32DeviceView), C.c_void_p, C.c_void_p, C.c_void_p,
                                               C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p,
                                               C.c_void_p, C.c_int]),
    "tcc_quantize_features_int8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]),
    "tcc_pack_features_int8x16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]),
    "tcc_quantize_pack_features_int8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                                  C.c_void_p]),
    "tcc_spmm_workspace_size": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, u64p, u64p]),
    "tcc_device_status": (C.c_int, [u32p, C.c_int]),
    "tcc_launch_spmm_int8_static_workspace": (C.c_int, [C.POINTER(Sw32DeviceView), C.c_void_p, C.c_void_p, C.c_void_p,
                                                        C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                                        C.c_void_p]),
    "tcc_spmm_launch_shape": (C.c_int, [C.c_uint32, C.c_int, u32p, u32p, u32p, C.POINTER(C.c_int)]),
    "tcc_make_canonical_csr": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, u32p, u32p, f32p,
                                         C.POINTER(C.c_void_p)]),
    "tcc_csr_arrays": (C.c_int, [C.c_void_p, u32p, C.POINTER(u32p), C.POINTER(u32p), C.POINTER(f32p), u64p]),
    "tcc_csr_free": (None, [C.c_void_p]),
    "tcc_load_matrix_market": (C.c_int, [C.c_char_p, u32p, C.POINTER(C.c_void_p)]),
    "tcc_convert_csr_to_sw32": (C.c_int, [C.c_uint32, C.c_uint32, u32p, u32p, f32p, C.c_uint64, C.c_int, C.c_uint32,
                                          C.POINTER(C.c_void_p)]),
    "tcc_sw32_host_sizes": (C.c_int, [C.c_void_p, C.POINTER(Sw32Sizes)]),
    "tcc_sw32_host_arrays": (C.c_int, [C.c_void_p, C.POINTER(Sw32Arrays)]),
    "tcc_sw32_host_free": (None, [C.c_void_p]),
    "tcc_partition_tasks": (C.c_int, [C.c_void_p, C.c_uint32, u32p, C.c_uint32, C.c_uint32, u32p]),
    "tcc_balance_tasks": (C.c_int, [C.c_void_p, C.c_uint32, u32p, C.c_uint32, C.c_uint32, C.c_void_p]),
    "tcc_balance_tasks_padded": (C.c_int, [C.c_void_p, C.c_uint32, u32p, C.c_uint32, C.c_uint32, C.c_uint32,
                                           C.c_void_p, C.c_uint64, C.POINTER(C.c_uint32)]),
    "tcc_convert_csr_to_sw32_device": (C.c_int, [C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                                                 C.c_uint64, C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]),
    "tcc_sw32_device_sizes": (C.c_int, [C.c_void_p, C.POINTER(Sw32Sizes)]),
    "tcc_sw32_device_arrays": (C.c_int, [C.c_void_p, C.POINTER(Sw32Arrays)]),
    "tcc_sw32_device_view_of": (C.c_int, [C.c_void_p, C.POINTER(Sw32DeviceView)]),
    "tcc_sw32_device_free": (None, [C.c_void_p]),
    "tcc_sw32_device_trim": (C.c_int, []),
    "tcc_device_matrix_upload": (C.c_int, [C.POINTER(Sw32Sizes), C.POINTER(Sw32Arrays), C.c_uint32, C.c_void_p,
                                           C.POINTER(C.c_void_p)]),
    "tcc_device_matrix_view": (C.c_int, [C.c_void_p, C.POINTER(Sw32DeviceView)]),
    "tcc_device_matrix_workspace": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    "tcc_device_matrix_free": (None, [C.c_void_p]),
}

# Failure-path test hooks of the library (exported, not declared in the public header).
TEST_SIGNATURES = {
    "tcc_test_launch_spmm_int8_stalled": (C.c_int, [C.POINTER(Sw32DeviceView), C.c_void_p, C.c_void_p, C.c_void_p,
                                                    C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p,
                                                    C.c_uint32, C.c_int, C.c_void_p]),
    "tcc_test_static_counters_nonzero": (C.c_int, [u64p]),
}

WL_SIGNATURES = {
    "tcc_wl_last_error": (C.c_char_p, []),
    "tcc_wl_free": (None, [C.POINTER(WlCsr)]),
    "tcc_wl_poisson": (C.c_int, [C.c_uint32, C.c_uint32, C.c_double, C.c_uint64, C.c_uint32,
                                 C.POINTER(C.POINTER(WlCsr))]),
    "tcc_wl_powerlaw": (C.c_int, [C.c_uint32, C.c_uint64, C.c_double, C.c_uint32, C.c_double, C.c_uint32, C.c_uint64,
                                  C.c_uint32, C.POINTER(C.POINTER(WlCsr))]),
    "tcc_wl_stress": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                C.c_uint64, C.c_uint32, C.POINTER(C.POINTER(WlCsr))]),
    "tcc_wl_rmat": (C.c_int, [C.c_uint32, C.c_uint64, C.c_double, C.c_double, C.c_double, C.c_uint64, C.c_uint32,
                              C.POINTER(C.POINTER(WlCsr))]),
    "tcc_wl_normal": (C.c_int, [f32p, C.c_uint64, C.c_uint64, C.c_uint32]),
    "tcc_wl_rmat_device": (C.c_int, [C.c_uint32, C.c_uint64, C.c_double, C.c_double, C.c_double, C.c_uint64,
                                     C.c_void_p, C.POINTER(C.c_void_p)]),
    "tcc_wl_device_csr_arrays": (C.c_int, [C.c_void_p, u32p, u32p, u64p, C.POINTER(C.c_void_p),
                                           C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    "tcc_wl_device_csr_free": (None, [C.c_void_p]),
}


def library_path() -> Path:
    return _LIBDIR / "libtcc_spmm_b200.so"


def _load(path: Path, signatures: dict) -> C.CDLL:
    if not path.exists():
        raise ImportError(f"native library {path} is missing; run `python -m tcc_spmm_b200.build` "
                          "(there is no fallback implementation)")
    handle = C.CDLL(str(path), mode=os.RTLD_LOCAL | os.RTLD_NOW)
    for name, (restype, argtypes) in signatures.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return handle


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = _load(library_path(), {**SIGNATURES, **TEST_SIGNATURES})
    return _lib


def workloads() -> C.CDLL:
    global _wl
    if _wl is None:
        _wl = _load(_LIBDIR / "libtcc_workloads.so", WL_SIGNATURES)
    return _wl
