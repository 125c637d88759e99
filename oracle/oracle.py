"""ORACLE - test infrastructure, not product code.

ctypes front end of oracle/_lib/libtcc_oracle.so (the C restatement) and of the reference
libraries compiled into oracle/_ref (see oracle/build.py). Nothing here imports the product
package; inputs and outputs are numpy arrays, device buffers are raw addresses.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
_o = None
_rh = None
_rc = {}

u32p = C.POINTER(C.c_uint32)
u64p = C.POINTER(C.c_uint64)
f32p = C.POINTER(C.c_float)
f64p = C.POINTER(C.c_double)
i8p = C.POINTER(C.c_int8)


def _lib() -> C.CDLL:
    global _o
    if _o is None:
        path = HERE / "_lib" / "libtcc_oracle.so"
        if not path.exists():
            raise ImportError(f"{path} missing; run `python oracle/build.py`")
        _o = C.CDLL(str(path), mode=os.RTLD_LOCAL)
        _o.oracle_tf32_rna.restype = C.c_float
        _o.oracle_tf32_rna.argtypes = [C.c_float]
        _o.oracle_tf32_bits.restype = C.c_float
        _o.oracle_tf32_bits.argtypes = [C.c_float]
        _o.oracle_tf32_rna_array.argtypes = [f32p, f32p, C.c_uint64]
        _o.oracle_quantize.argtypes = [f32p, i8p, f32p, C.c_uint32, C.c_uint32]
        _o.oracle_pack16.argtypes = [i8p, i8p, C.c_uint32, C.c_uint32]
        _o.oracle_spmm.restype = C.c_int
        _o.oracle_spmm.argtypes = [u32p, u32p, u64p, f32p, i8p, f32p, C.c_uint32, C.c_uint32, C.c_uint32, u32p,
                                   C.c_uint32, f32p, f64p, C.c_int]
        _o.oracle_max_threads.restype = C.c_int
    return _o


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(C.POINTER(t))


def max_threads() -> int:
    return int(_lib().oracle_max_threads())


def tf32_rna(x: np.ndarray) -> np.ndarray:
    """cvt.rna.tf32.f32 restated on exact values (reference src/kernel/spmm_kernel.cuh:7-11)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    _lib().oracle_tf32_rna_array(_p(x, C.c_float), _p(out, C.c_float), x.size)
    return out


def tf32_bits(x: np.ndarray) -> np.ndarray:
    """The same rounding done on the bit pattern (used inside the oracle's SpMM loop)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    special = (u & 0x7F800000) == 0x7F800000
    r = ((u + 0x1000) & 0xFFFFE000).astype(np.uint32)
    r = np.where(special, u.astype(np.uint32), r)
    return r.view(np.float32)


def quantize(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(q, scale) of reference src/format/int8_quantize.cu:4-25."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    sources, features = x.shape
    q = np.empty((sources, features), dtype=np.int8)
    s = np.empty(sources, dtype=np.float32)
    _lib().oracle_quantize(_p(x, C.c_float), _p(q, C.c_int8), _p(s, C.c_float), sources, features)
    return q, s


def pack16(q: np.ndarray) -> np.ndarray:
    """packed16 bytes of reference src/format/pack_int8.cu:6-15."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    out = np.empty_like(q)
    _lib().oracle_pack16(_p(q, C.c_int8), _p(out, C.c_int8), q.shape[0], q.shape[1])
    return out


def spmm(fmt, q: np.ndarray, scales: np.ndarray, sw_list: Optional[np.ndarray] = None, threads: int = 0,
         with_bound: bool = True) -> tuple[np.ndarray, Optional[np.ndarray], np.ndarray]:
    """Y rows of the listed 32-row windows (all windows by default) as [len*32, F] plus the
    bound sum|a q s| of the tolerance test. `fmt` needs window_offsets, source_ids,
    source_metadata, values, rows and cols. Returns (y, bound, row_index) where row_index maps
    output rows to matrix rows (-1 past the end)."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    features = q.shape[1]
    if sw_list is None:
        sw_list = np.arange(len(fmt.window_offsets) - 1, dtype=np.uint32)
    sw_list = np.ascontiguousarray(sw_list, dtype=np.uint32)
    n = sw_list.size
    y = np.empty((n * 32, features), dtype=np.float32)
    bound = np.empty((n * 32, features), dtype=np.float64) if with_bound else None
    wo = np.ascontiguousarray(fmt.window_offsets, dtype=np.uint32)
    si = np.ascontiguousarray(fmt.source_ids, dtype=np.uint32)
    sm = np.ascontiguousarray(fmt.source_metadata, dtype=np.uint64)
    va = np.ascontiguousarray(fmt.values, dtype=np.float32)
    status = _lib().oracle_spmm(_p(wo, C.c_uint32), _p(si, C.c_uint32), _p(sm, C.c_uint64), _p(va, C.c_float),
                                _p(q, C.c_int8), _p(scales, C.c_float), fmt.rows, fmt.cols, features,
                                _p(sw_list, C.c_uint32), n, _p(y, C.c_float),
                                _p(bound, C.c_double) if bound is not None else None, threads)
    if status != 0:
        raise ValueError("oracle_spmm rejected its arguments")
    rows = (sw_list.astype(np.int64)[:, None] * 32 + np.arange(32)[None, :]).reshape(-1)
    rows[rows >= fmt.rows] = -1
    return y, bound, rows


# ------------------------------------------------------------------------------------------
# The reference itself (oracle/_ref)
# ------------------------------------------------------------------------------------------
class RefError(Exception):
    def __init__(self, kind: int, message: str):
        super().__init__(message)
        self.kind = {1: "invalid_argument", 2: "overflow_error", 3: "runtime_error"}.get(kind, "exception")


def have_ref_host() -> bool:
    return (HERE / "_ref" / "libtcc_ref_host.so").exists()


def have_ref_cuda(tag: str = "sm100a") -> bool:
    return (HERE / "_ref" / f"libtcc_ref_cuda_{tag}.so").exists()


def _ref_host() -> C.CDLL:
    global _rh
    if _rh is None:
        path = HERE / "_ref" / "libtcc_ref_host.so"
        if not path.exists():
            raise ImportError(f"{path} missing; run `python oracle/build.py` where the reference tree exists")
        _rh = C.CDLL(str(path), mode=os.RTLD_LOCAL)
        _rh.ref_convert_csr_to_sw32.restype = C.c_int
        _rh.ref_convert_csr_to_sw32.argtypes = [C.c_uint32, C.c_uint32, u32p, C.c_uint64, u32p, f32p, C.c_uint64,
                                                C.c_int, C.POINTER(C.c_void_p), C.c_char_p, C.c_int]
        _rh.ref_sw32_sizes.argtypes = [C.c_void_p, u64p]
        _rh.ref_sw32_arrays.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
        _rh.ref_sw32_free.argtypes = [C.c_void_p]
        _rh.ref_make_canonical_csr.restype = C.c_int
        _rh.ref_make_canonical_csr.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, u32p, u32p, f32p,
                                               C.POINTER(C.c_void_p), C.c_char_p, C.c_int]
        _rh.ref_load_matrix_market.restype = C.c_int
        _rh.ref_load_matrix_market.argtypes = [C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_int]
        _rh.ref_csr_view.argtypes = [C.c_void_p, u64p, C.POINTER(C.c_void_p)]
        _rh.ref_csr_free.argtypes = [C.c_void_p]
    return _rh


def _copy(ptr, count, dtype):
    if count == 0 or not ptr:
        return np.zeros(0, dtype=dtype)
    nbytes = int(count) * np.dtype(dtype).itemsize
    return np.frombuffer((C.c_char * nbytes).from_address(ptr), dtype=dtype).copy()


REF_SW32_FIELDS = ("window_offsets", "source_ids", "row_group_masks", "source_metadata", "values", "bucket_offsets",
                   "tasks", "reductions", "partial_ids")
_REF_DTYPES = (np.uint32, np.uint32, np.uint32, np.uint64, np.float32, np.uint32, np.uint32, np.uint32, np.uint32)
_REF_WIDTH = (1, 1, 1, 1, 1, 1, 7, 2, 1)


def ref_convert_csr_to_sw32(rows, cols, row_offsets, source_ids, values, bucketed=True) -> dict:
    """The reference's convertCsrToSw32 (src/format/sw32.cpp:69-167) on these arrays. Returns
    a dict of numpy arrays (tasks as [T,7] u32, reductions as [R,2] u32) plus partial_count."""
    lib = _ref_host()
    ro = np.ascontiguousarray(row_offsets, dtype=np.uint32)
    si = np.ascontiguousarray(source_ids, dtype=np.uint32)
    va = np.ascontiguousarray(values, dtype=np.float32)
    handle = C.c_void_p()
    err = C.create_string_buffer(512)
    kind = lib.ref_convert_csr_to_sw32(rows, cols, _p(ro, C.c_uint32), ro.size, _p(si, C.c_uint32),
                                       _p(va, C.c_float), si.size, int(bucketed), C.byref(handle), err, 512)
    if kind:
        raise RefError(kind, err.value.decode())
    try:
        sizes = (C.c_uint64 * 10)()
        ptrs = (C.c_void_p * 9)()
        lib.ref_sw32_sizes(handle, sizes)
        lib.ref_sw32_arrays(handle, ptrs)
        out = {}
        for i, name in enumerate(REF_SW32_FIELDS):
            arr = _copy(ptrs[i], sizes[i] * _REF_WIDTH[i], _REF_DTYPES[i])
            out[name] = arr.reshape(-1, _REF_WIDTH[i]) if _REF_WIDTH[i] > 1 else arr
        out["partial_count"] = int(sizes[9])
        return out
    finally:
        lib.ref_sw32_free(handle)


def _ref_csr(handle) -> tuple:
    lib = _ref_host()
    dims = (C.c_uint64 * 3)()
    ptrs = (C.c_void_p * 3)()
    lib.ref_csr_view(handle, dims, ptrs)
    rows, cols, nnz = int(dims[0]), int(dims[1]), int(dims[2])
    res = (rows, cols, _copy(ptrs[0], rows + 1, np.uint32), _copy(ptrs[1], nnz, np.uint32),
           _copy(ptrs[2], nnz, np.float32))
    lib.ref_csr_free(handle)
    return res


def ref_make_canonical_csr(rows, cols, row_offsets, source_ids, values) -> tuple:
    """The reference's makeCanonicalCsr (src/format/csr.cpp:6-40): (rows, cols, ro, si, va)."""
    lib = _ref_host()
    ro = np.ascontiguousarray(row_offsets, dtype=np.uint32)
    si = np.ascontiguousarray(source_ids, dtype=np.uint32)
    va = np.ascontiguousarray(values, dtype=np.float32)
    handle = C.c_void_p()
    err = C.create_string_buffer(512)
    kind = lib.ref_make_canonical_csr(rows, cols, int(ro[-1]) if ro.size else 0, _p(ro, C.c_uint32),
                                      _p(si, C.c_uint32), _p(va, C.c_float), C.byref(handle), err, 512)
    if kind:
        raise RefError(kind, err.value.decode())
    return _ref_csr(handle)


def ref_load_matrix_market(path: str) -> tuple:
    """The reference's loadMatrixMarket (src/format/matrix_market.cpp:30-103)."""
    lib = _ref_host()
    handle = C.c_void_p()
    err = C.create_string_buffer(512)
    kind = lib.ref_load_matrix_market(str(path).encode(), C.byref(handle), err, 512)
    if kind:
        raise RefError(kind, err.value.decode())
    return _ref_csr(handle)


class RefCuda:
    """The reference's CUDA entry points (compute_80 PTX or sm_100a build)."""

    def __init__(self, tag: str = "sm100a"):
        path = HERE / "_ref" / f"libtcc_ref_cuda_{tag}.so"
        if not path.exists():
            raise ImportError(f"{path} missing")
        lib = C.CDLL(str(path), mode=os.RTLD_LOCAL)
        lib.ref_launch_spmm_int8.restype = C.c_int
        lib.ref_launch_spmm_int8.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                             C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_int]
        lib.ref_quantize_features_int8.restype = C.c_int
        lib.ref_quantize_features_int8.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                                   C.c_void_p, C.c_char_p, C.c_int]
        lib.ref_pack_features_int8x16.restype = C.c_int
        lib.ref_pack_features_int8x16.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p,
                                                  C.c_char_p, C.c_int]
        lib.ref_view_size.restype = C.c_int
        self.lib = lib
        self.tag = tag

    def _ok(self, kind, err):
        if kind:
            raise RefError(kind, err.value.decode())

    def launch_spmm_int8(self, view_addr: int, packed_x: int, scales: int, output: int, rows: int, cols: int,
                         features: int, partials: int, counters: int, stream: int) -> None:
        err = C.create_string_buffer(512)
        self._ok(self.lib.ref_launch_spmm_int8(view_addr, packed_x, scales, output, rows, cols, features, partials,
                                               counters, stream, err, 512), err)

    def quantize(self, x: int, q: int, scale: int, sources: int, features: int, stream: int) -> None:
        err = C.create_string_buffer(512)
        self._ok(self.lib.ref_quantize_features_int8(x, q, scale, sources, features, stream, err, 512), err)

    def pack(self, q: int, packed: int, sources: int, features: int, stream: int) -> None:
        err = C.create_string_buffer(512)
        self._ok(self.lib.ref_pack_features_int8x16(q, packed, sources, features, stream, err, 512), err)


def ref_cuda(tag: str = "sm100a") -> RefCuda:
    if tag not in _rc:
        _rc[tag] = RefCuda(tag)
    return _rc[tag]
