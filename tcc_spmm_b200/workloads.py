"""Seeded synthetic workloads with the shapes of the benchmark configurations.

The reference measures on ogbn-products (2,449,029 rows, 126,167,053 nnz), which is not
available here; the power-law configuration stands in for it with the same row and nnz
counts. All matrices come from libtcc_workloads (C++, counter-based RNG: the output does not
depend on the thread count).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N
from .api import CsrMatrix

FEATURE_SEED = 20261025


@dataclass(frozen=True)
class Config:
    name: str
    kind: str
    features: int
    params: tuple
    seed: int
    description: str


CONFIGS = {
    "cpu4096": Config("cpu4096", "poisson", 128, (4096, 4096, 16.0), 4096,
                      "4096x4096, row nnz ~ Poisson(16) at uniform columns, values U(-1,1), X N(0,1), F128"),
    "powerlaw128": Config("powerlaw128", "powerlaw", 128, (2449029, 126167053, 2.1, 17000, 0.6, 4096), 2449029,
                          "2,449,029 rows, 126,167,053 nnz, power-law degrees (alpha 2.1, max 17k), 60% of "
                          "neighbours within +-4096, values 1/sqrt(deg_i deg_j), X N(0,1), F128"),
    "powerlaw256": Config("powerlaw256", "powerlaw", 256, (2449029, 126167053, 2.1, 17000, 0.6, 4096), 2449029,
                          "the power-law matrix at F256 (two 128-feature slices)"),
    "stress": Config("stress", "stress", 128, (1048576, 4, 32, 524, 300, 20000, 60000), 1048576,
                     "1,048,576 rows, 99% with U[4,32] nnz, 524 rows with U[20k,60k] nnz in 300 windows, "
                     "values U(0,1], F128"),
    "rmat": Config("rmat", "rmat", 128, (24, 1 << 29, 0.57, 0.19, 0.19), 24,
                   "R-MAT(0.57,0.19,0.19,0.05), 2^24 rows, 2^29 edge samples, duplicates merged, values 1/deg_i, F128"),
    # A reduced power-law matrix for profiler captures: X (134 MB at F128) still exceeds L2.
    "powerlaw_profile": Config("powerlaw_profile", "powerlaw", 128, (1048576, 1048576 * 51, 2.1, 17000, 0.6, 4096),
                               1048576, "1,048,576-row power-law matrix, mean degree 51 (profiler captures)"),
    # Scaled-down shapes of the same generators (tests).
    "powerlaw_small": Config("powerlaw_small", "powerlaw", 128, (65536, 65536 * 51, 2.1, 4000, 0.6, 4096), 7,
                             "65,536-row power-law matrix, mean degree 51"),
    "stress_small": Config("stress_small", "stress", 128, (32768, 4, 32, 12, 6, 6000, 12000), 11,
                           "32,768 rows with 12 heavy rows in 6 windows (splits of up to ~10 chunks)"),
    "rmat_small": Config("rmat_small", "rmat", 128, (16, 1 << 20, 0.57, 0.19, 0.19), 16,
                         "R-MAT scale 16, 2^20 edge samples"),
}


def _take(ptr: C.POINTER(N.WlCsr)) -> CsrMatrix:
    lib = N.workloads()
    try:
        c = ptr.contents
        rows, nnz = c.rows, c.nnz
        ro = np.ctypeslib.as_array(c.rowOffsets, shape=(rows + 1,)).copy()
        si = np.ctypeslib.as_array(c.sourceIds, shape=(max(nnz, 1),))[:nnz].copy()
        va = np.ctypeslib.as_array(c.values, shape=(max(nnz, 1),))[:nnz].copy()
        return CsrMatrix(rows, c.cols, ro, si, va)
    finally:
        lib.tcc_wl_free(ptr)


def _call(fn, *args) -> CsrMatrix:
    out = C.POINTER(N.WlCsr)()
    if fn(*args, C.byref(out)) != 0:
        raise RuntimeError(N.workloads().tcc_wl_last_error().decode())
    return _take(out)


def poisson(rows: int, cols: int, mean: float, seed: int, threads: int = 0) -> CsrMatrix:
    return _call(N.workloads().tcc_wl_poisson, rows, cols, mean, seed, threads)


def powerlaw(rows: int, nnz: int, alpha: float, max_degree: int, local_fraction: float, local_radius: int, seed: int,
             threads: int = 0) -> CsrMatrix:
    return _call(N.workloads().tcc_wl_powerlaw, rows, nnz, alpha, max_degree, local_fraction, local_radius, seed,
                 threads)


def stress(rows: int, light_lo: int, light_hi: int, heavy_rows: int, heavy_windows: int, heavy_lo: int, heavy_hi: int,
           seed: int, threads: int = 0) -> CsrMatrix:
    return _call(N.workloads().tcc_wl_stress, rows, light_lo, light_hi, heavy_rows, heavy_windows, heavy_lo, heavy_hi,
                 seed, threads)


def rmat(scale: int, edges: int, a: float, b: float, c: float, seed: int, threads: int = 0) -> CsrMatrix:
    return _call(N.workloads().tcc_wl_rmat, scale, edges, a, b, c, seed, threads)


def generate(name: str, threads: int = 0) -> CsrMatrix:
    cfg = CONFIGS[name]
    fn = {"poisson": poisson, "powerlaw": powerlaw, "stress": stress, "rmat": rmat}[cfg.kind]
    return fn(*cfg.params, seed=cfg.seed, threads=threads)


@dataclass
class DeviceCsr:
    """A canonical CSR in device memory (torch tensors: row_offsets int32 [rows + 1], source_ids
    int32 [nnz], values float32 [nnz]; the int32 tensors hold the u32 arrays)."""

    rows: int
    cols: int
    row_offsets: object
    source_ids: object
    values: object

    @property
    def nnz(self) -> int:
        return int(self.values.numel())

    def to_host(self) -> CsrMatrix:
        return CsrMatrix(self.rows, self.cols, self.row_offsets.cpu().numpy().view(np.uint32),
                         self.source_ids.cpu().numpy().view(np.uint32), self.values.cpu().numpy())


def rmat_device(scale: int, edges: int, a: float, b: float, c: float, seed: int, device="cuda") -> DeviceCsr:
    """tcc_wl_rmat's matrix, bit for bit, generated on `device` (tcc_wl_rmat_device). The arrays
    are copied into torch tensors and the library's buffers freed before returning."""
    import torch

    device = torch.device(device)
    lib = N.workloads()
    handle = C.c_void_p()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        if lib.tcc_wl_rmat_device(scale, edges, a, b, c, seed, stream.cuda_stream, C.byref(handle)) != 0:
            raise RuntimeError(lib.tcc_wl_last_error().decode())
        try:
            rows, cols, nnz = C.c_uint32(), C.c_uint32(), C.c_uint64()
            ro, si, va = C.c_void_p(), C.c_void_p(), C.c_void_p()
            if lib.tcc_wl_device_csr_arrays(handle, C.byref(rows), C.byref(cols), C.byref(nnz), C.byref(ro),
                                            C.byref(si), C.byref(va)) != 0:
                raise RuntimeError(lib.tcc_wl_last_error().decode())

            def copy(ptr, count, dtype, typestr):
                out = torch.empty(int(count), dtype=dtype, device=device)
                if count:
                    src = torch.as_tensor(_DeviceBuffer(ptr.value, count, typestr), device=device)
                    out.copy_(src)
                return out

            result = DeviceCsr(rows.value, cols.value, copy(ro, rows.value + 1, torch.int32, "<i4"),
                               copy(si, nnz.value, torch.int32, "<i4"), copy(va, nnz.value, torch.float32, "<f4"))
            torch.cuda.current_stream(device).synchronize()
            return result
        finally:
            lib.tcc_wl_device_csr_free(handle)


class _DeviceBuffer:
    def __init__(self, ptr: int, count: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (int(count),), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def generate_device(name: str, device="cuda", threads: int = 0) -> DeviceCsr:
    """The configuration's matrix in device memory: R-MAT generated on the device, the others
    generated on the host (`threads`) and copied up. Identical to generate(name)."""
    import torch

    cfg = CONFIGS[name]
    if cfg.kind == "rmat":
        scale, edges, a, b, c = cfg.params
        return rmat_device(scale, edges, a, b, c, cfg.seed, device)
    csr = generate(name, threads=threads)
    up = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a).view(dt)).to(device)
    return DeviceCsr(csr.rows, csr.cols, up(csr.row_offsets, np.int32), up(csr.source_ids, np.int32),
                     up(csr.values, np.float32))


def normal_features(rows: int, features: int, seed: int = FEATURE_SEED, threads: int = 0) -> np.ndarray:
    """rows x features float32 N(0,1), row-major."""
    out = np.empty((rows, features), dtype=np.float32)
    if N.workloads().tcc_wl_normal(out.ctypes.data_as(N.f32p), out.size, seed, threads) != 0:
        raise RuntimeError(N.workloads().tcc_wl_last_error().decode())
    return out
