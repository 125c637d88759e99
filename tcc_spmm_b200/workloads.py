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


def normal_features(rows: int, features: int, seed: int = FEATURE_SEED, threads: int = 0) -> np.ndarray:
    """rows x features float32 N(0,1), row-major."""
    out = np.empty((rows, features), dtype=np.float32)
    if N.workloads().tcc_wl_normal(out.ctypes.data_as(N.f32p), out.size, seed, threads) != 0:
        raise RuntimeError(N.workloads().tcc_wl_last_error().decode())
    return out
