"""The oracle itself: its TF32 rounding, quantize, pack and SpMM restatements agree with
independent numpy formulations, so that a kernel checked against it is checked against the
reference's arithmetic."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tcc_spmm_b200 as T
from tests.cases import EDGE_CASES, random_csr


def test_tf32_rna_definition_vs_bit_form():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, size=2_000_000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    # values exactly on rounding ties and near binade edges
    ties = (np.arange(1, 20000, dtype=np.uint32) << 13 | 0x1000).view(np.float32)
    edges = np.array([0.0, -0.0, 1.0, 1.0009765625, 1.00048828125, -1.00048828125, 3.4e38, -3.4e38, 1e-40, -1e-40,
                      1.17549435e-38], dtype=np.float32)
    for v in (x, ties, -ties, edges):
        assert np.array_equal(O.tf32_rna(v).view(np.uint32), O.tf32_bits(v).view(np.uint32))


def test_tf32_rna_ties_go_away_from_zero():
    # 1 + 2^-11 is halfway between 1 and 1 + 2^-10
    assert O.tf32_rna(np.array([1 + 2**-11], np.float32))[0] == np.float32(1 + 2**-10)
    assert O.tf32_rna(np.array([-(1 + 2**-11)], np.float32))[0] == np.float32(-(1 + 2**-10))
    assert O.tf32_rna(np.array([1 + 2**-12], np.float32))[0] == np.float32(1.0)


def _numpy_quantize(x):
    m = np.max(np.abs(x), axis=1)
    s = np.where(m == 0, np.float32(1), (m / np.float32(127)).astype(np.float32)).astype(np.float32)
    v = np.rint(x / s[:, None])  # round half to even, as lrintf in the default mode
    return np.clip(v, -127, 127).astype(np.int8), s


@pytest.mark.parametrize("features", [16, 128, 256])
def test_quantize_restatement(features):
    rng = np.random.default_rng(features)
    x = rng.standard_normal((300, features)).astype(np.float32)
    x[0] = 0
    x[1] = np.float32(0.5)
    q, s = O.quantize(x)
    q2, s2 = _numpy_quantize(x)
    assert np.array_equal(s.view(np.uint32), s2.view(np.uint32))
    assert np.array_equal(q, q2)


def test_pack16_layout():
    q = np.arange(64, dtype=np.int8).reshape(2, 32)
    p = O.pack16(q)
    tile = [0, 8, 1, 9, 2, 10, 3, 11, 4, 12, 5, 13, 6, 14, 7, 15]
    assert list(p[0, :16]) == tile
    assert list(p[1, 16:]) == [48 + t for t in tile]


@pytest.mark.parametrize("name", ["every_mask", "random_small", "split_385", "empty"])
def test_spmm_restatement_vs_numpy(name):
    csr = EDGE_CASES[name]()
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((csr.cols, 32)).astype(np.float32)
    q, s = O.quantize(x)
    y, bound, rows = O.spmm(fmt, q, s)
    y, bound = y[rows >= 0], bound[rows >= 0]
    # numpy from the CSR: per row, terms tf32(a)*tf32(q*s) (exact in float64), summed in float64
    xh = O.tf32_rna((q.astype(np.float32) * s[:, None]).astype(np.float32)).astype(np.float64)
    ref = np.zeros((csr.rows, 32))
    bnd = np.zeros((csr.rows, 32))
    for r in range(csr.rows):
        lo, hi = csr.row_offsets[r], csr.row_offsets[r + 1]
        a = csr.values[lo:hi]
        cols = csr.source_ids[lo:hi]
        ref[r] = (O.tf32_rna(a).astype(np.float64)[:, None] * xh[cols]).sum(axis=0)
        bnd[r] = np.abs(a.astype(np.float64)[:, None] * (q[cols].astype(np.float64) * s[cols, None])).sum(axis=0)
    assert np.allclose(bound, bnd, rtol=1e-12, atol=0)
    assert np.all(np.abs(y - ref) <= 2.0**-20 * bnd + 1e-30)  # FP32 accumulation only


def test_spmm_restatement_window_subset():
    csr = random_csr(300, 300, 7.0, 2)
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    q, s = O.quantize(np.random.default_rng(2).standard_normal((300, 16)).astype(np.float32))
    full, _, rows_full = O.spmm(fmt, q, s)
    part, _, rows_part = O.spmm(fmt, q, s, sw_list=np.array([3, 1, 9], np.uint32))
    for i, r in enumerate(rows_part):
        if r >= 0:
            assert np.array_equal(part[i], full[r])
