"""Small seeded CSR cases that exercise the format's edge cases (the case list the reference
README describes: empty matrix, every row-group mask, tail rows and tail panels, long exclusive
and shared buckets, skewed load, split windows with 2 and 3 chunks, sources at cols-1)."""
from __future__ import annotations

import numpy as np

from tcc_spmm_b200.api import CsrMatrix


def from_rows(rows: int, cols: int, row_lists, rng: np.random.Generator, values="uniform") -> CsrMatrix:
    """Canonical CSR from per-row column lists (sorted, de-duplicated here)."""
    offsets = [0]
    cols_out, vals = [], []
    for r in range(rows):
        c = np.unique(np.asarray(row_lists[r] if r < len(row_lists) else [], dtype=np.int64))
        c = c[(c >= 0) & (c < cols)]
        cols_out.append(c.astype(np.uint32))
        if values == "uniform":
            v = rng.uniform(-1.0, 1.0, size=c.size).astype(np.float32)
            v[v == 0] = 0.5
        elif values == "ones":
            v = np.ones(c.size, dtype=np.float32)
        else:
            v = rng.uniform(0.25, 4.0, size=c.size).astype(np.float32) * np.where(rng.random(c.size) < 0.5, -1, 1)
            v = v.astype(np.float32)
        vals.append(v)
        offsets.append(offsets[-1] + c.size)
    return CsrMatrix(rows, cols, np.asarray(offsets, dtype=np.uint32),
                     np.concatenate(cols_out) if cols_out else np.zeros(0, np.uint32),
                     np.concatenate(vals) if vals else np.zeros(0, np.float32))


def random_csr(rows: int, cols: int, mean_degree: float, seed: int, local: float = 0.0, radius: int = 64) -> CsrMatrix:
    rng = np.random.default_rng(seed)
    lists = []
    for r in range(rows):
        d = rng.poisson(mean_degree)
        nl = int(round(local * d))
        loc = rng.integers(max(0, r - radius), min(cols, r + radius + 1), size=nl)
        glo = rng.integers(0, cols, size=d - nl)
        lists.append(np.concatenate([loc, glo]))
    return from_rows(rows, cols, lists, rng)


def every_mask_csr(seed: int = 1) -> CsrMatrix:
    """One 32-row window whose sources cover all 15 non-empty row-group masks, several
    sources per mask (long and short buckets, tail panels), plus a second partial window."""
    rng = np.random.default_rng(seed)
    rows, cols = 45, 512
    lists = [[] for _ in range(rows)]
    src = 0
    for mask in range(1, 16):
        for _ in range(int(rng.integers(1, 20))):
            for g in range(4):
                if mask & (1 << g):
                    for r in rng.choice(8, size=int(rng.integers(1, 4)), replace=False):
                        lists[8 * g + int(r)].append(src)
            src += 1
    for r in range(32, rows):  # tail window (rows % 32 != 0)
        lists[r] = list(rng.integers(0, cols, size=int(rng.integers(0, 30))))
    lists[3].append(cols - 1)  # source at the last column
    return from_rows(rows, cols, lists, rng)


def heavy_window_csr(panels_target: int, seed: int = 2, rows: int = 96, cols: int = 1 << 15) -> CsrMatrix:
    """Window 1 holds about `panels_target` panels of single-row sources (exclusive buckets of
    all four row groups plus some shared sources), windows 0 and 2 are light."""
    rng = np.random.default_rng(seed)
    lists = [list(rng.integers(0, cols, size=int(rng.integers(0, 6)))) for _ in range(rows)]
    slots = panels_target * 8
    srcs = rng.choice(cols, size=slots, replace=False)
    for i, s in enumerate(srcs):
        if i % 11 == 0:  # shared by two row groups
            lists[32 + int(rng.integers(0, 8))].append(int(s))
            lists[48 + int(rng.integers(0, 8))].append(int(s))
        else:
            lists[32 + int(rng.integers(0, 32))].append(int(s))
    return from_rows(rows, cols, lists, rng)


def empty_csr(rows: int = 70, cols: int = 33) -> CsrMatrix:
    return CsrMatrix(rows, cols, np.zeros(rows + 1, np.uint32), np.zeros(0, np.uint32), np.zeros(0, np.float32))


def single_term_csr(rows: int, cols: int, seed: int = 3) -> CsrMatrix:
    """Every row has exactly one nonzero: Y is then a single TF32 product per element, so the
    GPU result must equal the oracle bit for bit."""
    rng = np.random.default_rng(seed)
    lists = [[int(rng.integers(0, cols))] for _ in range(rows)]
    return from_rows(rows, cols, lists, rng, values="wide")


EDGE_CASES = {
    "every_mask": every_mask_csr,
    "empty": empty_csr,
    "random_small": lambda: random_csr(200, 300, 6.0, 5),
    "random_local": lambda: random_csr(1000, 1000, 20.0, 6, local=0.7, radius=40),
    "split_385": lambda: heavy_window_csr(385),
    "split_768": lambda: heavy_window_csr(768, seed=4),
    "split_769": lambda: heavy_window_csr(769, seed=5),
    "single_term": lambda: single_term_csr(300, 500),
    "one_row": lambda: random_csr(1, 40, 10.0, 9),
}


def bad_sw32_inputs():
    """Invalid inputs of convertCsrToSw32, one per check of the reference's merge and offsets."""
    good = random_csr(40, 50, 4.0, 3)
    ro, si, va = good.row_offsets.copy(), good.source_ids.copy(), good.values.copy()
    cases = {}
    bad = va.copy()
    bad[3] = 0.0
    cases["zero value"] = (40, 50, ro, si, bad)
    bad = va.copy()
    bad[5] = np.nan
    cases["nan value"] = (40, 50, ro, si, bad)
    bad = si.copy()
    bad[2] = 50
    cases["source out of range"] = (40, 50, ro, bad, va)
    bad = si.copy()
    r = int(np.argmax(np.diff(ro) >= 2))
    bad[ro[r]], bad[ro[r] + 1] = bad[ro[r] + 1], bad[ro[r]]
    cases["decreasing row sources"] = (40, 50, ro, bad, va)
    bad = ro.copy()
    bad[10], bad[11] = bad[11], bad[10]
    if bad[10] > bad[11]:
        cases["decreasing offsets"] = (40, 50, bad, si, va)
    cases["zero rows"] = (0, 50, np.zeros(1, np.uint32), si[:0], va[:0])
    cases["zero cols"] = (40, 0, ro, si, va)
    bad = ro.copy()
    bad[-1] -= 1
    cases["offsets end mismatch"] = (40, 50, bad, si, va)
    # Two failing windows: the error is the one of the first window in window order.
    big = random_csr(200, 60, 5.0, 8)
    bro, bsi, bva = big.row_offsets, big.source_ids.copy(), big.values.copy()
    bva[bro[110]] = 0.0                   # window 3
    bsi[bro[41] + 1] = 60                 # window 1: source out of range
    cases["two bad windows"] = (200, 60, bro, bsi, bva)
    return cases
