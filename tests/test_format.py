"""Host format parity: convertCsrToSw32 + buildPanelTasks and makeCanonicalCsr must be
byte-identical to the reference's own code (compiled from its sources into oracle/_ref), and
fail with the same exception type and message."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W
from tests.cases import EDGE_CASES, bad_sw32_inputs, random_csr

pytestmark = pytest.mark.skipif(not O.have_ref_host(), reason="oracle/_ref not built")


def assert_same_format(mine: T.Sw32HostFormat, ref: dict) -> None:
    for name in O.oracle.REF_SW32_FIELDS:
        a = getattr(mine, name)
        if name == "tasks":
            a = a.view(np.uint32).reshape(-1, 7)
        elif name == "reductions":
            a = a.view(np.uint32).reshape(-1, 2)
        b = ref[name]
        assert a.dtype.itemsize == b.dtype.itemsize, name
        assert a.shape == b.shape, (name, a.shape, b.shape)
        assert a.tobytes() == b.tobytes(), f"{name} differs from the reference"
    assert mine.partial_count == ref["partial_count"]


def convert_both(csr, bucketed=True, threads=0):
    mine = T.convert_csr_to_sw32(csr.rows, csr.cols, csr, bucketed, threads)
    ref = O.ref_convert_csr_to_sw32(csr.rows, csr.cols, csr.row_offsets, csr.source_ids, csr.values, bucketed)
    return mine, ref


@pytest.mark.parametrize("name", sorted(EDGE_CASES))
def test_edge_cases_byte_identical(name):
    csr = EDGE_CASES[name]()
    mine, ref = convert_both(csr)
    assert_same_format(mine, ref)


@pytest.mark.parametrize("name", ["cpu4096", "powerlaw_small", "stress_small", "rmat_small"])
def test_seeded_configs_byte_identical(name):
    csr = W.generate(name)
    mine, ref = convert_both(csr)
    assert_same_format(mine, ref)
    if name == "stress_small":
        assert mine.partial_count > 0 and int(mine.tasks["chunks"].max()) >= 3


@pytest.mark.parametrize("threads", [1, 3, 8])
def test_thread_count_does_not_change_bytes(threads):
    csr = W.generate("stress_small")
    mine = T.convert_csr_to_sw32(csr.rows, csr.cols, csr, True, threads)
    ref = O.ref_convert_csr_to_sw32(csr.rows, csr.cols, csr.row_offsets, csr.source_ids, csr.values)
    assert_same_format(mine, ref)


def test_unbucketed_mode_byte_identical():
    csr = random_csr(300, 700, 9.0, 21, local=0.5)
    mine, ref = convert_both(csr, bucketed=False)
    assert_same_format(mine, ref)
    assert mine.tasks.size == 0 and mine.bucket_offsets.size == 0


def test_split_tasks_cover_every_panel_once():
    csr = EDGE_CASES["split_769"]()
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    t = fmt.tasks
    assert (t["end"] - t["begin"]).max() <= T.TASK_PANEL_LIMIT
    # tasks tile [0, panels) in order, one or more per window
    assert t["begin"][0] == 0 and t["end"][-1] == fmt.panels
    assert np.all(t["begin"][1:] == t["end"][:-1])
    assert int(t["chunks"].max()) >= 3
    split = t[t["partial"] != T.NO_PARTIAL]
    assert fmt.partial_count == int(sum(bin(int(m)).count("1") for m in split["mask"]))


# --------------------------------------------------------------------------------------
# Error behaviour: same exception type and message as the reference.
# --------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", sorted(bad_sw32_inputs()))
def test_invalid_input_same_error_as_reference(case):
    rows, cols, ro, si, va = bad_sw32_inputs()[case]
    with pytest.raises(O.oracle.RefError) as ref_err:
        O.ref_convert_csr_to_sw32(rows, cols, ro, si, va)
    csr = T.CsrMatrix(rows, cols, ro, si, va)
    with pytest.raises((T.InvalidArgument, OverflowError)) as my_err:
        T.convert_csr_to_sw32(rows, cols, csr)
    assert ref_err.value.kind == "invalid_argument"
    assert isinstance(my_err.value, T.InvalidArgument)
    assert str(my_err.value) == str(ref_err.value)


# --------------------------------------------------------------------------------------
# makeCanonicalCsr
# --------------------------------------------------------------------------------------
def _raw_csr(seed, rows=60, cols=40, dup=True):
    rng = np.random.default_rng(seed)
    offsets, c, v = [0], [], []
    for _ in range(rows):
        n = int(rng.integers(0, 12))
        cc = rng.integers(0, cols, size=n)  # unsorted, with duplicates
        vv = rng.choice(np.array([-1.5, -0.5, 0.0, 0.25, 0.5, 1.0, 3.0], np.float32), size=n)
        c.append(cc)
        v.append(vv)
        offsets.append(offsets[-1] + n)
    return (rows, cols, np.asarray(offsets, np.uint32), np.concatenate(c).astype(np.uint32),
            np.concatenate(v).astype(np.float32))


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_canonical_csr_byte_identical(seed):
    rows, cols, ro, si, va = _raw_csr(seed)
    mine = T.make_canonical_csr(rows, cols, ro, si, va)
    r_rows, r_cols, r_ro, r_si, r_va = O.ref_make_canonical_csr(rows, cols, ro, si, va)
    assert mine.row_offsets.tobytes() == r_ro.tobytes()
    assert mine.source_ids.tobytes() == r_si.tobytes()
    assert mine.values.tobytes() == r_va.tobytes()


def test_canonical_csr_sums_in_stable_order_and_drops_zero():
    # 0.1 + 0.2 + -0.3 in float, in this order, is not exactly zero; the order must match.
    ro = np.array([0, 4, 6], np.uint32)
    si = np.array([7, 3, 7, 7, 1, 1], np.uint32)
    va = np.array([0.1, 2.0, 0.2, -0.3, 1.0, -1.0], np.float32)
    mine = T.make_canonical_csr(2, 10, ro, si, va)
    ref = O.ref_make_canonical_csr(2, 10, ro, si, va)
    assert mine.values.tobytes() == ref[4].tobytes() and mine.row_offsets.tobytes() == ref[2].tobytes()
    s = np.float32(0.1) + np.float32(0.2) + np.float32(-0.3)  # the same float sequence
    assert int(mine.row_offsets[1]) == (2 if s != 0 else 1)
    assert int(mine.row_offsets[2]) == int(mine.row_offsets[1])  # row 1 sums to zero and is dropped


@pytest.mark.parametrize("what", ["column", "nan", "offsets"])
def test_canonical_csr_errors_match(what):
    rows, cols, ro, si, va = _raw_csr(9)
    if what == "column":
        si = si.copy()
        si[4] = cols
    elif what == "nan":
        va = va.copy()
        va[6] = np.inf
    else:
        ro = ro.copy()
        ro[5] = ro[-1] + 1
    with pytest.raises(O.oracle.RefError) as ref_err:
        O.ref_make_canonical_csr(rows, cols, ro, si, va)
    with pytest.raises(T.InvalidArgument) as my_err:
        T.make_canonical_csr(rows, cols, ro, si, va)
    assert str(my_err.value) == str(ref_err.value)


def test_random_shapes_byte_identical():
    """Randomised shapes, degrees, locality and both bucket modes against the reference builder:
    ragged last windows (rows not a multiple of 32), few or many columns, empty rows, and
    windows dense enough to split into several tasks."""
    rng = np.random.default_rng(2024)
    for trial in range(40):
        rows = int(rng.integers(1, 400))
        cols = int(rng.choice([1, 3, 31, 33, 257, 4096, 1 << 16]))
        degree = float(rng.choice([0.0, 0.5, 2.0, 9.0, 40.0, 200.0]))
        # neighbours near the row index only where the columns reach that far
        local = float(rng.choice([0.0, 0.5, 0.95])) if cols >= rows else 0.0
        csr = random_csr(rows, cols, degree, 100 + trial, local=local, radius=int(rng.choice([4, 64, 4096])))
        for bucketed in (True, False):
            mine, ref = convert_both(csr, bucketed=bucketed, threads=int(rng.choice([1, 4])))
            assert_same_format(mine, ref)
