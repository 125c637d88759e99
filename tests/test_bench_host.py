"""Host-side logic of bench.py (no GPU): the algorithmic bytes of a task range (the roofline's
numerator), the window-aligned slices of the end-to-end leg, and the choice of the ncu traffic
entry that matches the running kernel."""
from __future__ import annotations

import numpy as np
import pytest

import bench
import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W


@pytest.fixture(scope="module")
def case():
    csr = W.generate("stress_small")
    return csr, T.convert_csr_to_sw32(csr.rows, csr.cols, csr)


@pytest.fixture(scope="module")
def fmt(case):
    return case[1]


def _bytes(case, lo, hi, features):
    """bench.range_bytes with host counters (the bench counts on the device arrays)."""
    csr, fmt = case
    ro = csr.row_offsets.astype(np.int64)
    return bench.range_bytes(fmt.tasks, lo, hi, fmt.rows, fmt.cols, features, fmt.partial_count,
                             lambda p0, p1: int(np.count_nonzero(fmt.source_ids[8 * p0:8 * p1] != T.PADDING_SOURCE)),
                             lambda r0, r1: int(ro[r1] - ro[r0]))


@pytest.mark.parametrize("features", [128, 256])
def test_whole_range_bytes_equal_format_bytes(case, features):
    fmt = case[1]
    got = _bytes(case, 0, fmt.tasks.size, features)
    want = fmt.algorithmic_bytes(features)
    for key in ("total", "compulsory", "merge_bytes"):
        assert got[key] == want[key], key


@pytest.mark.parametrize("parts", [2, 3, 8])
def test_shard_bytes_add_up(case, parts):
    fmt = case[1]
    bounds = T.partition_tasks(fmt, 128, parts)
    shards = [_bytes(case, int(bounds[r]), int(bounds[r + 1]), 128) for r in range(parts)]
    full = _bytes(case, 0, fmt.tasks.size, 128)
    for key in ("total", "a_bytes", "x_bytes", "y_bytes", "nnz", "rows", "valid_slots", "panels"):
        assert sum(s.get(key, 0) for s in shards) == full[key], key


def test_both_arms_print_the_same_config():
    """The reference arm and this arm describe the workload with the same dict (the driver
    compares them); neither carries arm-specific keys."""
    a = bench.workload_config("powerlaw128", 10, 20, 128, 3, 4, 5, 6)
    b = bench.workload_config("powerlaw128", 10, 20, 128, 3, 4, 5, 6)
    assert a == b and {"workload", "rows", "nnz", "features"} <= set(a)
    assert not {"kernel", "task_order", "prep", "format_from", "launch"} & set(a)


def test_timed_batches_split_steps():
    sizes = []
    for steps in (1, 4, 5, 7, 20, 100):
        parts = [steps // 5 + (1 if i < steps % 5 else 0) for i in range(5)]
        sizes.append(sum(p for p in parts if p > 0))
    assert sizes == [1, 4, 5, 7, 20, 100]


@pytest.mark.parametrize("parts", [1, 4, 8, 64])
def test_window_cuts_start_at_window_boundaries(fmt, parts):
    n = fmt.tasks.size
    cuts = bench.window_cuts(fmt.tasks, 0, n, parts)
    assert cuts[0] == 0 and cuts[-1] == n and cuts == sorted(set(cuts))
    sw = fmt.tasks["sw"]
    assert all(sw[c] != sw[c - 1] for c in cuts[1:-1])


def test_traffic_entry_matches_launch_shape():
    entry = bench.profile_traffic("powerlaw128", "default", "balanced")
    assert entry is not None and entry["dram_bytes_per_launch"] > 0
    same = dict(entry["launch"])
    assert bench.profile_traffic("powerlaw128", "default", "balanced", same) is not None
    other = dict(same, smem=same["smem"] + 128)
    assert bench.profile_traffic("powerlaw128", "default", "balanced", other) is None
    assert bench.profile_traffic("powerlaw128", "default", "format") is None
    assert bench.profile_traffic("powerlaw128", "default", "balanced-equal") is None  # another task order
    assert bench.profile_traffic("powerlaw128", "generic", "balanced") is None


def test_task_order_flags(monkeypatch):
    """The weighted task order is the default; --equal-count-order and --natural-order select
    the others."""
    monkeypatch.setattr("sys.argv", ["bench.py"])
    args = bench.parse_args()
    assert not args.equal_count_order and not args.natural_order
    monkeypatch.setattr("sys.argv", ["bench.py", "--equal-count-order"])
    assert bench.parse_args().equal_count_order


@pytest.mark.parametrize("cols,world", [(1, 2), (7, 2), (8, 4), (2_449_029, 4), (5, 8), (100, 3)])
def test_x_shards_tile_the_rows(cols, world):
    from tcc_spmm_b200 import shards

    padded, _, _ = shards.input_shard(cols, world, 0)
    assert padded % world == 0 and padded >= cols and padded - cols < world
    covered = []
    for r in range(world):
        p, a, b = shards.input_shard(cols, world, r)
        assert p == padded and 0 <= a <= b <= cols
        covered.extend(range(a, b))
    assert covered == list(range(cols))
