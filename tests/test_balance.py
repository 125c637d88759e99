"""Task order for the persistent launch (tcc_balance_tasks): a permutation of the tasks, equal
task counts per CTA (within one), and a more even estimated load per CTA than the natural
order. Y does not depend on the order (checked on the GPU in tests/test_gpu_spmm.py)."""
from __future__ import annotations

import numpy as np
import pytest

import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W


def _cost(tasks, masks, features):
    """The C++ cost estimate restated: panels weighted by the row-group MMAs, plus a fixed term."""
    pc = np.array([bin(int(m) & 15).count("1") for m in masks], dtype=np.float64)
    prefix = np.concatenate([[0.0], np.cumsum(8.0 + 2.0 * pc)])
    return 16.0 * features / 128 + prefix[tasks["end"]] - prefix[tasks["begin"]]


def _per_cta(costs, g):
    return np.array([costs[b::g].sum() for b in range(g)])


@pytest.fixture(scope="module")
def fmt():
    csr = W.generate("stress_small")
    return T.convert_csr_to_sw32(csr.rows, csr.cols, csr)


@pytest.mark.parametrize("ctas", [1, 7, 64, 592])
def test_permutation_and_equal_counts(fmt, ctas):
    out = T.balance_tasks(fmt.tasks, fmt.row_group_masks, 128, ctas)
    assert out.size == fmt.tasks.size
    key = lambda t: np.sort(np.ascontiguousarray(t).view(np.uint32).reshape(-1, 7).view(np.dtype((np.void, 28))).ravel())
    assert np.array_equal(key(out), key(fmt.tasks)), "not a permutation"


@pytest.mark.parametrize("ctas", [64, 592])
def test_load_is_more_even_than_natural_order(fmt, ctas):
    natural = _per_cta(_cost(fmt.tasks, fmt.row_group_masks, 128), ctas)
    out = T.balance_tasks(fmt.tasks, fmt.row_group_masks, 128, ctas)
    balanced = _per_cta(_cost(out, fmt.row_group_masks, 128), ctas)
    assert np.isclose(balanced.sum(), natural.sum())
    assert balanced.max() <= natural.max()
    assert balanced.max() / balanced.mean() < 1.05 + 1e-9 or balanced.max() < natural.max() * 0.9


def test_more_ctas_than_tasks_and_edge_cases():
    csr = W.generate("cpu4096")
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    out = T.balance_tasks(fmt.tasks, fmt.row_group_masks, 128, 10 ** 6)
    assert out.size == fmt.tasks.size
    empty = T.balance_tasks(fmt.tasks[:0], fmt.row_group_masks, 128, 8)
    assert empty.size == 0
    with pytest.raises(T.InvalidArgument):
        T.balance_tasks(fmt.tasks, fmt.row_group_masks, 128, 0)
