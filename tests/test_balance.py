"""Task order for the persistent launch (tcc_balance_tasks): a permutation of the tasks, equal
task counts per CTA (within one), and a more even estimated load per CTA than the natural
order. The speed-weighted order (tcc_balance_tasks_padded): the same tasks plus skip entries,
each CTA's list at b, b + G, ... with its skips last, and even estimated finish times when
each resident CTA of an SM counts at its speed. Y does not depend on the order (checked on the
GPU in tests/test_gpu_spmm.py)."""
from __future__ import annotations

import numpy as np
import pytest

import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W


SKIP = 0xFFFFFFFF
SPEED4 = [1.0, 0.94, 0.90, 0.82]  # the resident-CTA speeds of the C++ deal (4 CTAs per SM)


def _cost(tasks, masks, features):
    """The C++ cost estimate restated: the window epilogue, 80 per 8-panel chunk, 2 per extra
    row group a panel touches."""
    pc = np.array([bin(int(m) & 15).count("1") for m in masks], dtype=np.float64)
    prefix = np.concatenate([[0.0], np.cumsum(2.0 * np.maximum(pc - 1, 0))])
    panels = tasks["end"].astype(np.int64) - tasks["begin"]
    return 220.0 * 128 / max(128, features) + 80.0 * ((panels + 7) // 8) + prefix[tasks["end"]] - prefix[tasks["begin"]]


def _key(t):
    return np.sort(np.ascontiguousarray(t).view(np.uint32).reshape(-1, 7).view(np.dtype((np.void, 28))).ravel())


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
    assert np.array_equal(_key(out), _key(fmt.tasks)), "not a permutation"


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


@pytest.fixture(scope="module")
def big():
    csr = W.generate("powerlaw_small")
    return T.convert_csr_to_sw32(csr.rows, csr.cols, csr)


@pytest.mark.parametrize("ctas,per_sm", [(1, 1), (7, 1), (64, 4), (592, 4), (296, 2)])
def test_padded_order_layout(big, ctas, per_sm):
    out = T.balance_tasks_padded(big.tasks, big.row_group_masks, 128, ctas, per_sm)
    g = min(ctas, big.tasks.size)
    assert out.size % g == 0
    skip = out["sw"] == SKIP
    assert np.array_equal(_key(out[~skip]), _key(big.tasks)), "real entries are not a permutation"
    assert (out["begin"][skip] == 0).all() and (out["end"][skip] == 0).all()
    assert (out["partial"][skip] == SKIP).all()
    cols = skip.reshape(-1, g)  # row k = the k-th entry of every CTA
    assert (cols[1:] >= cols[:-1]).all(), "a CTA's skip entries must come after its tasks"
    assert not cols[-1].all(), "no row of skips only"


def test_padded_order_balances_weighted_finish_times(big):
    ctas, per_sm = 64, 4
    out = T.balance_tasks_padded(big.tasks, big.row_group_masks, 128, ctas, per_sm)
    real = out["sw"] != SKIP
    cost = np.where(real, _cost(np.where(real, out, big.tasks[:1].repeat(out.size)), big.row_group_masks, 128), 0.0)
    load = cost.reshape(-1, ctas).sum(axis=0)
    per_rank = ctas // per_sm
    cls = np.arange(ctas) // per_rank
    cls = np.minimum(cls + (np.arange(ctas) % per_rank >= per_rank - min(12, per_rank // 4)), per_sm - 1)
    finish = load / np.array(SPEED4)[cls]
    assert finish.max() / finish.mean() < 1.03
    rank = np.arange(ctas) // (ctas // per_sm)
    assert load[rank == 3].mean() < load[rank == 0].mean(), "the slowest resident CTAs get less work"
    even = T.balance_tasks_padded(big.tasks, big.row_group_masks, 128, ctas, 1)  # equal speeds
    real = even["sw"] != SKIP
    c = np.where(real, _cost(np.where(real, even, big.tasks[:1].repeat(even.size)), big.row_group_masks, 128), 0.0)
    l = c.reshape(-1, ctas).sum(axis=0)
    assert l.max() / l.mean() < 1.03


def test_padded_order_edge_cases(big):
    assert T.balance_tasks_padded(big.tasks[:0], big.row_group_masks, 128, 8, 4).size == 0
    out = T.balance_tasks_padded(big.tasks, big.row_group_masks, 128, 10 ** 6, 4)  # more CTAs than tasks
    assert out.size == big.tasks.size and not (out["sw"] == SKIP).any()
    with pytest.raises(T.InvalidArgument):
        T.balance_tasks_padded(big.tasks, big.row_group_masks, 128, 0, 4)
    with pytest.raises(T.InvalidArgument):
        T.balance_tasks_padded(big.tasks, big.row_group_masks, 128, 8, 0)
