"""Device-side failure paths of the SpMM kernel, made without faulting the GPU.

* A split matrix launched without a partial/counter workspace (the reference contract allows a
  null workspace only when partialCount is 0, include/spmm.cuh:8): the kernel records status
  bit 1, writes every unsplit window and leaves the split window alone.
* A bounded wait that runs out: a test hook stalls the MMA thread of every odd CTA on a barrier
  that nothing completes (about two seconds), so that CTA's waits run out one after another.
  The host sees status bit 0 (DeviceTimeout), the context stays usable, and once the caller has
  re-zeroed its counters the next launch is bit-identical to one that never failed.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import tcc_spmm_b200 as T
import tcc_spmm_b200._native as N
from tests.cases import EDGE_CASES
from tests.conftest import assert_within_tf32_bound
from tests.gpu_util import build_case, oracle_y, run_spmm

pytestmark = pytest.mark.gpu


def _stalled(case, y, workspace, static: bool) -> int:
    import torch

    view = case.dm.view()
    return N.lib().tcc_test_launch_spmm_int8_stalled(
        C.byref(view), case.packed_dev.data_ptr(), case.scales_dev.data_ptr(), y.data_ptr(), case.fmt.rows,
        case.fmt.cols, case.features, workspace.partials.data_ptr() if workspace.partials is not None else None,
        workspace.counters.data_ptr() if workspace.counters is not None else None, case.fmt.partial_count,
        int(static), torch.cuda.current_stream().cuda_stream)


def _window_rows(fmt, split: bool) -> np.ndarray:
    """Rows of the windows that are (split=True) or are not split into several tasks."""
    sw = fmt.tasks["sw"][fmt.tasks["partial"] != T.NO_PARTIAL]
    rows = np.arange(fmt.rows)
    return rows[np.isin(rows // 32, np.unique(sw)) == split]


@pytest.mark.parametrize("features", [128, 256])
def test_split_matrix_without_workspace_reports_status(features):
    import torch

    T.device_status(reset=True)
    case = build_case(EDGE_CASES["split_769"](), features, seed=21)
    assert case.fmt.partial_count > 0
    y = torch.full((case.fmt.rows, features), float("nan"), device="cuda")
    T.launch_spmm_int8(case.dm.view(), case.packed_dev, case.scales_dev, y, case.fmt.rows, case.fmt.cols, features,
                       T.SpmmWorkspace())
    with pytest.raises(T.InvalidArgument, match="workspace"):
        T.check_device()
    assert T.device_status() == 0  # check_device reset the word
    got = y.cpu().numpy()
    y_ref, bound = oracle_y(case)
    keep = _window_rows(case.fmt, split=False)
    assert keep.size > 0
    assert_within_tf32_bound(got[keep], y_ref[keep], bound[keep], "unsplit windows without workspace")
    assert np.isnan(got[_window_rows(case.fmt, split=True)]).all(), "split windows must be left alone"


@pytest.mark.parametrize("features", [128, 256])
def test_wait_that_runs_out_is_reported_and_recoverable(features):
    import torch

    T.device_status(reset=True)
    case = build_case(EDGE_CASES["split_769"](), features, seed=23)
    assert case.dm.task_count >= 4 and case.fmt.partial_count > 0
    good = run_spmm(case)
    torch.cuda.synchronize()
    ws = case.dm.workspace()
    y = torch.full_like(good, float("nan"))
    assert _stalled(case, y, ws, static=False) == 0
    with pytest.raises(T.DeviceTimeout):
        T.check_device()
    # The split window's tasks ran on even and odd CTAs: the even CTA's ticket was taken, the
    # odd ones' were not, so its counter is short of zero until the caller re-zeroes it.
    assert int(case.dm.counters.abs().sum()) > 0
    case.dm.counters.zero_()
    again = run_spmm(case)
    torch.cuda.synchronize()
    assert torch.equal(again.view(torch.int32), good.view(torch.int32))
    assert int(case.dm.counters.abs().sum()) == 0
    assert T.device_status() == 0
