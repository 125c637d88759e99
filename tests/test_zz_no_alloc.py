"""tcc_launch_spmm_int8_static_workspace: the SpMM with the split-window workspace in the
library's static device scratch (no allocation by caller or library), called through the C
ABI and compared with tcc_launch_spmm_int8 on two calls in a row. Collected last on purpose:
it must pass both alone and after every other test has used the device."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import tcc_spmm_b200 as T
import tcc_spmm_b200._native as N
from tests.cases import EDGE_CASES
from tests.conftest import assert_within_tf32_bound
from tests.gpu_util import build_case, oracle_y

pytestmark = pytest.mark.gpu


def _static_call(case, y) -> int:
    import torch

    view = case.dm.view()
    return N.lib().tcc_launch_spmm_int8_static_workspace(
        C.byref(view), case.packed_dev.data_ptr(), case.scales_dev.data_ptr(), y.data_ptr(), case.fmt.rows,
        case.fmt.cols, case.features, case.fmt.partial_count, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("features", [128, 256])
@pytest.mark.parametrize("name", ["split_769", "split_385", "random_local"])
def test_static_workspace_matches_caller_workspace(name, features):
    import torch

    case = build_case(EDGE_CASES[name](), features, seed=5)
    y_ref = torch.full((case.fmt.rows, features), float("nan"), device="cuda")
    T.launch_spmm_int8(case.dm.view(), case.packed_dev, case.scales_dev, y_ref, case.fmt.rows, case.fmt.cols,
                       features, case.dm.workspace())
    oracle, bound = oracle_y(case)
    for _ in range(2):  # the second call finds the counters back at zero
        y = torch.full_like(y_ref, float("nan"))
        assert _static_call(case, y) == 0, T.api.N.lib().tcc_last_error()
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert np.isfinite(got).all()
        # Same kernel, inputs and merge order as the caller-workspace call: the bits must match.
        assert np.array_equal(got.view(np.uint32), y_ref.cpu().numpy().view(np.uint32)), \
            f"{name}/F{features}: static workspace differs from caller workspace"
        assert_within_tf32_bound(got, oracle, bound, f"{name}/F{features} vs oracle")
    assert T.device_status() == 0


def test_static_workspace_rejects_oversized_partials():
    import torch

    case = build_case(EDGE_CASES["split_769"](), 128, seed=5)
    y = torch.empty((case.fmt.rows, 128), device="cuda")
    view = case.dm.view()
    status = N.lib().tcc_launch_spmm_int8_static_workspace(
        C.byref(view), case.packed_dev.data_ptr(), case.scales_dev.data_ptr(), y.data_ptr(), case.fmt.rows,
        case.fmt.cols, 128, 1 << 20, torch.cuda.current_stream().cuda_stream)
    assert status == 1  # TCC_INVALID_ARGUMENT
    assert b"static workspace" in N.lib().tcc_last_error()


def _static_nonzero_counters() -> int:
    n = C.c_uint64()
    assert N.lib().tcc_test_static_counters_nonzero(C.byref(n)) == 0, N.lib().tcc_last_error()
    return n.value


def test_static_workspace_recovers_after_a_wait_runs_out():
    """A launch whose bounded wait runs out leaves split-window counters short of zero. The
    static workspace belongs to the library, so the caller cannot re-zero it: the status reset
    (tcc_device_status with reset) does, and the next call is bit-identical to the caller-
    workspace call again."""
    import torch

    T.device_status(reset=True)
    case = build_case(EDGE_CASES["split_769"](), 128, seed=29)
    y_ref = torch.full((case.fmt.rows, 128), float("nan"), device="cuda")
    T.launch_spmm_int8(case.dm.view(), case.packed_dev, case.scales_dev, y_ref, case.fmt.rows, case.fmt.cols, 128,
                       case.dm.workspace())
    y = torch.full_like(y_ref, float("nan"))
    view = case.dm.view()
    status = N.lib().tcc_test_launch_spmm_int8_stalled(
        C.byref(view), case.packed_dev.data_ptr(), case.scales_dev.data_ptr(), y.data_ptr(), case.fmt.rows,
        case.fmt.cols, 128, None, None, case.fmt.partial_count, 1, torch.cuda.current_stream().cuda_stream)
    assert status == 0, N.lib().tcc_last_error()
    assert T.device_status() & T.api.STATUS_WAIT_TIMEOUT
    assert _static_nonzero_counters() > 0
    with pytest.raises(T.DeviceTimeout):
        T.check_device(reset=True)
    assert _static_nonzero_counters() == 0
    for _ in range(2):
        y = torch.full_like(y_ref, float("nan"))
        assert _static_call(case, y) == 0, N.lib().tcc_last_error()
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32))
    assert T.device_status() == 0
