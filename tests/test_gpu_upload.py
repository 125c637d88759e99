"""The library's upload helper (tcc_device_matrix_upload, the C counterpart of the reference's
DeviceMatrix constructor, src/device_matrix.cuh:18-28) through the C ABI: every device array
equals the Python DeviceMatrix upload bit for bit, the workspace has the reference's sizes with
zeroed counters, and an SpMM over its view and workspace gives the same bits."""
from __future__ import annotations

import numpy as np
import pytest

import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W
from tests.cases import EDGE_CASES
from tests.gpu_util import build_case, run_spmm

pytestmark = pytest.mark.gpu


class _Raw:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


def _bytes(ptr: int, nbytes: int):
    import torch

    if nbytes == 0:
        return torch.zeros(0, dtype=torch.uint8)
    return torch.as_tensor(_Raw(ptr, nbytes), device="cuda").cpu()


@pytest.mark.parametrize("features", [128, 256])
@pytest.mark.parametrize("name", ["every_mask", "split_769", "empty", "one_row", "stress_small"])
def test_upload_matches_device_matrix(name, features):
    import torch

    csr = W.generate(name) if name in W.CONFIGS else EDGE_CASES[name]()
    case = build_case(csr, features, seed=31)
    fmt, dm = case.fmt, case.dm
    up = T.UploadedMatrix(fmt, features)
    v, ref = up.view(), dm.view()
    assert v.taskCount == ref.taskCount == fmt.tasks.size
    for field, array in (("windowOffsets", fmt.window_offsets), ("sourceIds", fmt.source_ids),
                         ("rowGroupMasks", fmt.row_group_masks), ("sourceMetadata", fmt.source_metadata),
                         ("values", fmt.values), ("bucketOffsets", fmt.bucket_offsets), ("tasks", fmt.tasks),
                         ("reductions", fmt.reductions), ("partialIds", fmt.partial_ids)):
        ptr = getattr(v, field)
        assert ptr % 256 == 0, field
        got = _bytes(ptr, array.nbytes).numpy()
        want = _bytes(getattr(ref, field), array.nbytes).numpy()
        assert np.array_equal(got, want), field
        assert np.array_equal(got, np.ascontiguousarray(array).view(np.uint8).reshape(-1)), field
    partials, counters = up.workspace_pointers()
    pf, cw = T.workspace_size(fmt.rows, fmt.partial_count, features)
    assert bool(partials) == (pf > 0) and bool(counters) == (cw > 0)
    if cw:
        assert not _bytes(counters, 4 * cw).numpy().any(), "counters must start at zero"
    if fmt.tasks.size == 0:
        return
    y_ref = run_spmm(case)
    y = torch.full_like(y_ref, float("nan"))
    T.launch_spmm_int8(v, case.packed_dev, case.scales_dev, y, fmt.rows, fmt.cols, features,
                       T.SpmmWorkspace(partials or None, counters or None))
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32))
    if cw:
        assert not _bytes(counters, 4 * cw).numpy().any(), "counters must return to zero"
