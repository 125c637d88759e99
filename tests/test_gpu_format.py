"""SW32 construction on the GPU (tcc_convert_csr_to_sw32_device): every array byte-identical to
the host builder's (which tests/test_format.py pins to the reference's own code), the same
exception type and message on invalid input, and an SpMM over the GPU-built format
bit-identical to the one over the uploaded host format."""
from __future__ import annotations

import numpy as np
import pytest

import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W
from tests.cases import EDGE_CASES, bad_sw32_inputs, random_csr
from tests.gpu_util import build_case, run_spmm

pytestmark = pytest.mark.gpu

FIELDS = ("window_offsets", "source_ids", "row_group_masks", "source_metadata", "values", "bucket_offsets", "tasks",
          "reductions", "partial_ids")


def _device_csr(row_offsets, source_ids, values):
    import torch

    def up(a, dtype):
        a = np.ascontiguousarray(a, dtype=dtype)
        return torch.from_numpy(a.view(np.int32) if dtype == np.uint32 else a).cuda()

    return up(row_offsets, np.uint32), up(source_ids, np.uint32), up(values, np.float32)


def build_on_device(csr: T.CsrMatrix, bucketed: bool = True, stream=None) -> T.Sw32DeviceFormat:
    return T.convert_csr_to_sw32_device(csr.rows, csr.cols, *_device_csr(csr.row_offsets, csr.source_ids, csr.values),
                                        bucket_by_rw_mask=bucketed, stream=stream)


def assert_same_format(host: T.Sw32HostFormat, dev: T.Sw32DeviceFormat) -> None:
    got = dev.to_host()
    assert (got.rows, got.cols) == (host.rows, host.cols)
    for name in FIELDS:
        a, b = getattr(got, name), getattr(host, name)
        assert a.dtype.itemsize == b.dtype.itemsize and a.size == b.size, (name, a.size, b.size)
        assert a.tobytes() == b.tobytes(), f"{name} differs from the host builder"
    assert got.partial_count == host.partial_count
    assert dev.task_count == host.tasks.size


@pytest.mark.parametrize("bucketed", [True, False])
@pytest.mark.parametrize("name", sorted(EDGE_CASES))
def test_edge_cases_match_host_builder(name, bucketed):
    csr = EDGE_CASES[name]()
    assert_same_format(T.convert_csr_to_sw32(csr.rows, csr.cols, csr, bucketed), build_on_device(csr, bucketed))


@pytest.mark.parametrize("name", ["cpu4096", "powerlaw_small", "stress_small", "rmat_small"])
def test_seeded_configs_match_host_builder(name):
    csr = W.generate(name)
    host = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    dev = build_on_device(csr)
    assert_same_format(host, dev)
    if name == "stress_small":
        assert host.partial_count > 0 and int(host.tasks["chunks"].max()) >= 3


def test_unbucketed_random_local():
    csr = random_csr(300, 700, 9.0, 21, local=0.5)
    host = T.convert_csr_to_sw32(csr.rows, csr.cols, csr, False)
    assert host.tasks.size == 0 and host.bucket_offsets.size == 0
    assert_same_format(host, build_on_device(csr, False))


@pytest.mark.parametrize("cols", [1, 2, (1 << 27) + 3, 0xFFFFFFFF])
def test_source_id_widths(cols):
    """Source IDs of 0 to 32 bits (the device sort key packs window, source and row)."""
    rng = np.random.default_rng(cols % 1000)
    rows = 150
    lists = [np.unique(rng.integers(0, cols, size=int(rng.integers(0, 9)), dtype=np.uint64)).astype(np.uint32)
             for _ in range(rows)]
    ro = np.zeros(rows + 1, np.uint32)
    ro[1:] = np.cumsum([len(x) for x in lists])
    si = np.concatenate(lists).astype(np.uint32) if ro[-1] else np.zeros(0, np.uint32)
    va = (rng.random(si.size, dtype=np.float32) + np.float32(0.5)).astype(np.float32)
    csr = T.CsrMatrix(rows, cols, ro, si, va)
    assert_same_format(T.convert_csr_to_sw32(rows, cols, csr), build_on_device(csr))


@pytest.mark.parametrize("case", sorted(bad_sw32_inputs()))
def test_invalid_input_same_error_as_host(case):
    rows, cols, ro, si, va = bad_sw32_inputs()[case]
    with pytest.raises(T.InvalidArgument) as host_err:
        T.convert_csr_to_sw32(rows, cols, T.CsrMatrix(rows, cols, ro, si, va))
    with pytest.raises(T.InvalidArgument) as dev_err:
        T.convert_csr_to_sw32_device(rows, cols, *_device_csr(ro, si, va))
    assert str(dev_err.value) == str(host_err.value)


def test_side_stream_and_handle_lifetime():
    import torch

    csr = W.generate("stress_small")
    host = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dev = build_on_device(csr, stream=stream)
    stream.synchronize()
    values = dev.values  # keeps the library allocation alive on its own
    del dev
    import gc

    gc.collect()
    assert values.cpu().numpy().tobytes() == host.values.tobytes()


@pytest.mark.parametrize("features", [128, 256])
def test_spmm_over_device_format_bit_identical(features):
    import torch

    csr = W.generate("stress_small")
    case = build_case(csr, features, seed=4)
    y_host = run_spmm(case)
    dm = build_on_device(csr).device_matrix(features)
    y_dev = torch.full_like(y_host, float("nan"))
    T.launch_spmm_int8(dm.view(), case.packed_dev, case.scales_dev, y_dev, csr.rows, csr.cols, features,
                       dm.workspace())
    torch.cuda.synchronize()
    assert torch.equal(y_host.view(torch.int32), y_dev.view(torch.int32))
    assert int(dm.counters.abs().sum()) == 0
