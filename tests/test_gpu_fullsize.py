"""SpMM parity at the full benchmark sizes (power-law F128/F256, stress, R-MAT scale 24).

The whole-matrix oracle would take minutes at these sizes, so parity is checked through
properties that hold at any size plus the oracle on a sample of windows:
  * sampled windows (strided, plus every split window of the sample's heaviest kind) within
    the TF32 bound of the oracle restatement;
  * doubling every scale doubles Y bit-exactly: powers of two commute with the dequant
    product, TF32 rounding, the exact TF32 products and every FP32 sum;
  * a second launch is bit-identical and leaves every split-window counter at zero;
  * every element of Y is written (no NaN left from the NaN-filled output) and finite.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W

from tests.conftest import assert_within_tf32_bound

pytestmark = pytest.mark.gpu

CASES = [("powerlaw128", 128), ("powerlaw128", 256), ("stress", 128), ("rmat", 128)]


def _features(cols: int, features: int, seed: int):
    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, size=(cols, features), dtype=np.int8)
    s = (rng.random(cols, dtype=np.float32) * np.float32(0.05) + np.float32(0.001)).astype(np.float32)
    return q, s


def _sample_windows(fmt, count: int = 1500) -> np.ndarray:
    windows = fmt.window_offsets.size - 1
    strided = np.arange(0, windows, max(1, windows // count), dtype=np.int64)
    split = np.unique(fmt.tasks["sw"][fmt.tasks["chunks"] > 1].astype(np.int64)) if fmt.tasks.size else strided[:0]
    heavy = split[np.linspace(0, split.size - 1, min(split.size, 200)).astype(np.int64)] if split.size else split
    return np.unique(np.concatenate([strided, heavy])).astype(np.uint32)


@pytest.mark.parametrize("config,features", CASES)
def test_full_size_properties(config, features):
    import torch

    csr = W.generate(config)
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)
    del csr
    dm = T.DeviceMatrix(fmt, features, "cuda")
    q, s = _features(fmt.cols, features, 20261201)
    packed = torch.from_numpy(O.pack16(q).reshape(-1)).cuda()
    scales = torch.from_numpy(s).cuda()
    y = torch.full((fmt.rows, features), float("nan"), device="cuda")
    T.launch_spmm_int8(dm.view(), packed, scales, y, fmt.rows, fmt.cols, features, dm.workspace())
    torch.cuda.synchronize()
    assert bool(torch.isfinite(y).all()), "unwritten or non-finite output elements"

    # repeat: bit-identical, counters back to zero
    y2 = torch.full_like(y, float("nan"))
    T.launch_spmm_int8(dm.view(), packed, scales, y2, fmt.rows, fmt.cols, features, dm.workspace())
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int32), y2.view(torch.int32)), "repeated launch differs"
    if dm.counters is not None:
        assert int(dm.counters.abs().max()) == 0, "split-window counters not returned to zero"

    # doubled scales: exactly doubled output
    T.launch_spmm_int8(dm.view(), packed, scales * 2, y2, fmt.rows, fmt.cols, features, dm.workspace())
    torch.cuda.synchronize()
    assert torch.equal((y * 2).view(torch.int32), y2.view(torch.int32)), "doubling the scales did not double Y"
    del y2

    # sampled windows against the oracle
    sample = _sample_windows(fmt)
    ref, bound, rows = O.spmm(fmt, q, s, sample)
    keep = rows >= 0
    got = y[torch.from_numpy(rows[keep]).cuda()].cpu().numpy()
    assert_within_tf32_bound(got, ref[keep], bound[keep])


@pytest.mark.parametrize("config", ["powerlaw128", "stress", "rmat"])
def test_full_size_device_format_identical(config):
    """The GPU-built format of every full-size workload equals the host builder's, bit for bit."""
    import torch

    csr = W.generate(config)
    fmt = T.convert_csr_to_sw32(csr.rows, csr.cols, csr)

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).view(dtype)).cuda()

    dev = T.convert_csr_to_sw32_device(csr.rows, csr.cols, up(csr.row_offsets, np.int32),
                                       up(csr.source_ids, np.int32), up(csr.values, np.float32))
    assert dev.differences(fmt) == []
    if config == "rmat":  # the GPU generator the bench uses gives the same matrix
        gen = W.generate_device(config)
        assert gen.nnz == csr.nnz
        assert torch.equal(gen.row_offsets, up(csr.row_offsets, np.int32))
        assert torch.equal(gen.source_ids, up(csr.source_ids, np.int32))
        assert torch.equal(gen.values.view(torch.int32), up(csr.values, np.int32))
