"""SpMM parity on the B200 through the C ABI: Y within the reference's TF32 bound of the CPU
oracle (and of the reference kernel itself), bit-exact where Y is a single TF32 product,
counters back to zero, repeated launches identical, no writes outside Y and the workspace."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W
from tests.cases import EDGE_CASES, random_csr
from tests.conftest import assert_within_tf32_bound
from tests.gpu_util import build_case, oracle_y, run_spmm

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    return torch


@pytest.mark.parametrize("variant", ["default", "generic", "persistent32", "persistent64", "tmem8"])
@pytest.mark.parametrize("features", [128, 256])
@pytest.mark.parametrize("name", sorted(EDGE_CASES))
def test_edge_cases_within_tf32_bound(name, features, variant):
    torch = _torch()
    case = build_case(EDGE_CASES[name](), features)
    y = run_spmm(case, variant=variant)
    torch.cuda.synchronize()
    y_ref, bound = oracle_y(case)
    got = y.cpu().numpy()
    assert np.isfinite(got).all(), "every Y element must be written"
    assert_within_tf32_bound(got, y_ref, bound, f"{name}/F{features}")
    if case.dm.counters is not None:
        assert int(case.dm.counters.abs().sum()) == 0, "counters must return to zero"


@pytest.mark.parametrize("features", [128, 256])
@pytest.mark.parametrize("name", ["cpu4096", "powerlaw_small", "stress_small", "rmat_small"])
def test_seeded_configs_within_tf32_bound(name, features):
    torch = _torch()
    case = build_case(W.generate(name), features, seed=7)
    y = run_spmm(case)
    torch.cuda.synchronize()
    y_ref, bound = oracle_y(case)
    assert_within_tf32_bound(y.cpu().numpy(), y_ref, bound, f"{name}/F{features}")


@pytest.mark.parametrize("variant", ["generic", "persistent32", "persistent64"])
def test_single_term_rows_bit_exact(variant):
    """One nonzero per row: Y = tf32_rna(a) * tf32_rna(q*s) exactly, which pins the operand
    rounding (round-half-away on 10 mantissa bits) on the tensor cores of the kernels that
    dequantize X to TF32."""
    torch = _torch()
    case = build_case(EDGE_CASES["single_term"](), 128, seed=11)
    y = run_spmm(case, variant=variant)
    torch.cuda.synchronize()
    y_ref, _ = oracle_y(case)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("features", [128, 256])
@pytest.mark.parametrize("variant", ["default", "tmem8"])
def test_single_term_rows_within_half_bound(variant, features):
    """The tensor-memory kernel folds the scale into the values (q * (tf32(a) * s) to 22 bits):
    a single term is within 2^-11 relative of the reference's tf32_rna(a) * tf32_rna(q*s), half
    the stated bound."""
    torch = _torch()
    case = build_case(EDGE_CASES["single_term"](), features, seed=11)
    y = run_spmm(case, variant=variant)
    torch.cuda.synchronize()
    y_ref, bound = oracle_y(case)
    assert_within_tf32_bound(y.cpu().numpy(), y_ref, bound / 2, f"single-term rows/F{features}")


@pytest.mark.parametrize("features", [128, 256])
def test_repeated_launches_identical_and_counters_reset(features):
    torch = _torch()
    case = build_case(W.generate("stress_small"), features, seed=3)
    assert case.fmt.partial_count > 0
    stream = torch.cuda.Stream()  # non-default, non-blocking stream
    with torch.cuda.stream(stream):
        y1 = run_spmm(case, stream=stream)
        y2 = run_spmm(case, stream=stream)
    stream.synchronize()
    assert torch.equal(y1.view(torch.int32), y2.view(torch.int32))
    assert int(case.dm.counters.abs().sum()) == 0


def test_generic_and_pipelined_agree_within_bound():
    torch = _torch()
    case = build_case(W.generate("powerlaw_small"), 128, seed=5)
    a = run_spmm(case)
    b = run_spmm(case, variant="generic")
    torch.cuda.synchronize()
    _, bound = oracle_y(case)
    assert_within_tf32_bound(a.cpu().numpy(), b.cpu().numpy(), 2 * bound, "pipelined vs generic")


def test_no_writes_outside_outputs():
    """Canary words around Y and the partial workspace stay untouched."""
    torch = _torch()
    case = build_case(W.generate("stress_small"), 128, seed=9)
    rows, F = case.fmt.rows, 128
    pad = 4096
    canary = -7.77e30
    big = torch.full((rows * F + 2 * pad,), canary, device="cuda")
    y = big[pad:pad + rows * F].view(rows, F)
    pf = case.dm.partials.numel()
    pbig = torch.full((pf + 2 * pad,), canary, device="cuda")
    case.dm.partials = pbig[pad:pad + pf]
    run_spmm(case, out=y)
    torch.cuda.synchronize()
    for buf in (big, pbig):
        assert bool((buf[:pad] == canary).all()) and bool((buf[-pad:] == canary).all())


def test_misaligned_packed_x_uses_generic_path():
    torch = _torch()
    case = build_case(random_csr(500, 700, 8.0, 4), 128, seed=2)
    raw = torch.empty(case.packed_dev.numel() + 2, dtype=torch.int8, device="cuda")
    shifted = raw[2:]
    shifted.copy_(case.packed_dev)
    case.packed_dev = shifted  # 2-byte aligned only
    y = run_spmm(case)
    torch.cuda.synchronize()
    y_ref, bound = oracle_y(case)
    assert_within_tf32_bound(y.cpu().numpy(), y_ref, bound, "misaligned packedX")


@pytest.mark.parametrize("features", [128, 256])
def test_ids_and_metadata_only_4_byte_aligned(features):
    """IDs/metadata that are not 16-byte aligned (allowed by the reference's contract) take
    the kernel without bulk copies; results stay within the bound."""
    torch = _torch()
    case = build_case(random_csr(600, 900, 9.0, 5), features, seed=3)
    ids = torch.empty(case.dm.source_ids.numel() + 1, dtype=torch.int32, device="cuda")[1:]
    ids.copy_(case.dm.source_ids)
    meta = torch.empty(case.dm.source_metadata.numel() + 1, dtype=torch.int64, device="cuda")[1:]
    meta.copy_(case.dm.source_metadata)
    case.dm.source_ids, case.dm.source_metadata = ids, meta
    y = run_spmm(case)
    torch.cuda.synchronize()
    y_ref, bound = oracle_y(case)
    assert_within_tf32_bound(y.cpu().numpy(), y_ref, bound, "4-byte aligned IDs/metadata")


@pytest.mark.parametrize("features", [128, 256])
def test_values_only_4_byte_aligned(features):
    """Values that are not 16-byte aligned (the tensor-memory kernel copies each chunk's value
    range with one bulk copy) take the kernel without bulk copies; results stay within the
    bound."""
    torch = _torch()
    case = build_case(random_csr(600, 900, 9.0, 6), features, seed=4)
    vals = torch.empty(case.dm.values.numel() + 1, dtype=torch.float32, device="cuda")[1:]
    vals.copy_(case.dm.values)
    case.dm.values = vals
    y = run_spmm(case)
    torch.cuda.synchronize()
    y_ref, bound = oracle_y(case)
    assert_within_tf32_bound(y.cpu().numpy(), y_ref, bound, "4-byte aligned values")


def test_bad_feature_count_raises_invalid_argument():
    torch = _torch()
    case = build_case(random_csr(64, 64, 4.0, 1), 128)
    y = torch.empty(64, 128, device="cuda")
    with pytest.raises(T.InvalidArgument, match="128 or 256"):
        T.launch_spmm_int8(case.dm.view(), case.packed_dev, case.scales_dev, y, 64, 64, 64, case.dm.workspace())


REFERENCE_CASES = sorted(n for n in EDGE_CASES if n != "empty") + ["cpu4096", "powerlaw_small", "stress_small",
                                                                    "rmat_small"]


@pytest.mark.skipif(not O.have_ref_cuda("sm100a"), reason="reference kernel not built")
@pytest.mark.parametrize("tag", ["sm100a", "sm80"])
@pytest.mark.parametrize("features", [128, 256])
@pytest.mark.parametrize("name", REFERENCE_CASES)
def test_matches_reference_kernel(name, tag, features):
    """The reference's own kernel (its src/kernel/spmm.cu, built for sm_100a and as compute_80 PTX)
    on the same uploaded format, packed X and scales: Y within the stated bound of it, on every
    edge case and seeded configuration, and the shared counters back at zero after both."""
    torch = _torch()
    if not O.have_ref_cuda(tag):
        pytest.skip(f"reference {tag} build missing")
    ref = O.ref_cuda(tag)
    csr = W.generate(name) if name in W.CONFIGS else EDGE_CASES[name]()
    case = build_case(csr, features, seed=13)
    y = run_spmm(case)
    y_ref = torch.full_like(y, float("nan"))
    view = case.dm.view()
    import ctypes

    ws = case.dm.workspace()
    ref.launch_spmm_int8(ctypes.addressof(view), case.packed_dev.data_ptr(), case.scales_dev.data_ptr(),
                         y_ref.data_ptr(), case.fmt.rows, case.fmt.cols, features,
                         ws.partials.data_ptr() if ws.partials is not None else 0,
                         ws.counters.data_ptr() if ws.counters is not None else 0,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    _, bound = oracle_y(case)
    got, want = y.cpu().numpy(), y_ref.cpu().numpy()
    assert np.isfinite(want).all(), "the reference kernel must write every element"
    assert_within_tf32_bound(got, want, bound, f"{name}/F{features} vs reference {tag}")
    if case.dm.counters is not None:
        assert int(case.dm.counters.abs().sum()) == 0, "both kernels return the counters to zero"


@pytest.mark.parametrize("features", [128, 256])
@pytest.mark.parametrize("name", ["stress_small", "powerlaw_small"])
@pytest.mark.parametrize("variant", ["default", "generic", "persistent32", "persistent64"])
def test_balanced_task_order_bit_identical(name, features, variant):
    """Y does not depend on the task order: the speed-weighted order with its skip entries
    (tcc_balance_tasks_padded, what a balanced DeviceMatrix launches) gives the same bits as the
    format order in every kernel, which all skip the padding (split windows merge their
    partials in a fixed order)."""
    torch = _torch()
    case = build_case(W.generate(name), features, seed=17)
    y = run_spmm(case, variant=variant)
    balanced = T.DeviceMatrix(case.fmt, features, "cuda", balance=True)
    assert balanced.tasks_balanced is not None
    assert balanced.balanced_count > case.fmt.tasks.size, "the order has skip entries"
    y2 = torch.full_like(y, float("nan"))
    T.launch_spmm_int8(balanced.view(), case.packed_dev, case.scales_dev, y2, case.fmt.rows, case.fmt.cols,
                       features, balanced.workspace(), variant=variant)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int32), y2.view(torch.int32))
    assert int(balanced.counters.abs().sum()) == 0


