"""quantizeFeaturesInt8 / packFeaturesInt8x16 / fused quantize+pack on the B200: bytes
identical to the oracle restatement and to the reference's own kernels."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tcc_spmm_b200 as T
from tcc_spmm_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _x(sources, features, seed):
    x = W.normal_features(sources, features, seed)
    if sources > 4:
        x[0] = 0.0                                  # all-zero row -> scale 1
        x[1, :] = np.float32(0.5)                   # x/s hits exact ties of lrintf
        x[1, ::3] = -np.float32(1.5)
        x[2] *= np.float32(3e-30)                   # tiny but normal magnitudes
        x[3, 5 % features] = np.float32(-1e30)      # absmax from a negative value
    return x


SHAPES = [(1000, 128), (777, 256), (333, 48), (129, 1024), (64, 16), (50, 2048)]


@pytest.mark.parametrize("sources,features", SHAPES)
def test_quantize_and_pack_bytes(sources, features):
    import torch

    x = _x(sources, features, 3 + features)
    q_ref, s_ref = O.quantize(x)
    xd = torch.from_numpy(x).cuda()
    q = torch.empty(sources * features, dtype=torch.int8, device="cuda")
    s = torch.empty(sources, dtype=torch.float32, device="cuda")
    T.quantize_features_int8(xd, q, s, sources, features)
    packed = torch.empty_like(q)
    T.pack_features_int8x16(q, packed, sources, features)
    fused = torch.empty_like(q)
    s2 = torch.empty_like(s)
    T.quantize_pack_features_int8(xd, fused, s2, sources, features)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy().reshape(sources, features), q_ref)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    p_ref = O.pack16(q_ref)
    assert np.array_equal(packed.cpu().numpy().reshape(sources, features), p_ref)
    assert np.array_equal(fused.cpu().numpy().reshape(sources, features), p_ref)
    assert np.array_equal(s2.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_quantize_any_width_and_misaligned():
    import torch

    sources, features = 37, 19  # not a multiple of 16: generic path
    x = _x(sources, features, 5)
    q_ref, s_ref = O.quantize(x)
    raw = torch.empty(sources * features + 1, dtype=torch.float32, device="cuda")
    xd = raw[1:]  # 4-byte aligned only
    xd.copy_(torch.from_numpy(x.reshape(-1)))
    q = torch.empty(sources * features, dtype=torch.int8, device="cuda")
    s = torch.empty(sources, dtype=torch.float32, device="cuda")
    T.quantize_features_int8(xd, q, s, sources, features)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy().reshape(sources, features), q_ref)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_pack_two_byte_aligned_output():
    import torch

    sources, features = 100, 64
    q_ref, _ = O.quantize(_x(sources, features, 8))
    q = torch.from_numpy(q_ref.reshape(-1)).cuda()
    raw = torch.empty(sources * features + 2, dtype=torch.int8, device="cuda")
    out = raw[2:]
    T.pack_features_int8x16(q, out, sources, features)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().reshape(sources, features), O.pack16(q_ref))


def test_feature_errors():
    import torch

    q = torch.zeros(64, dtype=torch.int8, device="cuda")
    out = torch.zeros(64, dtype=torch.int8, device="cuda")
    with pytest.raises(T.InvalidArgument):
        T.pack_features_int8x16(q, out, 8, 8)  # features % 16 != 0
    with pytest.raises(T.CudaError):
        T.pack_features_int8x16(q, out, 0, 16)  # empty grid, as in the reference


@pytest.mark.skipif(not O.have_ref_cuda("sm100a"), reason="reference kernels not built")
@pytest.mark.parametrize("tag", ["sm100a", "sm80"])
def test_reference_kernels_bytes(tag):
    """The reference's quantize/pack kernels on the same X give the same bytes."""
    import torch

    if not O.have_ref_cuda(tag):
        pytest.skip(f"{tag} missing")
    ref = O.ref_cuda(tag)
    sources, features = 2048, 128
    x = _x(sources, features, 21)
    xd = torch.from_numpy(x).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    q = torch.empty(sources * features, dtype=torch.int8, device="cuda")
    s = torch.empty(sources, dtype=torch.float32, device="cuda")
    p = torch.empty_like(q)
    ref.quantize(xd.data_ptr(), q.data_ptr(), s.data_ptr(), sources, features, stream)
    ref.pack(q.data_ptr(), p.data_ptr(), sources, features, stream)
    mine_p = torch.empty_like(q)
    mine_s = torch.empty_like(s)
    T.quantize_pack_features_int8(xd, mine_p, mine_s, sources, features)
    torch.cuda.synchronize()
    assert torch.equal(p, mine_p)
    assert torch.equal(s.view(torch.int32), mine_s.view(torch.int32))
