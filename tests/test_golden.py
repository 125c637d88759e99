"""Golden fixtures made by the reference itself (tests/golden/make_golden.py): format arrays
from its convertCsrToSw32, q/scales/packed bytes from its quantize/pack kernels and Y from its
SpMM kernel. They pin both the oracle restatement and the product without needing the
reference tree or a GPU."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle as O
import tcc_spmm_b200 as T
from tests.conftest import assert_within_tf32_bound

GOLDEN = Path(__file__).resolve().parent / "golden"
FORMAT_FIXTURES = sorted(GOLDEN.glob("sw32_*.npz"))


@pytest.mark.parametrize("path", FORMAT_FIXTURES, ids=[p.stem for p in FORMAT_FIXTURES])
def test_format_matches_reference_fixture(path):
    g = np.load(path)
    rows, cols = int(g["rows"]), int(g["cols"])
    csr = T.CsrMatrix(rows, cols, g["row_offsets"], g["csr_source_ids"], g["csr_values"])
    mine = T.convert_csr_to_sw32(rows, cols, csr)
    for name in O.oracle.REF_SW32_FIELDS:
        a = getattr(mine, name)
        if name in ("tasks", "reductions"):
            a = a.view(np.uint32)
        assert a.tobytes() == g[name].tobytes(), name
    assert mine.partial_count == int(g["partial_count"])


def test_format_fixtures_exist():
    assert len(FORMAT_FIXTURES) >= 4


def _features_fixture():
    path = GOLDEN / "ref_features.npz"
    if not path.exists():
        pytest.skip("ref_features.npz not generated yet (needs a GPU run of make_golden.py gpu)")
    return np.load(path)


def _spmm_fixture():
    path = GOLDEN / "ref_spmm.npz"
    if not path.exists():
        pytest.skip("ref_spmm.npz not generated yet (needs a GPU run of make_golden.py gpu)")
    return np.load(path)


def test_oracle_quantize_pack_match_reference_kernels():
    g = _features_fixture()
    q, s = O.quantize(g["x"])
    assert np.array_equal(q, g["q"])
    assert np.array_equal(s.view(np.uint32), g["scales"].view(np.uint32))
    assert np.array_equal(O.pack16(q), g["packed"])


def test_oracle_spmm_matches_reference_kernel():
    g = _spmm_fixture()
    rows, cols = int(g["rows"]), int(g["cols"])
    csr = T.CsrMatrix(rows, cols, g["row_offsets"], g["source_ids"], g["values"])
    fmt = T.convert_csr_to_sw32(rows, cols, csr)
    y, bound, r = O.spmm(fmt, g["q"], g["scales"])
    assert_within_tf32_bound(g["y"], y[r >= 0], bound[r >= 0], "reference kernel vs oracle")


@pytest.mark.gpu
def test_product_matches_reference_fixtures():
    import torch

    g = _features_fixture()
    sources, features = g["x"].shape
    xd = torch.from_numpy(g["x"]).cuda()
    packed = torch.empty(sources * features, dtype=torch.int8, device="cuda")
    scales = torch.empty(sources, dtype=torch.float32, device="cuda")
    T.quantize_pack_features_int8(xd, packed, scales, sources, features)
    torch.cuda.synchronize()
    assert np.array_equal(packed.cpu().numpy().reshape(sources, features), g["packed"])
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), g["scales"].view(np.uint32))
    h = _spmm_fixture()
    rows, cols = int(h["rows"]), int(h["cols"])
    csr = T.CsrMatrix(rows, cols, h["row_offsets"], h["source_ids"], h["values"])
    fmt = T.convert_csr_to_sw32(rows, cols, csr)
    dm = T.DeviceMatrix(fmt, 128, "cuda")
    p = torch.from_numpy(O.pack16(h["q"]).reshape(-1)).cuda()
    s = torch.from_numpy(h["scales"]).cuda()
    y = torch.full((rows, 128), float("nan"), device="cuda")
    T.launch_spmm_int8(dm.view(), p, s, y, rows, cols, 128, dm.workspace())
    torch.cuda.synchronize()
    _, bound, r = O.spmm(fmt, h["q"], h["scales"])
    assert_within_tf32_bound(y.cpu().numpy(), h["y"], 2 * bound[r >= 0], "product vs reference kernel")
