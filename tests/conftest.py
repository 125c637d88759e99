"""Test configuration.

Markers: `gpu` tests need a B200 and call the operators through the C ABI
(libtcc_spmm_b200.so); everything else runs on the CPU. The oracle (oracle/) is the checker
only: the C restatement of the reference's arithmetic and the reference's own code compiled
into oracle/_ref.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

TOL_REL = 2.0 ** -10  # |dY| <= 2^-10 * sum|a_ij x_j| + 1e-6 (the reference's TF32 bound)
TOL_ABS = 1e-6


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running (full-size configurations)")


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def assert_within_tf32_bound(y: np.ndarray, y_ref: np.ndarray, bound: np.ndarray, what: str = "Y") -> None:
    """Element-wise |y - y_ref| <= 2^-10 * bound + 1e-6."""
    diff = np.abs(y.astype(np.float64) - y_ref.astype(np.float64))
    limit = TOL_REL * bound + TOL_ABS
    bad = diff > limit
    if bad.any():
        idx = np.argwhere(bad)[:5]
        detail = ", ".join(f"{tuple(i)}: got {y[tuple(i)]!r} want {y_ref[tuple(i)]!r} bound {bound[tuple(i)]!r}"
                           for i in idx)
        raise AssertionError(f"{what}: {int(bad.sum())} elements outside the TF32 bound; {detail}")


@pytest.fixture(scope="session")
def native():
    import tcc_spmm_b200._native as N

    return N.lib()
