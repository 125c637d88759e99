"""The GPU R-MAT generator (tcc_wl_rmat_device) produces the host generator's matrix bit for
bit: same row offsets, source IDs and 1/deg_i values, for several scales, edge counts and
quadrant probabilities (the full-size matrix is compared in test_gpu_fullsize.py)."""
from __future__ import annotations

import numpy as np
import pytest

from tcc_spmm_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("scale,edges,abc,seed", [
    (16, 1 << 20, (0.57, 0.19, 0.19), 16),          # rmat_small
    (18, (1 << 22) + 12345, (0.57, 0.19, 0.19), 3),  # two sampling blocks, a ragged last one
    (12, 1 << 16, (0.25, 0.25, 0.25), 9),            # uniform quadrants
    (5, 40, (0.45, 0.15, 0.15), 1),                  # fewer edges than rows
])
def test_device_rmat_equals_host(scale, edges, abc, seed):
    host = W.rmat(scale, edges, *abc, seed=seed)
    dev = W.rmat_device(scale, edges, *abc, seed=seed).to_host()
    assert (dev.rows, dev.cols) == (host.rows, host.cols)
    assert np.array_equal(dev.row_offsets, host.row_offsets)
    assert np.array_equal(dev.source_ids, host.source_ids)
    assert np.array_equal(dev.values.view(np.uint32), host.values.view(np.uint32))


def test_generate_device_matches_generate_for_host_configs():
    for name in ("stress_small", "powerlaw_small"):
        host = W.generate(name)
        dev = W.generate_device(name).to_host()
        assert np.array_equal(dev.row_offsets, host.row_offsets)
        assert np.array_equal(dev.source_ids, host.source_ids)
        assert np.array_equal(dev.values, host.values)
