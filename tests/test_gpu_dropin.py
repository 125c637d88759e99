"""Drop-in check: the reference's own CLI driver (its src/main.cu and src/device_matrix.cuh,
unmodified) built against this repository's headers and libtcc_spmm_b200.so
(oracle/_ref/tcc_spmm_run_dropin) runs the reference workflow end to end - Matrix Market file,
convertCsrToSw32, upload, quantize/pack, launchSpmmInt8 - and prints the same Y[0,0:8] as the
reference build of the same driver (oracle/_ref/tcc_spmm_run_ref) and as the oracle."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle as O
import tcc_spmm_b200 as T

ROOT = Path(__file__).resolve().parent.parent
DROPIN = ROOT / "oracle" / "_ref" / "tcc_spmm_run_dropin"
REF = ROOT / "oracle" / "_ref" / "tcc_spmm_run_ref"

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not DROPIN.exists(), reason="drop-in driver not built")]


def _write_mtx(path: Path, rows: int, seed: int) -> None:
    rng = np.random.default_rng(seed)
    lines = [f"%%MatrixMarket matrix coordinate real general", f"{rows} {rows} 0"]
    entries = []
    for r in range(rows):
        deg = int(rng.integers(0, 40)) if r % 97 else 4000  # a few heavy rows -> split windows
        cols = rng.integers(0, rows, size=deg)
        vals = rng.uniform(-1, 1, size=deg)
        entries += [f"{r + 1} {c + 1} {v:.6f}" for c, v in zip(cols, vals)]
    lines[1] = f"{rows} {rows} {len(entries)}"
    path.write_text("\n".join(lines + entries) + "\n")


def _run(binary: Path, mtx: Path, features: int):
    out = subprocess.run([str(binary), str(mtx), str(features), "0"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    ms = float(re.search(r"SpMM kernel average: ([0-9.]+) ms", out.stdout).group(1))
    y = np.array([float(v) for v in re.search(r"Output Y\[0,0:8\]:(.*)", out.stdout).group(1).split()])
    return ms, y


def _reference_features(rows: int, features: int) -> np.ndarray:
    """X of the reference driver: std::mt19937(20261025), (rng() >> 8) / 2^23 - 1."""
    raw = np.random.RandomState(20261025).randint(0, 2**32, size=rows * features, dtype=np.uint64)
    return ((raw >> 8).astype(np.float32) * np.float32(1.0 / 8388608.0) - np.float32(1.0)).reshape(rows, features)


@pytest.mark.parametrize("features", [128, 256])
def test_reference_driver_runs_on_new_library(tmp_path, features):
    mtx = tmp_path / "m.mtx"
    _write_mtx(mtx, 20000, features)
    ms_new, y_new = _run(DROPIN, mtx, features)
    m = T.load_matrix_market(str(mtx))
    fmt = T.convert_csr_to_sw32(m.rows, m.cols, m.csr)
    assert fmt.partial_count > 0
    q, s = O.quantize(_reference_features(m.cols, features))
    y, bound, rows = O.spmm(fmt, q, s, sw_list=np.array([0], np.uint32))
    tol = 2.0 ** -10 * bound[0, :8] + 1e-6 + 5e-7  # the driver prints 6 decimals
    assert np.all(np.abs(y_new - y[0, :8]) <= tol)
    if REF.exists():
        ms_ref, y_ref = _run(REF, mtx, features)
        assert np.all(np.abs(y_new - y_ref) <= 2 * tol)
