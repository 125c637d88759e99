"""loadMatrixMarket parity with the reference's own reader (oracle/_ref): same canonical CSR
bytes for general/symmetric, real/integer/pattern files and the same error messages."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import tcc_spmm_b200 as T

pytestmark = pytest.mark.skipif(not O.have_ref_host(), reason="oracle/_ref not built")


def _write(tmp_path, name, text):
    p = tmp_path / name
    p.write_text(text)
    return str(p)


def _random_mtx(seed, field="real", symmetry="general", n=40, m=30, entries=300):
    rng = np.random.default_rng(seed)
    if symmetry == "symmetric":
        m = n
    lines = [f"%%MatrixMarket matrix coordinate {field} {symmetry}", "% a comment", "", f"{n} {m} {entries}"]
    for _ in range(entries):
        r = int(rng.integers(1, n + 1))
        c = int(rng.integers(1, m + 1))
        if symmetry == "symmetric" and c > r:
            r, c = c, r
        if field == "pattern":
            lines.append(f"{r} {c}")
        elif field == "integer":
            lines.append(f"{r} {c} {int(rng.integers(-3, 4))}")
        else:
            lines.append(f"{r} {c} {rng.standard_normal():.7e}")
        if rng.random() < 0.05:
            lines.append("%interleaved comment")
    return "\n".join(lines) + "\n"


@pytest.mark.parametrize("field", ["real", "integer", "pattern"])
@pytest.mark.parametrize("symmetry", ["general", "symmetric"])
def test_same_csr_as_reference(tmp_path, field, symmetry):
    path = _write(tmp_path, "a.mtx", _random_mtx(hash((field, symmetry)) % 1000, field, symmetry))
    mine = T.load_matrix_market(path)
    rows, cols, ro, si, va = O.ref_load_matrix_market(path)
    assert (mine.rows, mine.cols) == (rows, cols)
    assert mine.csr.row_offsets.tobytes() == ro.tobytes()
    assert mine.csr.source_ids.tobytes() == si.tobytes()
    assert mine.csr.values.tobytes() == va.tobytes()


BAD = {
    "header": "%%MatrixMarket matrix array real general\n2 2\n1\n2\n3\n4\n",
    "dims": "%%MatrixMarket matrix coordinate real general\n0 3 1\n1 1 1.0\n",
    "truncated": "%%MatrixMarket matrix coordinate real general\n3 3 4\n1 1 1.0\n2 2 1.0\n",
    "entry": "%%MatrixMarket matrix coordinate real general\n3 3 1\n4 1 1.0\n",
    "nan": "%%MatrixMarket matrix coordinate real general\n3 3 1\n1 1 nan\n",
    "missing dims": "%%MatrixMarket matrix coordinate real general\n% only comments\n",
    "symmetric rect": "%%MatrixMarket matrix coordinate real symmetric\n3 4 1\n1 1 1.0\n",
}


@pytest.mark.parametrize("case", sorted(BAD))
def test_same_errors_as_reference(tmp_path, case):
    path = _write(tmp_path, "bad.mtx", BAD[case])
    with pytest.raises(O.oracle.RefError) as ref:
        O.ref_load_matrix_market(path)
    with pytest.raises(RuntimeError) as mine:
        T.load_matrix_market(path)
    assert str(mine.value) == str(ref.value)


def test_missing_file(tmp_path):
    with pytest.raises(RuntimeError, match="cannot open Matrix Market file"):
        T.load_matrix_market(str(tmp_path / "nope.mtx"))


def test_mtx_to_sw32_round_trip(tmp_path):
    path = _write(tmp_path, "b.mtx", _random_mtx(5, "real", "symmetric", n=100, entries=2000))
    m = T.load_matrix_market(path)
    fmt = T.convert_csr_to_sw32(m.rows, m.cols, m.csr)
    ref = O.ref_convert_csr_to_sw32(m.rows, m.cols, m.csr.row_offsets, m.csr.source_ids, m.csr.values)
    assert fmt.source_metadata.tobytes() == ref["source_metadata"].tobytes()
    assert fmt.values.tobytes() == ref["values"].tobytes()
