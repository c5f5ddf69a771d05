"""MatrixMarket reader (cove_mm_read) against the reference's own loader.

tests/golden/mm_cases.npz holds small coordinate files and the CSR that
structural::read_matrix_market_with_info (matrix_market.hpp:327-382)
returned for them, or the message it raised (tests/golden/make_mm_golden.py).
Host code only: runs without a GPU.
"""
import os

import numpy as np
import pytest

import cove_b200 as cb

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "mm_cases.npz")
FIELDS = ("real", "integer", "complex", "pattern")
SYMS = ("general", "symmetric", "skew-symmetric", "hermitian")


def _cases():
    d = np.load(GOLDEN)
    return d, sorted({k.split("/")[0] for k in d.files})


@pytest.mark.parametrize("name", _cases()[1])
def test_reader_matches_reference_loader(name, tmp_path):
    d, _ = _cases()
    path = tmp_path / f"{name}.mtx"
    path.write_bytes(bytes(d[f"{name}/text"]))
    dtype = np.float64 if int(d[f"{name}/esz"][0]) == 8 else np.float32
    if f"{name}/error" in d.files:
        want = bytes(d[f"{name}/error"]).decode()
        with pytest.raises(cb.CoveError, match=want):
            cb.read_matrix_market(str(path), dtype)
        return
    rows, cols, rp, ci, v, info = cb.read_matrix_market(str(path), dtype)
    assert (rows, cols) == tuple(int(x) for x in d[f"{name}/shape"])
    fs = d[f"{name}/field_symmetry"]
    assert (info["field"], info["symmetry"]) == (FIELDS[fs[0]], SYMS[fs[1]])
    c = d[f"{name}/counts"]
    assert (info["stored_entries"], info["expanded_entries"], info["coalesced_duplicates"]) == tuple(c)
    assert np.array_equal(rp, d[f"{name}/row_ptr"].astype(np.int64))
    assert np.array_equal(ci, d[f"{name}/col_idx"])
    assert v.dtype == dtype
    assert np.array_equal(v.view(np.uint8), d[f"{name}/values"].astype(dtype).view(np.uint8))


def test_reader_round_trips_a_generated_matrix(tmp_path):
    """A 2D Laplacian written with %.17g reads back bit for bit."""
    rows, cols, rp, ci, v = cb.synth_lapl2d(20, 17)
    v = v * (1.0 + np.arange(v.size) * 1e-7)  # many distinct values
    lines = [f"%%MatrixMarket matrix coordinate real general\n{rows} {cols} {v.size}\n"]
    for r in range(rows):
        for p in range(rp[r], rp[r + 1]):
            lines.append(f"{r + 1} {ci[p] + 1} {v[p]:.17g}\n")
    path = tmp_path / "l.mtx"
    path.write_text("".join(lines))
    r2, c2, rp2, ci2, v2, info = cb.read_matrix_market(str(path))
    assert (r2, c2) == (rows, cols) and info["coalesced_duplicates"] == 0
    assert np.array_equal(rp2, rp) and np.array_equal(ci2, ci) and np.array_equal(v2, v)


def test_reader_reports_missing_file(tmp_path):
    with pytest.raises(cb.CoveError, match="cannot open MatrixMarket file"):
        cb.read_matrix_market(str(tmp_path / "nope.mtx"))
