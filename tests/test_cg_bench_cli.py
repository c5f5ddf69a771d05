"""bench_cg_solve: the reference's CG solver comparison
(structural/src/bench_cg_solve.cu) over this library's operators.

CPU: the seeded SPD generators against hashes of the reference's own
generators (tests/golden/cg_synth.json, made by
tests/golden/make_cg_synth_golden.py) and the argument handling.  GPU: the
CSV contract -- six variants in the reference's order, the exact variants
reaching 1e-8 with the same solution, the low-precision floors, the nine
IR / FCG solves and append mode."""
import csv
import json
import os
import subprocess

import numpy as np
import pytest

import cove_b200 as cb

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
BIN = os.path.join(ROOT, "cove-spmv_b200", "bin", "bench_cg_solve")
HASH_SRC = os.path.join(ROOT, "tests", "cpp", "cg_synth_hash.cpp")
HASH_BIN = os.path.join(ROOT, "tests", "cpp", "_build", "cg_synth_hash")
VARIANTS = ["cusparse_double", "cusparse_float", "cove_lossless", "cove_bf16", "cove_bfp8", "cove_bfp8_outlier"]
SOLVERS = ["ir_bf16_k20", "ir_bf16_k40", "ir_bf16_k80", "fcg_bf16_k5", "fcg_bf16_k10", "fcg_bf16_k20",
           "fcg_bf16_k40", "fcg_bfp8_k5", "fcg_bfp8_k10"]


def _hash_bin():
    deps = [HASH_SRC, os.path.join(ROOT, "cove-spmv_b200", "include", "structural", "synthetic_spd.hpp")]
    if not os.path.exists(HASH_BIN) or os.path.getmtime(HASH_BIN) < max(map(os.path.getmtime, deps)):
        os.makedirs(os.path.dirname(HASH_BIN), exist_ok=True)
        subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off",
                        "-I" + os.path.join(ROOT, "cove-spmv_b200", "include"), "-o", HASH_BIN, HASH_SRC],
                       check=True, capture_output=True, text=True)
    return HASH_BIN


def test_synthetic_spd_matches_reference_generators():
    with open(os.path.join(ROOT, "tests", "golden", "cg_synth.json")) as f:
        golden = json.load(f)
    exe = _hash_bin()
    for row in golden:
        out = subprocess.run([exe, *map(str, row["case"])], capture_output=True, text=True, check=True).stdout
        got = dict(line.split(" ", 1) for line in out.strip().splitlines())
        assert got == {k: row[k] for k in ("nnz", "row_ptr", "col_idx", "values")}, row["case"]


def test_bench_cg_solve_usage():
    p = subprocess.run([BIN], capture_output=True, text=True, timeout=60)
    assert p.returncode == 2 and "usage:" in p.stderr and "synth:N:halfbw:delta" in p.stderr


def _run(*args):
    p = subprocess.run([BIN, *map(str, args)], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr
    return p.stdout


def _rows(path):
    with open(path) as f:
        return list(csv.DictReader(f))


@pytest.mark.gpu
def test_bench_cg_solve_synthetic(tmp_path):
    out_csv = tmp_path / "cg.csv"
    n, bw = 6000, 16
    text = _run(f"synth:{n}:{bw}:1.0", out_csv, 0, 3000, 7)
    assert f"== synth_n{n}_bw{bw}_d1 " in text and "seed=7 maxiter=3000" in text
    rows = _rows(out_csv)
    assert [r["variant"] for r in rows] == VARIANTS
    by = {r["variant"]: r for r in rows}
    nnz = n * (2 * bw + 1) - bw * (bw + 1)
    assert all(r["matrix"] == f"synth_n{n}_bw{bw}_d1" and int(r["n"]) == n and int(r["nnz"]) == nnz for r in rows)
    for v in ("cusparse_double", "cove_lossless"):  # exact fp64 matvecs
        r = by[v]
        assert r["spd_ok"] == "1" and int(r["iter_1e-8"]) > 0 and float(r["floor"]) <= 1e-8
        assert float(r["sol_err"]) < 1e-5 and float(r["ms_per_iter"]) > 0
        assert int(r["iter_1e-2"]) <= int(r["iter_1e-3"]) <= int(r["iter_1e-6"]) <= int(r["iter_1e-8"])
        assert float(r["time_1e-6_ms"]) == pytest.approx(int(r["iter_1e-6"]) * float(r["ms_per_iter"]), rel=1e-3,
                                                         abs=1e-3)
    assert abs(int(by["cusparse_double"]["iter_1e-8"]) - int(by["cove_lossless"]["iter_1e-8"])) <= 1
    assert float(by["cove_bf16"]["bytes_per_nnz"]) == 2.0 and float(by["cusparse_float"]["bytes_per_nnz"]) == 4.0
    assert 1.0 < float(by["cove_bfp8"]["bytes_per_nnz"]) < 1.5
    assert float(by["cove_bfp8_outlier"]["bytes_per_nnz"]) > float(by["cove_bfp8"]["bytes_per_nnz"])
    for v in ("cove_bf16", "cove_bfp8"):  # value rounding leaves a floor above fp64
        assert by[v]["spd_ok"] == "1" and float(by[v]["floor"]) > 1e-8 and by[v]["iter_1e-8"] == "-1"
        assert 0 < int(by[v]["iter_1e-2"])
    ir = _rows(tmp_path / "cg_ir.csv")
    assert [r["solver"] for r in ir] == SOLVERS
    for r in ir:
        assert r["reached"] == "1" and float(r["final_relres"]) <= 1e-8 and int(r["inner_total"]) > 0, r
        assert float(r["base_double_t1e8_ms"]) == pytest.approx(float(by["cusparse_double"]["iter_1e-8"])
                                                                * float(by["cusparse_double"]["ms_per_iter"]),
                                                                rel=1e-3, abs=1e-3)
    assert "--- IR vs FCG (target true relres 1e-08)" in text

    # append: the second matrix adds rows under the one header
    _run(f"lapl:4000:8:0.05", out_csv, 1, 3000, 7)
    rows = _rows(out_csv)
    assert len(rows) == 12 and [r["variant"] for r in rows[6:]] == VARIANTS
    assert rows[6]["matrix"] == "lapl_n4000_bw8_s0.05"
    lap = {r["variant"]: r for r in rows[6:]}
    assert lap["cove_lossless"]["spd_ok"] == "1" and int(lap["cove_lossless"]["iter_1e-8"]) > 0
    assert len(_rows(tmp_path / "cg_ir.csv")) == 18


@pytest.mark.gpu
def test_bench_cg_solve_matrix_market(tmp_path):
    rows, cols, rp, ci, v = cb.synth_lapl2d(40, 30)  # SPD
    path = tmp_path / "lap40x30.mtx"
    lines = [f"%%MatrixMarket matrix coordinate real general\n{rows} {cols} {len(v)}\n"]
    for r in range(rows):
        lines += [f"{r + 1} {ci[p] + 1} {v[p]:.17g}\n" for p in range(rp[r], rp[r + 1])]
    path.write_text("".join(lines))
    out_csv = tmp_path / "m.csv"
    text = _run(path, out_csv, 0, 2000)
    assert "== lap40x30 " in text and "seed=12345" in text
    got = {r["variant"]: r for r in _rows(out_csv)}
    assert got["cove_lossless"]["matrix"] == "lap40x30" and int(got["cove_lossless"]["iter_1e-8"]) > 0

    rect = tmp_path / "rect.mtx"
    rect.write_text("%%MatrixMarket matrix coordinate real general\n2 3 2\n1 1 1.0\n2 3 2.0\n")
    p = subprocess.run([BIN, str(rect), str(tmp_path / "r.csv")], capture_output=True, text=True, timeout=60)
    assert p.returncode == 0 and "rect not square -> CG N/A" in p.stderr
    assert not (tmp_path / "r.csv").exists()
