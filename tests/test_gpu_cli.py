"""struct_gpu_csr_bitbsr_spmv: the reference CLI's options and report.

The fused_lb checks of the reference's own CLI test
(structural/tests/test_gpu_csr_bitbsr_spmv_cli.sh:11-45, 61-67) on the same
4 x 8 matrix, and the joint-codec keys its sweep script reads
(structural/scripts/run_joint_sweep.py:74-101).  Option handling needs no
GPU; the runs do.
"""
import os
import subprocess

import numpy as np
import pytest

import cove_b200 as cb

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
BIN = os.path.join(ROOT, "cove-spmv_b200", "bin", "struct_gpu_csr_bitbsr_spmv")

KAT_4X8 = ("%%MatrixMarket matrix coordinate real general\n4 8 5\n"
           "1 1 1.0\n1 8 2.0\n2 4 3.0\n3 2 4.0\n4 7 5.0\n")


def run(*args):
    p = subprocess.run([BIN, *map(str, args)], capture_output=True, text=True, timeout=300)
    return p.returncode, p.stdout, p.stderr


def parse_kv(out):  # run_joint_sweep.py / parse_key_values
    d = {}
    for line in out.splitlines():
        if ": " in line:
            k, v = line.split(": ", 1)
            d[k.strip()] = v.strip()
    return d


@pytest.fixture
def kat(tmp_path):
    p = tmp_path / "kat.mtx"
    p.write_text(KAT_4X8)
    return p


def write_mtx(path, rows, cols, rp, ci, v):
    lines = [f"%%MatrixMarket matrix coordinate real general\n{rows} {cols} {len(v)}\n"]
    for r in range(rows):
        for p in range(rp[r], rp[r + 1]):
            lines.append(f"{r + 1} {ci[p] + 1} {v[p]:.17g}\n")
    path.write_text("".join(lines))


def test_cli_rejects_bad_options(kat):
    rc, _, err = run(kat, "--residual-threshold", "-1", "--warmup", "0", "--iters", "1")
    assert rc != 0 and "residual-threshold must be non-negative" in err
    rc, _, err = run(kat, "--bogus")
    assert rc != 0 and "unknown or incomplete argument: --bogus" in err
    rc, _, err = run(kat, "--mode", "two_pass")
    assert rc != 0 and "fused_lb only" in err
    rc, _, err = run(kat, "--iters", "0")
    assert rc != 0 and "iterations must be positive" in err
    rc, _, _ = run("--help")
    assert rc == 0


@pytest.mark.gpu
def test_cli_reference_kat_hybrid(kat):
    rc, out, err = run(kat, "--residual-threshold", "2", "--warmup", "0", "--iters", "1", "--verify-cpu")
    assert rc == 0, err
    lines = out.splitlines()
    for want in ("spmv_effective_layout: csr_bitbsr_fused_lb", "block: 8 x 4", "residual_threshold: 2",
                 "split_policy: cost_gated", "kept_blocks: 1", "residual_blocks: 1"):
        assert want in lines, want
    assert any(ln.startswith("verify_cpu: PASS,") for ln in lines)


@pytest.mark.gpu
def test_cli_reference_kat_cost_gated(kat):
    rc, out, err = run(kat, "--split-policy", "cost_gated", "--residual-threshold", "3",
                       "--cost-bitmap-block", "2", "--cost-csr-nnz", "1", "--warmup", "0", "--iters", "1",
                       "--verify-cpu")
    assert rc == 0, err
    d = parse_kv(out)
    assert (d["split_policy"], d["kept_blocks"], d["residual_blocks"], d["cost_skipped_blocks"]) == (
        "cost_gated", "2", "0", "2")
    assert d["verify_cpu"].startswith("PASS,")


@pytest.mark.gpu
@pytest.mark.parametrize("codec,route", [("auto", "dict_u8_lossless"), ("dict", "dict_u8_lossless"),
                                         ("bfp8", "bfp8_blocks+bf16_residual")])
def test_cli_joint_keys_lapl2d(tmp_path, codec, route):
    rows, cols, rp, ci, v = cb.synth_lapl2d(64, 48)
    m = tmp_path / "l.mtx"
    write_mtx(m, rows, cols, rp, ci, v)
    rc, out, err = run(m, "--mode", "fused_lb", "--long-row-split", "256", "--value-codec", codec,
                       "--warmup", "1", "--iters", "3", "--verify-cpu")
    assert rc == 0, err
    d = parse_kv(out)
    assert d["nnz"] == str(len(v)) and d["joint_value_codec"] == route
    assert d["joint_requested_codec"] == codec
    assert float(d["joint_min_ms"]) > 0 and float(d["joint_hybrid_fp64_min_ms"]) > 0
    rel = float(d["joint_rel_err"])
    assert 0 <= rel <= (1e-12 if route.startswith("dict") else 1e-2)
    assert d["joint_verify_pass_1e-2"] == "1"
    if codec != "bfp8":
        assert d["joint_value_cardinality"] == "2" and float(d["joint_bytes_per_nnz"]) > 0


@pytest.mark.gpu
def test_cli_bfp8_gate_report_fem_and_float(tmp_path):
    rows, cols, rp, ci, v = cb.synth_fem27(8, 8, 6, 3, seed=1)
    m = tmp_path / "f.mtx"
    write_mtx(m, rows, cols, rp, ci, v)
    rc, out, err = run(m, "--value-codec", "bfp8", "--warmup", "0", "--iters", "2", "--verify-cpu")
    assert rc == 0, err
    d = parse_kv(out)
    rel = float(d["joint_rel_err"])
    assert rel > 0 and d["joint_verify_pass_1e-2"] == ("1" if rel <= 1e-2 else "0")
    # the same matrix in fp32: lossless hybrid verified in float
    rc, out, err = run(m, "--precision", "float", "--warmup", "0", "--iters", "2", "--verify-cpu")
    assert rc == 0, err
    d = parse_kv(out)
    assert d["precision"] == "float" and d["verify_cpu"].startswith("PASS,")
    assert d["value_codec_effective"] == "raw_float"
