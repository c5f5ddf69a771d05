"""struct_gpu_spmv: the reference family runner's CLI (options, operator
contract, key: value report) over the BitBSR-only codecs and the cuSPARSE
CSR baseline.  The operator names, families, runners and verify gates are
the reference's (structural/include/structural/spmv_operator_plan.hpp), and
the report is read the way structural/scripts/run_gpu_spmv_family_sweep.py
reads it.  Option handling needs no GPU; the runs do."""
import os
import subprocess

import numpy as np
import pytest

import cove_b200 as cb

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
BIN = os.path.join(ROOT, "cove-spmv_b200", "bin", "struct_gpu_spmv")


def run(*args):
    p = subprocess.run([BIN, *map(str, args)], capture_output=True, text=True, timeout=300)
    return p.returncode, p.stdout, p.stderr


def parse(out):
    """key: value lines, the timing_ms line split into timing.<name> (the
    sweep script's parse_key_values)."""
    d = {}
    for line in out.splitlines():
        if ": " not in line:
            continue
        k, v = line.split(": ", 1)
        k, v = k.strip(), v.strip()
        if k == "timing_ms":
            for part in v.split(", "):
                name, val = part.split("=", 1)
                d["timing." + name] = val
        else:
            d[k] = v
    return d


def write_mtx(path, rows, cols, rp, ci, v):
    lines = [f"%%MatrixMarket matrix coordinate real general\n{rows} {cols} {len(v)}\n"]
    for r in range(rows):
        for p in range(rp[r], rp[r + 1]):
            lines.append(f"{r + 1} {ci[p] + 1} {v[p]:.17g}\n")
    path.write_text("".join(lines))
    return path


@pytest.fixture(scope="module")
def mats(tmp_path_factory):
    d = tmp_path_factory.mktemp("family")
    lap = write_mtx(d / "lap.mtx", *cb.synth_lapl2d(32, 24))
    rows, cols, rp, ci, v = cb.synth_lapl2d(40, 40)
    ones = write_mtx(d / "ones.mtx", rows, cols, rp, ci, np.ones_like(v))
    fem = write_mtx(d / "fem.mtx", *cb.synth_fem27(6, 5, 4, 3, seed=2))
    # nearly distinct values in [1, 2): every lossy codec but BFP4 stays inside
    # the 1e-2 gate, and the top 0.5% lie strictly above the outlier quantile
    rows, cols, rp, ci, v = cb.synth_lapl2d(48, 40)
    r = np.repeat(np.arange(rows), np.diff(rp))
    smooth = write_mtx(d / "smooth.mtx", rows, cols, rp, ci, 1.0 + ((r * 7919 + ci * 104729) % 9973) / 9973.0)
    return {"lap": lap, "ones": ones, "fem": fem, "smooth": smooth}


def test_family_cli_rejects_bad_options(tmp_path):
    m = write_mtx(tmp_path / "a.mtx", *cb.synth_lapl2d(4, 4))
    rc, _, err = run(m, "--layout", "sell")
    assert rc != 0 and "layout must be col_bitmap64, col_bitmap64_flag_lb, or cusparse_csr" in err
    rc, _, err = run(m, "--value-codec", "zip")
    assert rc != 0 and "value-codec must be original" in err
    rc, _, err = run(m, "--iters", "0")
    assert rc != 0 and "iterations must be positive" in err
    rc, _, err = run(m, "--lb-policy", "fast")
    assert rc != 0 and "lb-policy must be manual or binary_implicit_one" in err
    rc, _, err = run(m, "--cusparse-alg", "alg9")
    assert rc != 0 and "cusparse-alg must be default, csr_alg1, or csr_alg2" in err
    rc, _, err = run(m, "--bogus")
    assert rc != 0 and "unknown or incomplete argument: --bogus" in err
    rc, _, _ = run(m, "--help")
    assert rc == 0


CASES = [
    # matrix, layout, codec, operator_name, family, runner, gate, effective codec
    ("lap", "col_bitmap64_flag_lb", "original", "original_lb", "load_balanced_traversal",
     "bitbsr_original_traversal", "exact_abs_or_rel", "original"),
    ("lap", "col_bitmap64", "raw", "original_nolb", "non_load_balanced_traversal",
     "bitbsr_original_traversal", "exact_abs_or_rel", "original"),
    ("lap", "col_bitmap64_flag_lb", "auto_lossless", "dict2_lb", "lossless_value_specialized",
     "bitbsr_value_specialized", "exact_abs_or_rel", "dict2"),
    ("lap", "col_bitmap64", "dict16", "dict16_nolb", "lossless_value_specialized",
     "bitbsr_value_specialized", "exact_abs_or_rel", "dict16"),
    ("ones", "col_bitmap64_flag_lb", "all_one", "all_one_lb", "lossless_value_specialized",
     "bitbsr_value_specialized", "exact_abs_or_rel", "all_one"),
    ("smooth", "col_bitmap64_flag_lb", "bfp8_outlier", "bfp8_outlier_lb", "controlled_lossy_value_specialized",
     "bitbsr_value_specialized", "spmv_max_rel", "bfp8_outlier"),
    ("smooth", "col_bitmap64_flag_lb", "k256", "codebook256_u8_lb", "controlled_lossy_value_specialized",
     "bitbsr_value_specialized", "spmv_max_rel", "codebook256_u8"),
    ("smooth", "col_bitmap64", "global_logkmeans64", "global_logkmeans64_nolb", "controlled_lossy_value_specialized",
     "bitbsr_value_specialized", "spmv_max_rel", "global_logkmeans64"),
    ("smooth", "col_bitmap64_flag_lb", "bf16", "bf16_lb", "controlled_lossy_value_specialized",
     "bitbsr_value_specialized", "spmv_max_rel", "bf16"),
    ("smooth", "col_bitmap64_flag_lb", "bfp4", "bfp4_lb", "controlled_lossy_value_specialized",
     "bitbsr_value_specialized", "spmv_max_rel", "bfp4"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c[3] for c in CASES])
def test_family_cli_operators(mats, case):
    mat, layout, codec, name, family, runner, gate, effective = case
    rc, out, err = run(mats[mat], "--layout", layout, "--value-codec", codec, "--warmup", "1", "--iters", "3",
                       "--verify-cpu")
    d = parse(out)
    if effective == "bfp4":  # 15 levels a block: the gate decides, and the exit status follows it
        rel = float(d["spmv_output_rel_err"])
        assert (rc == 0) == (rel <= 1e-2) and d["verify_cpu"].startswith("PASS," if rel <= 1e-2 else "FAIL,")
        return
    assert rc == 0, err
    assert d["report_schema"] == "structural_spmv_cli_v3" and d["block"] == "8 x 4"
    assert (d["operator_name"], d["operator_family"], d["operator_runner"], d["verify_gate"]) == (
        name, family, runner, gate)
    assert d["value_codec_effective"] == effective and d["spmv_effective_layout"] == layout
    assert d["verify_cpu"].startswith("PASS,")
    assert float(d["spmv_output_rel_err"]) <= (1e-2 if gate == "spmv_max_rel" else 1e-12)
    assert float(d["timing.gpu_spmv_avg_event"]) > 0 and float(d["timing.gpu_spmv_min_event"]) > 0
    lb = layout.endswith("_lb")
    assert (int(d["gpu_work_items"]) > 0) == lb and int(d["gpu_num_blocks"]) > 0
    if effective != "original":
        assert int(d["value_codec_payload_bytes"]) < int(d["nnz"]) * 8 or effective == "bfp8_outlier"
    if codec == "auto_lossless":
        assert d["value_codec_auto_selected"] == "true" and d["value_codec_auto_unique_count"] == "2"
        assert int(d["value_codec_auto_candidate_payload_bytes"]) < int(d["value_codec_auto_raw_payload_bytes"])
    if effective == "bfp8_outlier":
        assert int(d["value_codec_num_outliers"]) > 0


@pytest.mark.gpu
def test_family_cli_binary_policy_and_cusparse_baseline(mats):
    rc, out, err = run(mats["ones"], "--value-codec", "all_one", "--lb-policy", "binary", "--iters", "2",
                       "--verify-cpu")
    assert rc == 0, err
    d = parse(out)
    assert d["load_balance_policy"] == "binary_implicit_one" and d["operator_promotion_status"] == "promoted"
    assert d["load_balance_chunk_blocks"] == "8"  # fewer than 30,000 blocks
    rc, _, err = run(mats["lap"], "--value-codec", "dict2", "--lb-policy", "binary", "--iters", "1")
    assert rc != 0 and "binary_implicit_one requires col_bitmap64_flag_lb layout and all_one" in err
    rc, out, err = run(mats["fem"], "--layout", "cusparse_alg2", "--iters", "3", "--verify-cpu")
    assert rc == 0, err
    d = parse(out)
    assert (d["operator_name"], d["operator_family"], d["operator_runner"]) == (
        "cusparse_csr", "external_baseline", "cusparse_csr")
    assert d["block"] == "csr" and d["cusparse_alg"] == "csr_alg2" and d["verify_cpu"].startswith("PASS,")
    rc, _, err = run(mats["fem"], "--layout", "cusparse_csr", "--value-codec", "bf16")
    assert rc != 0 and "compressed value codecs are only supported for BitBSR layouts" in err
