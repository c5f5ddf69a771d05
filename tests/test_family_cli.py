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


# ---- the reference CLI test's cases (structural/tests/test_gpu_spmv_cli.sh:17-553) ----
#
# Its five tiny matrices: a 4 x 8 general matrix with five distinct values
# (and the same pattern as a pattern file), and 8 x 4 dense matrices of
# +-1, 2.5, +-2.5 and three distinct values, 1-based (r + c) deciding the
# value.

def _dense84(value):
    return [(r, c, value(r, c)) for r in range(1, 9) for c in range(1, 5)]


REF_MATRICES = {
    "plain": [(1, 1, 1.0), (1, 8, 2.0), (2, 4, 3.0), (3, 2, 4.0), (4, 7, 5.0)],
    "sign": _dense84(lambda r, c: 1.0 if (r + c) % 2 == 0 else -1.0),
    "const": _dense84(lambda r, c: 2.5),
    "sign_scale": _dense84(lambda r, c: 2.5 if (r + c) % 2 == 0 else -2.5),
    "unique": _dense84(lambda r, c: {0: 2.0, 1: -3.0, 2: 5.0}[(r + c) % 3]),
}


@pytest.fixture(scope="module")
def ref_mats(tmp_path_factory):
    d = tmp_path_factory.mktemp("refcli")
    out = {}
    for name, entries in REF_MATRICES.items():
        shape = "4 8" if name == "plain" else "8 4"
        body = "".join(f"{r} {c} {v:.1f}\n" for r, c, v in entries)
        p = d / f"{name}.mtx"
        p.write_text(f"%%MatrixMarket matrix coordinate real general\n{shape} {len(entries)}\n{body}")
        out[name] = p
    p = d / "pattern.mtx"
    p.write_text("%%MatrixMarket matrix coordinate pattern general\n4 8 5\n"
                 + "".join(f"{r} {c}\n" for r, c, _ in REF_MATRICES["plain"]))
    out["pattern"] = p
    return out


def _op(codec, lb, kind, promotion="buildable_needs_report"):
    """The operator contract keys of a BitBSR run (spmv_operator_plan.hpp)."""
    family = {"original": "load_balanced_traversal" if lb else "non_load_balanced_traversal",
              "lossless": "lossless_value_specialized", "lossy": "controlled_lossy_value_specialized"}[kind]
    if kind == "original" and lb:
        promotion = "promoted"
    return {"operator_name": f"{codec}_{'lb' if lb else 'nolb'}", "operator_family": family,
            "operator_promotion_status": promotion,
            "operator_runner": "bitbsr_original_traversal" if kind == "original" else "bitbsr_value_specialized",
            "spmv_effective_layout": "col_bitmap64_flag_lb" if lb else "col_bitmap64",
            "verify_gate": "spmv_max_rel" if kind == "lossy" else "exact_abs_or_rel",
            "timing_scope": "event_excludes_output_init"}


def _payload(exact, codebook, payload, per_nnz):
    return {"value_codec_exact": exact, "value_codec_codebook_size": str(codebook),
            "value_codec_payload_bytes": str(payload), "value_codec_bytes_per_nnz": per_nnz}


def _auto(effective, unique, candidate):
    return {"value_codec": "auto_lossless", "value_codec_effective": effective, "value_codec_auto_selected": "true",
            "value_codec_auto_unique_count": str(unique),
            "value_codec_auto_candidate_payload_bytes": str(candidate)}


LAYOUTS = {True: "col_bitmap64_flag_lb", False: "col_bitmap64"}
REF_CASES = []  # (id, matrix, extra args, expected keys)
for lb in (False, True):
    REF_CASES.append((f"original_{lb}", "plain", ["--layout", LAYOUTS[lb]],
                      {**_op("original", lb, "original"), "value_codec": "original",
                       **_payload("true", 0, 40, "8")}))
    REF_CASES.append((f"k256_{lb}", "plain", ["--layout", LAYOUTS[lb], "--value-codec", "codebook256_u8"],
                      {**_op("codebook256_u8", lb, "lossy"), "value_codec": "codebook256_u8"}))
    for codec, book in (("fp16", 0), ("bf16", 0), ("global_logkmeans16", 2), ("global_logkmeans32", 2),
                        ("global_logkmeans64", 2), ("global_logkmeans128", 2)):
        REF_CASES.append((f"{codec}_{lb}", "sign", ["--layout", LAYOUTS[lb], "--value-codec", codec],
                          {**_op(codec, lb, "lossy"), "value_codec": codec, "value_codec_exact": "false",
                           "value_codec_codebook_size": str(book)}))
    for mat, codec, pay in (("pattern", "all_one", ("true", 0, 0, "0")), ("const", "const_c", ("true", 1, 8, "0.25")),
                            ("sign", "sign2", ("true", 0, 4, "0.125")),
                            ("sign_scale", "sign2_scale", ("true", 1, 12, "0.375")),
                            ("sign", "dict2", ("true", 2, 20, "0.625")), ("unique", "dict16", ("true", 3, 40, "1.25")),
                            ("unique", "dict4", ("true", 3, 32, "1")), ("unique", "dict256_u8", ("true", 3, 56, "1.75")),
                            ("unique", "dict65536_u16", ("true", 3, 88, "2.75"))):
        REF_CASES.append((f"{codec}_{lb}", mat, ["--layout", LAYOUTS[lb], "--value-codec", codec],
                          {**_op(codec, lb, "lossless"), "value_codec": codec, **_payload(*pay)}))
REF_CASES += [
    ("all_one_binary", "pattern",
     ["--layout", "col_bitmap64_flag_lb", "--value-codec", "all_one", "--lb-policy", "binary_implicit_one"],
     {**_op("all_one", True, "lossless", "promoted"), "load_balance_policy": "binary_implicit_one",
      "load_balance_chunk_blocks": "8", "load_balance_split_threshold_blocks": "8"}),
    ("all_one_binary_manual_chunk", "pattern",
     ["--layout", "col_bitmap64_flag_lb", "--value-codec", "all_one", "--lb-policy", "binary_implicit_one",
      "--lb-chunk-blocks", "64"],
     {**_op("all_one", True, "lossless"), "load_balance_policy": "manual", "load_balance_chunk_blocks": "64",
      "load_balance_split_threshold_blocks": "64"}),
    ("auto_pattern", "pattern", [], {**_op("all_one", True, "lossless"), **_auto("all_one", 1, 0)}),
    ("auto_const", "const", [], {**_op("const_c", True, "lossless"), **_auto("const_c", 1, 8)}),
    ("auto_sign", "sign", [], {**_op("sign2", True, "lossless"), **_auto("sign2", 2, 4)}),
    ("auto_sign_scale", "sign_scale", [], {**_op("sign2_scale", True, "lossless"), **_auto("sign2_scale", 2, 12)}),
    ("auto_unique", "unique", [],
     {**_op("dict4", True, "lossless"), **_auto("dict4", 3, 32), "value_codec_codebook_size": "3"}),
    ("auto_raw", "plain", [], {**_op("original", True, "original"), **_auto("original", 5, 40)}),
    ("cusparse", "plain", ["--layout", "cusparse_csr"],
     {"operator_name": "cusparse_csr", "operator_family": "external_baseline",
      "operator_promotion_status": "external_baseline", "operator_runner": "cusparse_csr",
      "spmv_effective_layout": "cusparse_csr", "value_codec": "original", **_payload("true", 0, 40, "8"),
      "verify_gate": "exact_abs_or_rel", "timing_scope": "cusparse_event_includes_beta_zero"}),
]
for i, (cid, mat, args, exp) in enumerate(REF_CASES):
    if cid.startswith("auto_"):
        REF_CASES[i] = (cid, mat, ["--layout", "col_bitmap64_flag_lb", "--value-codec", "auto_lossless"], exp)


@pytest.mark.gpu
@pytest.mark.parametrize("case", REF_CASES, ids=[c[0] for c in REF_CASES])
def test_family_cli_reference_cases(ref_mats, case):
    cid, mat, args, expected = case
    rc, out, err = run(ref_mats[mat], *args, "--warmup", "0", "--iters", "1", "--verify-cpu")
    assert rc == 0, err
    d = parse(out)
    assert d["report_schema"] == "structural_spmv_cli_v3" and d["verify_cpu"].startswith("PASS,")
    got = {k: d.get(k) for k in expected}
    assert got == expected
    if cid.startswith("auto_"):
        assert "timing.value_codec_auto_select_event" in d


def test_family_cli_rejects_before_loading(tmp_path):
    """Layout and load-balance-policy errors come before the matrix is read."""
    missing = tmp_path / "missing.mtx"
    for layout in ("block_meta", "col_delta_u16_raw_lb", "soa", "delta_u16", "delta_packed", "delta_packed_lb",
                   "delta_packed_lb_auto", "col_bitmap64_lb", "col_hybrid64", "col_hybrid64_flag_lb", "auto"):
        rc, _, err = run(missing, "--layout", layout, "--warmup", "0", "--iters", "1")
        assert rc != 0 and "layout must be col_bitmap64, col_bitmap64_flag_lb, or cusparse_csr" in err, layout
    for layout in ("col_bitmap64", "col_bitmap64_flag_lb"):
        rc, _, err = run(missing, "--layout", layout, "--value-codec", "original", "--lb-policy",
                         "binary_implicit_one", "--warmup", "0", "--iters", "1")
        assert rc != 0 and "binary_implicit_one requires col_bitmap64_flag_lb layout and all_one" in err


FLOAT_CASES = [
    ("original", "plain", ["--value-codec", "original"], {"operator_name": "original_lb",
                                                          **_payload("true", 0, 20, "4")}),
    ("dict2", "sign", ["--value-codec", "dict2"], {"operator_name": "dict2_lb", **_payload("true", 2, 12, "0.375")}),
    ("auto_unique", "unique", ["--value-codec", "auto_lossless"], {"value_codec_effective": "dict4"}),
    ("bf16", "sign", ["--value-codec", "bf16"], {"operator_name": "bf16_lb", "verify_gate": "spmv_max_rel"}),
    ("cusparse", "plain", ["--layout", "cusparse_csr"], {"operator_name": "cusparse_csr",
                                                         **_payload("true", 0, 20, "4")}),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", FLOAT_CASES, ids=[c[0] for c in FLOAT_CASES])
def test_family_cli_float_precision(ref_mats, case):
    """--precision float: 4-byte values and codebooks, the fp32 gates."""
    _, mat, args, expected = case
    rc, out, err = run(ref_mats[mat], "--precision", "float", *args, "--warmup", "0", "--iters", "1", "--verify-cpu")
    assert rc == 0, err
    d = parse(out)
    assert d["precision"] == "float" and d["verify_cpu"].startswith("PASS,")
    assert {k: d.get(k) for k in expected} == expected
