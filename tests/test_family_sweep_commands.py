"""Every command the reference's family sweep script builds (all operators
of its catalog, fp64 and fp32; tests/golden/family_sweep_commands.json from
tests/golden/make_family_sweep_golden.py) is accepted by this build's
binaries: each run gets past option handling and stops only at the missing
matrix, so the sweep drives these binaries unchanged."""
import json
import os
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
BIN_DIR = os.path.join(ROOT, "cove-spmv_b200", "bin")


def test_sweep_commands_pass_option_handling(tmp_path):
    with open(os.path.join(ROOT, "tests", "golden", "family_sweep_commands.json")) as f:
        rows = json.load(f)
    assert len(rows) == 86
    missing = str(tmp_path / "absent.mtx")
    bad = []
    for r in rows:
        argv = [a.replace("BIN/", BIN_DIR + "/") if a.startswith("BIN/") else (missing if a == "MATRIX" else a)
                for a in r["argv"]]
        p = subprocess.run(argv, capture_output=True, text=True, timeout=60)
        if p.returncode == 0 or "cannot open MatrixMarket file" not in p.stderr:
            bad.append((r["operator"], r["precision"], p.returncode, p.stderr.strip()[-200:]))
    assert not bad, bad[:5]


def test_joint_sweep_commands_pass_option_handling(tmp_path):
    """run_joint_sweep.py:75-79 builds [bin, matrix, --mode fused_lb,
    --long-row-split 256, --value-codec C, --warmup W, --iters I, --verify-cpu]
    for its default codecs bfp8, bfp8_outlier and auto (:35)."""
    exe = os.path.join(BIN_DIR, "struct_gpu_csr_bitbsr_spmv")
    for codec in ("bfp8", "bfp8_outlier", "auto"):
        p = subprocess.run([exe, str(tmp_path / "absent.mtx"), "--mode", "fused_lb", "--long-row-split", "256",
                            "--value-codec", codec, "--warmup", "5", "--iters", "30", "--verify-cpu"],
                           capture_output=True, text=True, timeout=60)
        assert p.returncode != 0 and "cannot open MatrixMarket file" in p.stderr, (codec, p.stderr)
