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
