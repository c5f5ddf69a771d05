"""Both CLIs answer argument lists exactly as the reference's own CLIs do
when the matrix does not exist -- exit status and stderr, usage text and
every option check made before the matrix is read
(tests/golden/cli_errors.json, from tests/golden/make_cli_errors_golden.py,
which ran the reference's main_gpu_spmv.cu and main_gpu_csr_bitbsr_spmv.cu
built from its own sources).  No GPU is touched on these paths."""
import json
import os
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
MATRIX = "/nonexistent/cove_cli_case.mtx"


def test_cli_errors_match_reference():
    with open(os.path.join(ROOT, "tests", "golden", "cli_errors.json")) as f:
        golden = json.load(f)
    bad, n = [], 0
    for cli, rows in golden.items():
        exe = os.path.join(ROOT, "cove-spmv_b200", "bin", cli)
        for r in rows:
            p = subprocess.run([exe] + [MATRIX if a == "M" else a for a in r["args"]], capture_output=True,
                               text=True, timeout=60)
            got = (p.returncode, p.stderr.replace(exe, "PROG").replace(MATRIX, "MATRIX"))
            n += 1
            if got != (r["rc"], r["stderr"]):
                bad.append((cli, r["args"], got, (r["rc"], r["stderr"])))
    assert n == 48 and not bad, bad[:3]
