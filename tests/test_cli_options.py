"""The shim's family-CLI option handling (structural/spmv_cli_options.hpp)
against the reference's: tests/cpp/cli_options_table.cu built against the
shim must answer tests/golden/cli_options_inputs.txt exactly as the same
program built against the reference's headers did
(tests/golden/cli_options.txt, from tests/golden/make_cli_options_golden.py)."""
import os
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
SRC = os.path.join(ROOT, "tests", "cpp", "cli_options_table.cu")
BIN = os.path.join(ROOT, "tests", "cpp", "_build", "cli_options_table")
DEPS = [SRC] + [os.path.join(ROOT, "cove-spmv_b200", "include", "structural", f)
                for f in ("spmv_cli_options.hpp", "load_balance_policy.hpp")]


def _build():
    if os.path.exists(BIN) and os.path.getmtime(BIN) >= max(map(os.path.getmtime, DEPS)):
        return
    os.makedirs(os.path.dirname(BIN), exist_ok=True)
    subprocess.run(["nvcc", "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I" + os.path.join(ROOT, "cove-spmv_b200", "include"), "-I" + os.path.join(ROOT, "include"),
                    "-o", BIN, SRC], check=True, capture_output=True, text=True, timeout=600)


def test_cli_options_match_reference():
    _build()
    golden = os.path.join(ROOT, "tests", "golden")
    with open(os.path.join(golden, "cli_options_inputs.txt")) as f:
        cases = f.read()
    got = subprocess.run([BIN], input=cases, capture_output=True, text=True, check=True, timeout=60).stdout
    with open(os.path.join(golden, "cli_options.txt")) as f:
        want = f.read()
    got_lines, want_lines = got.splitlines(), want.splitlines()
    assert len(got_lines) == len(want_lines) == len(cases.splitlines()) > 900
    bad = [(g, w) for g, w in zip(got_lines, want_lines) if g != w]
    assert not bad, bad[:5]
