"""The shim's operator contract (structural/spmv_operator_plan.hpp) and
load-balance policy table (structural/load_balance_policy.hpp) against the
reference's headers: tests/cpp/operator_plan_table.cu built against the shim
must print exactly tests/golden/operator_plan.txt, the same program's output
built against the reference (tests/golden/make_operator_plan_golden.py)."""
import os
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
SRC = os.path.join(ROOT, "tests", "cpp", "operator_plan_table.cu")
BIN = os.path.join(ROOT, "tests", "cpp", "_build", "operator_plan_table")
SHIM = os.path.join(ROOT, "cove-spmv_b200", "include", "structural")


def _build():
    deps = [SRC] + [os.path.join(SHIM, f) for f in ("spmv_operator_plan.hpp", "load_balance_policy.hpp",
                                                    os.path.join("operators", "bitbsr_spmv_8x4_dispatch.cuh"))]
    if os.path.exists(BIN) and os.path.getmtime(BIN) >= max(map(os.path.getmtime, deps)):
        return
    os.makedirs(os.path.dirname(BIN), exist_ok=True)
    subprocess.run(["nvcc", "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I" + os.path.join(ROOT, "cove-spmv_b200", "include"), "-I" + os.path.join(ROOT, "include"),
                    "-o", BIN, SRC], check=True, capture_output=True, text=True, timeout=600)


def test_operator_contract_matches_reference():
    _build()
    got = subprocess.run([BIN], capture_output=True, text=True, check=True, timeout=60).stdout.splitlines()
    with open(os.path.join(ROOT, "tests", "golden", "operator_plan.txt")) as f:
        want = f.read().splitlines()
    assert len(got) == len(want) == 481
    bad = [(g, w) for g, w in zip(got, want) if g != w]
    assert not bad, bad[:5]
