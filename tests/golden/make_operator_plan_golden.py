"""Writes tests/golden/operator_plan.txt: the reference's SpMV operator
contract (make_spmv_operator_spec over every layout, value codec and
load-balance policy) and its binary all-one load-balance decisions.

Runs oracle/_ref/ref_operator_plan, which oracle/Makefile builds from
tests/cpp/operator_plan_table.cu against the reference's headers.
Usage: make -C oracle && python tests/golden/make_operator_plan_golden.py
"""
import os
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))


def main():
    out = subprocess.run([os.path.join(ROOT, "oracle", "_ref", "ref_operator_plan")], capture_output=True,
                         text=True, check=True, timeout=60).stdout
    path = os.path.join(ROOT, "tests", "golden", "operator_plan.txt")
    with open(path, "w") as f:
        f.write(out)
    print(f"wrote {path}: {len(out.splitlines())} lines")


if __name__ == "__main__":
    main()
