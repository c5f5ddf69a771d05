"""Writes tests/golden/cg_synth.json: hashes of the CG bench's synthetic SPD
matrices as the reference's own generators build them.

Runs oracle/_ref/ref_cg_synth (oracle/Makefile compiles it from the
reference's structural/src/bench_cg_solve.cu, so it exists only where the
reference checkout does).  Usage: python tests/golden/make_cg_synth_golden.py
"""
import json
import os
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
REF = os.path.join(ROOT, "oracle", "_ref", "ref_cg_synth")

# kind, n, half bandwidth, seed, delta (synth) or sigma (lapl)
CASES = [
    ("synth", 20000, 32, 12345, 1.0),
    ("lapl", 20000, 32, 12345, 0.01),
    ("synth", 4097, 5, 7, 0.25),
    ("lapl", 777, 3, 99, 0.1),
    ("synth", 1000, 8, 12345, 1.0),
    ("synth", 10, 32, 1, 1.0),
    ("lapl", 1, 4, 3, 0.5),
    ("synth", 64, 0, 5, 2.0),
]


def run(exe, case):
    out = subprocess.run([exe, *map(str, case)], capture_output=True, text=True, check=True, timeout=300).stdout
    return dict(line.split(" ", 1) for line in out.strip().splitlines())


def main():
    rows = [{"case": list(c), **run(REF, c)} for c in CASES]
    path = os.path.join(os.path.dirname(__file__), "cg_synth.json")
    with open(path, "w") as f:
        json.dump(rows, f, indent=1)
        f.write("\n")
    print(f"wrote {path}: {len(rows)} cases")


if __name__ == "__main__":
    main()
