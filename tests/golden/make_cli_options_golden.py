"""Writes tests/golden/cli_options_inputs.txt and tests/golden/cli_options.txt:
the reference's answers for the family CLI's option handling.

The spellings are every string literal of the reference's
structural/include/structural/spmv_cli_options.hpp (read as text), each tried
as a layout, codec, policy and algorithm, plus a few that must fail; the
argument lists cover each option, alias and check.  The answers come from
oracle/_ref/ref_cli_options (tests/cpp/cli_options_table.cu built against
the reference's headers by oracle/Makefile).
Usage: make -C oracle && [REF_ROOT=<reference checkout>] python tests/golden/make_cli_options_golden.py
"""
import os
import re
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
REF_ROOT = os.environ.get("REF_ROOT", "/root/reference")  # the reference checkout, as oracle/Makefile
REF_HEADER = os.path.join(REF_ROOT, "structural/include/structural/spmv_cli_options.hpp")

ARGS = [
    "m.mtx",
    "m.mtx --precision float --layout col_bitmap --value-codec raw",
    "m.mtx --precision half",
    "m.mtx --layout cusparse_alg2",
    "m.mtx --layout cusparse_csr_alg1 --cusparse-alg alg2",
    "m.mtx --cusparse-alg alg2 --layout cusparse",
    "m.mtx --value-codec k256 --lb-policy binary",
    "m.mtx --lb-chunk-blocks 64",
    "m.mtx --chunk-blocks 16 --split-threshold-blocks 48",
    "m.mtx --lb-split-threshold 7",
    "m.mtx --lb-chunk-blocks 0",
    "m.mtx --lb-chunk-blocks -3",
    "m.mtx --lb-split-threshold-blocks 0",
    "m.mtx --warmup -1",
    "m.mtx --iters 0",
    "m.mtx --iterations 3 --warmup 0 --verify-cpu",
    "m.mtx --iters abc",
    "m.mtx --layout",
    "m.mtx --bogus",
    "m.mtx extra",
    "m.mtx --lb-policy fast",
    "m.mtx --cusparse-alg alg3",
    "m.mtx --value-codec zip",
    "m.mtx --layout sell",
]


def inputs():
    with open(REF_HEADER) as f:
        words = sorted(set(re.findall(r'"([A-Za-z0-9_]+)"', f.read())))
    words += ["", "none", "Original", "col_bitmap64_lb", "auto"]
    lines = []
    for kind in ("layout", "codec", "policy", "alg"):
        lines += [f"N {kind} {w}" if w else f"N {kind}" for w in words]
    for kind in ("layout", "codec", "policy"):
        lines += [f"K {kind} {w}" for w in words if w]
    lines += [f"P {a}" for a in ARGS]
    return lines


def main():
    lines = inputs()
    text = "\n".join(lines) + "\n"
    out = subprocess.run([os.path.join(ROOT, "oracle", "_ref", "ref_cli_options")], input=text,
                         capture_output=True, text=True, check=True, timeout=60).stdout
    with open(os.path.join(ROOT, "tests", "golden", "cli_options_inputs.txt"), "w") as f:
        f.write(text)
    with open(os.path.join(ROOT, "tests", "golden", "cli_options.txt"), "w") as f:
        f.write(out)
    print(f"wrote {len(lines)} cases")


if __name__ == "__main__":
    main()
