"""Writes tests/golden/cli_errors.json: how the reference's own CLIs answer
argument lists whose matrix does not exist -- exit status and stderr (the
program name replaced by PROG, the matrix path by MATRIX).  Everything they
check before reading the matrix shows up here; none of it needs a GPU.

Runs oracle/_ref/ref_struct_gpu_spmv and oracle/_ref/ref_struct_gpu_csr_bitbsr_spmv
(the reference's main_gpu_spmv.cu and main_gpu_csr_bitbsr_spmv.cu built
from its own sources and headers by oracle/Makefile).
Usage: make -C oracle && python tests/golden/make_cli_errors_golden.py
"""
import json
import os
import subprocess

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
MATRIX = "/nonexistent/cove_cli_case.mtx"

FAMILY = [
    [], ["M"], ["M", "--layout", "sell"], ["M", "--value-codec", "zip"],
    ["M", "--layout", "col_bitmap64", "--lb-policy", "binary"], ["M", "--value-codec", "all_one", "--lb-policy", "binary"],
    ["M", "--layout", "cusparse_csr", "--value-codec", "bf16"], ["M", "--layout", "cusparse_csr", "--value-codec", "auto_lossless"],
    ["M", "--layout", "cusparse_alg2", "--value-codec", "original"], ["M", "--precision", "half"], ["M", "--iters", "0"],
    ["M", "--warmup", "-1"], ["M", "--lb-chunk-blocks", "0"], ["M", "--value-codec", "auto_lossless", "--lb-policy", "binary"],
    ["M", "--layout", "col_bitmap64", "--value-codec", "k256"], ["M", "--bogus"], ["M", "--cusparse-alg", "alg9"],
    ["M", "--lb-policy", "binary", "--lb-chunk-blocks", "16", "--layout", "col_bitmap64"],
    ["M", "--precision", "float", "--value-codec", "bfp4", "--verify-cpu"], ["M", "--value-codec", "bfp8_outlier"],
    ["M", "--layout"], ["M", "--iters", "x"],
]
JOINT = [
    [], ["M"], ["M", "--mode", "fused_lb", "--long-row-split", "256", "--value-codec", "bfp8"],
    ["M", "--value-codec", "bfp8_outlier"], ["M", "--value-codec", "auto"], ["M", "--value-codec", "dict"],
    ["M", "--value-codec", "zip"], ["M", "--mode", "warp"], ["M", "--split-policy", "threshold", "--residual-threshold", "2"],
    ["M", "--split-policy", "none"], ["M", "--residual-threshold", "-1"], ["M", "--long-row-split", "-5"],
    ["M", "--cost-bitmap-block", "-1"], ["M", "--lb-chunk-blocks", "0"], ["M", "--lb-split-threshold-blocks", "0"],
    ["M", "--precision", "half"], ["M", "--iters", "0"], ["M", "--bogus"], ["M", "--operator-label", "hybrid_lb"],
    ["M", "--cusparse-alg", "alg2"], ["M", "--cusparse-alg", "alg9"], ["M", "--br", "4"], ["M", "--residual-format", "csr"],
    ["M", "--mode", "two_pass"], ["M", "--residual-format", "sell"], ["M", "--residual-format", "brcoo"],
]


def answer(exe, args):
    argv = [exe] + [MATRIX if a == "M" else a for a in args]
    p = subprocess.run(argv, capture_output=True, text=True, timeout=60)
    return {"args": args, "rc": p.returncode,
            "stderr": p.stderr.replace(exe, "PROG").replace(MATRIX, "MATRIX")}


def main():
    ref = os.path.join(ROOT, "oracle", "_ref")
    out = {"struct_gpu_spmv": [answer(os.path.join(ref, "ref_struct_gpu_spmv"), a) for a in FAMILY],
           "struct_gpu_csr_bitbsr_spmv": [answer(os.path.join(ref, "ref_struct_gpu_csr_bitbsr_spmv"), a)
                                          for a in JOINT]}
    path = os.path.join(ROOT, "tests", "golden", "cli_errors.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
