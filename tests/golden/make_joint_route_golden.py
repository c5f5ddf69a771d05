"""Writes tests/golden/ref_joint_routes.json: the reference's own joint
operator's route choice and gate on the benchmark matrices.

Each matrix is written as a MatrixMarket file (values with %.17g / %.9g, so
they read back exactly) and run through the reference's CLI
oracle/_ref/ref_struct_gpu_csr_bitbsr_spmv (its main_gpu_csr_bitbsr_spmv.cu
compiled for sm_100a by oracle/Makefile) the way its sweep script drives it
(scripts/run_joint_sweep.py:75-79):

    <bin> M.mtx --mode fused_lb --long-row-split 256 --value-codec C --verify-cpu

and the report keys joint_value_codec, joint_value_cardinality,
joint_rel_err and joint_verify_pass_1e-2 (main_gpu_csr_bitbsr_spmv.cu:
1360-1376) are stored with the split counters.  The CLI needs a GPU: run
this on a B200 box, then copy the JSON into tests/golden/.

Usage: python tests/golden/make_joint_route_golden.py [out.json] [workdir]
"""
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "cove-spmv_b200")):
    sys.path.insert(0, p)

import oracle as O  # noqa: E402

BIN = os.path.join(ROOT, "oracle", "_ref", "ref_struct_gpu_csr_bitbsr_spmv")

# (case, precision, codecs): configs 1-3 at full size, config 4 at n = 2^16
CASES = [
    ("lapl2d_512", "double", ["auto", "bfp8"]),
    ("fem27_64", "double", ["auto", "bfp8_outlier"]),
    ("rmat_22", "float", ["auto", "bfp8_outlier"]),
    ("blocksparse_2e16", "double", ["auto", "bfp8_outlier"]),
]
KEYS = ("joint_value_codec", "joint_requested_codec", "joint_value_cardinality", "joint_rel_err",
        "joint_verify_pass_1e-2", "kept_blocks", "residual_nnz", "kept_nnz", "nnz", "shape")


def matrix(case):
    """(rows, cols, row_ptr, col_idx, values) of a case."""
    if case == "lapl2d_512":
        rp, ci, v = O.lapl2d(512, 512)
        return 512 * 512, 512 * 512, rp, ci, v
    if case == "fem27_64":
        rp, ci, v = O.fem27_rows(64, 64, 64, 3, 1, 0, 786432)
        return 786432, 786432, rp, ci, v
    import cove_b200 as cb  # R-MAT and block-sparse: the library's host generators

    if case == "rmat_22":
        n, _, rp, ci, v = cb.synth_rmat(22, 16, seed=2)
        return n, n, rp, ci, v
    n = 1 << 16
    rp, ci, v = cb.synth_blocksparse_rows(n, 0, n, 2e-3, 0.6, 1e-3, 3)
    return n, n, rp, ci, v


def parse(out):
    d = {}
    for ln in out.splitlines():
        if ": " in ln:
            k, v = ln.split(": ", 1)
            d[k.strip()] = v.strip()
    return d


def main():
    out_path = sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden", "ref_joint_routes.json")
    work = sys.argv[2] if len(sys.argv) > 2 else tempfile.mkdtemp(prefix="joint_routes_")
    result = {"_about": __doc__.split("\n\n")[0].replace("\n", " "),
              "_command": "--mode fused_lb --long-row-split 256 --value-codec C --verify-cpu", "cases": {}}
    for case, precision, codecs in CASES:
        t0 = time.time()
        rows, cols, rp, ci, v = matrix(case)
        if precision == "float":
            v = v.astype("float32", copy=False)
        path = os.path.join(work, case + ".mtx")
        O.write_mtx(path, rows, cols, rp, ci, v)
        entry = {"rows": rows, "cols": cols, "nnz": int(ci.size), "precision": precision, "runs": {}}
        for codec in codecs:
            cmd = [BIN, path, "--mode", "fused_lb", "--long-row-split", "256", "--value-codec", codec,
                   "--precision", precision, "--warmup", "1", "--iters", "2", "--verify-cpu"]
            p = subprocess.run(cmd, capture_output=True, text=True, timeout=1800)
            if p.returncode != 0:
                raise RuntimeError(f"{case} {codec}: rc {p.returncode}: {p.stderr[-2000:]}")
            d = parse(p.stdout)
            entry["runs"][codec] = {k: d.get(k) for k in KEYS}
        os.remove(path)
        result["cases"][case] = entry
        print(case, f"{time.time() - t0:.1f}s", json.dumps(entry["runs"]), flush=True)
    with open(out_path, "w") as f:
        json.dump(result, f, indent=1)
    print("wrote", out_path)


if __name__ == "__main__":
    main()
