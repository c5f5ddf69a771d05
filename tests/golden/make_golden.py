"""Generate tests/golden/ref_cases.npz from the reference's own host code.

Runs oracle/_ref/libcove_ref.so -- the reference's convert_to_bitbsr, CSR+BitBSR
split (threshold and cost-gated), storage_stats, BFP8 and BFP8+outlier
encoders, spmv_csr and make_input_vector, compiled from its headers by
oracle/Makefile -- on seeded random CSR matrices, and stores inputs and
outputs.  The CPU test suite checks the plain-C oracle against these arrays
(tests/test_oracle_golden.py) and the GPU suite checks the CUDA path against
them (tests/test_gpu_parity.py), so both stay pinned to the reference even
where the reference checkout is absent.

Usage:  python tests/golden/make_golden.py      (needs oracle/_ref built)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402


def random_csr(rng, rows, cols, density, dtype, zeros=0.0, long_rows=0, dense_band=0):
    """Sorted CSR with optional stored zeros, a few long rows and a dense band."""
    rp = [0]
    ci = []
    vals = []
    for r in range(rows):
        k = rng.binomial(cols, density)
        cs = set(rng.choice(cols, size=min(k, cols), replace=False).tolist()) if k else set()
        if long_rows and r % max(1, rows // long_rows) == 0:
            cs |= set(rng.choice(cols, size=min(cols, 40 + int(rng.integers(0, 40))), replace=False).tolist())
        if dense_band:
            lo = max(0, r - dense_band)
            hi = min(cols, r + dense_band + 1)
            cs |= set(range(lo, hi))
        cs = sorted(cs)
        v = rng.standard_normal(len(cs)).astype(dtype)
        v[v == 0] = 1
        if zeros > 0 and len(cs):
            z = rng.random(len(cs)) < zeros
            v[z] = 0
        ci.extend(cs)
        vals.extend(v.tolist())
        rp.append(len(ci))
    return (np.array(rp, np.int64), np.array(ci, np.int32), np.array(vals, dtype))


CASES = [
    # name, rows, cols, density, dtype, zeros, long_rows, dense_band
    ("sparse_f64", 203, 157, 0.03, np.float64, 0.0, 0, 0),
    ("band_f64", 300, 300, 0.01, np.float64, 0.0, 0, 3),
    ("zeros_f64", 97, 130, 0.08, np.float64, 0.2, 0, 0),
    ("longrows_f64", 260, 900, 0.005, np.float64, 0.0, 6, 1),
    ("empty_rows_f64", 129, 64, 0.004, np.float64, 0.0, 0, 0),
    ("band_f32", 211, 211, 0.02, np.float32, 0.0, 0, 2),
    ("sparse_f32", 64, 301, 0.06, np.float32, 0.1, 2, 0),
]

SPLITS = [
    # key, threshold, use_cost, cost
    ("cost32", 32, True, (10.0, 0.0, 0.0, 1.0)),
    ("thr2", 2, False, (10.0, 0.0, 0.0, 1.0)),
    ("cost_b2", 3, True, (2.0, 0.0, 0.0, 1.0)),
]


def main():
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libcove_ref.so is not built (make -C oracle)")
    rng = np.random.default_rng(20261201)
    out = {}
    for name, rows, cols, dens, dt, zeros, lr, band in CASES:
        rp, ci, v = random_csr(rng, rows, cols, dens, dt, zeros, lr, band)
        p = f"{name}/"
        out[p + "shape"] = np.array([rows, cols], np.int64)
        out[p + "row_ptr"] = rp
        out[p + "col_idx"] = ci
        out[p + "values"] = v
        for key, thr, use_cost, cost in SPLITS:
            R = O.RefSplit(rows, cols, rp, ci, v, 8, 4, thr, use_cost, cost)
            q = f"{p}{key}/"
            if key == "cost32":
                fb = R.bitbsr(0)
                for k, a in zip(["block_row_ptr", "block_col_idx", "bitmap", "block_val_ptr", "values"], fb):
                    out[p + "full/" + k] = a
            kb = R.bitbsr(1)
            for k, a in zip(["block_row_ptr", "block_col_idx", "bitmap", "block_val_ptr", "values"], kb):
                out[q + "kept/" + k] = a
            rr = R.residual()
            for k, a in zip(["row_ptr", "col_idx", "values"], rr):
                out[q + "res/" + k] = a
            c = R.counters()
            out[q + "counters"] = np.array([c[k] for k in sorted(c)], np.int64)
            out[q + "counter_names"] = np.array(sorted(c))
            if key == "cost32":
                q8, sc, *_ = R.bfp8(1, -1.0)
                out[q + "bfp8/q"] = q8
                out[q + "bfp8/scale"] = sc
                qo, so, orow, ocol, oval = R.bfp8(1, 0.005)
                out[q + "bfp8o/q"] = qo
                out[q + "bfp8o/scale"] = so
                out[q + "bfp8o/rows"] = orow
                out[q + "bfp8o/cols"] = ocol
                out[q + "bfp8o/vals"] = oval
                qo, so, orow, ocol, oval = R.bfp8(1, 0.05)
                out[q + "bfp8o5/q"] = qo
                out[q + "bfp8o5/rows"] = orow
                out[q + "bfp8o5/vals"] = oval
        x = O.ref_canonical_x(cols, dt)
        y, _ = O.ref_spmv_csr(rows, cols, rp, ci, v, x)
        out[p + "canonical_x"] = x
        out[p + "y_canonical"] = y
    path = os.path.join(HERE, "ref_cases.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    main()
