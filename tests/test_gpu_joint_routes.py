"""Route choice and gate against the reference's own joint operator.

tests/golden/ref_joint_routes.json holds what the reference's CLI
(structural/src/main_gpu_csr_bitbsr_spmv.cu, compiled for sm_100a by
oracle/Makefile and run on a B200 by tests/golden/make_joint_route_golden.py)
reports for the benchmark matrices with `--mode fused_lb --long-row-split
256 --value-codec C --verify-cpu`: the codec it chose, its value
cardinality, its gate error on the canonical x and whether the gate passed
(main_gpu_csr_bitbsr_spmv.cu:1222-1246, 1360-1376).  The same matrices,
planned by this library with the same codec, must choose the same route,
take the same gate decision and, on the BFP8 routes (both fp32
accumulations), report the same gate error up to summation order.
"""
import json
import os

import numpy as np
import pytest

import cove_b200 as cb

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
GOLD = os.path.join(ROOT, "tests", "golden", "ref_joint_routes.json")


def _cases():
    with open(GOLD) as f:
        d = json.load(f)
    out = []
    for case, e in d["cases"].items():
        for codec, run in e["runs"].items():
            out.append((case, e, codec, run))
    return out


CASES = _cases() if os.path.exists(GOLD) else []


def _matrix(case):
    if case == "lapl2d_512":
        return cb.synth_lapl2d(512, 512)
    if case == "fem27_64":
        return cb.synth_fem27(64, 64, 64, 3, seed=1)
    if case == "rmat_22":
        return cb.synth_rmat(22, 16, seed=2)
    n = 1 << 16
    rp, ci, v = cb.synth_blocksparse_rows(n, 0, n, 2e-3, 0.6, 1e-3, 3)
    return n, n, rp, ci, v


_PLANS = {}


def _plan(case, codec):
    key = (case, codec)
    if key not in _PLANS:
        _PLANS.clear()
        rows, cols, rp, ci, v = _matrix(case)
        _PLANS[key] = cb.Plan(cb.DeviceCsr.from_numpy(rows, cols, rp, ci, v), value_codec=codec,
                              long_row_split=256)
    return _PLANS[key]


def test_fixture_covers_configs_1_to_4():
    assert {c[0] for c in CASES} == {"lapl2d_512", "fem27_64", "rmat_22", "blocksparse_2e16"}


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{c[2]}" for c in CASES])
def test_route_and_gate_match_reference_binary(case):
    name, entry, codec, ref = case
    info = _plan(name, codec).info
    assert int(info.nnz) == entry["nnz"] == int(ref["nnz"])
    assert int(info.kept_blocks) == int(ref["kept_blocks"])
    assert int(info.residual_nnz) == int(ref["residual_nnz"])
    assert cb.ROUTE_NAMES[info.joint_route] == ref["joint_value_codec"]
    ref_pass = ref["joint_verify_pass_1e-2"] == "1"
    ref_err = float(ref["joint_rel_err"])
    assert bool(info.gate_pass) == ref_pass, (info.joint_rel_err, ref_err)
    if ref["joint_value_codec"].startswith("bfp8"):
        # both accumulate in fp32; only the summation order differs (the
        # reference prints 6 significant digits; near 1e-7 the error is the
        # fp32 summation noise itself)
        assert abs(info.joint_rel_err - ref_err) <= 2e-3 * ref_err + 2e-6, (info.joint_rel_err, ref_err)
    else:
        # exact dictionary: this library accumulates in T (the reference in fp32)
        assert info.joint_rel_err <= max(ref_err, 1e-12)
    # the dispatched route is the joint one when the gate passes, else the
    # lossless hybrid (the reference's evaluation, plot_eval_performance.py:216-219)
    expect = info.joint_route if ref_pass else cb.ROUTE_HYBRID
    assert info.dispatched_route == expect
