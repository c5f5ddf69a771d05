"""Mixed-precision iterative refinement and flexible CG (needs a B200).

The recurrences are the reference's run_ir / run_fcg
(structural/src/bench_cg_solve.cu:280-448): an exact (lossless) outer level
and a bounded inner CG on a cheaper route.  With a BFP8 inner route both
must reach fp64 accuracy; with the exact route inside, iterative refinement
must follow a numpy run of the same recurrence step for step.
"""
import ctypes as C

import numpy as np
import pytest

import cove_b200 as cb

pytestmark = pytest.mark.gpu


def fem_plan(nx=14, ny=12, nz=10):
    rows, cols, rp, ci, v = cb.synth_fem27(nx, ny, nz, 3, seed=1)
    p = cb.Plan(cb.DeviceCsr.from_numpy(rows, cols, rp, ci, v), value_codec="bfp8", gate_enable=0,
                keep_lossless=1)
    return p, (rows, cols, rp, ci, v)


def relres(csr, x, b):
    import scipy.sparse as sp

    rows, cols, rp, ci, v = csr
    A = sp.csr_matrix((v, ci, rp), shape=(rows, cols))
    return np.linalg.norm(b - A @ x) / np.linalg.norm(b)


def numpy_ir(csr, b, tol, k_inner, max_outer):
    import scipy.sparse as sp

    rows, cols, rp, ci, v = csr
    A = sp.csr_matrix((v, ci, rp), shape=(rows, cols))
    x = np.zeros(rows)
    r = b.copy()
    bn = np.linalg.norm(b)
    inner = 0
    outer = 0
    for outer in range(max_outer):
        if np.linalg.norm(r) / bn < tol:
            break
        d = np.zeros(rows)
        ri = r.copy()
        p = r.copy()
        rs = ri @ ri
        for _ in range(k_inner):
            ap = A @ p
            pap = p @ ap
            if not pap > 0:
                break
            a = rs / pap
            d += a * p
            ri -= a * ap
            rsn = ri @ ri
            inner += 1
            p = ri + (rsn / rs) * p
            rs = rsn
        x += d
        r = b - A @ x
    else:
        outer = max_outer
    return x, outer, inner, np.linalg.norm(r) / bn


@pytest.mark.parametrize("flexible", [False, True])
def test_mixed_precision_bfp8_inner_reaches_fp64(flexible):
    import torch

    p, csr = fem_plan()
    b = cb.synth_vector("uniform_pm1", csr[0], seed=4)
    bd = torch.from_numpy(b).cuda()
    xd = torch.full_like(bd, float("nan"))
    res = p.mp_solve(bd, xd, cb.ROUTE_BFP8, tol=1e-10, k_inner=20, max_outer=40, flexible=flexible)
    torch.cuda.synchronize()
    x = xd.cpu().numpy()
    assert res.reached == 1 and res.final_relres <= 1e-10
    assert res.outer >= 1 and res.inner_total >= res.outer
    assert relres(csr, x, b) <= 2e-10  # the reported residual is the true one
    assert res.ms_total > 0


def test_iterative_refinement_follows_numpy_with_exact_inner():
    import torch

    p, csr = fem_plan(10, 9, 8)
    b = cb.synth_vector("uniform_pm1", csr[0], seed=7)
    bd = torch.from_numpy(b).cuda()
    xd = torch.empty_like(bd)
    res = p.mp_solve(bd, xd, cb.ROUTE_HYBRID, tol=1e-11, k_inner=6, max_outer=30)
    torch.cuda.synchronize()
    x_ref, outer, inner, rr = numpy_ir(csr, b, 1e-11, 6, 30)
    assert (res.outer, res.inner_total) == (outer, inner)
    assert abs(res.final_relres - rr) <= 1e-3 * rr + 1e-15
    assert np.abs(xd.cpu().numpy() - x_ref).max() <= 1e-9 * np.abs(x_ref).max()


def test_partition_entry_point_matches_single_plan():
    """cove_dist_mp_solve on two row shards of one rank (world 1) against the
    single-plan solver on the whole matrix."""
    import torch

    nx, ny, nz = 12, 10, 8
    rows, cols, rp, ci, v = cb.synth_fem27(nx, ny, nz, 3, seed=1)
    b = cb.synth_vector("uniform_pm1", rows, seed=5)
    whole = cb.Plan(cb.DeviceCsr.from_numpy(rows, cols, rp, ci, v), value_codec="bfp8", gate_enable=0,
                    keep_lossless=1)
    bd = torch.from_numpy(b).cuda()
    x1 = torch.empty_like(bd)
    r1 = whole.mp_solve(bd, x1, cb.ROUTE_BFP8, tol=1e-10, k_inner=15, max_outer=40, flexible=True)
    # two shards at a z-plane cut (window = all columns)
    cut = (nz // 2) * nx * ny * 3
    shards = []
    for lo, hi in ((0, cut), (cut, rows)):
        srp = rp[lo:hi + 1] - rp[lo]
        shards.append(cb.Plan(cb.DeviceCsr.from_numpy(hi - lo, cols, srp, ci[rp[lo]:rp[hi]], v[rp[lo]:rp[hi]]),
                              value_codec="bfp8", gate_enable=0, keep_lossless=1))
    L = cb.lib()
    idbuf = np.zeros(L.cove_dist_id_bytes(), np.uint8)
    cb.check(L.cove_dist_make_id(idbuf.ctypes.data_as(C.c_void_p)))
    D = C.c_void_p()
    arr = (C.c_void_p * 2)(shards[0].handle.value, shards[1].handle.value)
    cb.check(L.cove_dist_create(0, 1, idbuf.ctypes.data_as(C.c_void_p), arr, 2, rows, 0, rows, 0, cols,
                                60000, C.byref(D)))
    x2 = torch.empty_like(bd)
    r2 = cb.IrResult()
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    cb.check(L.cove_dist_mp_solve(D, 1, cb.ROUTE_BFP8, C.c_void_p(bd.data_ptr()), C.c_void_p(x2.data_ptr()),
                                  1e-10, 15, 40, C.byref(r2), s))
    torch.cuda.synchronize()
    cb.check(L.cove_dist_destroy(D))
    assert r1.reached == 1 and r2.reached == 1
    assert abs(r1.outer - r2.outer) <= 1
    assert np.abs(x1.cpu().numpy() - x2.cpu().numpy()).max() <= 1e-8 * np.abs(x1.cpu().numpy()).max()


def test_solver_argument_errors():
    import torch

    p, csr = fem_plan(6, 6, 6)
    bd = torch.ones(csr[0], dtype=torch.float64, device="cuda")
    xd = torch.empty_like(bd)
    with pytest.raises(cb.CoveError, match="inner route"):
        p.mp_solve(bd, xd, cb.ROUTE_DICT_U8)
    with pytest.raises(cb.CoveError, match="tol must be positive"):
        p.mp_solve(bd, xd, cb.ROUTE_BFP8, tol=0.0)
