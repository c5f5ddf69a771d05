"""Conjugate gradient over the fused SpMV (needs a B200).

The recurrence is the reference's timed CG (structural/src/bench_cg_solve.cu:
165-197); the device solve must follow a numpy run of the same recurrence.
"""
import ctypes as C

import numpy as np
import pytest

import cove_b200 as cb

pytestmark = pytest.mark.gpu


def numpy_cg(rows, rp, ci, v, b, iters):
    import scipy.sparse as sp

    A = sp.csr_matrix((v, ci, rp), shape=(rows, rows))
    x = np.zeros(rows)
    r = b.copy()
    p = b.copy()
    rs = r @ r
    rs0 = rs
    for _ in range(iters):
        ap = A @ p
        pap = p @ ap
        alpha = rs / pap if pap != 0 else 0.0
        x += alpha * p
        r -= alpha * ap
        rs_new = r @ r
        beta = rs_new / rs if rs != 0 else 0.0
        p = r + beta * p
        rs = rs_new
    return x, rs0, rs


def test_single_plan_cg_matches_numpy():
    import torch

    rows, n, rp, ci, v = cb.synth_lapl3d(24, 20, 16)
    b = cb.synth_vector("uniform_pm1", rows, seed=4)
    p = cb.Plan(cb.DeviceCsr.from_numpy(rows, n, rp, ci, v), value_codec="auto")
    assert p.info.dispatched_route == cb.ROUTE_DICT_U8
    bd = torch.from_numpy(b).cuda()
    xd = torch.empty_like(bd)
    res = p.cg(bd, xd, 30)
    torch.cuda.synchronize()
    x_ref, rs0, rs = numpy_cg(rows, rp, ci, v, b, 30)
    assert abs(res.rs_initial - rs0) <= 1e-12 * rs0
    assert abs(res.rs_final - rs) <= 1e-8 * rs0
    assert np.abs(xd.cpu().numpy() - x_ref).max() <= 1e-9 * np.abs(x_ref).max()
    assert res.ms_total > 0 and res.ms_spmv > 0


def test_sharded_dist_cg_world1_matches_numpy():
    """Two row shards on one rank (the layout the 768^3 problem uses on one GPU)."""
    import torch

    L = cb.lib()
    nx, ny, nz = 16, 16, 24
    n = nx * ny * nz
    plane = nx * ny
    shards = [(0, 10 * plane), (10 * plane, n)]
    plans = []
    for sb, se in shards:
        rows, _, rp, ci, v = cb.synth_lapl3d(nx, ny, nz, sb, se, 0)
        plans.append(cb.Plan(cb.DeviceCsr.from_numpy(rows, n, rp, ci, v), value_codec="auto",
                             keep_lossless=0))
    idbuf = np.zeros(L.cove_dist_id_bytes(), np.uint8)
    cb.check(L.cove_dist_make_id(idbuf.ctypes.data_as(C.c_void_p)))
    D = C.c_void_p()
    arr = (C.c_void_p * 2)(*[p.handle.value for p in plans])
    cb.check(L.cove_dist_create(0, 1, idbuf.ctypes.data_as(C.c_void_p), arr, 2, n, 0, n, 0, n,
                                60000, C.byref(D)))
    try:
        b = cb.synth_vector("uniform_pm1", n, seed=4)
        bd = torch.from_numpy(b).cuda()
        xd = torch.empty_like(bd)
        res = cb.CgResult()
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        cb.check(L.cove_dist_cg_solve(D, C.c_void_p(bd.data_ptr()), C.c_void_p(xd.data_ptr()), 25,
                                      C.byref(res), stream))
        torch.cuda.synchronize()
        rows, _, rp, ci, v = cb.synth_lapl3d(nx, ny, nz)
        x_ref, rs0, rs = numpy_cg(rows, rp, ci, v, b, 25)
        assert abs(res.rs_final - rs) <= 1e-8 * rs0
        assert np.abs(xd.cpu().numpy() - x_ref).max() <= 1e-9 * np.abs(x_ref).max()
        # distributed SpMV through the same handle (no halo with one rank)
        yd = torch.empty_like(bd)
        cb.check(L.cove_dist_spmv(D, C.c_void_p(bd.data_ptr()), C.c_void_p(yd.data_ptr()), stream))
        torch.cuda.synchronize()
        import scipy.sparse as sp

        A = sp.csr_matrix((v, ci, rp), shape=(n, n))
        assert np.abs(yd.cpu().numpy() - A @ b).max() <= 1e-12 * np.abs(A @ b).max()
    finally:
        L.cove_dist_destroy(D)


def test_device_generator_matches_host_generator():
    import torch

    L = cb.lib()
    nx, ny, nz = 10, 12, 9
    sb, se, shift = 240, 960, 120
    rows = se - sb
    nnz = C.c_int64(0)
    cb.check(L.cove_synth_lapl3d_device(nx, ny, nz, sb, se, shift, None, None, None,
                                        C.byref(nnz), None))
    rp = torch.empty(rows + 1, dtype=torch.int32, device="cuda")
    ci = torch.empty(nnz.value, dtype=torch.int32, device="cuda")
    v = torch.empty(nnz.value, dtype=torch.float64, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    cb.check(L.cove_synth_lapl3d_device(nx, ny, nz, sb, se, shift, C.c_void_p(rp.data_ptr()),
                                        C.c_void_p(ci.data_ptr()), C.c_void_p(v.data_ptr()),
                                        C.byref(nnz), stream))
    torch.cuda.synchronize()
    hr, _, hrp, hci, hv = cb.synth_lapl3d(nx, ny, nz, sb, se, shift)
    assert np.array_equal(rp.cpu().numpy(), hrp)
    assert np.array_equal(ci.cpu().numpy(), hci)
    assert np.array_equal(v.cpu().numpy(), hv)
    out = torch.empty(100, dtype=torch.float64, device="cuda")
    cb.check(L.cove_synth_vector_device(0, 4, 7, 50, 100, C.c_void_p(out.data_ptr()), stream))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), cb.synth_vector("uniform_pm1", 150, seed=4)[50:])
