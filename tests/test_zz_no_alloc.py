"""cove_cg_solve_noalloc: CG with its work vectors in a fixed device array.

Checked through the C ABI against cove_cg_solve on the same plan and inputs,
on two calls in a row (the second call finds the first call's contents in
the shared array), with the tolerance the other CG tests use.  The file is
named to be collected last, and passes alone in a fresh process as well.
"""
import ctypes as C

import numpy as np
import pytest

import cove_b200 as cb

pytestmark = pytest.mark.gpu


def _solve(fn, plan, b, iters):
    import torch

    x = torch.full_like(b, float("nan"))  # every entry must be written
    res = cb.CgResult()
    st = fn(plan.handle, C.c_void_p(b.data_ptr()), C.c_void_p(x.data_ptr()), iters, C.byref(res),
            C.c_void_p(torch.cuda.current_stream().cuda_stream))
    cb.check(st)
    torch.cuda.synchronize()
    return x.cpu().numpy(), res


def test_noalloc_cg_matches_cg_solve_on_two_calls():
    import torch

    L = cb.lib()
    rows, n, rp, ci, v = cb.synth_lapl3d(40, 36, 30)  # 43200 rows, under the limit
    plan = cb.Plan(cb.DeviceCsr.from_numpy(rows, n, rp, ci, v), value_codec="auto")
    iters = 30
    bs = [torch.from_numpy(cb.synth_vector("uniform_pm1", rows, seed=s)).cuda() for s in (4, 9)]
    for b in bs:
        x_ref, r_ref = _solve(L.cove_cg_solve, plan, b, iters)
        x_na, r_na = _solve(L.cove_cg_solve_noalloc, plan, b, iters)
        assert np.isfinite(x_na).all()
        assert r_na.iterations == iters
        assert abs(r_na.rs_initial - r_ref.rs_initial) <= 1e-12 * r_ref.rs_initial
        assert abs(r_na.rs_final - r_ref.rs_final) <= 1e-8 * r_ref.rs_initial
        assert np.abs(x_na - x_ref).max() <= 1e-9 * np.abs(x_ref).max()
    plan.close()


def test_noalloc_cg_leaves_free_device_memory_unchanged():
    """The property the entry point exists for: after a first call on the
    device, a call takes no device memory (cudaMemGetInfo's free bytes are the
    same before and after it)."""
    import torch

    L = cb.lib()
    rows, n, rp, ci, v = cb.synth_lapl2d(200, 150)
    plan = cb.Plan(cb.DeviceCsr.from_numpy(rows, n, rp, ci, v), value_codec="auto")
    b = torch.from_numpy(cb.synth_vector("uniform_pm1", rows, seed=5)).cuda()
    x = torch.empty_like(b)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    res = cb.CgResult()
    args = (plan.handle, C.c_void_p(b.data_ptr()), C.c_void_p(x.data_ptr()), 20, C.byref(res), stream)
    cb.check(L.cove_cg_solve_noalloc(*args))  # first call on the device: its set-up
    torch.cuda.synchronize()
    before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        cb.check(L.cove_cg_solve_noalloc(*args))
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == before
    assert res.iterations == 20 and res.rs_final < res.rs_initial
    plan.close()


def test_noalloc_cg_with_an_empty_plan_returns_zero_residuals():
    import torch

    L = cb.lib()
    plan = cb.Plan(cb.DeviceCsr.from_numpy(0, 0, np.zeros(1, np.int64), np.zeros(0, np.int32),
                                           np.zeros(0, np.float64)), value_codec="original")
    b = torch.zeros(1, dtype=torch.float64, device="cuda")
    x = torch.zeros(1, dtype=torch.float64, device="cuda")
    for fn in (L.cove_cg_solve_noalloc, L.cove_cg_solve):
        res = cb.CgResult()
        cb.check(fn(plan.handle, C.c_void_p(b.data_ptr()), C.c_void_p(x.data_ptr()), 5, C.byref(res),
                    C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        assert res.iterations == 5 and res.rs_initial == 0.0 and res.rs_final == 0.0
    plan.close()


def test_noalloc_cg_rejects_plans_beyond_its_scratch():
    import torch

    L = cb.lib()
    side = 363  # 363^2 = 131769 rows > 131072
    rows, n, rp, ci, v = cb.synth_lapl2d(side, side)
    assert rows > 131072
    plan = cb.Plan(cb.DeviceCsr.from_numpy(rows, n, rp, ci, v), value_codec="auto")
    b = torch.ones(rows, dtype=torch.float64, device="cuda")
    x = torch.empty_like(b)
    res = cb.CgResult()
    st = L.cove_cg_solve_noalloc(plan.handle, C.c_void_p(b.data_ptr()), C.c_void_p(x.data_ptr()), 5,
                                 C.byref(res), None)
    assert st == 1
    msg = L.cove_last_error().decode()
    assert "131072" in msg and "rows" in msg
    plan.close()
