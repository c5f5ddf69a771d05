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
