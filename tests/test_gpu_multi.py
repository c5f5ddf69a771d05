"""Row-block partition over 2+ GPUs: NCCL halo exchange and CG allreduce.

Needs at least two visible GPUs (skipped otherwise).  Each rank is its own
process with its own GPU; the NCCL id travels over a gloo process group.
Results are compared with a single-process numpy run of the same recurrence.
"""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _gpus():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q, nx, ny, nz, iters):
    sys.path.insert(0, os.path.join(ROOT, "cove-spmv_b200"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import ctypes as C
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import cove_b200 as cb

    try:
        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        plane = nx * ny
        n = plane * nz
        cuts = [round(r * nz / world) for r in range(world + 1)]
        rb, re = cuts[rank] * plane, cuts[rank + 1] * plane
        wb, we = max(0, rb - plane), min(n, re + plane)
        rows, _, rp, ci, v = cb.synth_lapl3d(nx, ny, nz, rb, re, wb)
        plan = cb.Plan(cb.DeviceCsr.from_numpy(rows, we - wb, rp, ci, v), value_codec="auto")
        L = cb.lib()
        idbuf = np.zeros(L.cove_dist_id_bytes(), np.uint8)
        if rank == 0:
            cb.check(L.cove_dist_make_id(idbuf.ctypes.data_as(C.c_void_p)))
        obj = [idbuf.tobytes()]
        dist.broadcast_object_list(obj, src=0)
        idbuf = np.frombuffer(obj[0], np.uint8).copy()
        D = C.c_void_p()
        arr = (C.c_void_p * 1)(plan.handle.value)
        cb.check(L.cove_dist_create(rank, world, idbuf.ctypes.data_as(C.c_void_p), arr, 1, n, rb, re,
                                    wb, we - wb, 60000, C.byref(D)))
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        xg = cb.synth_vector("uniform_pm1", n, seed=4)
        xw = torch.zeros(we - wb, dtype=torch.float64, device="cuda")
        xw[rb - wb: re - wb] = torch.from_numpy(xg[rb:re]).cuda()
        y = torch.empty(rows, dtype=torch.float64, device="cuda")
        cb.check(L.cove_dist_spmv(D, C.c_void_p(xw.data_ptr()), C.c_void_p(y.data_ptr()), stream))
        b = torch.from_numpy(xg[rb:re].copy()).cuda()
        x = torch.empty_like(b)
        res = cb.CgResult()
        cb.check(L.cove_dist_cg_solve(D, C.c_void_p(b.data_ptr()), C.c_void_p(x.data_ptr()), iters,
                                      C.byref(res), stream))
        torch.cuda.synchronize()
        q.put((rank, rb, re, y.cpu().numpy(), x.cpu().numpy(), res.rs_final, xw.cpu().numpy(), wb))
        cb.check(L.cove_dist_destroy(D))
        plan.close()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_rank_halo_spmv_and_cg():
    import scipy.sparse as sp
    import torch.multiprocessing as mp

    import cove_b200 as cb

    nx, ny, nz, iters, world = 24, 20, 18, 20, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, nx, ny, nz, iters)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert all(o[1] != "error" for o in out), out
    rows, n, rp, ci, v = cb.synth_lapl3d(nx, ny, nz)
    A = sp.csr_matrix((v, ci, rp), shape=(n, n))
    xg = cb.synth_vector("uniform_pm1", n, seed=4)
    yg = A @ xg
    x = np.zeros(n)
    r = xg.copy()
    p = xg.copy()
    rs = r @ r
    for _ in range(iters):
        ap = A @ p
        alpha = rs / (p @ ap)
        x += alpha * p
        r -= alpha * ap
        rs_new = r @ r
        p = r + rs_new / rs * p
        rs = rs_new
    for rank, rb, re, y, xl, rs_d, xw, wb in out:
        # the halo arrived: the window holds the neighbours' rows of x
        assert np.array_equal(xw, xg[wb: wb + xw.size])
        assert np.abs(y - yg[rb:re]).max() <= 1e-12 * np.abs(yg).max()
        assert np.abs(xl - x[rb:re]).max() <= 1e-9 * np.abs(x).max()
        assert abs(rs_d - rs) <= 1e-8 * (xg @ xg)
