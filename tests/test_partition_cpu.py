"""Row-block partition, halo plan and distributed CG on CPU ranks (gloo).

The multi-GPU path (cove_dist_*) exchanges x halos with ncclSend/ncclRecv
according to cove_dist_halo_plan and allreduces the CG dot products.  Here
the same plan drives gloo point-to-point transfers between world_size 2-3
CPU processes, with scipy standing in for the per-rank SpMV, and the result
is compared with the single-process answer.  A rank that dies before a
collective makes the others fail within the process-group timeout.
"""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def slab_blocks(nx, ny, nz, world):
    plane = nx * ny
    n = plane * nz
    cuts = [round(r * nz / world) for r in range(world + 1)]
    blocks = []
    for r in range(world):
        rb, re = cuts[r] * plane, cuts[r + 1] * plane
        wb, we = max(0, rb - plane), min(n, re + plane)
        blocks.append((rb, re, wb, we - wb))
    return blocks


def test_halo_plan_covers_windows():
    import cove_b200 as cb

    blocks = slab_blocks(5, 4, 9, 3)
    p0 = cb.halo_plan(0, blocks)
    p1 = cb.halo_plan(1, blocks)
    assert [t[0] for t in p0] == [1]
    assert sorted(t[0] for t in p1) == [0, 2]
    # rank 1 receives one plane (20 rows) from each side and sends one to each
    assert all(t[2] == 20 and t[4] == 20 for t in p1)
    bad = [(0, 40, 0, 80), (60, 100, 20, 80)]  # rows 40..60 owned by nobody
    with pytest.raises(cb.CoveError):
        cb.halo_plan(0, bad)


def test_halo_plan_for_a_window_of_all_columns():
    """A general matrix partitioned by rows (every rank's window is all of
    x): each rank receives every other rank's rows where they sit in x and
    sends its own rows to each peer."""
    import cove_b200 as cb

    n = 1000
    cuts = [0, 336, 664, n]
    blocks = [(cuts[r], cuts[r + 1], 0, n) for r in range(3)]
    for rank in range(3):
        got = sorted(cb.halo_plan(rank, blocks))
        peers = [q for q in range(3) if q != rank]
        assert [t[0] for t in got] == peers
        for peer, so, sn, ro, rn in got:
            assert (so, sn) == (cuts[rank], cuts[rank + 1] - cuts[rank])
            assert (ro, rn) == (cuts[peer], cuts[peer + 1] - cuts[peer])


def _worker(rank, world, port, nx, ny, nz, iters, out_q, mode):
    sys.path.insert(0, os.path.join(ROOT, "cove-spmv_b200"))
    import scipy.sparse as sp
    import torch
    import torch.distributed as dist

    import cove_b200 as cb

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=6))
    try:
        if mode == "die" and rank == world - 1:
            os._exit(3)  # leaves before any collective
        blocks = slab_blocks(nx, ny, nz, world)
        rb, re, wb, wl = blocks[rank]
        rows, n, rp, ci, v = cb.synth_lapl3d(nx, ny, nz, rb, re, wb)
        A = sp.csr_matrix((v, ci, rp), shape=(rows, wl))
        plan = cb.halo_plan(rank, blocks)

        def halo(xw):
            reqs = []
            for peer, so, sn, ro, rn in plan:
                if sn:
                    reqs.append(dist.isend(torch.from_numpy(xw[so:so + sn].copy()), peer))
            bufs = []
            for peer, so, sn, ro, rn in plan:
                if rn:
                    t = torch.empty(rn, dtype=torch.float64)
                    reqs.append(dist.irecv(t, peer))
                    bufs.append((ro, rn, t))
            for r in reqs:
                r.wait()
            for ro, rn, t in bufs:
                xw[ro:ro + rn] = t.numpy()

        def allsum(v):
            t = torch.tensor([v], dtype=torch.float64)
            dist.all_reduce(t)
            return float(t[0])

        # one distributed SpMV of a global vector
        xg = cb.synth_vector("uniform_pm1", n, seed=4)
        xw = np.zeros(wl)
        xw[rb - wb: re - wb] = xg[rb:re]
        halo(xw)
        y_local = A @ xw
        # textbook CG (bench_cg_solve.cu:165-197), b = U[-1,1]
        b = xg[rb:re].copy()
        x = np.zeros(rows)
        r = b.copy()
        pw = np.zeros(wl)
        off = rb - wb
        pw[off:off + rows] = b
        rs = allsum(float(r @ r))
        for _ in range(iters):
            halo(pw)
            ap = A @ pw
            p = pw[off:off + rows]
            pap = allsum(float(p @ ap))
            alpha = rs / pap if pap != 0 else 0.0
            x += alpha * p
            r -= alpha * ap
            rs_new = allsum(float(r @ r))
            beta = rs_new / rs if rs != 0 else 0.0
            pw[off:off + rows] = r + beta * p
            rs = rs_new
        out_q.put((rank, rb, re, y_local, x, rs))
    except Exception as e:  # reported to the parent
        out_q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, mode="ok", nx=6, ny=5, nz=8, iters=15):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, nx, ny, nz, iters, q, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    results = []
    expect = world if mode == "ok" else world - 1
    for _ in range(expect):
        results.append(q.get(timeout=120))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world", [2, 3])
def test_distributed_spmv_and_cg_match_single_process(world):
    import scipy.sparse as sp

    import cove_b200 as cb

    nx, ny, nz, iters = 6, 5, 8, 15
    res = _run(world, nx=nx, ny=ny, nz=nz, iters=iters)
    assert all(r[1] != "error" for r in res), res
    rows, n, rp, ci, v = cb.synth_lapl3d(nx, ny, nz)
    A = sp.csr_matrix((v, ci, rp), shape=(n, n))
    xg = cb.synth_vector("uniform_pm1", n, seed=4)
    y = A @ xg
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
    for rank, rb, re, y_local, x_local, rs_d in res:
        assert np.allclose(y_local, y[rb:re], rtol=0, atol=1e-13)
        assert np.allclose(x_local, x[rb:re], rtol=1e-9, atol=1e-12)
        assert abs(rs_d - rs) <= 1e-9 * abs(rs)


def test_rank_that_dies_fails_the_others_within_the_timeout():
    res = _run(2, mode="die")
    assert len(res) == 1
    rank, status, msg = res[0]
    assert status == "error"
