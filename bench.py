#!/usr/bin/env python3
"""Benchmark of the COVE SpMV hot path on B200 (one process per GPU).

Workload (default, `--workload lapl3d_cg`): the 3D 7-point Laplacian on a
768^3 grid (n = 452,984,832, nnz = 3,167,354,880, fp64, diagonal 6 and
neighbours -1), b ~ U[-1,1] seed 4, x0 = 0.  One step = one solve of 50
textbook CG iterations (the recurrence of the reference's CG bench) with the
SpMV on the plan's dispatched route.  Rows are cut into z-slabs across the
ranks (strong scaling: the same matrix at every N); each rank's slab is one
or more int32-safe row-block plans, the x halo (one grid plane to each
neighbour) arrives by NCCL send/recv overlapped with the interior rows, and
the two dot products per iteration are NCCL allreduces.  `value` is the SpMV
throughput inside the solve: 2 nnz / (device time of one SpMV, halo
included), max over ranks, aggregated over the whole job.

Other workloads: `--workload fem27` (config 2, the FEM 64^3 x 3 dof matrix;
one step = one SpMV; N > 1: weak-scaling z-slabs with an NCCL halo),
`lapl2d_512` / `rmat_22` (configs 1 and 3, one SpMV per step; N > 1:
independent replicas), `blocksparse` (config 4, 5.3e9 nnz in row-block
plans).

Timing: W warm-up steps, then K steps bracketed by barrier + synchronize;
device times from CUDA events on the launching stream, the max over ranks
per step.  `e2e` repeats the step through the C ABI with pinned host
buffers (inputs copied in and the result copied out every step).
`--impl reference` times the reference's own CPU SpMV (structural::spmv_csr,
OpenMP, every host core) on a bounded sample of the same workload; its input
is built by the oracle's restatement of the generators, so that arm never
loads this repository's library.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
import warnings

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cove-spmv_b200"))

import numpy as np  # noqa: E402

FEM = dict(nx=64, ny=64, nz=64, dof=3, seed=1)
GRAPH_SPMVS = 100  # SpMVs per CUDA graph in the warm-L2 timing
STEP_SLEEP_CYCLES = 600_000  # about 0.3 ms of device sleep ahead of each multi-rank step


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def fem_partition(rank, world):
    """Rows, window and generator arguments of one z-slab of the FEM grid."""
    nx, ny, nzl, dof = FEM["nx"], FEM["ny"], FEM["nz"], FEM["dof"]
    nz = nzl * world
    plane = nx * ny * dof
    row_begin = rank * nzl * plane
    row_end = row_begin + nzl * plane
    wb = max(0, row_begin - plane)
    we = min(nz * plane, row_end + plane)
    return dict(nx=nx, ny=ny, nz=nz, dof=dof, row_begin=row_begin, row_end=row_end,
                window_begin=wb, window_len=we - wb)


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    return O


def cpu_reference_time(rows, cols, rp, ci, v, x, reps):
    """The reference's spmv_csr (OpenMP, every host core) on this host;
    (best ms, threads, kind)."""
    O = _oracle()
    if O.ref_available():
        cores = O.ref_use_all_cores()
        t = O.RefCsrTimer(rows, cols, rp, ci, v, x)
        t.run(1)
        _, ms = t.run(reps)
        t.close()
        return ms, cores, "reference"
    best = 1e300
    for _ in range(reps):
        t0 = time.perf_counter()
        O.spmv_csr(rows, rp, ci, v, x)
        best = min(best, (time.perf_counter() - t0) * 1e3)
    return best, 1, "port"


LAPL3D = dict(n=768, seed=4, iters=50, stream=7, sample_planes=8)
L2_NOTE_CG = "inputs larger than L2 (every CG vector is n x 8 B, the matrix 10s of GB); no flush"
L2_NOTE_FLUSH = "flushed between steps (256 MiB write, outside the timed events)"


def lapl3d_nnz(g):
    return 7 * g ** 3 - 6 * g ** 2


def lapl3d_workload(g, iters):
    return (f"3D 7-point Laplacian {g}^3 (n={g ** 3}, nnz={lapl3d_nnz(g)}), "
            f"{iters} textbook CG iterations per step")


def bench_config(args):
    """The `config` object, identical in both arms for one workload."""
    if args.workload == "lapl3d_cg":
        g = args.grid or LAPL3D["n"]
        return {"workload": lapl3d_workload(g, args.cg_iters), "l2": L2_NOTE_CG}
    if args.workload == "fem27":
        return {"workload": "fem27 64x64x64 nodes x3 dof (n=786432, nnz=61731000), one SpMV per step",
                "l2": L2_NOTE_FLUSH}
    if args.workload == "blocksparse":
        n = args.bs_n or BLOCKSPARSE["n"]
        return {"workload": f"block-sparse 8x4 n={n} (p_block {BLOCKSPARSE['p_block']}, "
                            f"p_entry {BLOCKSPARSE['p_entry']}, {BLOCKSPARSE['outlier_fraction']:g} outliers),"
                            f" one SpMV per step", "l2": L2_NOTE_FLUSH}
    return {"workload": f"{args.workload}, one SpMV per step", "l2": L2_NOTE_FLUSH}


def reference_sample(args):
    """Bounded CPU sample of the workload: (rows, cols, rp, ci, v, x, description)."""
    O = _oracle()
    if args.workload == "lapl3d_cg":
        # 3.2e9 nnz do not fit host memory: the SpMV of the first grid planes
        # (their columns reach one plane further), x = b's first entries
        g = args.grid or LAPL3D["n"]
        planes = min(LAPL3D["sample_planes"], g)
        rows = planes * g * g
        rp, ci, v = O.lapl3d_rows(g, g, g, 0, rows)
        cols = min(g, planes + 1) * g * g
        x = O.vector("uniform_pm1", LAPL3D["seed"], LAPL3D["stream"], 0, cols)
        return rows, cols, rp, ci, v, x, f"the SpMV of grid planes [0, {planes}) ({ci.size} nnz)"
    if args.workload == "fem27":
        rp, ci, v = O.fem27_rows(64, 64, 64, 3, FEM["seed"], 0, 786432)
        x = O.vector("uniform_pm1", FEM["seed"], 7, 0, 786432)
        return 786432, 786432, rp, ci, v, x, "the whole matrix"
    if args.workload == "lapl2d_512":
        rp, ci, v = O.lapl2d(512, 512)
        x = O.vector("uniform_pm1", 0, 7, 0, 512 * 512)
        return 512 * 512, 512 * 512, rp, ci, v, x, "the whole matrix"
    if args.workload == "rmat_22":
        rp, ci, v = O.rmat(22, 16, seed=2)
        n = 1 << 22
        x = O.vector("uniform01", 2, 7, 0, n).astype(np.float32)
        return n, n, rp, ci, v, x, "the whole matrix"
    bs = BLOCKSPARSE
    n = args.bs_n or bs["n"]
    rp, ci, v = O.blocksparse_rows(n, 0, min(n, 32768), bs["p_block"], bs["p_entry"],
                                   bs["outlier_fraction"], bs["seed"])
    x = O.vector("normal", bs["seed"], 7, 0, n)
    return len(rp) - 1, n, rp, ci, v, x, f"rows [0, {len(rp) - 1}) ({ci.size} nnz)"


def run_reference_arm(args):
    """The reference's own CPU SpMV (structural::spmv_csr compiled from its
    headers into oracle/_ref, OpenMP over every host core), one bounded
    sample of the workload per step; rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    O = _oracle()
    rows, n, rp, ci, v, x, sample = reference_sample(args)
    nnz = int(ci.size)
    kind = "reference" if O.ref_available() else "port"
    times = []
    if kind == "reference":
        cores = O.ref_use_all_cores()
        t = O.RefCsrTimer(rows, n, rp, ci, v, x)
        for _ in range(args.warmup):
            t.run(1)
        for _ in range(args.steps):
            _, ms = t.run(1)
            times.append(ms)
        t.close()
    else:
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            O.spmv_csr(rows, rp, ci, v, x)
            if i >= args.warmup:
                times.append((time.perf_counter() - t0) * 1e3)
        cores = 1
    ms = sum(times) / len(times)
    gflops = 2.0 * nnz / (ms * 1e-3) / 1e9
    cg = args.workload == "lapl3d_cg"
    line = {
        "impl": "reference", "metric": "spmv_gflops", "value": round(gflops, 3),
        "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong" if args.workload in ("lapl3d_cg", "blocksparse") else "weak",
        "vs_baseline": None, "dtype": "f64" if v.dtype == np.float64 else "f32", "data": "synthetic",
        "config": bench_config(args),
        "cpu_baseline": {"value": round(gflops, 3), "unit": "GFLOP/s", "cores": cores,
                         "kind": kind,
                         "sample": f"structural::spmv_csr, one SpMV per step of {sample}"},
        "e2e": {"value": round(gflops, 3), "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_fem(args):
    import torch
    import torch.distributed as dist

    import cove_b200 as cb

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    fem = args.workload == "fem27"
    if fem:
        part = fem_partition(rank, world)
        rows, n, rp, ci, v = cb.synth_fem27_rows(part["nx"], part["ny"], part["nz"], part["dof"],
                                                 FEM["seed"], part["row_begin"], part["row_end"],
                                                 part["window_begin"])
        wl = part["window_len"]
        xg = cb.synth_vector("uniform_pm1", n, seed=FEM["seed"])
        x_window = xg[part["window_begin"]: part["window_begin"] + wl].copy()
    else:  # one named matrix, a replica per rank
        rows, n, rp, ci, v, x_window = cb.workload(args.workload)
        wl = n
    vt = torch.float64 if v.dtype == np.float64 else torch.float32
    esz = v.itemsize
    csr = cb.DeviceCsr.from_numpy(rows, wl, rp, ci, v, device=dev)
    t0 = time.perf_counter()
    plan = cb.Plan(csr, value_codec=args.codec, long_row_split=256)
    build_s = time.perf_counter() - t0
    del csr
    info = plan.info
    route = info.dispatched_route if args.route is None else cb.ROUTE_NAMES_INV[args.route]
    nnz_local = int(info.nnz)

    stream = torch.cuda.current_stream()
    xw = torch.from_numpy(x_window).to(dev)
    y = torch.empty(rows, dtype=vt, device=dev)
    D = None
    if world > 1 and fem:
        import ctypes as C

        idb = cb.lib().cove_dist_id_bytes()
        idbuf = np.zeros(idb, np.uint8)
        if rank == 0:
            cb.check(cb.lib().cove_dist_make_id(idbuf.ctypes.data_as(C.c_void_p)))
        obj = [idbuf.tobytes()]
        dist.broadcast_object_list(obj, src=0)
        idbuf = np.frombuffer(obj[0], np.uint8).copy()
        D = C.c_void_p()
        arr = (C.c_void_p * 1)(plan.handle.value)
        cb.check(cb.lib().cove_dist_create(rank, world, idbuf.ctypes.data_as(C.c_void_p), arr, 1,
                                           n, part["row_begin"], part["row_end"],
                                           part["window_begin"], wl, 120000, C.byref(D)))

    def step(xbuf, ybuf):
        if D is not None:
            cb.check(cb.lib().cove_dist_spmv(D, C.c_void_p(xbuf.data_ptr()),
                                             C.c_void_p(ybuf.data_ptr()),
                                             C.c_void_p(stream.cuda_stream)))
        else:
            plan.spmv(xbuf, ybuf, route=route, stream=stream)

    # parity check of this very plan against a CPU SpMV of the same rows
    step(xw, y)
    torch.cuda.synchronize()
    import scipy.sparse as sp

    A = sp.csr_matrix((v, ci, rp), shape=(rows, wl))
    y_ref = A @ x_window
    yh = y.cpu().numpy()
    rel = float(np.abs(yh - y_ref).max() / max(np.abs(y_ref).max(), 1e-300))

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        step(xw, y)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    clk = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk.start()
    time.sleep(0.3)
    w0 = time.perf_counter()
    for i in range(args.steps):
        flush.zero_()
        if world > 1:
            # every rank starts the step together: a barrier, then a short
            # device sleep that covers the host's enqueue of the whole step
            # (the NCCL halo included), so the events time the GPU's work and
            # not a rank's host falling behind
            dist.barrier()
            torch.cuda._sleep(STEP_SLEEP_CYCLES)
        ev[i][0].record(stream)
        step(xw, y)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    if world > 1:
        dist.barrier()
    clocks = clk.stop()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    ms = sum(step_ms) / len(step_ms)
    launches = plan.launches(route) if D is None else cb.lib().cove_dist_spmv_launches(D)

    # end to end through the public C ABI with host buffers (pinned)
    xh = torch.from_numpy(x_window).pin_memory()
    yh_t = torch.empty(rows, dtype=vt).pin_memory()
    xd2 = torch.empty(wl, dtype=vt, device=dev)
    e2e_ms = []
    for i in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        if D is None:
            plan.spmv_host(xh.numpy(), yh_t.numpy(), stream=stream)
        else:
            xd2.copy_(xh, non_blocking=True)
            step(xd2, y)
            yh_t.copy_(y, non_blocking=True)
            torch.cuda.synchronize()
        if i >= args.warmup:
            e2e_ms.append((time.perf_counter() - t0) * 1e3)

    e2e_median = float(np.median(e2e_ms))
    # the L2-resident matrices (2D Laplacian 512^2: ~10 MB of streams) are also
    # timed warm, as one CUDA graph of GRAPH_SPMVS back-to-back SpMVs (no
    # launch gaps); the per-step numbers above are the cold-L2 ones
    warm_graph_ms = None
    if not fem and D is None:
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            plan.spmv(xw, y, route=route, stream=cap)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=cap):
            for _ in range(GRAPH_SPMVS):
                plan.spmv(xw, y, route=route, stream=torch.cuda.current_stream())
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        reps = []
        for _ in range(10):
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            g.replay()
            c1.record(stream)
            torch.cuda.synchronize()
            reps.append(c0.elapsed_time(c1) / GRAPH_SPMVS)
        warm_graph_ms = float(np.median(reps))
        del g
    # vendor library context: cuSPARSE CSR SpMV (through torch) of the same matrix
    vendor_ms = None
    try:
        with warnings.catch_warnings():  # torch's beta-state notes on sparse CSR tensors
            warnings.simplefilter("ignore", UserWarning)
            A_csr = torch.sparse_csr_tensor(torch.from_numpy(rp.astype(np.int64)),
                                            torch.from_numpy(ci.astype(np.int64)),
                                            torch.from_numpy(v), size=(rows, wl), device=dev)
        xv = xw.view(-1, 1)
        for _ in range(3):
            A_csr.matmul(xv)
        vt = []
        for _ in range(10):
            flush.zero_()
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record()
            A_csr.matmul(xv)
            c1.record()
            torch.cuda.synchronize()
            vt.append(c0.elapsed_time(c1))
        vendor_ms = float(np.median(vt))
        del A_csr
    except Exception:
        vendor_ms = None
    # the host link on its own: plain pinned copies of the same x and y bytes
    copy_ms = {}
    for name, dst, src in (("h2d", xd2, xh), ("d2h", yh_t, y)):
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(10):
            dst.copy_(src, non_blocking=True)
        c1.record()
        torch.cuda.synchronize()
        copy_ms[name] = c0.elapsed_time(c1) / 10
    tot = torch.tensor(step_ms + [float(np.mean(e2e_ms)), float(nnz_local), rel, wall],
                       dtype=torch.float64, device=dev)
    K = args.steps
    if world > 1:
        allv = [torch.empty_like(tot) for _ in range(world)]
        dist.all_gather(allv, tot)
        M = torch.stack(allv).cpu().numpy()
    else:
        M = tot.cpu().numpy()[None, :]
    step_max = M[:, :K].max(axis=0)  # per step, the slowest rank
    ms_all = float(step_max.mean())
    e2e_all, rel_all = float(M[:, K].max()), float(M[:, K + 2].max())
    nnz_total = float(M[:, K + 1].sum())

    if rank == 0:
        hbm, peak_kind = peaks()
        alg_bytes = int(info.algorithmic_bytes[route])
        achieved = alg_bytes / (ms_all * 1e-3) / 1e9  # every rank holds the same rows
        gflops = 2.0 * nnz_total / (ms_all * 1e-3) / 1e9
        e2e_gflops = 2.0 * nnz_total / (e2e_all * 1e-3) / 1e9
        tr = load_traffic("fem27_64" if fem else args.workload, cb.ROUTE_NAMES[route])
        traffic = int(round(tr["bytes"] * nnz_local / tr["nnz"])) if tr and tr.get("nnz") else None
        # the reference's CPU SpMV on the same matrix, bounded sample
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cms, cores, kind = cpu_reference_time(rows, wl, rp, ci, v, x_window, 5)
            cpu = {"value": round(2.0 * nnz_local / (cms * 1e-3) / 1e9, 3), "unit": "GFLOP/s",
                   "cores": cores, "kind": kind,
                   "sample": "best of 5 full SpMVs (structural::spmv_csr, OpenMP) of the same matrix"}
        line = {
            "metric": "spmv_gflops", "value": round(gflops, 3), "unit": "GFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_all, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": ("f64" if esz == 8 else "f32") if route in (0, 1, 2)
                     else f"f32 accumulate, {'f64' if esz == 8 else 'f32'} in/out",
            "data": "synthetic",
            "config": {"workload": (f"fem27 {FEM['nx']}x{FEM['ny']}x{FEM['nz'] * world} nodes x3 dof"
                                    f" ({'z-slab per rank, ' if world > 1 else ''}nnz={int(nnz_total)})")
                                   if fem else f"{args.workload} (rows={rows}, nnz={nnz_local}"
                                               f"{', a replica per rank' if world > 1 else ''})",
                       "route": cb.ROUTE_NAMES[route], "requested_codec": args.codec,
                       "dispatched_route": cb.ROUTE_NAMES[info.dispatched_route],
                       "joint_route": cb.ROUTE_NAMES[info.joint_route],
                       "gate_rel_err": info.joint_rel_err, "gate_pass": bool(info.gate_pass),
                       "l2": "flushed between steps (256 MiB write, outside the timed events)",
                       "parallelism": ("1 GPU" if world == 1 else f"row-block z-slabs x{world}, NCCL halo"
                                       if fem else f"{world} independent replicas"),
                       "plan_build_s": round(build_s, 3), "kernel_slots": info.kernel_slots,
                       "e2e_ms_mean": round(e2e_all, 4), "e2e_ms_median_rank0": round(e2e_median, 4),
                       "ms_per_step_median": round(float(np.median(step_max)), 5),
                       "ms_per_step_max": round(float(step_max.max()), 5),
                       "host_copy_ms_rank0": {k: round(v, 4) for k, v in copy_ms.items()},
                       "cusparse_csr_ms_rank0": round(vendor_ms, 5) if vendor_ms else None,
                       "warm_l2_graph_ms_per_spmv_rank0": round(warm_graph_ms, 5) if warm_graph_ms else None,
                       "warm_l2_graph_gflops_rank0": round(2.0 * nnz_local / (warm_graph_ms * 1e-3) / 1e9, 3)
                       if warm_graph_ms else None,
                       "parity_rel_vs_cpu": rel_all},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                         "algorithmic_bytes": alg_bytes, "traffic": traffic,
                         "traffic_source": (f"ncu DRAM bytes of one launch on {tr['case']} "
                                            f"(profiles/traffic.json)") if traffic else None},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_gflops, 3), "unit": "GFLOP/s",
                    "h2d_bytes_per_step": wl * esz, "d2h_bytes_per_step": rows * esz},
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if D is not None:
        cb.lib().cove_dist_destroy(D)
    plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


MAX_SHARD_NNZ = 2_000_000_000  # one plan per shard keeps the int32 offsets of the format


def lapl3d_partition(rank, world, nx, ny, nz):
    """z-slab rows [row_begin, row_end) of rank, its window (one plane of halo
    each side) and its shards (whole planes, < MAX_SHARD_NNZ nnz each)."""
    plane = nx * ny
    cuts = [round(r * nz / world) for r in range(world + 1)]
    k0, k1 = cuts[rank], cuts[rank + 1]
    per_shard = max(1, MAX_SHARD_NNZ // (7 * plane))
    shards = [(k * plane, min(k1, k + per_shard) * plane) for k in range(k0, k1, per_shard)]
    wb = max(0, k0 - 1) * plane
    we = min(nz, k1 + 1) * plane
    return dict(row_begin=k0 * plane, row_end=k1 * plane, window_begin=wb, window_len=we - wb,
                shards=shards)


def load_traffic(key, route):
    """ncu DRAM bytes of one launch of the dominant kernel on a captured case,
    with the nnz of that case (profiles/traffic.json), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
        e = t.get(key, {}).get(route)
    except Exception:
        return None
    return e


def run_lapl3d_cg(args):
    """3D 7-point Laplacian CG, rows partitioned across the ranks (strong scaling)."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    import cove_b200 as cb

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    g = args.grid or LAPL3D["n"]
    nx = ny = nz = g
    n_global = g ** 3
    iters = args.cg_iters
    part = lapl3d_partition(rank, world, nx, ny, nz)
    stream = torch.cuda.current_stream()
    sh = C.c_void_p(stream.cuda_stream)
    L = cb.lib()
    plans = []
    nnz_local = 0
    t0 = time.perf_counter()
    for (sb, se) in part["shards"]:
        rows = se - sb
        nnz = C.c_int64(0)
        cb.check(L.cove_synth_lapl3d_device(nx, ny, nz, sb, se, part["window_begin"], None, None,
                                            None, C.byref(nnz), sh))
        rp = torch.empty(rows + 1, dtype=torch.int32, device=dev)
        ci = torch.empty(nnz.value, dtype=torch.int32, device=dev)
        v = torch.empty(nnz.value, dtype=torch.float64, device=dev)
        cb.check(L.cove_synth_lapl3d_device(nx, ny, nz, sb, se, part["window_begin"],
                                            C.c_void_p(rp.data_ptr()), C.c_void_p(ci.data_ptr()),
                                            C.c_void_p(v.data_ptr()), C.byref(nnz), sh))
        csr = cb.DeviceCsr(rows, part["window_len"], rp, ci, v)
        plans.append(cb.Plan(csr, value_codec=args.codec, keep_lossless=0, stream=stream))
        nnz_local += int(plans[-1].info.nnz)
        del csr, rp, ci, v
        torch.cuda.empty_cache()
    build_s = time.perf_counter() - t0
    route = plans[0].info.dispatched_route
    # every plan's algorithmic bytes count its x window once; the rank's shards
    # share one window, read once per SpMV
    alg_local = sum(int(p.info.algorithmic_bytes[p.info.dispatched_route]) - 8 * int(p.info.cols)
                    for p in plans) + 8 * part["window_len"]
    rows_local = part["row_end"] - part["row_begin"]
    p_off = part["row_begin"] - part["window_begin"]
    b = torch.empty(rows_local, dtype=torch.float64, device=dev)
    cb.check(L.cove_synth_vector_device(0, LAPL3D["seed"], LAPL3D["stream"], part["row_begin"], rows_local,
                                        C.c_void_p(b.data_ptr()), sh))
    x = torch.zeros(rows_local, dtype=torch.float64, device=dev)

    idb = L.cove_dist_id_bytes()
    idbuf = np.zeros(idb, np.uint8)
    if rank == 0:
        cb.check(L.cove_dist_make_id(idbuf.ctypes.data_as(C.c_void_p)))
    if world > 1:
        obj = [idbuf.tobytes()]
        dist.broadcast_object_list(obj, src=0)
        idbuf = np.frombuffer(obj[0], np.uint8).copy()
    D = C.c_void_p()
    arr = (C.c_void_p * len(plans))(*[p.handle.value for p in plans])
    cb.check(L.cove_dist_create(rank, world, idbuf.ctypes.data_as(C.c_void_p), arr, len(plans),
                                n_global, part["row_begin"], part["row_end"],
                                part["window_begin"], part["window_len"], 300000, C.byref(D)))

    def solve(bd, xd):
        res = cb.CgResult()
        cb.check(L.cove_dist_cg_solve(D, C.c_void_p(bd.data_ptr()), C.c_void_p(xd.data_ptr()), iters,
                                      C.byref(res), sh))
        return res

    for _ in range(args.warmup):
        res = solve(b, x)
    torch.cuda.synchronize()
    # check of the solve: the true residual ||b - A x||^2 (one more distributed
    # SpMV) against the recurrence's r.r, relative to r0.r0
    xw = torch.zeros(part["window_len"], dtype=torch.float64, device=dev)
    xw[p_off:p_off + rows_local].copy_(x)
    yv = torch.empty(rows_local, dtype=torch.float64, device=dev)
    cb.check(L.cove_dist_spmv(D, C.c_void_p(xw.data_ptr()), C.c_void_p(yv.data_ptr()), sh))
    chk = ((b - yv) ** 2).sum().reshape(1)
    del xw, yv
    if world > 1:
        dist.all_reduce(chk)
    true_rs = float(chk[0])  # res.rs_final is already the global r.r
    residual_gap = abs(true_rs - res.rs_final) / res.rs_initial if res.rs_initial else None

    clk = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk.start()
    time.sleep(0.3)
    step_total, step_spmv, launches = [], [], 0
    for _ in range(args.steps):
        if world > 1:
            dist.barrier()
        res = solve(b, x)
        step_total.append(res.ms_total)
        step_spmv.append(res.ms_spmv)
        launches += int(res.launches)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = clk.stop()
    rs_ratio = res.rs_final / res.rs_initial if res.rs_initial else None

    # end to end through the C ABI: b from pinned host memory in, the solution
    # x out to pinned host memory, every step
    e2e_steps = max(1, min(args.steps, 5))
    bh = b.cpu().pin_memory()
    xh = torch.empty(rows_local, dtype=torch.float64).pin_memory()
    bd2 = torch.empty_like(b)
    xd2 = torch.empty_like(x)
    e2e = []
    for i in range(1 + e2e_steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t1 = time.perf_counter()
        bd2.copy_(bh, non_blocking=True)
        solve(bd2, xd2)
        xh.copy_(xd2, non_blocking=True)
        torch.cuda.synchronize()
        if i >= 1:
            e2e.append((time.perf_counter() - t1) * 1e3)
    e2e_ok = bool(torch.equal(xh, x.cpu()))  # the same solve as the device-resident one

    # per-step times of every rank; the step time is the max over ranks
    loc = torch.tensor(step_total + step_spmv + e2e + [float(nnz_local), float(alg_local), float(launches),
                                                       float(e2e_ok)], dtype=torch.float64, device=dev)
    if world > 1:
        allv = [torch.empty_like(loc) for _ in range(world)]
        dist.all_gather(allv, loc)
        M = torch.stack(allv).cpu().numpy()
    else:
        M = loc.cpu().numpy()[None, :]
    K, E = args.steps, e2e_steps
    tot = M[:, :K].max(axis=0)
    spm = M[:, K:2 * K].max(axis=0)
    e2e_max = M[:, 2 * K:2 * K + E].max(axis=0)
    nnz_total = float(M[:, 2 * K + E].sum())
    alg_total = float(M[:, 2 * K + E + 1].sum())
    launches_total = int(M[:, 2 * K + E + 2].sum())
    e2e_all_ok = bool(M[:, 2 * K + E + 3].min() > 0)

    if rank == 0:
        hbm, peak_kind = peaks()
        ms_step = float(np.mean(tot))
        ms_spmv = float(np.mean(spm)) / iters
        gflops = 2.0 * nnz_total / (ms_spmv * 1e-3) / 1e9
        achieved = alg_total / world / (ms_spmv * 1e-3) / 1e9
        rname = cb.ROUTE_NAMES[route]
        tr = load_traffic("lapl3d", rname)
        traffic = None
        if tr and tr.get("nnz"):
            traffic = int(round(tr["bytes"] * (nnz_total / world) / tr["nnz"]))
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            rows_s, cols_s, rp_s, ci_s, v_s, x_s, sample = reference_sample(args)
            cms, cores, kind = cpu_reference_time(rows_s, cols_s, rp_s, ci_s, v_s, x_s, 5)
            cpu = {"value": round(2.0 * ci_s.size / (cms * 1e-3) / 1e9, 3), "unit": "GFLOP/s", "cores": cores,
                   "kind": kind, "sample": f"best of 5 runs of structural::spmv_csr (OpenMP) on {sample}"}
        e2e_ms = float(np.mean(e2e_max))
        line = {
            "metric": "spmv_gflops", "value": round(gflops, 3), "unit": "GFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": bench_config(args),
            "details": {
                "step": f"one solve of {iters} textbook CG iterations from x0 = 0",
                "route": rname, "ms_per_iteration": round(ms_step / iters, 5),
                "ms_per_spmv": round(ms_spmv, 5),
                "ms_per_step_median": round(float(np.median(tot)), 4),
                "ms_per_step_max": round(float(np.max(tot)), 4),
                "iteration_gflops": round((2.0 * nnz_total + 10.0 * n_global) / (ms_step / iters * 1e-3) / 1e9, 3),
                "rs_ratio": rs_ratio, "true_vs_recurrence_residual_gap": residual_gap,
                "shards_per_rank": len(plans), "plan_build_s_rank0": round(build_s, 2),
                "parallelism": "1 GPU" if world == 1 else f"z-slab row blocks x{world}, NCCL halo + allreduce",
                "e2e_ms_per_step": round(e2e_ms, 3), "e2e_steps": E,
                "e2e_result_equals_device_run": e2e_all_ok,
                "gpu_launches_per_rank": launches // max(1, args.steps),
            },
            "roofline": {"bound": "hbm", "kernel": "the SpMV of one CG iteration (all its launches)",
                         "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                         "algorithmic_bytes": int(alg_total / world), "traffic": traffic,
                         "traffic_source": (f"ncu DRAM bytes of one launch on {tr['case']}, scaled by nnz "
                                            f"(profiles/traffic.json)") if traffic else None},
            "cpu_baseline": cpu,
            "e2e": {"value": round(2.0 * nnz_total * iters / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GFLOP/s",
                    "h2d_bytes_per_step": n_global * 8, "d2h_bytes_per_step": n_global * 8},
            "gpu_launches": launches_total,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    L.cove_dist_destroy(D)
    for p in plans:
        p.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


BLOCKSPARSE = dict(n=1 << 21, p_block=2e-3, p_entry=0.6, outlier_fraction=1e-3, seed=3)
SHARD_NNZ_TARGET = 1_800_000_000  # expected nnz per plan (int32 offsets, with margin)


def blocksparse_shards(rank, world, n):
    """Rows [row_begin, row_end) of rank (whole 8-row block rows) and its shards."""
    bs = BLOCKSPARSE
    nbr = (n + 7) // 8
    cuts = [round(r * nbr / world) * 8 for r in range(world + 1)]
    rb, re = cuts[rank], min(cuts[rank + 1], n)
    per_row = ((n + 3) // 4) * bs["p_block"] * 4 * bs["p_entry"]
    k = max(1, int(np.ceil((re - rb) * per_row / SHARD_NNZ_TARGET)))
    sb = [rb + round(i * (re - rb) / (8 * k)) * 8 for i in range(k)] + [re]
    return rb, re, [(sb[i], sb[i + 1]) for i in range(k) if sb[i + 1] > sb[i]]


def run_blocksparse(args):
    """Random 8x4 block-sparse n = 2^21 with outliers (5.3e9 nnz): row blocks
    of int32-safe plans generated in HBM; with N > 1 the same matrix's rows
    are split across the ranks (strong scaling) and each rank receives the
    other ranks' x rows (every rank reads all of x)."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    import cove_b200 as cb

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=dev)
    bs = BLOCKSPARSE
    n = args.bs_n or bs["n"]
    gen = (bs["p_block"], bs["p_entry"], bs["outlier_fraction"], bs["seed"])
    codec = args.codec or "bfp8_outlier"
    rb, re, shards = blocksparse_shards(rank, world, n)
    stream = torch.cuda.current_stream()
    sh = C.c_void_p(stream.cuda_stream)
    L = cb.lib()
    plans = []
    t0 = time.perf_counter()
    for (sb, se) in shards:
        rp, ci, v = cb.synth_blocksparse_device(n, sb, se, *gen, device=dev, stream=stream)
        plans.append(cb.Plan(cb.DeviceCsr(se - sb, n, rp, ci, v), value_codec=codec, keep_lossless=1,
                             stream=stream))
        del rp, ci, v
        torch.cuda.empty_cache()
    build_s = time.perf_counter() - t0
    nnz_local = sum(int(p.info.nnz) for p in plans)
    route = plans[0].info.dispatched_route
    x_host = cb.synth_vector("normal", n, seed=bs["seed"])
    xd = torch.from_numpy(x_host).to(dev)
    y = torch.empty(re - rb, dtype=torch.float64, device=dev)

    idbuf = np.zeros(L.cove_dist_id_bytes(), np.uint8)
    if rank == 0:
        cb.check(L.cove_dist_make_id(idbuf.ctypes.data_as(C.c_void_p)))
    if world > 1:
        obj = [idbuf.tobytes()]
        dist.broadcast_object_list(obj, src=0)
        idbuf = np.frombuffer(obj[0], np.uint8).copy()
    D = C.c_void_p()
    arr = (C.c_void_p * len(plans))(*[p.handle.value for p in plans])
    cb.check(L.cove_dist_create(rank, world, idbuf.ctypes.data_as(C.c_void_p), arr, len(plans), n, rb, re,
                                0, n, 300000, C.byref(D)))

    def step(xbuf, ybuf):
        cb.check(L.cove_dist_spmv(D, C.c_void_p(xbuf.data_ptr()), C.c_void_p(ybuf.data_ptr()), sh))

    # parity on 16 block rows of this rank, regenerated on the host
    step(xd, y)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    nbr_local = (re - rb + 7) // 8
    worst = 0.0
    ymax = 0.0
    for q in np.linspace(0, nbr_local - 1, 16).astype(np.int64):
        r0 = rb + int(q) * 8
        r1 = min(r0 + 8, re)
        srp, sci, sv = cb.synth_blocksparse_rows(n, r0, r1, *gen)
        for i in range(r1 - r0):
            ref = float(np.dot(sv[srp[i]:srp[i + 1]], x_host[sci[srp[i]:srp[i + 1]]]))
            worst = max(worst, abs(ref - yh[r0 - rb + i]))
            ymax = max(ymax, abs(ref))
    rel = worst / max(ymax, 1e-300)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        step(xd, y)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    clk = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk.start()
    time.sleep(0.3)
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record(stream)
        step(xd, y)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = clk.stop()
    ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    launches = int(L.cove_dist_spmv_launches(D))

    # end to end: pinned host x in, y out, every step
    xh = torch.from_numpy(x_host).pin_memory()
    yh_t = torch.empty(re - rb, dtype=torch.float64).pin_memory()
    xd2 = torch.empty(n, dtype=torch.float64, device=dev)
    e2e = []
    for i in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t1 = time.perf_counter()
        xd2.copy_(xh, non_blocking=True)
        step(xd2, y)
        yh_t.copy_(y, non_blocking=True)
        torch.cuda.synchronize()
        if i >= args.warmup:
            e2e.append((time.perf_counter() - t1) * 1e3)
    alg_local = sum(int(p.info.algorithmic_bytes[p.info.dispatched_route]) for p in plans)
    tot = torch.tensor([ms, float(np.mean(e2e)), float(nnz_local), rel, float(alg_local)], dtype=torch.float64,
                       device=dev)
    if world > 1:
        mx = tot.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = tot.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms_all, e2e_all, rel_all, nnz_total = float(mx[0]), float(mx[1]), float(mx[3]), float(sm[2])
        alg_total = float(sm[4])
    else:
        ms_all, e2e_all, rel_all, nnz_total = ms, float(np.mean(e2e)), rel, float(nnz_local)
        alg_total = float(alg_local)
    if rank == 0:
        hbm, peak_kind = peaks()
        alg = int(alg_total / world)  # per GPU
        achieved = alg / (ms_all * 1e-3) / 1e9
        tr = load_traffic("blocksparse", cb.ROUTE_NAMES[route])
        traffic = int(round(tr["bytes"] * (nnz_total / world) / tr["nnz"])) if tr and tr.get("nnz") else None
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            # bounded sample: the first 32,768 rows (~8e7 nnz) through the reference's spmv_csr
            srp, sci, sv = _oracle().blocksparse_rows(n, 0, min(n, 32768), *gen)
            cms, cores, kind = cpu_reference_time(len(srp) - 1, n, srp, sci, sv, x_host, 5)
            cpu = {"value": round(2.0 * len(sv) / (cms * 1e-3) / 1e9, 3), "unit": "GFLOP/s", "cores": cores,
                   "kind": kind, "sample": f"best of 5 SpMVs of rows [0, {len(srp) - 1}) ({len(sv)} nnz)"}
        line = {
            "metric": "spmv_gflops", "value": round(2.0 * nnz_total / (ms_all * 1e-3) / 1e9, 3),
            "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_all, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64" if route in (0, 1, 2) else "f32 accumulate, f64 in/out",
            "data": "synthetic",
            "config": {"workload": f"block-sparse 8x4 n={n} (p_block {bs['p_block']}, p_entry {bs['p_entry']},"
                                   f" {bs['outlier_fraction']:g} outliers; nnz={int(nnz_total)})",
                       "requested_codec": codec, "route": cb.ROUTE_NAMES[route],
                       "joint_route": cb.ROUTE_NAMES[plans[0].info.joint_route],
                       "gate_rel_err": plans[0].info.joint_rel_err, "gate_pass": bool(plans[0].info.gate_pass),
                       "plans_per_rank": len(plans), "plan_build_s": round(build_s, 2),
                       "l2": "flushed between steps (256 MiB write, outside the timed events)",
                       "parallelism": "1 GPU" if world == 1 else f"row blocks x{world}, x rows exchanged by NCCL",
                       "parity_rel_sampled_rows": rel_all},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_kind": peak_kind, "algorithmic_bytes": alg,
                         "traffic": traffic,
                         "traffic_source": (f"ncu DRAM bytes of one main-pass launch on {tr['case']}, scaled by "
                                            f"nnz to a rank's plans (profiles/traffic.json)") if traffic else None},
            "cpu_baseline": cpu,
            "e2e": {"value": round(2.0 * nnz_total / (e2e_all * 1e-3) / 1e9, 3), "unit": "GFLOP/s",
                    "h2d_bytes_per_step": n * 8, "d2h_bytes_per_step": (re - rb) * 8},
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    L.cove_dist_destroy(D)
    for p in plans:
        p.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="lapl3d_cg",
                    choices=["fem27", "lapl3d_cg", "lapl2d_512", "rmat_22", "blocksparse"])
    ap.add_argument("--bs-n", type=int, default=0, help="blocksparse: n (default 2^21)")
    ap.add_argument("--grid", type=int, default=0, help="lapl3d_cg: grid edge (default 768)")
    ap.add_argument("--cg-iters", type=int, default=50)
    ap.add_argument("--codec", default=None, help="value codec (default auto; blocksparse: bfp8_outlier)")
    ap.add_argument("--route", default=None,
                    help="time this route instead of the dispatched one (analysis only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.workload == "blocksparse":
        return run_blocksparse(args)
    if args.codec is None:
        args.codec = "auto"
    if args.workload == "lapl3d_cg":
        return run_lapl3d_cg(args)
    return run_fem(args)


if __name__ == "__main__":
    sys.exit(main())
