"""Config 5 at full size: the 3D 7-point Laplacian on the 768^3 grid
(n = 452,984,832, nnz = 3,167,354,880, beyond int32 offsets), held on one
GPU as two row-block plans of whole grid planes, the way the benchmark holds
it.  The whole SpMV y = A x runs on the device; sampled grid planes (the
first and last planes, the planes on both sides of the plan boundary and one
in the middle) are checked against the reference's own CPU SpMV
(structural::spmv_csr, spmv.hpp:12-29) of the same rows, regenerated on the
host with the oracle's restated generator.  Lossless route: 1e-12 normwise
per plane."""
import ctypes as C

import numpy as np
import pytest

import bench
import cove_b200 as cb
import oracle as O

pytestmark = pytest.mark.gpu

G = 768
SEED, STREAM = 4, 7


def _ref_spmv(rows, cols, rp, ci, v, x):
    if O.ref_available():
        return O.ref_spmv_csr(rows, cols, rp, ci, v, x)[0]
    return O.spmv_csr(rows, rp, ci, v, x)


def test_full_size_lapl3d_spmv_on_sampled_planes():
    import torch

    L = cb.lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    sh = C.c_void_p(stream.cuda_stream)
    n = G ** 3
    plane = G * G
    part = bench.lapl3d_partition(0, 1, G, G, G)
    assert len(part["shards"]) == 2
    plans = []
    nnz_total = 0
    for sb, se in part["shards"]:
        nnz = C.c_int64(0)
        cb.check(L.cove_synth_lapl3d_device(G, G, G, sb, se, 0, None, None, None, C.byref(nnz), sh))
        rp = torch.empty(se - sb + 1, dtype=torch.int32, device=dev)
        ci = torch.empty(nnz.value, dtype=torch.int32, device=dev)
        v = torch.empty(nnz.value, dtype=torch.float64, device=dev)
        cb.check(L.cove_synth_lapl3d_device(G, G, G, sb, se, 0, C.c_void_p(rp.data_ptr()),
                                            C.c_void_p(ci.data_ptr()), C.c_void_p(v.data_ptr()),
                                            C.byref(nnz), sh))
        plans.append(cb.Plan(cb.DeviceCsr(se - sb, n, rp, ci, v), value_codec="auto", keep_lossless=0,
                             stream=stream))
        nnz_total += nnz.value
        del rp, ci, v
        torch.cuda.empty_cache()
    assert nnz_total == bench.lapl3d_nnz(G) == 3167354880
    assert all(cb.ROUTE_NAMES[p.info.dispatched_route] == "dict_u8_lossless" for p in plans)
    x = torch.empty(n, dtype=torch.float64, device=dev)
    cb.check(L.cove_synth_vector_device(0, SEED, STREAM, 0, n, C.c_void_p(x.data_ptr()), sh))
    y = torch.full((n,), float("nan"), dtype=torch.float64, device=dev)
    off = 0
    for (sb, se), p in zip(part["shards"], plans):
        p.spmv(x, y[sb:se], stream=stream)
        off = se
    torch.cuda.synchronize()
    assert off == n
    boundary = part["shards"][0][1] // plane
    for k in sorted({0, 1, boundary - 1, boundary, G // 2, G - 2, G - 1}):
        r0, r1 = k * plane, (k + 1) * plane
        c0 = max(0, k - 1) * plane
        c1 = min(G, k + 2) * plane
        rp, ci, v = O.lapl3d_rows(G, G, G, r0, r1, c0)
        xw = O.vector("uniform_pm1", SEED, STREAM, c0, c1 - c0)
        ref = _ref_spmv(r1 - r0, c1 - c0, rp, ci, v, xw)
        got = y[r0:r1].cpu().numpy()
        assert np.isfinite(got).all(), k
        rel = np.abs(got - ref).max() / np.abs(ref).max()
        assert rel <= 1e-12, (k, rel)
    for p in plans:
        p.close()
