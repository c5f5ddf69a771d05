"""The 8x4 block-sparse workload with outliers at sizes beyond one plan (needs a B200).

The full matrix (n = 2^21, 5.3e9 nnz) exceeds the int32 offsets of the
format, so it is generated in HBM row block by row block and held as several
plans.  Here: the device generator against the host one (bit for bit), and a
three-plan partition of a smaller instance against a SciPy product of the
host-generated matrix, lossless and through the BFP8 outlier route.
"""
import ctypes as C

import numpy as np
import pytest

import cove_b200 as cb

pytestmark = pytest.mark.gpu

GEN = dict(p_block=0.05, p_entry=0.6, outlier_fraction=0.01, seed=11)


@pytest.mark.parametrize("rows", [(0, 4099), (1024, 2048), (4096, 4099)])
def test_device_generator_matches_host(rows):
    n = 4099
    rb, re = rows
    rp, ci, v = cb.synth_blocksparse_rows(n, rb, re, **GEN)
    drp, dci, dv = cb.synth_blocksparse_device(n, rb, re, **GEN)
    assert np.array_equal(drp.cpu().numpy(), rp.astype(np.int32))
    assert np.array_equal(dci.cpu().numpy(), ci)
    assert np.array_equal(dv.cpu().numpy(), v)  # outliers and bf16 redraws included
    assert (np.abs(v) >= 1e5).any()


def test_generator_rejects_ragged_row_ranges():
    with pytest.raises(cb.CoveError, match="whole 8-row block rows"):
        cb.synth_blocksparse_device(4099, 4, 64, **GEN)
    with pytest.raises(cb.CoveError, match="whole 8-row block rows"):
        cb.synth_blocksparse_rows(4099, 0, 100, **GEN)


@pytest.mark.parametrize("codec", ["original", "bfp8_outlier"])
def test_three_plan_partition_matches_scipy(codec):
    import scipy.sparse as sp
    import torch

    n = 1 << 15
    g = dict(GEN, p_block=0.01)
    _, _, rp, ci, v = cb.synth_blocksparse(n, **g)
    A = sp.csr_matrix((v, ci, rp), shape=(n, n))
    x = cb.synth_vector("normal", n, seed=3)
    ref = A @ x
    cuts = [0, 10000, 20000, n]  # whole block rows
    plans = []
    for sb, se in zip(cuts[:-1], cuts[1:]):
        drp, dci, dv = cb.synth_blocksparse_device(n, sb, se, **g)
        plans.append(cb.Plan(cb.DeviceCsr(se - sb, n, drp, dci, dv), value_codec=codec, gate_enable=0,
                             keep_lossless=1))
    L = cb.lib()
    idbuf = np.zeros(L.cove_dist_id_bytes(), np.uint8)
    cb.check(L.cove_dist_make_id(idbuf.ctypes.data_as(C.c_void_p)))
    D = C.c_void_p()
    arr = (C.c_void_p * 3)(*[p.handle.value for p in plans])
    cb.check(L.cove_dist_create(0, 1, idbuf.ctypes.data_as(C.c_void_p), arr, 3, n, 0, n, 0, n, 60000,
                                C.byref(D)))
    xd = torch.from_numpy(x).cuda()
    y = torch.full((n,), float("nan"), dtype=torch.float64, device="cuda")
    cb.check(L.cove_dist_spmv(D, C.c_void_p(xd.data_ptr()), C.c_void_p(y.data_ptr()),
                              C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    cb.check(L.cove_dist_destroy(D))
    rel = np.abs(y.cpu().numpy() - ref).max() / np.abs(ref).max()
    if codec == "original":
        assert rel <= 1e-12
    else:
        assert plans[0].info.dispatched_route == cb.ROUTE_BFP8_OUTLIER
        assert rel <= 1e-2  # the route's gate bound; outliers are exact
