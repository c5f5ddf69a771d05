"""CUDA path vs the oracle / the reference's own outputs (needs a B200).

Position and value streams are compared bit for bit; SpMV outputs are
compared normwise with the reference's global_rel metric
(max|y - y0| / max|y0|, structural/include/structural/spmv.hpp:73-89):
lossless routes within 1e-12 (fp64) / 1e-6 (fp32), lossy routes within the
reference's joint gate (1e-2) and within fp32-summation noise of the
oracle's emulation of the same decoded values.
"""
import numpy as np
import pytest

import cove_b200 as cb
import oracle as O
from conftest import case_names

pytestmark = pytest.mark.gpu

LOSSLESS_TOL = {np.float64: 1e-12, np.float32: 1e-6}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    yield


def plan_for(rows, cols, rp, ci, v, **opts):
    csr = cb.DeviceCsr.from_numpy(rows, cols, rp, ci, v)
    return cb.Plan(csr, **opts)


def gpu_spmv(plan, x, route=None):
    import torch

    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    yd = torch.full((plan.info.rows,), float("nan"), dtype=xd.dtype, device="cuda")
    plan.spmv(xd, yd, route=route)
    torch.cuda.synchronize()
    return yd.cpu().numpy()


def assert_streams_equal_split(p, s, dtype):
    assert np.array_equal(p.stream("kept_block_row_ptr"), s.kept.block_row_ptr)
    assert np.array_equal(p.stream("kept_block_col_idx"), s.kept.block_col_idx)
    assert np.array_equal(p.stream("kept_bitmap"), s.kept.bitmap_words)
    assert np.array_equal(p.stream("kept_values"), s.kept.values.astype(dtype))
    assert np.array_equal(p.stream("kept_block_val_ptr"), s.kept.block_val_ptr)
    assert np.array_equal(p.stream("res_row_ptr"), s.res_row_ptr)
    assert np.array_equal(p.stream("res_col_idx"), s.res_col_idx)
    assert np.array_equal(p.stream("res_values"), s.res_values.astype(dtype))
    i = p.info
    assert (i.kept_blocks, i.residual_blocks, i.cost_skipped_blocks) == (
        s.kept_blocks, s.residual_blocks, s.cost_skipped_blocks)
    assert (i.kept_nnz, i.residual_nnz, i.cost_skipped_nnz) == (
        s.kept_nnz, s.residual_nnz, s.cost_skipped_nnz)


def assert_lossless(y, rows, rp, ci, v, x, y_ref=None):
    """Lossless bound: normwise 1e-12 (fp64) / 1e-6 (fp32) against the exact
    product of the stored values (evaluated in fp64).  For fp32 the
    reference's own fp32-summed output is further off on long rows; it is
    checked against its float summation bound instead."""
    tol = LOSSLESS_TOL[v.dtype.type]
    y_exact = O.spmv_csr(rows, rp, ci, v.astype(np.float64), np.asarray(x, np.float64))
    rel = O.compare_vectors(y_exact, np.asarray(y, np.float64))[2]
    assert rel <= tol, rel
    if y_ref is not None:
        lens = np.diff(np.asarray(rp))
        bound = 1e-14 if v.dtype == np.float64 else 1e-7 * max(8.0, float(np.sqrt(lens.max())) * 4)
        assert O.compare_vectors(np.asarray(y_ref, np.float64), np.asarray(y, np.float64))[2] <= max(tol, bound)


def _kat_csr(k):
    return (k["rows"], k["cols"], np.array(k["row_ptr"], np.int64),
            np.array(k["col_idx"], np.int32), np.array(k["values"], np.float64))


@pytest.mark.parametrize("name", ["gpu_warp_direct_9x10", "gpu_warp_direct_empty_block_row",
                                  "gpu_workspace_second", "gpu_wide_block_span",
                                  "gpu_flag_lb_chunk2"])
def test_kat_full_bitbsr_matches_cpu_converter(kats, name):
    """test_gpu_convert.cu:124-296: GPU converter == convert_to_bitbsr(8x4)."""
    rows, cols, rp, ci, v = _kat_csr(kats[name])
    p = plan_for(rows, cols, rp, ci, v, keep_full_bitbsr=1)
    b = O.convert_to_bitbsr(rows, cols, rp, ci, v)
    assert np.array_equal(p.stream("full_block_row_ptr"), b.block_row_ptr)
    assert np.array_equal(p.stream("full_block_col_idx"), b.block_col_idx)
    assert np.array_equal(p.stream("full_bitmap"), b.bitmap_words)
    assert np.array_equal(p.stream("full_values"), b.values)
    assert np.array_equal(p.stream("full_block_row_val_ptr"), b.block_val_ptr[b.block_row_ptr])
    if name == "gpu_warp_direct_9x10":
        assert p.stream("full_block_row_val_ptr").tolist() == kats[name]["expect"]["block_row_val_ptr"]


@pytest.mark.parametrize("name,style", [("gpu_flag_lb_chunk2", "device"),
                                        ("gpu_split_threshold_chunking", "device"),
                                        ("gpu_flag_lb_chunk2", "hybrid")])
def test_kat_work_items(kats, name, style):
    k = kats[name]
    rows, cols, rp, ci, v = _kat_csr(k)
    p = plan_for(rows, cols, rp, ci, v, split_policy="none", lb_chunk_blocks=k["chunk"],
                 lb_split_threshold_blocks=k["split"], lb_style=style)
    b = O.convert_to_bitbsr(rows, cols, rp, ci, v)
    words, items, irp = O.lb_layout(b, k["chunk"], k["split"], style=style)
    assert np.array_equal(p.stream("words"), words)
    assert np.array_equal(p.stream("work_items"), items)
    assert np.array_equal(p.stream("work_item_row_ptr"), irp)
    if style == "device":
        assert p.stream("work_items").tolist() == k["expect"]["items"]
    y = gpu_spmv(p, np.arange(cols) % 13 * 0.25 - 1.5)
    y0 = O.spmv_csr(rows, rp, ci, v, np.arange(cols) % 13 * 0.25 - 1.5)
    assert O.compare_vectors(y0, y)[2] <= 1e-12


@pytest.mark.parametrize("name", ["cli_hybrid_4x8_thr2", "cli_hybrid_4x8_cost_b2"])
def test_kat_cli_counts(kats, name):
    k = kats[name]
    rows, cols, rp, ci, v = _kat_csr(k)
    c = k["cost"]
    p = plan_for(rows, cols, rp, ci, v, residual_threshold=k["threshold"], cost_bitmap_block=c[0],
                 cost_bitmap_nnz=c[1], cost_csr_block=c[2], cost_csr_nnz=c[3])
    for key, val in k["expect"].items():
        assert getattr(p.info, key) == val, key
    x = O.canonical_x(cols)
    assert O.compare_vectors(O.spmv_csr(rows, rp, ci, v, x), gpu_spmv(p, x))[2] <= 1e-12


SPLIT_OPTS = {"cost32": dict(residual_threshold=32),
              "thr2": dict(residual_threshold=2, split_policy="threshold"),
              "cost_b2": dict(residual_threshold=3, cost_bitmap_block=2.0)}


@pytest.mark.parametrize("split_key", sorted(SPLIT_OPTS))
def test_reference_cases_position_streams(ref_cases, split_key):
    d = ref_cases
    for name in case_names(d):
        rows, cols = (int(v) for v in d[f"{name}/shape"])
        rp, ci, v = d[f"{name}/row_ptr"], d[f"{name}/col_idx"], d[f"{name}/values"]
        p = plan_for(rows, cols, rp, ci, v, keep_full_bitbsr=1, long_row_split=16,
                     **SPLIT_OPTS[split_key])
        q = f"{name}/{split_key}/"
        assert np.array_equal(p.stream("kept_block_row_ptr"), d[q + "kept/block_row_ptr"]), name
        assert np.array_equal(p.stream("kept_block_col_idx"), d[q + "kept/block_col_idx"]), name
        assert np.array_equal(p.stream("kept_bitmap"), d[q + "kept/bitmap"]), name
        assert np.array_equal(p.stream("kept_block_val_ptr"), d[q + "kept/block_val_ptr"]), name
        assert np.array_equal(p.stream("kept_values"), d[q + "kept/values"]), name
        assert np.array_equal(p.stream("res_row_ptr"), d[q + "res/row_ptr"]), name
        assert np.array_equal(p.stream("res_col_idx"), d[q + "res/col_idx"]), name
        assert np.array_equal(p.stream("res_values"), d[q + "res/values"]), name
        if split_key == "cost32":
            assert np.array_equal(p.stream("full_block_row_ptr"), d[f"{name}/full/block_row_ptr"])
            assert np.array_equal(p.stream("full_block_col_idx"), d[f"{name}/full/block_col_idx"])
            assert np.array_equal(p.stream("full_bitmap"), d[f"{name}/full/bitmap"])
            assert np.array_equal(p.stream("full_values"), d[f"{name}/full/values"])
        # packed words, work items and long chunks against the oracle
        s = O.split(rows, cols, rp, ci, v, threshold=p.opts.residual_threshold,
                    use_cost=p.opts.split_policy == 0,
                    cost=(p.opts.cost_bitmap_block, 0.0, 0.0, 1.0))
        words, items, irp = O.lb_layout(s.kept, 32, 32, style="hybrid")
        assert np.array_equal(p.stream("words"), words), name
        assert np.array_equal(p.stream("work_items"), items), name
        assert np.array_equal(p.stream("work_item_row_ptr"), irp), name
        cr, cpb, cpc, nl = O.long_chunks(s.res_row_ptr, 16)
        assert np.array_equal(p.stream("chunk_row"), cr), name
        assert np.array_equal(p.stream("chunk_pbegin"), cpb), name
        assert np.array_equal(p.stream("chunk_pcount"), cpc), name
        assert p.info.long_rows == nl
        # lossless SpMV on the canonical x vs the reference's spmv_csr output
        x = d[f"{name}/canonical_x"]
        y = gpu_spmv(p, x)
        assert_lossless(y, rows, rp, ci, v, x, d[f"{name}/y_canonical"])


def _mask_for(opts):
    """CsrBitBsrSplitCostModel::should_move_to_residual (csr_bitbsr_split.hpp:66-73)
    tabulated over block populations 0..32, as the split API's predicate."""
    if opts.get("split_policy") == "threshold":
        return (1 << 33) - 1
    bb, bn, cb, cn = opts.get("cost_bitmap_block", 10.0), 0.0, 0.0, 1.0
    return sum(1 << p for p in range(33) if cb + cn * p < bb + bn * p)


@pytest.mark.parametrize("split_key", sorted(SPLIT_OPTS))
def test_reference_cases_mask_policy(ref_cases, split_key):
    """COVE_SPLIT_MASK with the tabulated predicate gives the reference's split."""
    d = ref_cases
    opts = SPLIT_OPTS[split_key]
    for name in case_names(d):
        rows, cols = (int(v) for v in d[f"{name}/shape"])
        rp, ci, v = d[f"{name}/row_ptr"], d[f"{name}/col_idx"], d[f"{name}/values"]
        p = plan_for(rows, cols, rp, ci, v, split_policy="mask", move_mask=_mask_for(opts),
                     residual_threshold=opts["residual_threshold"])
        ref = plan_for(rows, cols, rp, ci, v, **opts)
        q = f"{name}/{split_key}/"
        for stream, key in (("kept_block_row_ptr", "kept/block_row_ptr"), ("kept_block_col_idx", "kept/block_col_idx"),
                            ("kept_bitmap", "kept/bitmap"), ("kept_block_val_ptr", "kept/block_val_ptr"),
                            ("kept_values", "kept/values"), ("res_row_ptr", "res/row_ptr"),
                            ("res_col_idx", "res/col_idx"), ("res_values", "res/values")):
            assert np.array_equal(p.stream(stream), d[q + key]), (name, stream)
        for k in ("kept_blocks", "residual_blocks", "cost_skipped_blocks", "kept_nnz", "residual_nnz",
                  "cost_skipped_nnz"):
            assert getattr(p.info, k) == getattr(ref.info, k), (name, k)


def test_reference_cases_value_codecs(ref_cases):
    d = ref_cases
    for name in case_names(d):
        rows, cols = (int(v) for v in d[f"{name}/shape"])
        rp, ci, v = d[f"{name}/row_ptr"], d[f"{name}/col_idx"], d[f"{name}/values"]
        q = f"{name}/cost32/"
        p8 = plan_for(rows, cols, rp, ci, v, value_codec="bfp8")
        assert np.array_equal(p8.stream("bfp8_int8"), d[q + "bfp8/q"]), name
        assert np.array_equal(p8.stream("bfp8_scale"), d[q + "bfp8/scale"]), name
        assert np.array_equal(p8.stream("res_bf16"), O.bf16_half_up(d[q + "res/values"])), name
        po = plan_for(rows, cols, rp, ci, v, value_codec="bfp8_outlier")
        assert np.array_equal(po.stream("bfp8_int8"), d[q + "bfp8o/q"]), name
        assert np.array_equal(po.stream("bfp8_scale"), d[q + "bfp8o/scale"]), name
        assert np.array_equal(po.stream("outlier_rows"), d[q + "bfp8o/rows"]), name
        assert np.array_equal(po.stream("outlier_cols"), d[q + "bfp8o/cols"]), name
        assert np.array_equal(po.stream("outlier_vals"), d[q + "bfp8o/vals"]), name
        po5 = plan_for(rows, cols, rp, ci, v, value_codec="bfp8_outlier", outlier_fraction=0.05)
        assert np.array_equal(po5.stream("bfp8_int8"), d[q + "bfp8o5/q"]), name
        assert np.array_equal(po5.stream("outlier_rows"), d[q + "bfp8o5/rows"]), name
        pd = plan_for(rows, cols, rp, ci, v, value_codec="dict")
        uniq, cbk, kc, rc = O.dict_intern(d[q + "kept/values"], d[q + "res/values"])
        assert pd.info.value_cardinality == uniq
        if uniq <= 65536:
            assert np.array_equal(pd.stream("dict_codebook"), cbk), name
            assert np.array_equal(pd.stream("dict_kept_idx").astype(np.int32), kc), name
            assert np.array_equal(pd.stream("dict_res_idx").astype(np.int32), rc), name


def _joint_oracle(rows, cols, rp, ci, v, x, fraction=None):
    s = O.split(rows, cols, rp, ci, v)
    if fraction is None:
        q, sc = O.bfp8_encode(s.kept)
        orow = ocol = np.zeros(0, np.int32)
        oval = np.zeros(0, v.dtype)
    else:
        q, sc, orow, ocol, oval, _ = O.bfp8_outlier_encode(s.kept, fraction)
    rb = O.bf16_half_up(s.res_values)
    return O.joint_bfp8_spmv(s.kept, q, sc, s.res_row_ptr, s.res_col_idx, rb, orow, ocol, oval, x)


@pytest.mark.parametrize("codec", ["bfp8", "bfp8_outlier", "dict", "auto"])
def test_routes_spmv_and_gate(ref_cases, codec):
    d = ref_cases
    for name in case_names(d):
        rows, cols = (int(v) for v in d[f"{name}/shape"])
        rp, ci, v = d[f"{name}/row_ptr"], d[f"{name}/col_idx"], d[f"{name}/values"]
        p = plan_for(rows, cols, rp, ci, v, value_codec=codec, long_row_split=16)
        x = d[f"{name}/canonical_x"]
        y0 = d[f"{name}/y_canonical"]
        jr = p.info.joint_route
        y = gpu_spmv(p, x, route=jr)
        rel = O.compare_vectors(y0, y)[2]
        if jr in (cb.ROUTE_DICT_U8, cb.ROUTE_DICT_U16):
            assert_lossless(y, rows, rp, ci, v, x, y0)
        else:
            frac = 0.005 if jr == cb.ROUTE_BFP8_OUTLIER else None
            ye = _joint_oracle(rows, cols, rp, ci, v, x, frac)
            scale = max(np.abs(ye).max(), 1e-30)
            assert np.abs(ye - y).max() / scale <= 2e-6, name
            # the plan's gate value is this same global_rel (up to fp32 summation order)
            assert abs(p.info.joint_rel_err - rel) <= 1e-5 + 1e-3 * rel, name
            assert p.info.gate_pass == (rel <= 1e-2), name
            want = jr if p.info.gate_pass else cb.ROUTE_HYBRID
            assert p.info.dispatched_route == want


@pytest.mark.parametrize("codec", ["auto", "bfp8", "bfp8_outlier"])
def test_blocksparse_outlier_config_scaled(codec):
    """The block-sparse outlier matrix family at n = 2^16 (same block / entry densities,
    bf16-representable values in [-8, 8] with 0.1 % outliers of 1e5-1e6):
    position and value streams bit-exact, route choice and gate as the
    oracle decides them, and the dispatched SpMV within its route's bound."""
    rows, cols, rp, ci, v = cb.synth_blocksparse(1 << 16)
    assert np.abs(v).max() >= 1e5  # the outliers are there
    p = plan_for(rows, cols, rp, ci, v, value_codec=codec, long_row_split=256)
    s = O.split(rows, cols, rp, ci, v)
    assert_streams_equal_split(p, s, v.dtype)
    if codec == "auto":  # only auto and dict intern the values (the reference's menu)
        assert p.info.value_cardinality == -1 or p.info.value_cardinality > 256
    want_joint = cb.ROUTE_BFP8_OUTLIER if codec == "bfp8_outlier" else cb.ROUTE_BFP8
    assert p.info.joint_route == want_joint
    if codec == "bfp8_outlier":
        q, sc, orow, ocol, oval, _ = O.bfp8_outlier_encode(s.kept, 0.005)
        assert np.array_equal(p.stream("outlier_rows"), orow)
        assert np.array_equal(p.stream("outlier_cols"), ocol)
        assert np.array_equal(p.stream("outlier_vals"), oval)
    else:
        q, sc = O.bfp8_encode(s.kept)
    assert np.array_equal(p.stream("bfp8_int8"), q)
    assert np.array_equal(p.stream("bfp8_scale"), sc)
    # gate on the canonical x, as the reference evaluates it
    xc = O.canonical_x(cols)
    y0 = O.spmv_csr(rows, rp, ci, v, xc)
    ye = _joint_oracle(rows, cols, rp, ci, v, xc, 0.005 if codec == "bfp8_outlier" else None)
    rel = O.compare_vectors(y0, ye)[2]
    assert abs(p.info.joint_rel_err - rel) <= 1e-5 + 1e-3 * rel
    assert p.info.gate_pass == (rel <= 1e-2)
    assert p.info.dispatched_route == (want_joint if p.info.gate_pass else cb.ROUTE_HYBRID)
    # the dispatched route on the config's own x (N(0,1), seed 3)
    x = cb.synth_vector("normal", cols, seed=3)
    y = gpu_spmv(p, x)
    ref = O.spmv_csr(rows, rp, ci, v, x)
    bound = 1e-12 if p.info.dispatched_route == cb.ROUTE_HYBRID else 1e-2
    assert O.compare_vectors(ref, y)[2] <= bound


@pytest.mark.parametrize("dtype", ["f64", "f32"])
@pytest.mark.parametrize("codec", ["bfp8", "bfp8_outlier"])
def test_bfp8_long_block_rows(codec, dtype):
    """Block rows of more than 64 kept blocks (several 32-block batches each)
    take the segment-decoding BFP8 kernel: its output equals the oracle's
    emulation of the same codes within fp32 summation noise, for x read as
    32-byte, 16-byte and element loads (three alignments of the same x)."""
    import torch

    rows, cols, rp, ci, v = cb.synth_blocksparse(1 << 14, p_block=0.03, outlier_fraction=0.002, seed=5)
    if dtype == "f32":
        v = v.astype(np.float32)
    p = plan_for(rows, cols, rp, ci, v, value_codec=codec, long_row_split=256)
    assert p.info.kept_blocks >= 64 * ((rows + 7) // 8)  # the segment kernel's rule
    frac = 0.005 if codec == "bfp8_outlier" else None
    x = cb.synth_vector("normal", cols, seed=3).astype(v.dtype)
    ye = _joint_oracle(rows, cols, rp, ci, v, x, frac)
    scale = max(np.abs(ye).max(), 1e-30)
    tdt = torch.float64 if v.dtype == np.float64 else torch.float32
    for off in (0, 1, 2, 4):  # elements past a 512-byte aligned allocation
        buf = torch.zeros(cols + 8, dtype=tdt, device="cuda")
        xd = buf[off:off + cols]
        xd.copy_(torch.from_numpy(x))
        yd = torch.full((rows,), float("nan"), dtype=tdt, device="cuda")
        p.spmv(xd, yd, route=p.info.joint_route)
        torch.cuda.synchronize()
        y = yd.cpu().numpy().astype(np.float64)
        assert np.abs(ye - y).max() / scale <= 2e-6, off


@pytest.mark.parametrize("codec", ["bfp8", "bfp8_outlier"])
def test_bfp8_long_block_rows_heavy_and_ragged(codec):
    """The segment-decoding BFP8 kernel with a ragged last block row (n not a
    multiple of 8) and one block row of 3000 kept blocks, beyond the heavy
    limit, whose tail the overflow launch finishes: output equals the
    oracle's emulation of the same codes within fp32 summation noise."""
    rng = np.random.default_rng(7)
    rows, cols, rp, ci, v = cb.synth_blocksparse(16387, p_block=0.03, outlier_fraction=0.002, seed=7)
    heavy = range(800, 808)  # block row 100
    blocks = np.sort(rng.choice((cols + 3) // 4, 3000, replace=False))
    cells = (blocks[:, None] * 4 + np.arange(4)[None, :]).ravel()
    cells = cells[cells < cols]
    new_rp, new_ci, new_v = [0], [], []
    for r in range(rows):
        if r in heavy:
            c = np.sort(cells[rng.random(cells.size) < 0.6]).astype(np.int32)
            val = rng.integers(1, 64, c.size) * rng.choice([-0.125, 0.125], c.size)  # bf16-exact, nonzero
        else:
            c, val = ci[rp[r]:rp[r + 1]], v[rp[r]:rp[r + 1]]
        new_ci.append(c)
        new_v.append(val)
        new_rp.append(new_rp[-1] + c.size)
    rp = np.array(new_rp, np.int64)
    ci = np.concatenate(new_ci).astype(np.int32)
    v = np.concatenate(new_v).astype(np.float64)
    x = cb.synth_vector("normal", cols, seed=3)
    frac = 0.005 if codec == "bfp8_outlier" else None
    for dt in (np.float64, np.float32):
        vv, xx = v.astype(dt), x.astype(dt)
        p = plan_for(rows, cols, rp, ci, vv, value_codec=codec, long_row_split=256, gate_enable=0)
        assert p.info.kept_blocks >= 64 * ((rows + 7) // 8)  # the segment kernel's rule
        assert p.info.kernel_overflow_tasks > 0  # the heavy block row's tail
        ye = _joint_oracle(rows, cols, rp, ci, vv, xx, frac)
        y = gpu_spmv(p, xx, route=p.info.joint_route).astype(np.float64)
        assert np.abs(ye - y).max() / max(np.abs(ye).max(), 1e-30) <= 2e-6, dt


def test_auto_route_choice_matches_reference_rule():
    # uniq <= 256 -> dict_u8; > 256 -> bfp8 (main_gpu_csr_bitbsr_spmv.cu:1244-1245)
    rows, cols, rp, ci, v = cb.synth_lapl2d(64, 64)
    p = plan_for(rows, cols, rp, ci, v, value_codec="auto")
    assert p.info.value_cardinality == 2 and p.info.joint_route == cb.ROUTE_DICT_U8
    assert p.info.dispatched_route == cb.ROUTE_DICT_U8
    assert p.stream("dict_codebook").tolist() == [4.0, -1.0]
    v2 = v.copy()
    v2[::3] = np.arange(v2[::3].size) + 5.0  # many distinct values
    p2 = plan_for(rows, cols, rp, ci, v2, value_codec="auto")
    assert p2.info.value_cardinality > 256 and p2.info.joint_route == cb.ROUTE_BFP8
    p3 = plan_for(rows, cols, rp, ci, v2, value_codec="dict")
    assert p3.info.joint_route == cb.ROUTE_DICT_U16
    x = O.canonical_x(cols)
    assert O.compare_vectors(O.spmv_csr(rows, rp, ci, v2, x), gpu_spmv(p3, x))[2] <= 1e-12


def test_gate_failure_falls_back_to_lossless():
    # each row holds a cancelling pair 1000 + d, -1000 in two sparse blocks whose x
    # entries are equal (columns 136 = 8 * 17 apart): bf16 cannot hold d, so the
    # joint output loses the whole row value and the gate must reject it
    rows, cols = 256, 400
    rp = np.arange(0, 2 * rows + 1, 2, dtype=np.int64)
    ci = np.stack([np.arange(rows), np.arange(rows) + 136], 1).reshape(-1).astype(np.int32)
    v = np.stack([1000.0 + 0.123 + 1e-3 * np.arange(rows), -1000.0 * np.ones(rows)], 1).reshape(-1)
    p = plan_for(rows, cols, rp, ci, v, value_codec="bfp8")
    assert p.info.gate_evaluated == 1 and p.info.joint_rel_err > 1e-2
    assert p.info.gate_pass == 0 and p.info.dispatched_route == cb.ROUTE_HYBRID
    x = O.canonical_x(cols)
    y = np.empty(rows)
    p.spmv_host(x, y)
    assert O.compare_vectors(O.spmv_csr(rows, rp, ci, v, x), y)[2] <= 1e-12


def test_edge_cases():
    import torch

    # empty matrix
    p = plan_for(3, 4, np.zeros(4, np.int64), np.zeros(0, np.int32), np.zeros(0))
    y = gpu_spmv(p, np.ones(4))
    assert np.all(y == 0)
    # stored zeros only
    p = plan_for(2, 4, np.array([0, 2, 3]), np.array([0, 1, 2], np.int32), np.zeros(3))
    assert p.info.nnz == 0 and np.all(gpu_spmv(p, np.ones(4)) == 0)
    # int32 row_ptr input
    rows, cols, rp, ci, v = cb.synth_lapl2d(16, 16)
    csr = cb.DeviceCsr(rows, cols, torch.from_numpy(rp.astype(np.int32)).cuda(),
                       torch.from_numpy(ci).cuda(), torch.from_numpy(v).cuda())
    p = cb.Plan(csr)
    x = O.canonical_x(cols)
    assert O.compare_vectors(O.spmv_csr(rows, rp, ci, v, x), gpu_spmv(p, x))[2] <= 1e-12
    # invalid inputs return status codes (validation on the device)
    bad = [
        (np.array([0, 2, 1, 3]), np.array([0, 1, 2], np.int32), "monotonic"),
        (np.array([0, 2, 2, 3]), np.array([1, 0, 2], np.int32), "strictly increasing"),
        (np.array([0, 2, 2, 3]), np.array([1, 1, 2], np.int32), "strictly increasing"),
        (np.array([0, 2, 2, 3]), np.array([0, 9, 2], np.int32), "out of range"),
        # an offset above nnz is a non-monotonic row_ptr; the row is not read
        (np.array([0, 5000, 1, 3]), np.array([0, 1, 2], np.int32), "monotonic"),
        # an order error before a range error in one row: the range error is reported
        (np.array([0, 3, 3, 3]), np.array([1, 0, 9], np.int32), "out of range"),
    ]
    for rp_b, ci_b, msg in bad:
        with pytest.raises(cb.CoveError, match=msg):
            plan_for(3, 4, rp_b, ci_b, np.ones(3))


def _heavy_rows_csr(seed=31):
    """64 x 200000 with three 6000-entry rows (two in one block row), 300-entry
    rows and 7-entry rows; 5 % stored zeros, columns in order."""
    rng = np.random.default_rng(seed)
    rows, cols = 64, 200000
    lists = [np.unique(rng.integers(0, cols, 6000 if r in (3, 17, 18) else (300 if r % 5 == 0 else 7)))
             for r in range(rows)]
    rp = np.zeros(rows + 1, np.int64)
    rp[1:] = np.cumsum([len(c) for c in lists])
    ci = np.concatenate(lists).astype(np.int32)
    v = rng.standard_normal(ci.size)
    v[rng.random(ci.size) < 0.05] = 0.0
    return rows, cols, rp, ci, v


def _step_api_full(rows, cols, rp, ci, v):
    """cove_bitbsr8x4_count + cove_bitbsr8x4_fill into caller buffers."""
    import ctypes as C

    import torch

    csr = cb.DeviceCsr.from_numpy(rows, cols, rp, ci, v)
    d = csr.desc()
    nbr = (rows + 7) // 8
    brp = torch.empty(nbr + 1, dtype=torch.int32, device="cuda")
    brvp = torch.empty(nbr + 1, dtype=torch.int32, device="cuda")
    nb, nz = C.c_int64(), C.c_int64()
    L = cb.lib()
    cb.check(L.cove_bitbsr8x4_count(C.byref(d), C.c_void_p(brp.data_ptr()), C.c_void_p(brvp.data_ptr()),
                                    C.byref(nb), C.byref(nz), None))
    col = torch.empty(max(nb.value, 1), dtype=torch.int32, device="cuda")
    bm = torch.empty(max(nb.value, 1), dtype=torch.int32, device="cuda")
    vals = torch.empty(max(nz.value, 1), dtype=csr.values.dtype, device="cuda")
    cb.check(L.cove_bitbsr8x4_fill(C.byref(d), C.c_void_p(brp.data_ptr()), C.c_void_p(brvp.data_ptr()),
                                   C.c_void_p(col.data_ptr()), C.c_void_p(bm.data_ptr()),
                                   C.c_void_p(vals.data_ptr()), None))
    torch.cuda.synchronize()
    return (brp.cpu().numpy(), brvp.cpu().numpy(), col.cpu().numpy()[: nb.value],
            bm.cpu().numpy().view(np.uint32)[: nb.value], vals.cpu().numpy()[: nz.value])


@pytest.mark.parametrize("zeros", ["in_order", "out_of_order"])
def test_heavy_block_rows_convert_in_pieces(zeros):
    """Block rows with more than 1024 CSR entries are converted as
    column-range pieces (each row binary-searched for the range); with a
    stored zero out of column order the converter keeps one piece per block
    row.  Both give the reference converter's streams bit for bit, through
    the plan and through the step-by-step count / fill calls."""
    rows, cols, rp, ci, v = _heavy_rows_csr()
    if zeros == "out_of_order":
        q = rp[17] + 10  # a stored zero whose column goes back: valid CSR, zeros are ignored
        v[q] = 0.0
        ci[q] = ci[rp[17]]
    b = O.convert_to_bitbsr(rows, cols, rp, ci, v)
    p = plan_for(rows, cols, rp, ci, v, keep_full_bitbsr=1, value_codec="original")
    assert np.array_equal(p.stream("full_block_row_ptr"), b.block_row_ptr)
    assert np.array_equal(p.stream("full_block_col_idx"), b.block_col_idx)
    assert np.array_equal(p.stream("full_bitmap"), b.bitmap_words)
    assert np.array_equal(p.stream("full_values"), b.values)
    assert np.array_equal(p.stream("full_block_row_val_ptr"), b.block_val_ptr[b.block_row_ptr])
    # the split of these block rows (more than 2048 blocks: split in pieces)
    assert_streams_equal_split(p, O.split(rows, cols, rp, ci, v), v.dtype)
    pt = plan_for(rows, cols, rp, ci, v, split_policy="threshold", residual_threshold=2, value_codec="original")
    assert_streams_equal_split(pt, O.split(rows, cols, rp, ci, v, threshold=2, use_cost=False), v.dtype)
    brp, brvp, col, bm, vals = _step_api_full(rows, cols, rp, ci, v)
    assert np.array_equal(brp, b.block_row_ptr) and np.array_equal(brvp, b.block_val_ptr[b.block_row_ptr])
    assert np.array_equal(col, b.block_col_idx) and np.array_equal(bm, b.bitmap_words)
    assert np.array_equal(vals, b.values)
    x = cb.synth_vector("uniform_pm1", cols, seed=9)
    y = gpu_spmv(p, x)
    assert O.compare_vectors(O.spmv_csr(rows, rp, ci, v, x), y)[2] <= 1e-12


def test_long_row_validation_follows_the_reference_priority():
    """Rows longer than 256 entries are validated in 2048-entry units, a lane
    per entry.  As in the reference (every column's range is checked before
    the converter meets a duplicate), a range error anywhere outranks an
    order error."""
    rows, cols, rp, ci, v = _heavy_rows_csr(seed=5)
    v[:] = 1.0
    r = 3  # a 6000-entry row
    dup = ci.copy()
    dup[rp[r] + 100] = dup[rp[r] + 99]  # duplicate at entry 100 ...
    with pytest.raises(cb.CoveError, match="strictly increasing"):
        plan_for(rows, cols, rp, dup, v)
    dup[rp[r] + 5000] = cols + 5  # ... and out of range at entry 5000, in another unit
    with pytest.raises(cb.CoveError, match="out of range"):
        plan_for(rows, cols, rp, dup, v)
    oor = ci.copy()
    oor[rp[r] + 4000] = -1
    with pytest.raises(cb.CoveError, match="out of range"):
        plan_for(rows, cols, rp, oor, v)
    z = v.copy()  # a zero between two equal columns is fine; the equal nonzeros are not
    eq = ci.copy()
    eq[rp[r] + 301] = eq[rp[r] + 300]
    z[rp[r] + 300] = 0.0
    plan_for(rows, cols, rp, eq, z)
    z[rp[r] + 300] = 1.0
    with pytest.raises(cb.CoveError, match="strictly increasing"):
        plan_for(rows, cols, rp, eq, z)


def test_long_rows_and_heavy_block_rows_overflow_path():
    """Residual rows beyond the kernel's row split and block rows beyond the
    heavy limit go through the second launch; results stay exact."""
    rng = np.random.default_rng(11)
    rows, cols = 4096, 40000
    rp = [0]
    ci = []
    for r in range(rows):
        if r == 5:
            cs = np.arange(0, cols, 3)  # very long residual-ish row
        elif 64 <= r < 72:
            cs = np.arange(0, cols, 1)[: 20000]  # one block row with 5000 dense blocks
        else:
            cs = np.unique(rng.integers(0, cols, 6))
        ci.extend(cs.tolist())
        rp.append(len(ci))
    rp = np.array(rp, np.int64)
    ci = np.array(ci, np.int32)
    v = rng.standard_normal(ci.size)
    # the dense block row (5000 kept blocks) is split in pieces
    assert_streams_equal_split(plan_for(rows, cols, rp, ci, v, value_codec="original"),
                               O.split(rows, cols, rp, ci, v), v.dtype)
    for codec in ("original", "bfp8_outlier"):
        p = plan_for(rows, cols, rp, ci, v, value_codec=codec, gate_enable=0)
        assert p.info.kernel_overflow_tasks > 0
        assert p.launches() == 2
        x = O.canonical_x(cols)
        y0 = O.spmv_csr(rows, rp, ci, v, x)
        y = gpu_spmv(p, x, route=p.info.joint_route)
        if codec == "original":
            assert O.compare_vectors(y0, y)[2] <= 1e-12
        else:
            assert O.compare_vectors(y0, y)[2] <= 1e-2


def test_lane_per_row_kernel_with_overflow_pieces():
    """A 5-point Laplacian selects the one-lane-per-row kernel; a long residual
    row and a dense block row added to it go to the overflow pass."""
    import scipy.sparse as sp

    rows, cols, rp, ci, v = cb.synth_lapl2d(256, 256)
    A = sp.csr_matrix((v, ci, rp), shape=(rows, cols)).tolil()
    rng = np.random.default_rng(5)
    A[77, np.arange(0, cols, 21)] = rng.standard_normal(len(range(0, cols, 21)))  # long residual row
    for r in range(800, 808):  # one block row with 300 dense 8x4 blocks
        A[r, 4000:5200] = rng.standard_normal(1200)
    A = A.tocsr()
    A.sort_indices()
    p = plan_for(rows, cols, A.indptr.astype(np.int64), A.indices.astype(np.int32), A.data,
                 value_codec="original", gate_enable=0)
    assert p.info.kernel_slots == 0
    assert p.info.kernel_overflow_tasks > 0 and p.launches() == 2
    x = cb.synth_vector("uniform_pm1", cols, seed=8)
    y = gpu_spmv(p, x)
    ref = A @ x
    assert np.abs(y - ref).max() <= 1e-12 * np.abs(ref).max()


def _slot_matrix(kind):
    import scipy.sparse as sp

    rng = np.random.default_rng(21)
    n = 1 << 16
    if kind.startswith("random"):  # k random columns a row, no 8x4 structure
        k = int(kind[6:])
        rows = np.repeat(np.arange(n), k)
        A = sp.csr_matrix((rng.uniform(-1, 1, n * k), (rows, rng.integers(0, n, n * k))), shape=(n, n))
    elif kind == "banded":  # 24 scattered diagonals: neighbouring rows read neighbouring x
        offs = [0, 1, -1, 3, -3, 7, -7, 9, -9, 20, -20, 33, -33, 64, -64, 77, 200, -200, 513, -513,
                1000, -1000, 4096, -4096]
        A = sp.diags([rng.uniform(-1, 1, n - abs(o)) for o in offs], offs, shape=(n, n), format="csr")
    else:  # power law: 400 rows of 400 entries hold most of the residual, the rest 2 a row
        heavy = rng.choice(n, 400, replace=False)
        lens = np.full(n, 2)
        lens[heavy] = 400
        rows = np.repeat(np.arange(n), lens)
        A = sp.csr_matrix((rng.uniform(-1, 1, rows.size), (rows, rng.integers(0, n, rows.size))), shape=(n, n))
    A.sum_duplicates()
    A.sort_indices()
    return A


@pytest.mark.parametrize("kind,slots", [("random8", 0), ("banded", 0), ("powerlaw", 0), ("random16", 2),
                                        ("random40", 4)])
def test_slot_rule_from_residual_profile(kind, slots):
    """The kernel choice follows the residual rows' shape: short light rows, a
    diagonal structure or long heavy rows take one lane per row; longer
    random rows take 2 or 4 lanes per block row.  Every choice stays exact."""
    A = _slot_matrix(kind)
    n = A.shape[0]
    p = plan_for(n, n, A.indptr.astype(np.int64), A.indices.astype(np.int32), A.data,
                 value_codec="original", gate_enable=0)
    assert p.info.kernel_slots == slots
    x = cb.synth_vector("uniform_pm1", n, seed=3)
    y = gpu_spmv(p, x)
    ref = A @ x
    assert np.abs(y - ref).max() <= 1e-12 * np.abs(ref).max()


def test_spmv_rejects_mismatched_vectors():
    """The C ABI takes bare pointers; the Python plan checks element type,
    device and length before the call."""
    import torch

    rows, cols, rp, ci, v = cb.synth_lapl2d(32, 32)
    p = plan_for(rows, cols, rp, ci, v.astype(np.float32), value_codec="original")
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    with pytest.raises(cb.CoveError, match="plan computes in"):
        p.spmv(torch.zeros(cols, dtype=torch.float64, device="cuda"), y)
    with pytest.raises(cb.CoveError, match="at least"):
        p.spmv(torch.zeros(cols - 1, dtype=torch.float32, device="cuda"), y)
    with pytest.raises(cb.CoveError, match="CUDA tensor"):
        p.spmv(torch.zeros(cols, dtype=torch.float32), y)


def test_spmv_host_matches_device():
    rows, cols, rp, ci, v = cb.synth_fem27(12, 10, 9, 3, seed=5)
    p = plan_for(rows, cols, rp, ci, v, value_codec="auto")
    x = cb.synth_vector("uniform_pm1", cols, seed=1)
    yh = p.spmv_host(x)
    yd = gpu_spmv(p, x)
    assert np.array_equal(yh, yd)  # same kernel, deterministic stores


def _pinned(n):
    import torch

    return torch.empty(n, dtype=torch.float64, pin_memory=True).numpy()


@pytest.mark.parametrize("long_row", [False, True])
def test_spmv_host_sliced_overlap_matches_device(long_row):
    """Pinned host buffers of a few MB take the sliced path (x slices in, block-row
    slices of the main pass, y slices out on a second copy stream); with a long
    residual row the y copy waits for the overflow pass instead."""
    rows, cols, rp, ci, v = cb.synth_lapl3d(100, 100, 100)
    if long_row:
        lc = np.arange(0, cols, 3, dtype=np.int32)
        a, b = rp[5], rp[6]
        ci = np.concatenate([ci[:a], lc, ci[b:]])
        v = np.concatenate([v[:a], np.linspace(-1.0, 1.0, lc.size), v[b:]])
        rp = rp.astype(np.int64)
        rp[6:] += lc.size - (b - a)
    p = plan_for(rows, cols, rp, ci, v, value_codec="auto", long_row_split=256)
    assert (p.info.kernel_overflow_tasks > 0) == long_row
    x = cb.synth_vector("uniform_pm1", cols, seed=3)
    yd = gpu_spmv(p, x)
    xh = _pinned(cols)
    xh[:] = x
    for _ in range(2):  # first call builds the slices, second reuses them
        yh = _pinned(rows)
        yh[:] = np.nan
        p.spmv_host(xh, yh)
        if long_row:  # the long row's chunks add in any order
            assert np.abs(yh - yd).max() <= 1e-12 * np.abs(yd).max()
        else:
            assert np.array_equal(yh, yd)
    assert np.array_equal(p.spmv_host(x), yd) or long_row  # pageable buffers: one-shot path


def test_spmv_host_sliced_segment_kernel_matches_device():
    """The host path's block-row slices run the segment-decoding BFP8 kernel
    from each slice's first block row: the same rows, bit for bit."""
    rows, cols, rp, ci, v = cb.synth_blocksparse(1 << 18, outlier_fraction=0.0)  # 131 kept blocks a block row
    p = plan_for(rows, cols, rp, ci, v, value_codec="bfp8", long_row_split=256, gate_enable=0)
    assert p.info.kept_blocks >= 64 * ((rows + 7) // 8)
    assert p.info.dispatched_route == cb.ROUTE_BFP8 and p.launches() == 1
    x = cb.synth_vector("normal", cols, seed=3)
    yd = gpu_spmv(p, x)
    xh = _pinned(cols)
    xh[:] = x
    for _ in range(2):
        yh = _pinned(rows)
        yh[:] = np.nan
        p.spmv_host(xh, yh)
        assert np.array_equal(yh, yd)


@pytest.mark.parametrize("cfg", ["lapl2d_512", "fem27_64", "rmat_22"])
def test_full_size_configs(cfg):
    """2D Laplacian 512^2, FEM 27-point 64^3 and R-MAT 2^22 at full size:
    streams bit-exact, routes, SpMV."""
    rows, cols, rp, ci, v, x = cb.workload(cfg)
    opts = dict(value_codec="auto", long_row_split=256)
    p = plan_for(rows, cols, rp, ci, v, **opts)
    s = O.split(rows, cols, rp, ci, v)
    assert_streams_equal_split(p, s, v.dtype)
    words, items, irp = O.lb_layout(s.kept, 32, 32, style="hybrid")
    assert np.array_equal(p.stream("words"), words)
    assert np.array_equal(p.stream("work_items"), items)
    cr, cpb, cpc, nl = O.long_chunks(s.res_row_ptr, 256)
    assert np.array_equal(p.stream("chunk_row"), cr) and np.array_equal(p.stream("chunk_pbegin"), cpb)
    want_route = {"lapl2d_512": cb.ROUTE_DICT_U8, "fem27_64": cb.ROUTE_BFP8,
                  "rmat_22": cb.ROUTE_BFP8}[cfg]
    assert p.info.joint_route == want_route
    y0 = O.spmv_csr(rows, rp, ci, v, x)
    yl = gpu_spmv(p, x, route=cb.ROUTE_HYBRID)
    assert_lossless(yl, rows, rp, ci, v, x, y0)
    yj = gpu_spmv(p, x, route=want_route)
    if want_route == cb.ROUTE_DICT_U8:
        assert_lossless(yj, rows, rp, ci, v, x, y0)
    else:
        q, sc = O.bfp8_encode(s.kept)
        assert np.array_equal(p.stream("bfp8_int8"), q) and np.array_equal(p.stream("bfp8_scale"), sc)
        ye = O.joint_bfp8_spmv(s.kept, q, sc, s.res_row_ptr, s.res_col_idx,
                               O.bf16_half_up(s.res_values), np.zeros(0, np.int32),
                               np.zeros(0, np.int32), np.zeros(0, v.dtype), x)
        # fp32 sums in two different orders: bounded by the longest row's
        # float summation error (R-MAT rows reach ~10^5 entries)
        lens = np.diff(rp)
        bound = 1e-7 * max(16.0, 4.0 * float(np.sqrt(lens.max())))
        assert np.abs(ye - yj).max() / np.abs(ye).max() <= bound
        # gate decision = the oracle's on the canonical x
        xc = O.canonical_x(cols, v.dtype)
        yc0 = O.spmv_csr(rows, rp, ci, v, xc)
        yce = O.joint_bfp8_spmv(s.kept, q, sc, s.res_row_ptr, s.res_col_idx,
                                O.bf16_half_up(s.res_values), np.zeros(0, np.int32),
                                np.zeros(0, np.int32), np.zeros(0, v.dtype), xc)
        rel = O.compare_vectors(yc0, yce)[2]
        assert p.info.gate_pass == (rel <= 1e-2)
        assert abs(p.info.joint_rel_err - rel) <= 1e-4 * max(rel, 1e-6) + 1e-6
