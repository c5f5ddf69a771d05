"""The CPU oracle, pinned to the reference (no GPU).

1. Known-answer vectors transcribed from the reference's own tests
   (tests/golden/reference_kats.json, each with its source lines).
2. Outputs of the reference's own host code on seeded random matrices
   (tests/golden/ref_cases.npz, made by tests/golden/make_golden.py).
3. When oracle/_ref is built here, a live comparison on fresh inputs.
"""
import numpy as np
import pytest

import oracle as O
from conftest import case_names


def _csr(k, dtype=np.float64):
    return (k["rows"], k["cols"], np.array(k["row_ptr"], np.int64),
            np.array(k["col_idx"], np.int32), np.array(k["values"], dtype))


def test_kat_bitbsr_2x2_offsets(kats):
    k = kats["bitbsr_2x2_offsets"]
    b = O.convert_to_bitbsr(*_csr(k), br=k["br"], bc=k["bc"])
    e = k["expect"]
    assert b.num_blocks == e["num_blocks"]
    assert b.block_row_ptr.tolist() == e["block_row_ptr"]
    assert b.block_col_idx.tolist() == e["block_col_idx"]
    assert b.block_val_ptr.tolist() == e["block_val_ptr"]
    assert b.bitmap_words.tolist() == e["bitmap_words"]
    assert b.values.tolist() == e["values"]


def test_kat_spmv(kats):
    k = kats["bitbsr_2x2_spmv"]
    rows, cols, rp, ci, v = _csr(k)
    y = O.spmv_csr(rows, rp, ci, v, np.array(k["x"], np.float64))
    assert y.tolist() == k["expect"]["y"]


def test_kat_drops_zeros(kats):
    k = kats["bitbsr_drops_zeros"]
    b = O.convert_to_bitbsr(*_csr(k), br=k["br"], bc=k["bc"])
    assert b.nnz == k["expect"]["nnz"]
    assert b.values.tolist() == k["expect"]["values"]


@pytest.mark.parametrize("name", ["split_threshold_2x2", "split_cost_gated_2x2",
                                  "cli_hybrid_4x8_thr2", "cli_hybrid_4x8_cost_b2"])
def test_kat_split(kats, name):
    k = kats[name]
    br, bc = k.get("br", 8), k.get("bc", 4)
    cost = tuple(k.get("cost", O.DEFAULT_COST))
    s = O.split(*_csr(k), br=br, bc=bc, threshold=k["threshold"], use_cost=k["use_cost"], cost=cost)
    e = k["expect"]
    got = {"kept_blocks": s.kept_blocks, "residual_blocks": s.residual_blocks,
           "cost_skipped_blocks": s.cost_skipped_blocks, "kept_nnz": s.kept_nnz,
           "residual_nnz": s.residual_nnz, "cost_skipped_nnz": s.cost_skipped_nnz,
           "kept_block_row_ptr": s.kept.block_row_ptr.tolist(),
           "kept_block_col_idx": s.kept.block_col_idx.tolist(),
           "res_row_ptr": s.res_row_ptr.tolist(), "res_col_idx": s.res_col_idx.tolist(),
           "res_values": s.res_values.tolist()}
    for key, val in e.items():
        assert got[key] == val, key


def test_kat_block_row_val_ptr(kats):
    k = kats["gpu_warp_direct_9x10"]
    b = O.convert_to_bitbsr(*_csr(k))
    brvp = b.block_val_ptr[b.block_row_ptr]
    assert brvp.tolist() == k["expect"]["block_row_val_ptr"]


@pytest.mark.parametrize("name", ["gpu_flag_lb_chunk2", "gpu_split_threshold_chunking"])
def test_kat_device_layout(kats, name):
    k = kats[name]
    b = O.convert_to_bitbsr(*_csr(k))
    words, items, _ = O.lb_layout(b, k["chunk"], k["split"], style=k["style"])
    assert items.tolist() == k["expect"]["items"]
    flagged = [i for i, w in enumerate(words) if int(w) & 0x80000000]
    assert flagged == k["expect"]["flagged_blocks"]


def test_kat_wide_block_span(kats):
    k = kats["gpu_wide_block_span"]
    b = O.convert_to_bitbsr(*_csr(k))
    assert b.block_col_idx.tolist() == k["expect"]["block_col_idx"]
    words, items, _ = O.lb_layout(b, 32, 32, style="hybrid")
    want = [(bm << 32) | col for bm, col in k["expect"]["words_unflagged"]]
    assert [int(w) for w in words] == want
    words, items, _ = O.lb_layout(b, 1, 1, style="device")
    assert items[:, 2].tolist() == k["expect"]["device_layout_chunk1"]["block_counts"]
    assert all(int(w) & 0x80000000 for w in words)


def test_hybrid_layout_empty_rows_and_flags():
    """Host layout (main_gpu_csr_bitbsr_spmv.cu:429-458): empty block rows emit an
    item with count 0, long block rows are cut and flagged on every piece."""
    rows, cols = 24, 400
    rp = [0] * 9 + [0] * 8 + [0] * 8
    ci, v = [], []
    # block row 0: 5 blocks in row 0; block row 1 empty; block row 2: 2 blocks
    rowsets = {0: [0, 4, 8, 12, 16], 16: [0, 100]}
    rp = [0]
    for r in range(rows):
        cs = rowsets.get(r, [])
        ci += cs
        v += [1.0] * len(cs)
        rp.append(len(ci))
    b = O.convert_to_bitbsr(rows, cols, np.array(rp), np.array(ci, np.int32), np.array(v))
    words, items, irp = O.lb_layout(b, 2, 2, style="hybrid")
    assert items.tolist() == [[0, 0, 2, 0], [0, 2, 2, 2], [0, 4, 1, 4], [1, 5, 0, 5], [2, 5, 2, 5]]
    assert irp.tolist() == [0, 3, 4, 5]
    flags = [bool(int(w) & 0x80000000) for w in words]
    assert flags == [True, False, True, False, True, False, False]


def test_cost_model_table():
    """should_move_to_residual with the default model moves blocks of <= 9 nnz."""
    moves = [bool(O._lib().oc_cost_model_moves(10.0, 0.0, 0.0, 1.0, n)) for n in range(0, 33)]
    assert moves == [n < 10 for n in range(0, 33)]


def test_bf16_rounding_matches_reference_helper():
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.standard_normal(200), [1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -0.0]])
    for v in vals.astype(np.float32):
        want = O.ref_float_to_bf16_bits(float(v)) if O.ref_available() else None
        got = O.float_to_bf16_bits(float(v))
        if want is not None:
            assert got == want


def test_bf16_half_up_residual_rule():
    # (u + 0x8000) >> 16: halves round away on the magnitude, no tie-to-even
    v = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -(1.0 + 2 ** -8)], np.float32)
    got = O.bf16_half_up(v)
    assert got.tolist() == [0x3F81, 0x3F82, 0xBF81]


@pytest.mark.parametrize("split_key", ["cost32", "thr2", "cost_b2"])
def test_oracle_matches_reference_outputs(ref_cases, split_key):
    d = ref_cases
    costs = {"cost32": (32, True, (10.0, 0.0, 0.0, 1.0)), "thr2": (2, False, O.DEFAULT_COST),
             "cost_b2": (3, True, (2.0, 0.0, 0.0, 1.0))}
    thr, use_cost, cost = costs[split_key]
    for name in case_names(d):
        rows, cols = (int(v) for v in d[f"{name}/shape"])
        rp, ci, v = d[f"{name}/row_ptr"], d[f"{name}/col_idx"], d[f"{name}/values"]
        s = O.split(rows, cols, rp, ci, v, threshold=thr, use_cost=use_cost, cost=cost)
        q = f"{name}/{split_key}/"
        assert np.array_equal(s.kept.block_row_ptr, d[q + "kept/block_row_ptr"]), name
        assert np.array_equal(s.kept.block_col_idx, d[q + "kept/block_col_idx"]), name
        assert np.array_equal(s.kept.bitmap_words, d[q + "kept/bitmap"]), name
        assert np.array_equal(s.kept.block_val_ptr, d[q + "kept/block_val_ptr"]), name
        assert np.array_equal(s.kept.values, d[q + "kept/values"]), name
        assert np.array_equal(s.res_row_ptr, d[q + "res/row_ptr"]), name
        assert np.array_equal(s.res_col_idx, d[q + "res/col_idx"]), name
        assert np.array_equal(s.res_values, d[q + "res/values"]), name
        names = list(d[q + "counter_names"])
        cnt = dict(zip(names, d[q + "counters"].tolist()))
        assert cnt["kept_blocks"] == s.kept_blocks and cnt["residual_blocks"] == s.residual_blocks
        assert cnt["cost_skipped_blocks"] == s.cost_skipped_blocks
        assert cnt["kept_nnz"] == s.kept_nnz and cnt["residual_nnz"] == s.residual_nnz
        assert cnt["cost_skipped_nnz"] == s.cost_skipped_nnz
        if split_key == "cost32":
            assert np.array_equal(s.full.block_row_ptr, d[f"{name}/full/block_row_ptr"])
            assert np.array_equal(s.full.bitmap_words, d[f"{name}/full/bitmap"])
            assert np.array_equal(s.full.values, d[f"{name}/full/values"])
            q8, sc = O.bfp8_encode(s.kept)
            assert np.array_equal(q8, d[q + "bfp8/q"]), name
            assert np.array_equal(sc, d[q + "bfp8/scale"]), name
            qo, so, orow, ocol, oval, _ = O.bfp8_outlier_encode(s.kept, 0.005)
            assert np.array_equal(qo, d[q + "bfp8o/q"]), name
            assert np.array_equal(so, d[q + "bfp8o/scale"]), name
            assert np.array_equal(orow, d[q + "bfp8o/rows"]), name
            assert np.array_equal(ocol, d[q + "bfp8o/cols"]), name
            assert np.array_equal(oval, d[q + "bfp8o/vals"]), name
            qo5, *_rest = O.bfp8_outlier_encode(s.kept, 0.05)
            assert np.array_equal(qo5, d[q + "bfp8o5/q"]), name
            assert np.array_equal(_rest[1], d[q + "bfp8o5/rows"]), name


def test_oracle_spmv_and_canonical_x(ref_cases):
    d = ref_cases
    for name in case_names(d):
        rows, cols = (int(v) for v in d[f"{name}/shape"])
        v = d[f"{name}/values"]
        x = O.canonical_x(cols, v.dtype)
        assert np.array_equal(x, d[f"{name}/canonical_x"])
        y = O.spmv_csr(rows, d[f"{name}/row_ptr"], d[f"{name}/col_idx"], v, x)
        # the reference sums each row in the same order: bit-identical
        assert np.array_equal(y, d[f"{name}/y_canonical"]), name


def test_dict_first_occurrence_order():
    kept = np.array([3.0, -1.0, 3.0, 7.0])
    res = np.array([-1.0, 9.0, 3.0])
    uniq, cb, kc, rc = O.dict_intern(kept, res)
    assert uniq == 4
    assert cb.tolist() == [3.0, -1.0, 7.0, 9.0]
    assert kc.tolist() == [0, 1, 0, 2] and rc.tolist() == [1, 3, 0]


def test_long_chunks():
    rp = np.array([0, 3, 3, 2000, 2100, 4100], np.int64)
    r, pb, pc, nl = O.long_chunks(rp, 256)
    assert nl == 2
    assert r.tolist() == [2, 2, 4, 4]
    assert pb.tolist() == [3, 1027, 2100, 3124]
    assert pc.tolist() == [1024, 973, 1024, 976]
    assert O.long_chunks(rp, 0)[0].size == 0


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")
def test_live_reference_random():
    """Fresh random inputs, oracle vs the reference compiled here."""
    rng = np.random.default_rng(7)
    for trial in range(4):
        rows, cols = int(rng.integers(20, 200)), int(rng.integers(20, 200))
        dens = float(rng.uniform(0.01, 0.2))
        mask = rng.random((rows, cols)) < dens
        vals = rng.standard_normal((rows, cols))
        rp = np.concatenate([[0], np.cumsum(mask.sum(1))]).astype(np.int64)
        ci = np.nonzero(mask)[1].astype(np.int32)
        v = vals[mask]
        R = O.RefSplit(rows, cols, rp, ci, v)
        s = O.split(rows, cols, rp, ci, v)
        brp, bci, bm, bvp, kv = R.bitbsr(1)
        assert np.array_equal(s.kept.block_col_idx, bci)
        assert np.array_equal(s.kept.bitmap_words, bm)
        assert np.array_equal(s.kept.values, kv)
        rrp, rci, rv = R.residual()
        assert np.array_equal(s.res_col_idx, rci) and np.array_equal(s.res_values, rv)
