"""The C-ABI library loads and exports what include/*.h declares (no GPU)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import cove_b200 as cb

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _declared_symbols():
    names = set()
    for fn in ("cove_b200.h", "cove_synth.h"):
        with open(os.path.join(ROOT, "include", fn)) as f:
            text = f.read()
        names |= set(re.findall(r"COVE_API\s+[\w\s\*]+?\b(cove_\w+)\s*\(", text))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    L = cb.lib()
    declared = _declared_symbols()
    assert len(declared) >= 30
    for name in sorted(declared):
        assert hasattr(L, name), f"{name} is declared in include/ but not exported"
    assert set(cb.EXPORTED) == declared


def test_version_and_status_strings():
    L = cb.lib()
    assert b"sm_100a" in L.cove_version()
    assert L.cove_status_string(0) == b"ok"
    assert L.cove_status_string(3) == b"int32 offset overflow"


def test_default_options_are_the_reference_defaults():
    o = cb.default_opts()
    assert o.residual_threshold == 32
    assert (o.cost_bitmap_block, o.cost_bitmap_nnz, o.cost_csr_block, o.cost_csr_nnz) == (10, 0, 0, 1)
    assert o.lb_chunk_blocks == 32 and o.lb_split_threshold_blocks == -1
    assert o.long_row_split == 0 and o.outlier_fraction == 0.005 and o.gate_tolerance == 1e-2
    assert o.value_codec == cb.CODEC["original"]


def test_null_arguments_are_rejected_without_a_device():
    L = cb.lib()
    h = C.c_void_p()
    st = L.cove_plan_build(None, None, None, C.byref(h))
    assert st == 1
    assert b"null" in L.cove_last_error()
    assert L.cove_plan_get_info(None, None) == 1
    assert L.cove_spmv(None, None, None, None) == 1


def test_bad_options_are_rejected_before_any_device_work():
    L = cb.lib()
    d = cb.CsrDesc()
    d.rows = d.cols = 4
    d.dtype = cb.F64
    for field, val, msg in [("residual_threshold", -1, b"residual-threshold must be non-negative"),
                            ("lb_chunk_blocks", 0, b"lb-chunk-blocks must be positive"),
                            ("cost_csr_nnz", -1.0, b"cost model must be non-negative")]:
        o = cb.default_opts(**{field: val})
        h = C.c_void_p()
        assert L.cove_plan_build(C.byref(d), C.byref(o), None, C.byref(h)) == 1
        assert msg in L.cove_last_error()
    d.dtype = 7
    h = C.c_void_p()
    assert L.cove_plan_build(C.byref(d), None, None, C.byref(h)) == 6


def test_route_names():
    L = cb.lib()
    assert [L.cove_route_name(i).decode() for i in range(5)] == [
        "original", "dict_u8_lossless", "dict_u16_lossless", "bfp8_blocks+bf16_residual",
        "bfp8_outlier_blocks+bf16_residual"]


def test_counter_rng_is_stable():
    # splitmix64 chain: fixed values pin the generator across builds
    a = [cb.lib().cove_rng_u64(1, 0, i) for i in range(3)]
    assert a == [cb.lib().cove_rng_u64(1, 0, i) for i in range(3)]
    u = np.array([cb.rng_uniform01(3, 2, i) for i in range(1000)])
    assert 0.0 <= u.min() and u.max() < 1.0 and abs(u.mean() - 0.5) < 0.05


def test_generators_are_deterministic_and_valid():
    r1 = cb.synth_fem27(6, 5, 4, 3, seed=11)
    r2 = cb.synth_fem27(6, 5, 4, 3, seed=11)
    for a, b in zip(r1[2:], r2[2:]):
        assert np.array_equal(a, b)
    rows, cols, rp, ci, v = r1
    assert rp[-1] == ci.size == 9 * (3 * 6 - 2) * (3 * 5 - 2) * (3 * 4 - 2)
    for r in range(rows):
        seg = ci[rp[r]:rp[r + 1]]
        assert np.all(np.diff(seg) > 0)
    assert np.all(v != 0)


def test_lapl3d_window_columns():
    rows, n, rp, ci, v = cb.synth_lapl3d(4, 4, 8, row_begin=32, row_end=96, col_shift=16)
    assert rows == 64 and n == 128
    assert ci.min() >= 0 and ci.max() < 128 - 16
    full = cb.synth_lapl3d(4, 4, 8)
    # the same rows with shifted columns
    assert np.array_equal(full[3][full[2][32]:full[2][96]] - 16, ci)


def test_rmat_duplicates_are_merged_by_summation():
    rows, cols, rp, ci, v = cb.synth_rmat(10, 16, seed=2)
    assert rows == 1024 and ci.size < 16 * 1024
    assert v.dtype == np.float32 and np.all(v > 0)
    assert abs(float(v.sum()) - 16 * 1024 * 0.5) < 0.05 * 16 * 1024
