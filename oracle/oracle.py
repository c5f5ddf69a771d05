"""ctypes front end of the CPU oracle (test infrastructure only).

Loads ``oracle/liboracle.so`` (the plain-C restatement in ``cove_oracle.c``)
and, when present, ``oracle/_ref/libcove_ref.so`` (the reference's own host
code compiled from its headers).  Only the tests, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` import this module, as the checker.

Every function returns numpy arrays.  Offsets are int64 in the oracle; the
reference's own types are int32 (structural/include/structural/types.hpp:7-8).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None


def build() -> None:
    """Compile liboracle.so (and _ref/ when the reference checkout exists)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _LIB = C.CDLL(path)
        _setup(_LIB)
    return _LIB


def ref_available() -> bool:
    return os.path.exists(os.path.join(_HERE, "_ref", "libcove_ref.so"))


def _ref():
    global _REF
    if _REF is None:
        _REF = C.CDLL(os.path.join(_HERE, "_ref", "libcove_ref.so"))
        _setup_ref(_REF)
    return _REF


class _OcBitBsr(C.Structure):
    _fields_ = [
        ("rows", C.c_int32), ("cols", C.c_int32), ("block_rows", C.c_int32),
        ("block_cols", C.c_int32), ("num_block_rows", C.c_int32),
        ("num_block_cols", C.c_int32), ("words_per_block", C.c_int32), ("esz", C.c_int32),
        ("num_blocks", C.c_int64), ("nnz", C.c_int64),
        ("block_row_ptr", C.POINTER(C.c_int64)), ("block_col_idx", C.POINTER(C.c_int32)),
        ("bitmap_words", C.POINTER(C.c_uint32)), ("block_val_ptr", C.POINTER(C.c_int64)),
        ("values", C.c_void_p),
    ]


class _OcSplit(C.Structure):
    _fields_ = [
        ("kept", C.POINTER(_OcBitBsr)), ("rows", C.c_int32), ("cols", C.c_int32),
        ("esz", C.c_int32),
        ("res_row_ptr", C.POINTER(C.c_int64)), ("res_col_idx", C.POINTER(C.c_int32)),
        ("res_values", C.c_void_p),
        ("kept_blocks", C.c_int64), ("residual_blocks", C.c_int64), ("kept_nnz", C.c_int64),
        ("residual_nnz", C.c_int64), ("cost_skipped_blocks", C.c_int64),
        ("cost_skipped_nnz", C.c_int64),
    ]


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def _setup(L):
    vp, i32, i64, f64 = C.c_void_p, C.c_int32, C.c_int64, C.c_double
    L.oc_convert_to_bitbsr.restype = C.POINTER(_OcBitBsr)
    L.oc_convert_to_bitbsr.argtypes = [i32, i32, vp, vp, vp, i32, i32, i32, C.c_char_p, i32]
    L.oc_bitbsr_free.argtypes = [C.POINTER(_OcBitBsr)]
    L.oc_split_bitbsr.restype = C.POINTER(_OcSplit)
    L.oc_split_bitbsr.argtypes = [C.POINTER(_OcBitBsr), i32, i32, f64, f64, f64, f64,
                                  C.c_char_p, i32]
    L.oc_split_free.argtypes = [C.POINTER(_OcSplit)]
    L.oc_cost_model_moves.restype = C.c_int
    L.oc_cost_model_moves.argtypes = [f64, f64, f64, f64, i64]
    L.oc_lb_layout.restype = i64
    L.oc_lb_layout.argtypes = [C.POINTER(_OcBitBsr), i32, i32, i32, vp, vp, vp]
    L.oc_long_chunks.restype = i64
    L.oc_long_chunks.argtypes = [i32, vp, i32, i32, vp, vp, vp, vp]
    L.oc_float_to_bf16_bits.restype = C.c_uint16
    L.oc_float_to_bf16_bits.argtypes = [C.c_float]
    L.oc_bfp8_encode.argtypes = [C.POINTER(_OcBitBsr), vp, vp]
    L.oc_bfp8_outlier_encode.restype = i64
    L.oc_bfp8_outlier_encode.argtypes = [C.POINTER(_OcBitBsr), f64, vp, vp, vp, vp, vp,
                                         C.POINTER(C.c_double)]
    L.oc_bf16_half_up.argtypes = [vp, i64, i32, vp]
    L.oc_dict_intern.restype = i64
    L.oc_dict_intern.argtypes = [vp, i64, vp, i64, i32, vp, vp, vp, i64]
    L.oc_spmv_csr.argtypes = [i32, vp, vp, vp, vp, vp, i32]
    L.oc_compare_vectors.argtypes = [vp, vp, i64, i32, vp]
    L.oc_canonical_x.argtypes = [i64, i32, vp]
    L.oc_joint_bfp8_spmv.argtypes = [C.POINTER(_OcBitBsr), vp, vp, vp, vp, vp, i64, vp, vp,
                                     vp, vp, vp]
    u64 = C.c_uint64
    L.oc_vector.argtypes = [i32, u64, u64, i64, i64, vp]
    L.oc_lapl3d_rows.restype = i64
    L.oc_lapl3d_rows.argtypes = [i32, i32, i32, i64, i64, i64, vp, vp, vp]
    L.oc_lapl2d.restype = i64
    L.oc_lapl2d.argtypes = [i32, i32, vp, vp, vp]
    L.oc_fem27_rows.restype = i64
    L.oc_write_mtx.restype = C.c_int
    L.oc_write_mtx.argtypes = [C.c_char_p, i64, i64, vp, vp, vp, i32]
    L.oc_fem27_rows.argtypes = [i32, i32, i32, i32, u64, i64, i64, i64, vp, vp, vp]
    L.oc_blocksparse_rows.restype = i64
    L.oc_blocksparse_rows.argtypes = [i32, f64, f64, f64, u64, i64, i64, vp, vp, vp]
    L.oc_rmat.restype = i64
    L.oc_rmat.argtypes = [i32, i32, f64, f64, f64, u64, vp, vp, vp]


def _setup_ref(R):
    vp, i32, i64, f64 = C.c_void_p, C.c_int32, C.c_int64, C.c_double
    R.ref_last_error.restype = C.c_char_p
    R.ref_split_build.restype = vp
    R.ref_split_build.argtypes = [i32, i32, vp, vp, vp, i32, i32, i32, i32, i32, vp]
    R.ref_split_free.argtypes = [vp]
    R.ref_split_counters.argtypes = [vp, vp, vp]
    R.ref_split_bitbsr.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp]
    R.ref_split_residual.argtypes = [vp, vp, vp, vp, vp]
    R.ref_bfp8.restype = i64
    R.ref_bfp8.argtypes = [vp, i32, f64, vp, vp, vp, vp, vp]
    R.ref_float_to_bf16_bits.restype = C.c_uint16
    R.ref_float_to_bf16_bits.argtypes = [C.c_float]
    R.ref_spmv_csr.restype = f64
    R.ref_spmv_csr.argtypes = [i32, i32, vp, vp, vp, i32, vp, vp]
    R.ref_csr_create.restype = vp
    R.ref_csr_create.argtypes = [i32, i32, vp, vp, vp, i32, vp]
    R.ref_csr_free.argtypes = [vp]
    R.ref_csr_spmv_timed.restype = f64
    R.ref_csr_spmv_timed.argtypes = [vp, i32, vp]
    R.ref_omp_max_threads.restype = i32
    R.ref_omp_set_threads.argtypes = [i32]
    R.ref_compare_vectors.argtypes = [vp, vp, i64, i32, vp]
    R.ref_canonical_x.argtypes = [i32, i32, vp]


@dataclass
class BitBsr:
    rows: int
    cols: int
    block_rows: int
    block_cols: int
    num_block_rows: int
    num_block_cols: int
    words_per_block: int
    block_row_ptr: np.ndarray
    block_col_idx: np.ndarray
    bitmap_words: np.ndarray
    block_val_ptr: np.ndarray
    values: np.ndarray
    _handle: object = None

    @property
    def num_blocks(self):
        return int(self.block_col_idx.size)

    @property
    def nnz(self):
        return int(self.values.size)


def _arr(ptr, n, dtype):
    if n == 0:
        return np.zeros(0, dtype=dtype)
    return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(np.ctypeslib.as_ctypes_type(dtype))),
                                 shape=(n,)).copy()


def _bitbsr_from(h, dtype) -> BitBsr:
    m = h.contents
    nb, nnz = m.num_blocks, m.nnz
    return BitBsr(
        rows=m.rows, cols=m.cols, block_rows=m.block_rows, block_cols=m.block_cols,
        num_block_rows=m.num_block_rows, num_block_cols=m.num_block_cols,
        words_per_block=m.words_per_block,
        block_row_ptr=_arr(m.block_row_ptr, m.num_block_rows + 1, np.int64),
        block_col_idx=_arr(m.block_col_idx, nb, np.int32),
        bitmap_words=_arr(m.bitmap_words, nb * m.words_per_block, np.uint32),
        block_val_ptr=_arr(m.block_val_ptr, nb + 1, np.int64),
        values=_arr(m.values, nnz, dtype),
    )


def _csr_args(rows, row_ptr, col_idx, values):
    row_ptr = np.ascontiguousarray(row_ptr, dtype=np.int64)
    col_idx = np.ascontiguousarray(col_idx, dtype=np.int32)
    values = np.ascontiguousarray(values)
    assert values.dtype in (np.float64, np.float32)
    assert row_ptr.size == rows + 1
    return row_ptr, col_idx, values


def convert_to_bitbsr(rows, cols, row_ptr, col_idx, values, br=8, bc=4) -> BitBsr:
    """convert_to_bitbsr (convert.hpp:13-165)."""
    L = _lib()
    row_ptr, col_idx, values = _csr_args(rows, row_ptr, col_idx, values)
    err = C.create_string_buffer(256)
    h = L.oc_convert_to_bitbsr(rows, cols, _p(row_ptr), _p(col_idx), _p(values),
                               values.itemsize, br, bc, err, 256)
    if not h:
        raise RuntimeError(err.value.decode())
    try:
        return _bitbsr_from(h, values.dtype)
    finally:
        L.oc_bitbsr_free(h)


@dataclass
class Split:
    kept: BitBsr
    res_row_ptr: np.ndarray
    res_col_idx: np.ndarray
    res_values: np.ndarray
    kept_blocks: int
    residual_blocks: int
    kept_nnz: int
    residual_nnz: int
    cost_skipped_blocks: int
    cost_skipped_nnz: int
    full: BitBsr = None


DEFAULT_COST = (10.0, 0.0, 0.0, 1.0)  # csr_bitbsr_split.hpp:53-58


def split(rows, cols, row_ptr, col_idx, values, br=8, bc=4, threshold=32, use_cost=True,
          cost=DEFAULT_COST) -> Split:
    """convert_to_bitbsr + convert_bitbsr_to_csr_bitbsr_split{_cost_gated}."""
    L = _lib()
    row_ptr, col_idx, values = _csr_args(rows, row_ptr, col_idx, values)
    err = C.create_string_buffer(256)
    fh = L.oc_convert_to_bitbsr(rows, cols, _p(row_ptr), _p(col_idx), _p(values),
                                values.itemsize, br, bc, err, 256)
    if not fh:
        raise RuntimeError(err.value.decode())
    try:
        full = _bitbsr_from(fh, values.dtype)
        sh = L.oc_split_bitbsr(fh, threshold, 1 if use_cost else 0, *cost, err, 256)
        if not sh:
            raise RuntimeError(err.value.decode())
        try:
            s = sh.contents
            kept = _bitbsr_from(s.kept, values.dtype)
            rn = int(s.residual_nnz)
            out = Split(
                kept=kept,
                res_row_ptr=_arr(s.res_row_ptr, rows + 1, np.int64),
                res_col_idx=_arr(s.res_col_idx, rn, np.int32),
                res_values=_arr(s.res_values, rn, values.dtype),
                kept_blocks=int(s.kept_blocks), residual_blocks=int(s.residual_blocks),
                kept_nnz=int(s.kept_nnz), residual_nnz=rn,
                cost_skipped_blocks=int(s.cost_skipped_blocks),
                cost_skipped_nnz=int(s.cost_skipped_nnz),
                full=full,
            )
            return out
        finally:
            L.oc_split_free(sh)
    finally:
        L.oc_bitbsr_free(fh)


def _to_oc(m: BitBsr):
    """Build a temporary oc_bitbsr view over numpy arrays (kept alive by caller)."""
    s = _OcBitBsr()
    s.rows, s.cols = m.rows, m.cols
    s.block_rows, s.block_cols = m.block_rows, m.block_cols
    s.num_block_rows, s.num_block_cols = m.num_block_rows, m.num_block_cols
    s.words_per_block = m.words_per_block
    s.esz = m.values.itemsize
    s.num_blocks, s.nnz = m.num_blocks, m.nnz
    keep = [np.ascontiguousarray(m.block_row_ptr, np.int64),
            np.ascontiguousarray(m.block_col_idx, np.int32),
            np.ascontiguousarray(m.bitmap_words, np.uint32),
            np.ascontiguousarray(m.block_val_ptr, np.int64),
            np.ascontiguousarray(m.values)]
    s.block_row_ptr = keep[0].ctypes.data_as(C.POINTER(C.c_int64))
    s.block_col_idx = keep[1].ctypes.data_as(C.POINTER(C.c_int32))
    s.bitmap_words = keep[2].ctypes.data_as(C.POINTER(C.c_uint32))
    s.block_val_ptr = keep[3].ctypes.data_as(C.POINTER(C.c_int64))
    s.values = keep[4].ctypes.data
    return s, keep


def lb_layout(kept: BitBsr, chunk_blocks=32, split_threshold_blocks=None, style="hybrid"):
    """Packed words + work items (hybrid host layout or device layout)."""
    if split_threshold_blocks is None or split_threshold_blocks < 0:
        split_threshold_blocks = chunk_blocks
    L = _lib()
    s, keep = _to_oc(kept)
    words = np.zeros(max(kept.num_blocks, 1), np.uint64)
    items = np.zeros((kept.num_block_rows + kept.num_blocks + 1) * 4, np.uint32)
    irp = np.zeros(kept.num_block_rows + 1, np.int64)
    n = L.oc_lb_layout(C.byref(s), chunk_blocks, split_threshold_blocks,
                       0 if style == "hybrid" else 1, _p(words), _p(items), _p(irp))
    return words[: kept.num_blocks], items[: 4 * n].reshape(n, 4), irp


def long_chunks(res_row_ptr, tau, chunk_nnz=1024):
    L = _lib()
    rp = np.ascontiguousarray(res_row_ptr, np.int64)
    rows = rp.size - 1
    n = L.oc_long_chunks(rows, _p(rp), tau, chunk_nnz, None, None, None, None)
    r = np.zeros(max(n, 1), np.int32)
    pb = np.zeros(max(n, 1), np.int64)
    pc = np.zeros(max(n, 1), np.int32)
    nl = C.c_int64(0)
    L.oc_long_chunks(rows, _p(rp), tau, chunk_nnz, _p(r), _p(pb), _p(pc), C.byref(nl))
    return r[:n], pb[:n], pc[:n], int(nl.value)


def float_to_bf16_bits(v: float) -> int:
    return int(_lib().oc_float_to_bf16_bits(C.c_float(v)))


def bfp8_encode(kept: BitBsr):
    L = _lib()
    s, keep = _to_oc(kept)
    q = np.zeros(max(kept.nnz, 1), np.int8)
    sc = np.zeros(max(kept.num_blocks, 1), np.uint16)
    L.oc_bfp8_encode(C.byref(s), _p(q), _p(sc))
    return q[: kept.nnz], sc[: kept.num_blocks]


def bfp8_outlier_encode(kept: BitBsr, fraction=0.005):
    L = _lib()
    s, keep = _to_oc(kept)
    n = max(kept.nnz, 1)
    q = np.zeros(n, np.int8)
    sc = np.zeros(max(kept.num_blocks, 1), np.uint16)
    orow = np.zeros(n, np.int32)
    ocol = np.zeros(n, np.int32)
    oval = np.zeros(n, kept.values.dtype)
    thr = C.c_double(0)
    k = L.oc_bfp8_outlier_encode(C.byref(s), fraction, _p(q), _p(sc), _p(orow), _p(ocol),
                                 _p(oval), C.byref(thr))
    return (q[: kept.nnz], sc[: kept.num_blocks], orow[:k], ocol[:k], oval[:k],
            float(thr.value))


def bf16_half_up(values):
    v = np.ascontiguousarray(values)
    out = np.zeros(max(v.size, 1), np.uint16)
    _lib().oc_bf16_half_up(_p(v), v.size, v.itemsize, _p(out))
    return out[: v.size]


def dict_intern(kept_values, res_values, cap=65536):
    """First-occurrence exact-value codebook over kept then residual values."""
    kv = np.ascontiguousarray(kept_values)
    rv = np.ascontiguousarray(res_values, dtype=kv.dtype)
    cb = np.zeros(cap, kv.dtype)
    kc = np.zeros(max(kv.size, 1), np.int32)
    rc = np.zeros(max(rv.size, 1), np.int32)
    uniq = _lib().oc_dict_intern(_p(kv), kv.size, _p(rv), rv.size, kv.itemsize, _p(cb),
                                 _p(kc), _p(rc), cap)
    return int(uniq), cb[: min(uniq, cap)], kc[: kv.size], rc[: rv.size]


def spmv_csr(rows, row_ptr, col_idx, values, x):
    rp = np.ascontiguousarray(row_ptr, np.int64)
    ci = np.ascontiguousarray(col_idx, np.int32)
    v = np.ascontiguousarray(values)
    xx = np.ascontiguousarray(x, dtype=v.dtype)
    y = np.zeros(rows, v.dtype)
    _lib().oc_spmv_csr(rows, _p(rp), _p(ci), _p(v), _p(xx), _p(y), v.itemsize)
    return y


def compare_vectors(ref, got):
    """(max_abs, max_rel, global_rel) in the element type (spmv.hpp:73-89)."""
    r = np.ascontiguousarray(ref)
    g = np.ascontiguousarray(got, dtype=r.dtype)
    out = np.zeros(3, np.float64)
    _lib().oc_compare_vectors(_p(r), _p(g), r.size, r.itemsize, _p(out))
    return float(out[0]), float(out[1]), float(out[2])


def canonical_x(n, dtype=np.float64):
    x = np.zeros(n, dtype)
    _lib().oc_canonical_x(n, x.itemsize, _p(x))
    return x


def joint_bfp8_spmv(kept: BitBsr, q, scale, res_row_ptr, res_col, res_bf16, orow, ocol, oval,
                    x):
    L = _lib()
    s, keep = _to_oc(kept)
    rp = np.ascontiguousarray(res_row_ptr, np.int64)
    rc = np.ascontiguousarray(res_col, np.int32)
    rb = np.ascontiguousarray(res_bf16, np.uint16)
    q = np.ascontiguousarray(q, np.int8)
    sc = np.ascontiguousarray(scale, np.uint16)
    orow = np.ascontiguousarray(orow, np.int32)
    ocol = np.ascontiguousarray(ocol, np.int32)
    oval = np.ascontiguousarray(oval, kept.values.dtype)
    xx = np.ascontiguousarray(x, kept.values.dtype)
    y = np.zeros(kept.rows, kept.values.dtype)
    L.oc_joint_bfp8_spmv(C.byref(s), _p(q), _p(sc), _p(rp), _p(rc), _p(rb), orow.size,
                         _p(orow), _p(ocol), _p(oval), _p(xx), _p(y))
    return y


# ---------------------------------------------------------------------------
# the reference itself (oracle/_ref), for pinning the restatement
# ---------------------------------------------------------------------------

class RefSplit:
    """Results of the reference's own convert_to_bitbsr + split on a CSR."""

    def __init__(self, rows, cols, row_ptr, col_idx, values, br=8, bc=4, threshold=32,
                 use_cost=True, cost=DEFAULT_COST):
        R = _ref()
        self.R = R
        rp = np.ascontiguousarray(row_ptr, np.int32)
        ci = np.ascontiguousarray(col_idx, np.int32)
        v = np.ascontiguousarray(values)
        c4 = np.ascontiguousarray(cost, np.float64)
        self.dtype = v.dtype
        self.rows = rows
        self.h = R.ref_split_build(rows, cols, _p(rp), _p(ci), _p(v), v.itemsize, br, bc,
                                   threshold, 1 if use_cost else 0, _p(c4))
        if not self.h:
            raise RuntimeError(R.ref_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.R.ref_split_free(self.h)
            self.h = None

    def counters(self):
        c = np.zeros(7, np.int64)
        b = np.zeros(4, np.int64)
        self.R.ref_split_counters(self.h, _p(c), _p(b))
        keys = ["full_blocks", "kept_blocks", "residual_blocks", "cost_skipped_blocks",
                "kept_nnz", "residual_nnz", "cost_skipped_nnz"]
        out = dict(zip(keys, (int(v) for v in c)))
        out.update(zip(["full_bitbsr_position_bits", "kept_bitbsr_position_bits",
                        "residual_csr_position_bits", "split_position_bits"],
                       (int(v) for v in b)))
        return out

    def bitbsr(self, which):
        sizes = np.zeros(4, np.int64)
        self.R.ref_split_bitbsr(self.h, which, _p(sizes), None, None, None, None, None)
        nbr, nb, nnz, wpb = (int(v) for v in sizes)
        brp = np.zeros(nbr + 1, np.int32)
        bci = np.zeros(max(nb, 1), np.int32)
        bm = np.zeros(max(nb * wpb, 1), np.uint32)
        bvp = np.zeros(nb + 1, np.int32)
        vals = np.zeros(max(nnz, 1), self.dtype)
        self.R.ref_split_bitbsr(self.h, which, _p(sizes), _p(brp), _p(bci), _p(bm), _p(bvp),
                                _p(vals))
        return brp, bci[:nb], bm[: nb * wpb], bvp, vals[:nnz]

    def residual(self):
        sizes = np.zeros(2, np.int64)
        self.R.ref_split_residual(self.h, _p(sizes), None, None, None)
        rows, nnz = (int(v) for v in sizes)
        rp = np.zeros(rows + 1, np.int32)
        ci = np.zeros(max(nnz, 1), np.int32)
        v = np.zeros(max(nnz, 1), self.dtype)
        self.R.ref_split_residual(self.h, _p(sizes), _p(rp), _p(ci), _p(v))
        return rp, ci[:nnz], v[:nnz]

    def bfp8(self, which=1, outlier_fraction=-1.0):
        sizes = np.zeros(4, np.int64)
        self.R.ref_split_bitbsr(self.h, which, _p(sizes), None, None, None, None, None)
        nb, nnz = int(sizes[1]), int(sizes[2])
        q = np.zeros(max(nnz, 1), np.int8)
        sc = np.zeros(max(nb, 1), np.uint16)
        orow = np.zeros(max(nnz, 1), np.int32)
        ocol = np.zeros(max(nnz, 1), np.int32)
        oval = np.zeros(max(nnz, 1), self.dtype)
        k = self.R.ref_bfp8(self.h, which, outlier_fraction, _p(q), _p(sc), _p(orow), _p(ocol),
                            _p(oval))
        if k < 0:
            raise RuntimeError(self.R.ref_last_error().decode())
        return q[:nnz], sc[:nb], orow[:k], ocol[:k], oval[:k]


def ref_spmv_csr(rows, cols, row_ptr, col_idx, values, x):
    """The reference's OpenMP spmv_csr; returns (y, milliseconds)."""
    R = _ref()
    rp = np.ascontiguousarray(row_ptr, np.int32)
    ci = np.ascontiguousarray(col_idx, np.int32)
    v = np.ascontiguousarray(values)
    xx = np.ascontiguousarray(x, v.dtype)
    y = np.zeros(rows, v.dtype)
    ms = R.ref_spmv_csr(rows, cols, _p(rp), _p(ci), _p(v), v.itemsize, _p(xx), _p(y))
    if ms < 0:
        raise RuntimeError(R.ref_last_error().decode())
    return y, ms


class RefCsrTimer:
    """Reference spmv_csr over a resident copy of the matrix, for timing."""

    def __init__(self, rows, cols, row_ptr, col_idx, values, x):
        self.R = _ref()
        rp = np.ascontiguousarray(row_ptr, np.int32)
        ci = np.ascontiguousarray(col_idx, np.int32)
        v = np.ascontiguousarray(values)
        xx = np.ascontiguousarray(x, v.dtype)
        self.rows = rows
        self.dtype = v.dtype
        self.h = self.R.ref_csr_create(rows, cols, _p(rp), _p(ci), _p(v), v.itemsize, _p(xx))

    def run(self, reps=1):
        y = np.zeros(self.rows, self.dtype)
        ms = self.R.ref_csr_spmv_timed(self.h, reps, _p(y))
        return y, ms

    def close(self):
        if self.h:
            self.R.ref_csr_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def ref_threads() -> int:
    return int(_ref().ref_omp_max_threads())


def ref_use_all_cores() -> int:
    """Give the reference's OpenMP loops every core this process may run on,
    whatever OMP_NUM_THREADS a launcher set (torchrun sets 1); returns the
    thread count now in force."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    _ref().ref_omp_set_threads(max(1, n))
    return ref_threads()


def ref_float_to_bf16_bits(v: float) -> int:
    return int(_ref().ref_float_to_bf16_bits(C.c_float(v)))


def ref_compare_vectors(ref, got):
    r = np.ascontiguousarray(ref)
    g = np.ascontiguousarray(got, dtype=r.dtype)
    out = np.zeros(3, np.float64)
    _ref().ref_compare_vectors(_p(r), _p(g), r.size, r.itemsize, _p(out))
    return float(out[0]), float(out[1]), float(out[2])


def ref_canonical_x(n, dtype=np.float64):
    x = np.zeros(n, dtype)
    _ref().ref_canonical_x(n, x.itemsize, _p(x))
    return x


# ---- seeded benchmark inputs (oracle_workloads.c) ------------------------------

def vector(kind, seed, stream, begin, n):
    """Seeded vector of global indices [begin, begin + n): kind "uniform_pm1"
    (U[-1,1]), "uniform01" or "normal"; float64."""
    k = {"uniform_pm1": 0, "uniform01": 1, "normal": 2}[kind]
    out = np.empty(n, np.float64)
    _lib().oc_vector(k, seed, stream, begin, n, _p(out))
    return out


def _gen_csr(count, fill, rows):
    nnz = count()
    rp = np.zeros(rows + 1, np.int64)
    ci = np.empty(nnz, np.int32)
    v = np.empty(nnz, np.float64)
    fill(_p(rp), _p(ci), _p(v))
    return rp, ci, v


def lapl3d_rows(nx, ny, nz, row_begin, row_end, col_shift=0):
    """Rows [row_begin, row_end) of the 3D 7-point Laplacian: (rp, ci, v)."""
    L = _lib()
    return _gen_csr(lambda: L.oc_lapl3d_rows(nx, ny, nz, row_begin, row_end, col_shift, None, None, None),
                    lambda a, b, c: L.oc_lapl3d_rows(nx, ny, nz, row_begin, row_end, col_shift, a, b, c),
                    row_end - row_begin)


def lapl2d(nx, ny):
    """The 2D 5-point Laplacian on nx x ny: (rp, ci, v)."""
    L = _lib()
    return _gen_csr(lambda: L.oc_lapl2d(nx, ny, None, None, None),
                    lambda a, b, c: L.oc_lapl2d(nx, ny, a, b, c), nx * ny)


def fem27_rows(nx, ny, nz, dof, seed, row_begin, row_end, col_shift=0):
    """Rows [row_begin, row_end) of the FEM-like 27-point stencil: (rp, ci, v)."""
    L = _lib()
    return _gen_csr(lambda: L.oc_fem27_rows(nx, ny, nz, dof, seed, row_begin, row_end, col_shift,
                                            None, None, None),
                    lambda a, b, c: L.oc_fem27_rows(nx, ny, nz, dof, seed, row_begin, row_end, col_shift,
                                                    a, b, c),
                    row_end - row_begin)


def blocksparse_rows(n, row_begin, row_end, p_block=2e-3, p_entry=0.6, outlier_fraction=1e-3, seed=3):
    """Rows [row_begin, row_end) of the random 8x4 block-sparse n x n matrix
    (row_ptr relative to row_begin, global columns): (rp, ci, v)."""
    L = _lib()
    args = (n, p_block, p_entry, outlier_fraction, seed, row_begin, row_end)
    nnz = L.oc_blocksparse_rows(*args, None, None, None)
    if nnz < 0:
        raise ValueError("block-sparse rows must start and end on whole 8-row block rows")
    rp = np.zeros(row_end - row_begin + 1, np.int64)
    ci = np.empty(nnz, np.int32)
    v = np.empty(nnz, np.float64)
    L.oc_blocksparse_rows(*args, _p(rp), _p(ci), _p(v))
    return rp, ci, v


def rmat(scale, edge_factor=16, a=0.57, b=0.19, c=0.19, seed=2):
    """The R-MAT graph with 2^scale rows and float values: (rp, ci, v)."""
    L = _lib()
    n = 1 << scale
    nnz = L.oc_rmat(scale, edge_factor, a, b, c, seed, None, None, None)
    if nnz < 0:
        raise MemoryError("R-MAT generation failed")
    rp = np.zeros(n + 1, np.int64)
    ci = np.empty(nnz, np.int32)
    v = np.empty(nnz, np.float32)
    L.oc_rmat(scale, edge_factor, a, b, c, seed, _p(rp), _p(ci), _p(v))
    return rp, ci, v


def write_mtx(path, rows, cols, row_ptr, col_idx, values):
    """MatrixMarket file of a CSR; values round-trip exactly (%.17g / %.9g)."""
    rp = np.ascontiguousarray(row_ptr, np.int64)
    ci = np.ascontiguousarray(col_idx, np.int32)
    v = np.ascontiguousarray(values)
    if _lib().oc_write_mtx(str(path).encode(), rows, cols, _p(rp), _p(ci), _p(v), v.itemsize) != 0:
        raise OSError(f"cannot write {path}")
