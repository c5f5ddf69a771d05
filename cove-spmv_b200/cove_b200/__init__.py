"""Python binding of the B200 COVE SpMV library (ctypes over the C ABI).

The product is ``libcove_b200.so`` (sm_100a kernels behind the ``extern "C"``
interface in ``include/cove_b200.h``).  This module only marshals arguments:
device memory and streams come from PyTorch tensors, every computation is a
call into the library, and importing fails loudly when the library is
missing -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcove_b200.so")

F64, F32 = 0, 1
CODEC = {"original": 0, "auto": 1, "dict": 2, "bfp8": 3, "bfp8_outlier": 4}
ROUTE_HYBRID, ROUTE_DICT_U8, ROUTE_DICT_U16, ROUTE_BFP8, ROUTE_BFP8_OUTLIER = range(5)
# value codecs of the BitBSR-only family runner (cove_hybrid_spmv)
(ROUTE_TILE_CODE, ROUTE_BF16_NNZ, ROUTE_IMPLICIT_ONE, ROUTE_CONST_C, ROUTE_SIGN2,
 ROUTE_FP16_NNZ, ROUTE_BFP4) = range(5, 12)
ROUTE_NAMES = {0: "original", 1: "dict_u8_lossless", 2: "dict_u16_lossless",
               3: "bfp8_blocks+bf16_residual", 4: "bfp8_outlier_blocks+bf16_residual"}
ROUTE_NAMES_INV = {v: k for k, v in ROUTE_NAMES.items()}
ROUTE_NAMES_INV.update({"hybrid": 0, "dict_u8": 1, "dict_u16": 2, "bfp8": 3, "bfp8_outlier": 4})
SPLIT = {"cost_gated": 0, "threshold": 1, "none": 2, "mask": 3}
LB_STYLE = {"hybrid": 0, "device": 1}

STREAM = {
    "full_block_row_ptr": (0, np.int32), "full_block_col_idx": (1, np.int32),
    "full_bitmap": (2, np.uint32), "full_values": (3, None),
    "full_block_row_val_ptr": (4, np.int32),
    "kept_block_row_ptr": (10, np.int32), "kept_block_col_idx": (11, np.int32),
    "kept_bitmap": (12, np.uint32), "kept_values": (13, None),
    "kept_block_val_ptr": (14, np.int32), "kept_block_row_val_ptr": (15, np.int32),
    "res_row_ptr": (20, np.int32), "res_col_idx": (21, np.int32), "res_values": (22, None),
    "words": (30, np.uint64), "work_items": (31, np.uint32), "work_item_row_ptr": (32, np.int32),
    "chunk_row": (40, np.int32), "chunk_pbegin": (41, np.int32), "chunk_pcount": (42, np.int32),
    "dict_codebook": (50, None), "dict_kept_idx": (51, "dict"), "dict_res_idx": (52, "dict"),
    "bfp8_int8": (60, np.int8), "bfp8_scale": (61, np.uint16), "res_bf16": (62, np.uint16),
    "outlier_rows": (63, np.int32), "outlier_cols": (64, np.int32), "outlier_vals": (65, None),
}


class CoveError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{msg} (status {status})")
        self.status = status


class CsrDesc(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("nnz", C.c_int64),
                ("row_ptr", C.c_void_p), ("col_idx", C.c_void_p), ("values", C.c_void_p),
                ("dtype", C.c_int32), ("row_ptr_i32", C.c_int32)]


class PlanOpts(C.Structure):
    _fields_ = [("residual_threshold", C.c_int32), ("split_policy", C.c_int32),
                ("cost_bitmap_block", C.c_double), ("cost_bitmap_nnz", C.c_double),
                ("cost_csr_block", C.c_double), ("cost_csr_nnz", C.c_double),
                ("lb_chunk_blocks", C.c_int32), ("lb_split_threshold_blocks", C.c_int32),
                ("lb_style", C.c_int32), ("long_row_split", C.c_int32),
                ("value_codec", C.c_int32), ("outlier_fraction", C.c_double),
                ("gate_tolerance", C.c_double), ("gate_enable", C.c_int32),
                ("keep_full_bitbsr", C.c_int32), ("keep_lossless", C.c_int32),
                ("move_mask", C.c_uint64)]


class PlanInfo(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("dtype", C.c_int32),
                ("nnz", C.c_int64),
                ("full_blocks", C.c_int64), ("kept_blocks", C.c_int64),
                ("residual_blocks", C.c_int64), ("cost_skipped_blocks", C.c_int64),
                ("kept_nnz", C.c_int64), ("residual_nnz", C.c_int64),
                ("cost_skipped_nnz", C.c_int64),
                ("work_items", C.c_int64), ("long_rows", C.c_int64),
                ("long_row_chunks", C.c_int64), ("num_outliers", C.c_int64),
                ("value_cardinality", C.c_int64),
                ("full_bitbsr_position_bits", C.c_int64), ("kept_bitbsr_position_bits", C.c_int64),
                ("residual_csr_position_bits", C.c_int64), ("split_position_bits", C.c_int64),
                ("requested_codec", C.c_int32), ("joint_route", C.c_int32),
                ("dispatched_route", C.c_int32), ("gate_evaluated", C.c_int32),
                ("gate_pass", C.c_int32),
                ("joint_rel_err", C.c_double), ("joint_bytes_per_nnz", C.c_double),
                ("outlier_threshold", C.c_double),
                ("algorithmic_bytes", C.c_int64 * 5),
                ("kernel_slots", C.c_int32), ("kernel_overflow_tasks", C.c_int32)]


class HybridDesc(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("num_block_rows", C.c_int32),
                ("dtype", C.c_int32), ("kept_blocks", C.c_int64), ("kept_nnz", C.c_int64),
                ("residual_nnz", C.c_int64), ("block_row_ptr", C.c_void_p),
                ("block_row_val_ptr", C.c_void_p), ("words", C.c_void_p),
                ("res_row_ptr", C.c_void_p), ("res_col_idx", C.c_void_p),
                ("long_row_tau", C.c_int32), ("num_chunks", C.c_int64), ("chunk_row", C.c_void_p),
                ("chunk_pbegin", C.c_void_p), ("chunk_pcount", C.c_void_p)]


class ValuesDesc(C.Structure):
    _fields_ = [("route", C.c_int32), ("kept", C.c_void_p), ("res", C.c_void_p),
                ("block_scale", C.c_void_p), ("codebook", C.c_void_p),
                ("codebook_size", C.c_int64), ("num_outliers", C.c_int64),
                ("outlier_rows", C.c_void_p), ("outlier_cols", C.c_void_p),
                ("outlier_vals", C.c_void_p), ("tile_code_words", C.c_void_p),
                ("tile_bits", C.c_int32), ("value_scale", C.c_double), ("sign_masks", C.c_void_p)]


class CgResult(C.Structure):
    _fields_ = [("iterations", C.c_int32), ("rs_initial", C.c_double),
                ("rs_final", C.c_double), ("ms_total", C.c_double), ("ms_spmv", C.c_double),
                ("launches", C.c_int64)]


class IrResult(C.Structure):
    _fields_ = [("outer", C.c_int32), ("inner_total", C.c_int32), ("final_relres", C.c_double),
                ("reached", C.c_int32), ("ms_total", C.c_double)]


class MmMatrix(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("nnz", C.c_int64),
                ("row_ptr", C.POINTER(C.c_int64)), ("col_idx", C.POINTER(C.c_int32)),
                ("values", C.c_void_p), ("dtype", C.c_int32), ("field", C.c_int32),
                ("symmetry", C.c_int32), ("stored_entries", C.c_int64),
                ("expanded_entries", C.c_int64), ("coalesced_duplicates", C.c_int64)]


MM_FIELDS = ("real", "integer", "complex", "pattern")
MM_SYMMETRIES = ("general", "symmetric", "skew-symmetric", "hermitian")


# every symbol include/cove_b200.h and include/cove_synth.h declare
EXPORTED = [
    "cove_last_error", "cove_status_string", "cove_version", "cove_plan_opts_default",
    "cove_plan_build", "cove_plan_destroy", "cove_plan_get_info", "cove_route_name",
    "cove_plan_stream", "cove_bitbsr8x4_count", "cove_bitbsr8x4_fill", "cove_pack_words",
    "cove_lb_layout_count", "cove_lb_layout_fill",
    "cove_hybrid_spmv", "cove_spmv", "cove_spmv_route", "cove_spmv_host",
    "cove_spmv_launches", "cove_compare_vectors", "cove_canonical_x", "cove_cg_solve",
    "cove_mm_read", "cove_mm_free", "cove_ir_solve", "cove_fcg_solve", "cove_dist_mp_solve",
    "cove_cg_solve_noalloc",
    "cove_dist_halo_plan", "cove_dist_id_bytes", "cove_dist_make_id", "cove_dist_create", "cove_dist_destroy",
    "cove_dist_halo", "cove_dist_cg_solve", "cove_dist_spmv", "cove_dist_spmv_launches",
    "cove_rng_u64", "cove_rng_uniform01", "cove_synth_lapl2d", "cove_synth_lapl3d",
    "cove_synth_fem27", "cove_synth_fem27_rows", "cove_synth_rmat", "cove_synth_blocksparse", "cove_synth_vector",
    "cove_synth_lapl3d_device", "cove_synth_vector_device", "cove_synth_blocksparse_rows",
    "cove_synth_blocksparse_device",
]

_lib = None


def lib():
    """Load libcove_b200.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C cove-spmv_b200`")
        L = C.CDLL(LIB_PATH)
        _setup(L)
        _lib = L
    return _lib


def _setup(L):
    vp, i32, i64, u64, f64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_double
    L.cove_last_error.restype = C.c_char_p
    L.cove_status_string.restype = C.c_char_p
    L.cove_status_string.argtypes = [C.c_int]
    L.cove_version.restype = C.c_char_p
    L.cove_plan_opts_default.argtypes = [C.POINTER(PlanOpts)]
    L.cove_plan_build.argtypes = [C.POINTER(CsrDesc), C.POINTER(PlanOpts), vp, C.POINTER(vp)]
    L.cove_plan_destroy.argtypes = [vp]
    L.cove_plan_get_info.argtypes = [vp, C.POINTER(PlanInfo)]
    L.cove_route_name.restype = C.c_char_p
    L.cove_route_name.argtypes = [i32]
    L.cove_plan_stream.argtypes = [vp, i32, vp, C.c_size_t, C.POINTER(C.c_size_t), vp]
    L.cove_hybrid_spmv.argtypes = [C.POINTER(HybridDesc), C.POINTER(ValuesDesc), vp, vp, vp]
    L.cove_bitbsr8x4_count.argtypes = [C.POINTER(CsrDesc), vp, vp, C.POINTER(C.c_int64),
                                       C.POINTER(C.c_int64), vp]
    L.cove_bitbsr8x4_fill.argtypes = [C.POINTER(CsrDesc), vp, vp, vp, vp, vp, vp]
    L.cove_pack_words.argtypes = [i64, vp, vp, vp, vp]
    L.cove_lb_layout_count.argtypes = [i32, vp, i32, i32, i32, vp, C.POINTER(C.c_int64), vp]
    L.cove_lb_layout_fill.argtypes = [i32, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp]
    L.cove_spmv.argtypes = [vp, vp, vp, vp]
    L.cove_spmv_route.argtypes = [vp, i32, vp, vp, vp]
    L.cove_spmv_host.argtypes = [vp, vp, vp, vp]
    L.cove_spmv_launches.restype = i32
    L.cove_spmv_launches.argtypes = [vp, i32]
    L.cove_compare_vectors.argtypes = [vp, vp, i64, i32, vp, vp]
    L.cove_canonical_x.argtypes = [vp, i64, i32, vp]
    L.cove_cg_solve.argtypes = [vp, vp, vp, i32, C.POINTER(CgResult), vp]
    L.cove_mm_read.argtypes = [C.c_char_p, i32, C.POINTER(MmMatrix)]
    L.cove_ir_solve.argtypes = [vp, i32, vp, vp, C.c_double, i32, i32, C.POINTER(IrResult), vp]
    L.cove_fcg_solve.argtypes = [vp, i32, vp, vp, C.c_double, i32, i32, C.POINTER(IrResult), vp]
    L.cove_dist_mp_solve.argtypes = [vp, i32, i32, vp, vp, C.c_double, i32, i32, C.POINTER(IrResult), vp]
    L.cove_mm_free.restype = None
    L.cove_mm_free.argtypes = [C.POINTER(MmMatrix)]
    L.cove_cg_solve_noalloc.argtypes = [vp, vp, vp, i32, C.POINTER(CgResult), vp]
    L.cove_dist_halo_plan.restype = i32
    L.cove_dist_halo_plan.argtypes = [i32, i32, vp, vp, i32]
    L.cove_dist_id_bytes.restype = C.c_size_t
    L.cove_dist_make_id.argtypes = [vp]
    L.cove_dist_create.argtypes = [i32, i32, vp, vp, i32, i64, i64, i64, i64, i64, i32,
                                   C.POINTER(vp)]
    L.cove_dist_destroy.argtypes = [vp]
    L.cove_dist_halo.argtypes = [vp, vp, vp]
    L.cove_dist_cg_solve.argtypes = [vp, vp, vp, i32, C.POINTER(CgResult), vp]
    L.cove_dist_spmv.argtypes = [vp, vp, vp, vp]
    L.cove_dist_spmv_launches.restype = i32
    L.cove_dist_spmv_launches.argtypes = [vp]
    L.cove_rng_u64.restype = u64
    L.cove_rng_u64.argtypes = [u64, u64, u64]
    L.cove_rng_uniform01.restype = f64
    L.cove_rng_uniform01.argtypes = [u64, u64, u64]
    L.cove_synth_lapl2d.restype = i64
    L.cove_synth_lapl2d.argtypes = [i32, i32, vp, vp, vp]
    L.cove_synth_lapl3d.restype = i64
    L.cove_synth_lapl3d.argtypes = [i32, i32, i32, i64, i64, i64, vp, vp, vp]
    L.cove_synth_fem27.restype = i64
    L.cove_synth_fem27.argtypes = [i32, i32, i32, i32, u64, vp, vp, vp]
    L.cove_synth_fem27_rows.restype = i64
    L.cove_synth_fem27_rows.argtypes = [i32, i32, i32, i32, u64, i64, i64, i64, vp, vp, vp]
    L.cove_synth_rmat.restype = i64
    L.cove_synth_rmat.argtypes = [i32, i32, f64, f64, f64, u64, vp, vp, vp]
    L.cove_synth_blocksparse.restype = i64
    L.cove_synth_blocksparse.argtypes = [i32, f64, f64, f64, u64, vp, vp, vp]
    L.cove_synth_blocksparse_rows.restype = i64
    L.cove_synth_blocksparse_rows.argtypes = [i32, f64, f64, f64, u64, i64, i64, vp, vp, vp]
    L.cove_synth_blocksparse_device.restype = C.c_int
    L.cove_synth_blocksparse_device.argtypes = [i32, f64, f64, f64, u64, i64, i64, vp, vp, vp,
                                                C.POINTER(C.c_int64), vp]
    L.cove_synth_vector.argtypes = [i32, u64, u64, i64, i32, vp]
    L.cove_synth_lapl3d_device.restype = C.c_int
    L.cove_synth_lapl3d_device.argtypes = [i32, i32, i32, i64, i64, i64, vp, vp, vp,
                                           C.POINTER(C.c_int64), vp]
    L.cove_synth_vector_device.restype = C.c_int
    L.cove_synth_vector_device.argtypes = [i32, u64, u64, i64, i64, vp, vp]
    for fn in ("cove_plan_build", "cove_plan_destroy", "cove_plan_get_info", "cove_plan_stream",
               "cove_hybrid_spmv", "cove_bitbsr8x4_count", "cove_bitbsr8x4_fill", "cove_pack_words",
               "cove_lb_layout_count", "cove_lb_layout_fill",
               "cove_spmv", "cove_spmv_route", "cove_spmv_host", "cove_compare_vectors",
               "cove_canonical_x", "cove_cg_solve", "cove_dist_make_id", "cove_dist_create",
               "cove_dist_destroy", "cove_dist_halo", "cove_dist_cg_solve", "cove_dist_spmv"):
        getattr(L, fn).restype = C.c_int


def check(status):
    if status != 0:
        raise CoveError(status, lib().cove_last_error().decode())


def _np_ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def _stream_handle(stream):
    if stream is None:
        import torch

        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(stream.cuda_stream)


def _dptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _vec(t, n, dtype, name):
    """Device pointer of a contiguous CUDA vector of at least n `dtype` entries;
    the C ABI takes bare pointers, so a wrong element type would be read as
    the plan's type."""
    import torch

    want = torch.float64 if dtype == np.float64 else torch.float32
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise CoveError(1, f"{name} must be a CUDA tensor")
    if t.dtype != want:
        raise CoveError(1, f"{name} is {t.dtype}, the plan computes in {want}")
    if not t.is_contiguous() or t.numel() < n:
        raise CoveError(1, f"{name} must be contiguous with at least {n} entries")
    return C.c_void_p(t.data_ptr())


def default_opts(**kw) -> PlanOpts:
    o = PlanOpts()
    lib().cove_plan_opts_default(C.byref(o))
    for k, v in kw.items():
        if k == "value_codec" and isinstance(v, str):
            v = CODEC[v]
        if k == "split_policy" and isinstance(v, str):
            v = SPLIT[v]
        if k == "lb_style" and isinstance(v, str):
            v = LB_STYLE[v]
        setattr(o, k, v)
    return o


# ---------------------------------------------------------------------------
# plan
# ---------------------------------------------------------------------------

@dataclass
class DeviceCsr:
    """A CSR held in torch CUDA tensors (row_ptr int64 or int32, col int32)."""
    rows: int
    cols: int
    row_ptr: object
    col_idx: object
    values: object

    @classmethod
    def from_numpy(cls, rows, cols, row_ptr, col_idx, values, device="cuda"):
        import torch

        rp = torch.from_numpy(np.ascontiguousarray(row_ptr, dtype=np.int64)).to(device)
        ci = torch.from_numpy(np.ascontiguousarray(col_idx, dtype=np.int32)).to(device)
        v = torch.from_numpy(np.ascontiguousarray(values)).to(device)
        return cls(rows, cols, rp, ci, v)

    def desc(self) -> CsrDesc:
        import torch

        d = CsrDesc()
        d.rows, d.cols = self.rows, self.cols
        d.nnz = int(self.col_idx.numel())
        d.row_ptr = self.row_ptr.data_ptr()
        d.col_idx = self.col_idx.data_ptr() if d.nnz else None
        d.values = self.values.data_ptr() if d.nnz else None
        d.dtype = F64 if self.values.dtype == torch.float64 else F32
        d.row_ptr_i32 = 1 if self.row_ptr.dtype == torch.int32 else 0
        return d


class Plan:
    """A built COVE plan: position streams, value streams, routes, gate."""

    def __init__(self, csr: DeviceCsr, opts: PlanOpts | None = None, stream=None, **kw):
        self._h = C.c_void_p()
        if opts is None:
            opts = default_opts(**kw)
        d = csr.desc()
        check(lib().cove_plan_build(C.byref(d), C.byref(opts), _stream_handle(stream),
                                    C.byref(self._h)))
        self.opts = opts
        self.info = self.get_info()
        self.dtype = np.float64 if self.info.dtype == F64 else np.float32

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            lib().cove_plan_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def get_info(self) -> PlanInfo:
        info = PlanInfo()
        check(lib().cove_plan_get_info(self._h, C.byref(info)))
        return info

    def report(self) -> dict:
        i = self.info
        out = {f: getattr(i, f) for f, _ in PlanInfo._fields_ if f != "algorithmic_bytes"}
        out["algorithmic_bytes"] = list(i.algorithmic_bytes)
        out["joint_value_codec"] = ROUTE_NAMES[i.joint_route]
        out["dispatched_route_name"] = ROUTE_NAMES[i.dispatched_route]
        return out

    def stream(self, name: str, stream=None) -> np.ndarray:
        sid, dt = STREAM[name]
        if dt is None:
            dt = self.dtype
        if dt == "dict":
            dt = np.uint8 if self.info.joint_route == ROUTE_DICT_U8 else np.uint16
        nbytes = C.c_size_t(0)
        check(lib().cove_plan_stream(self._h, sid, None, 0, C.byref(nbytes), _stream_handle(stream)))
        itemsize = np.dtype(dt).itemsize
        out = np.zeros(max(nbytes.value // itemsize, 1), dtype=dt)
        check(lib().cove_plan_stream(self._h, sid, _np_ptr(out), out.nbytes, C.byref(nbytes),
                                     _stream_handle(stream)))
        out = out[: nbytes.value // itemsize]
        if name == "work_items":
            out = out.reshape(-1, 4)
        return out

    def spmv(self, x, y, route=None, stream=None):
        """y = A x on device tensors (dispatched route unless `route` given)."""
        xp = _vec(x, self.info.cols, self.dtype, "x")
        yp = _vec(y, self.info.rows, self.dtype, "y")
        if route is None:
            check(lib().cove_spmv(self._h, xp, yp, _stream_handle(stream)))
        else:
            check(lib().cove_spmv_route(self._h, route, xp, yp, _stream_handle(stream)))
        return y

    def spmv_host(self, x_host: np.ndarray, y_host: np.ndarray | None = None, stream=None):
        """End-to-end call on host arrays (copies in and out; synchronizes)."""
        x_host = np.ascontiguousarray(x_host, dtype=self.dtype)
        if y_host is None:
            y_host = np.empty(self.info.rows, dtype=self.dtype)
        check(lib().cove_spmv_host(self._h, _np_ptr(x_host), _np_ptr(y_host),
                                   _stream_handle(stream)))
        return y_host

    def launches(self, route=None) -> int:
        return int(lib().cove_spmv_launches(self._h, self.info.dispatched_route if route is None
                                            else route))

    def mp_solve(self, b, x, inner_route, tol=1e-10, k_inner=20, max_outer=50, flexible=False,
                 stream=None) -> IrResult:
        """Mixed-precision iterative refinement (flexible=False) or flexible CG."""
        res = IrResult()
        fn = lib().cove_fcg_solve if flexible else lib().cove_ir_solve
        n = self.info.rows
        check(fn(self._h, inner_route, _vec(b, n, self.dtype, "b"), _vec(x, n, self.dtype, "x"), tol,
                 k_inner, max_outer, C.byref(res), _stream_handle(stream)))
        return res

    def cg(self, b, x, iters, stream=None) -> CgResult:
        res = CgResult()
        n = self.info.rows
        check(lib().cove_cg_solve(self._h, _vec(b, n, self.dtype, "b"), _vec(x, n, self.dtype, "x"),
                                  iters, C.byref(res), _stream_handle(stream)))
        return res


def halo_plan(rank, blocks):
    """Transfer plan of `rank` given every rank's (row_begin, row_end,
    window_begin, window_len); list of (peer, send_off, send_n, recv_off, recv_n)."""
    b = np.ascontiguousarray(np.array(blocks, np.int64).reshape(-1))
    world = b.size // 4
    out = np.zeros(5 * max(world, 1), np.int64)
    n = lib().cove_dist_halo_plan(rank, world, _np_ptr(b), _np_ptr(out), world)
    if n < 0:
        raise CoveError(1, "halo is not covered by other ranks' row blocks")
    return [tuple(int(v) for v in out[5 * i: 5 * i + 5]) for i in range(n)]


def compare_vectors(ref, got, stream=None):
    """(max_abs, max_rel, global_rel) on device tensors, computed in T."""
    import torch

    out = np.zeros(3, np.float64)
    dt = F64 if ref.dtype == torch.float64 else F32
    check(lib().cove_compare_vectors(_dptr(ref), _dptr(got), ref.numel(), dt, _np_ptr(out),
                                     _stream_handle(stream)))
    return float(out[0]), float(out[1]), float(out[2])


def canonical_x(t, stream=None):
    import torch

    dt = F64 if t.dtype == torch.float64 else F32
    check(lib().cove_canonical_x(_dptr(t), t.numel(), dt, _stream_handle(stream)))
    return t


# ---------------------------------------------------------------------------
# synthetic workloads (host generators in the library)
# ---------------------------------------------------------------------------

def _two_call(fn, rows, args, vdtype, rows_arr=None):
    nnz = fn(*args, None, None, None)
    rp = np.zeros(rows + 1, np.int64)
    ci = np.zeros(max(nnz, 1), np.int32)
    v = np.zeros(max(nnz, 1), vdtype)
    got = fn(*args, _np_ptr(rp), _np_ptr(ci), _np_ptr(v))
    assert got == nnz
    return rp, ci[:nnz], v[:nnz]


def synth_lapl2d(nx, ny):
    n = nx * ny
    rp, ci, v = _two_call(lib().cove_synth_lapl2d, n, (nx, ny), np.float64)
    return n, n, rp, ci, v


def synth_lapl3d(nx, ny, nz, row_begin=0, row_end=None, col_shift=0):
    n = nx * ny * nz
    if row_end is None:
        row_end = n
    rows = row_end - row_begin
    rp, ci, v = _two_call(lib().cove_synth_lapl3d, rows,
                          (nx, ny, nz, row_begin, row_end, col_shift), np.float64)
    return rows, n, rp, ci, v


def synth_fem27(nx, ny, nz, dof=3, seed=1):
    n = nx * ny * nz * dof
    rp, ci, v = _two_call(lib().cove_synth_fem27, n, (nx, ny, nz, dof, seed), np.float64)
    return n, n, rp, ci, v


def synth_fem27_rows(nx, ny, nz, dof, seed, row_begin, row_end, col_shift=0):
    rows = row_end - row_begin
    rp, ci, v = _two_call(lib().cove_synth_fem27_rows, rows,
                          (nx, ny, nz, dof, seed, row_begin, row_end, col_shift), np.float64)
    return rows, nx * ny * nz * dof, rp, ci, v


def synth_rmat(scale, edge_factor=16, a=0.57, b=0.19, c=0.19, seed=2):
    n = 1 << scale
    rp, ci, v = _two_call(lib().cove_synth_rmat, n, (scale, edge_factor, a, b, c, seed), np.float32)
    return n, n, rp, ci, v


def synth_blocksparse(n, p_block=2e-3, p_entry=0.6, outlier_fraction=1e-3, seed=3):
    rp, ci, v = _two_call(lib().cove_synth_blocksparse, n,
                          (n, p_block, p_entry, outlier_fraction, seed), np.float64)
    return n, n, rp, ci, v


def synth_blocksparse_rows(n, row_begin, row_end, p_block=2e-3, p_entry=0.6, outlier_fraction=1e-3, seed=3):
    """Rows [row_begin, row_end) of synth_blocksparse(n): (row_ptr relative, cols, values)."""
    if lib().cove_synth_blocksparse_rows(n, p_block, p_entry, outlier_fraction, seed, row_begin, row_end,
                                         None, None, None) < 0:
        raise CoveError(1, "row range must cover whole 8-row block rows of [0, n)")
    rp, ci, v = _two_call(lib().cove_synth_blocksparse_rows, row_end - row_begin,
                          (n, p_block, p_entry, outlier_fraction, seed, row_begin, row_end), np.float64)
    return rp, ci, v


def synth_blocksparse_device(n, row_begin, row_end, p_block=2e-3, p_entry=0.6, outlier_fraction=1e-3,
                             seed=3, device="cuda", stream=None):
    """The same rows generated in HBM: (row_ptr int32 relative, cols int32, values f64) tensors."""
    import torch

    L = lib()
    nnz = C.c_int64(0)
    check(L.cove_synth_blocksparse_device(n, p_block, p_entry, outlier_fraction, seed, row_begin, row_end,
                                          None, None, None, C.byref(nnz), _stream_handle(stream)))
    rows = row_end - row_begin
    rp = torch.empty(rows + 1, dtype=torch.int32, device=device)
    ci = torch.empty(max(nnz.value, 1), dtype=torch.int32, device=device)
    v = torch.empty(max(nnz.value, 1), dtype=torch.float64, device=device)
    check(L.cove_synth_blocksparse_device(n, p_block, p_entry, outlier_fraction, seed, row_begin, row_end,
                                          C.c_void_p(rp.data_ptr()), C.c_void_p(ci.data_ptr()),
                                          C.c_void_p(v.data_ptr()), C.byref(nnz), _stream_handle(stream)))
    return rp, ci[: nnz.value], v[: nnz.value]


def read_matrix_market(path, dtype=np.float64):
    """CSR of a coordinate MatrixMarket file (structural::read_matrix_market_with_info):
    (rows, cols, row_ptr int64, col_idx int32, values, info dict)."""
    m = MmMatrix()
    check(lib().cove_mm_read(os.fsencode(path), F64 if dtype == np.float64 else F32, C.byref(m)))
    try:
        rp = np.ctypeslib.as_array(m.row_ptr, (m.rows + 1,)).copy()
        ci = np.ctypeslib.as_array(m.col_idx, (max(m.nnz, 1),))[: m.nnz].copy()
        vt = C.c_double if dtype == np.float64 else C.c_float
        v = np.ctypeslib.as_array(C.cast(m.values, C.POINTER(vt)), (max(m.nnz, 1),))[: m.nnz].copy()
        info = {"field": MM_FIELDS[m.field], "symmetry": MM_SYMMETRIES[m.symmetry],
                "stored_entries": m.stored_entries, "expanded_entries": m.expanded_entries,
                "coalesced_duplicates": m.coalesced_duplicates}
        return m.rows, m.cols, rp, ci, v.astype(dtype, copy=False), info
    finally:
        lib().cove_mm_free(C.byref(m))


def synth_vector(kind, n, seed, stream=7, dtype=np.float64):
    """kind 'uniform_pm1' (U[-1,1]), 'uniform01' (U[0,1]) or 'normal' (N(0,1))."""
    k = {"uniform_pm1": 0, "uniform01": 1, "normal": 2}[kind]
    out = np.zeros(n, dtype)
    lib().cove_synth_vector(k, seed, stream, n, 0 if dtype == np.float64 else 1, _np_ptr(out))
    return out


def rng_uniform01(seed, stream, index):
    return float(lib().cove_rng_uniform01(seed, stream, index))


# The five seeded workloads (sizes scale with `scale` for tests).
def workload(name: str):
    """Full-size CSR of a named workload as (rows, cols, row_ptr, col_idx, values, x)."""
    if name == "lapl2d_512":
        rows, cols, rp, ci, v = synth_lapl2d(512, 512)
        x = synth_vector("uniform_pm1", cols, seed=0)
    elif name == "fem27_64":
        rows, cols, rp, ci, v = synth_fem27(64, 64, 64, 3, seed=1)
        x = synth_vector("uniform_pm1", cols, seed=1)
    elif name == "rmat_22":
        rows, cols, rp, ci, v = synth_rmat(22, 16, seed=2)
        x = synth_vector("uniform01", cols, seed=2, dtype=np.float32)
    else:
        raise KeyError(name)
    return rows, cols, rp, ci, v, x
