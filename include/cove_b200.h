/*
 * cove_b200.h -- C ABI of the B200 (sm_100a) COVE SpMV hot path.
 *
 * Plain C: raw pointers, sizes, status codes, a cudaStream_t passed as
 * void*.  Device pointers are device-resident buffers on the current CUDA
 * device; host pointers are noted as such.  Every call is stream-ordered on
 * the given stream; calls that return host data synchronize that stream.
 *
 * Each entry point names the reference interface it replaces
 * (fanna1234/cove-spmv, paths under structural/).  The reference throws
 * std::runtime_error; this layer returns a cove_status and keeps the message
 * for cove_last_error().  The C++ header shim in
 * cove-spmv_b200/include/structural/ maps both back onto the reference's
 * own function names and exceptions.
 */
#ifndef COVE_B200_H
#define COVE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define COVE_API __attribute__((visibility("default")))
#else
#define COVE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    COVE_OK = 0,
    COVE_ERR_INVALID_ARGUMENT = 1, /* bad pointer, size or option (reference: validate() throws) */
    COVE_ERR_INVALID_INPUT = 2,    /* CSR not monotonic / unsorted / duplicate / out of range */
    COVE_ERR_OVERFLOW = 3,         /* a stream exceeds the reference's int32 offsets */
    COVE_ERR_CUDA = 4,             /* a CUDA runtime call failed (reference: cuda_check) */
    COVE_ERR_OUT_OF_MEMORY = 5,
    COVE_ERR_UNSUPPORTED = 6,      /* block shape other than 8x4, unknown codec, ... */
    COVE_ERR_NCCL = 7,             /* a collective failed or timed out */
    COVE_ERR_TIMEOUT = 8           /* a partition wait (NCCL or stream) passed its deadline */
} cove_status;

typedef enum { COVE_F64 = 0, COVE_F32 = 1 } cove_dtype;

/* Requested joint value codec (main_gpu_csr_bitbsr_spmv.cu:49, :1222-1246). */
typedef enum {
    COVE_CODEC_ORIGINAL = 0,     /* lossless hybrid, raw T values ("original") */
    COVE_CODEC_AUTO = 1,         /* dict if <= 256 distinct values, else bfp8 */
    COVE_CODEC_DICT = 2,         /* dict (u8 / u16), bfp8 if > 65536 distinct values */
    COVE_CODEC_BFP8 = 3,         /* int8 x per-block bf16 scale + bf16 residual */
    COVE_CODEC_BFP8_OUTLIER = 4  /* bfp8 + exact global top-P% outlier side list */
} cove_codec;

/* Effective route of a plan (the joint_value_codec report string). */
typedef enum {
    COVE_ROUTE_HYBRID = 0,        /* lossless fp64/fp32 hybrid ("original") */
    COVE_ROUTE_DICT_U8 = 1,       /* "dict_u8_lossless" */
    COVE_ROUTE_DICT_U16 = 2,      /* "dict_u16_lossless" */
    COVE_ROUTE_BFP8 = 3,          /* "bfp8_blocks+bf16_residual" */
    COVE_ROUTE_BFP8_OUTLIER = 4,  /* "bfp8_outlier_blocks+bf16_residual" */
    /* BitBSR-only value codecs of the family runner, cove_hybrid_spmv only: */
    COVE_ROUTE_TILE_CODE = 5,     /* per-cell tile codes + codebook: dict2, unique4/16, dict256,
                                     dict65536, k256, log-k-means (common.cuh:270-319) */
    COVE_ROUTE_BF16_NNZ = 6,      /* per-nnz bf16 values (common.cuh:632-687) */
    COVE_ROUTE_IMPLICIT_ONE = 7,  /* every value 1 (bitbsr_spmv_8x4_lossless.cuh:10-105) */
    COVE_ROUTE_CONST_C = 8,       /* every value value_scale */
    COVE_ROUTE_SIGN2 = 9,         /* +-value_scale by sign_masks (common.cuh:119-125) */
    COVE_ROUTE_FP16_NNZ = 10,     /* per-nnz fp16 values, fp32 accumulate (common.cuh:626-687) */
    COVE_ROUTE_BFP4 = 11          /* packed int4 x per-block bf16 scale (common.cuh:780-835) */
} cove_route;

/* Split policy (main_gpu_csr_bitbsr_spmv.cu:35, :1087-1093). */
typedef enum {
    COVE_SPLIT_COST_GATED = 0,
    COVE_SPLIT_THRESHOLD = 1,
    COVE_SPLIT_NONE = 2,          /* BitBSR only, no residual (family runner operators) */
    COVE_SPLIT_MASK = 3           /* move a block of population p <= threshold iff bit p of
                                     move_mask is set: any predicate of
                                     convert_bitbsr_to_csr_bitbsr_split_if
                                     (csr_bitbsr_split.hpp:405-471), tabulated */
} cove_split_policy;

/* Work-item layout flavour. */
typedef enum {
    COVE_LB_HYBRID = 0,   /* make_fused_8x4_load_balance_layout_host, main_gpu_csr_bitbsr_spmv.cu:387-475 */
    COVE_LB_DEVICE = 1    /* count/fill_bitbsr_8x4_load_balance_work_items, bitbsr_spmv_8x4_common.cuh:199-267 */
} cove_lb_style;

/*
 * CSR input (device pointers).  Column indices must be strictly increasing
 * within a row; stored zeros are dropped (convert.hpp:45, matrix_market.hpp
 * drops them at load).  row_ptr is int64 unless row_ptr_i32 is non-zero.
 */
typedef struct {
    int32_t rows;
    int32_t cols;
    int64_t nnz;
    const void* row_ptr;    /* rows + 1 entries, int64 (or int32 if row_ptr_i32) */
    const int32_t* col_idx; /* nnz */
    const void* values;     /* nnz, double or float */
    int32_t dtype;          /* cove_dtype */
    int32_t row_ptr_i32;
} cove_csr_desc;

/*
 * Plan options.  cove_plan_opts_default() fills the reference defaults:
 * residual_threshold 32, cost model {10, 0, 0, 1} (csr_bitbsr_split.hpp:53-58,
 * main_gpu_csr_bitbsr_spmv.cu:40), lb chunk 32 / split = chunk (:42-43,
 * :175-177), long_row_split 0 (:41), codec "original", outlier fraction
 * 0.005 (:1291), gate 1e-2 (:1375).
 */
typedef struct {
    int32_t residual_threshold;
    int32_t split_policy;              /* cove_split_policy */
    double cost_bitmap_block;
    double cost_bitmap_nnz;
    double cost_csr_block;
    double cost_csr_nnz;
    int32_t lb_chunk_blocks;
    int32_t lb_split_threshold_blocks; /* < 0: equal to lb_chunk_blocks */
    int32_t lb_style;                  /* cove_lb_style */
    int32_t long_row_split;            /* tau; 0 = no long-row chunks */
    int32_t value_codec;               /* cove_codec */
    double outlier_fraction;
    double gate_tolerance;             /* joint route passes iff 0 <= rel <= tolerance */
    int32_t gate_enable;               /* evaluate the gate and fall back on failure */
    int32_t keep_full_bitbsr;          /* keep the un-split BitBSR for cove_plan_stream */
    int32_t keep_lossless;             /* keep raw values after a joint route passes */
    uint64_t move_mask;                /* COVE_SPLIT_MASK only: bits 0..32, by block population */
} cove_plan_opts;

typedef struct cove_plan cove_plan;

/* Plan report: the counters and keys the reference CLI prints
 * (main_gpu_csr_bitbsr_spmv.cu:1366-1476). */
typedef struct {
    int32_t rows, cols, dtype;
    int64_t nnz;                 /* after dropping stored zeros */
    int64_t full_blocks, kept_blocks, residual_blocks, cost_skipped_blocks;
    int64_t kept_nnz, residual_nnz, cost_skipped_nnz;
    int64_t work_items, long_rows, long_row_chunks, num_outliers;
    int64_t value_cardinality;   /* distinct values, or -1 if > 65536 (not counted) */
    int64_t full_bitbsr_position_bits, kept_bitbsr_position_bits;
    int64_t residual_csr_position_bits, split_position_bits;
    int32_t requested_codec;     /* cove_codec */
    int32_t joint_route;         /* cove_route chosen by the codec menu */
    int32_t dispatched_route;    /* joint_route if the gate passed, else COVE_ROUTE_HYBRID */
    int32_t gate_evaluated;
    int32_t gate_pass;
    double joint_rel_err;        /* global_rel on the canonical x, -1 if not evaluated */
    double joint_bytes_per_nnz;  /* reference formula, :1261-1263 / :1322-1325 / :1354-1356 */
    double outlier_threshold;
    int64_t algorithmic_bytes[5];/* bytes one SpMV of each cove_route must move (0 if absent) */
    int32_t kernel_slots;        /* lanes per block row / 8 in the fused kernel; 0: one lane per row */
    int32_t kernel_overflow_tasks;
} cove_plan_info;

/* Streams that cove_plan_stream can copy out (bit-exact parity checks). */
typedef enum {
    COVE_STREAM_FULL_BLOCK_ROW_PTR = 0,   /* int32  nbr+1            DeviceBitBsrMatrix::block_row_ptr */
    COVE_STREAM_FULL_BLOCK_COL_IDX = 1,   /* int32  full blocks */
    COVE_STREAM_FULL_BITMAP = 2,          /* uint32 full blocks */
    COVE_STREAM_FULL_VALUES = 3,          /* T      nnz */
    COVE_STREAM_FULL_BLOCK_ROW_VAL_PTR = 4,/* int32 nbr+1 */
    COVE_STREAM_KEPT_BLOCK_ROW_PTR = 10,  /* int32  nbr+1            split.bitbsr */
    COVE_STREAM_KEPT_BLOCK_COL_IDX = 11,  /* int32  kept blocks */
    COVE_STREAM_KEPT_BITMAP = 12,         /* uint32 kept blocks */
    COVE_STREAM_KEPT_VALUES = 13,         /* T      kept nnz */
    COVE_STREAM_KEPT_BLOCK_VAL_PTR = 14,  /* int32  kept blocks + 1  BitBsrMatrix::block_val_ptr */
    COVE_STREAM_KEPT_BLOCK_ROW_VAL_PTR = 15, /* int32 nbr+1 */
    COVE_STREAM_RES_ROW_PTR = 20,         /* int32  rows+1           split.residual */
    COVE_STREAM_RES_COL_IDX = 21,         /* int32  residual nnz */
    COVE_STREAM_RES_VALUES = 22,          /* T      residual nnz */
    COVE_STREAM_WORDS = 30,               /* uint64 kept blocks      packed col/flag/bitmap */
    COVE_STREAM_WORK_ITEMS = 31,          /* uint32x4 work items */
    COVE_STREAM_WORK_ITEM_ROW_PTR = 32,   /* int32  nbr+1 */
    COVE_STREAM_CHUNK_ROW = 40,           /* int32  long-row chunks */
    COVE_STREAM_CHUNK_PBEGIN = 41,        /* int32 */
    COVE_STREAM_CHUNK_PCOUNT = 42,        /* int32 */
    COVE_STREAM_DICT_CODEBOOK = 50,       /* T      distinct values, first-occurrence order */
    COVE_STREAM_DICT_KEPT_IDX = 51,       /* uint8 or uint16 per kept nnz */
    COVE_STREAM_DICT_RES_IDX = 52,        /* uint8 or uint16 per residual nnz */
    COVE_STREAM_BFP8_INT8 = 60,           /* int8   kept nnz */
    COVE_STREAM_BFP8_SCALE = 61,          /* uint16 kept blocks (bf16 bits) */
    COVE_STREAM_RES_BF16 = 62,            /* uint16 residual nnz */
    COVE_STREAM_OUTLIER_ROWS = 63,        /* int32  outliers */
    COVE_STREAM_OUTLIER_COLS = 64,        /* int32 */
    COVE_STREAM_OUTLIER_VALS = 65         /* T */
} cove_stream_id;

/* ---- errors ---------------------------------------------------------- */

/* Message of the last failing call on this host thread ("" if none). */
COVE_API const char* cove_last_error(void);
COVE_API const char* cove_status_string(cove_status s);
/* Library version string.  0.2: cove_plan_opts ends with move_mask
 * (COVE_SPLIT_MASK); callers built against 0.1 must be rebuilt. */
COVE_API const char* cove_version(void);

/* ---- plan (converter + split + layout + codecs + gate) --------------- */

COVE_API void cove_plan_opts_default(cove_plan_opts* opts);

/*
 * Build a plan from a device CSR on the current device.  Replaces the host
 * pipeline of the hybrid/joint operator: convert_to_bitbsr +
 * convert_bitbsr_to_csr_bitbsr_split_cost_gated (main_gpu_csr_bitbsr_spmv.cu:1083-1097),
 * copy_bitbsr_to_device (:1099-1105), make_fused_8x4_load_balance_layout_host
 * (:1113-1122), the residual upload and long-row chunks (:1142-1184), the
 * joint value menu (:1222-1358) and the joint gate (:1360-1376, with the
 * fall-back of structural/scripts/plot_eval_performance.py:216-219).
 * All stages run as sm_100a kernels on `stream`.
 */
COVE_API cove_status cove_plan_build(const cove_csr_desc* csr, const cove_plan_opts* opts, void* stream,
                            cove_plan** out);
COVE_API cove_status cove_plan_destroy(cove_plan* plan);
COVE_API cove_status cove_plan_get_info(const cove_plan* plan, cove_plan_info* info);
/* Report name of a route ("dict_u8_lossless", ...); "original" for HYBRID. */
COVE_API const char* cove_route_name(int32_t route);

/*
 * Copy a stream to host memory (synchronizes `stream`).  With dst == NULL
 * only *bytes is set.  Returns COVE_ERR_INVALID_ARGUMENT if the plan does not
 * hold that stream or capacity is short.
 */
COVE_API cove_status cove_plan_stream(const cove_plan* plan, int32_t which, void* dst_host,
                             size_t capacity, size_t* bytes, void* stream);

/* ---- step-by-step device API on caller-owned buffers ------------------- */

/*
 * CSR -> BitBSR 8x4, first step: validates the CSR and writes
 * block_row_ptr and block_row_val_ptr (both num_block_rows + 1 int32) and
 * the block and nnz totals, so the caller can size the next step.
 * With cove_bitbsr8x4_fill this replaces
 * convert_to_bitbsr_gpu_warp_direct_8x4_device (gpu_convert.cuh:406-512).
 */
COVE_API cove_status cove_bitbsr8x4_count(const cove_csr_desc* csr, int32_t* block_row_ptr,
                                          int32_t* block_row_val_ptr, int64_t* num_blocks,
                                          int64_t* nnz, void* stream);
/* Second step: block_col_idx (int32), bitmap (uint32) per block, values (T) per nnz. */
COVE_API cove_status cove_bitbsr8x4_fill(const cove_csr_desc* csr, const int32_t* block_row_ptr,
                                         const int32_t* block_row_val_ptr, int32_t* block_col_idx,
                                         uint32_t* bitmap, void* values, void* stream);
/* Packed words without flags: make_bitbsr_8x4_col_bitmap_packed (common.cuh:1024-1050). */
COVE_API cove_status cove_pack_words(int64_t num_blocks, const int32_t* block_col_idx,
                                     const uint32_t* bitmap, uint64_t* words, void* stream);
/*
 * Work items, first step: item_row_ptr (num_block_rows + 1) and the item
 * count.  style = cove_lb_style.  Second step fills the 16-byte items and
 * sets the flag bit of `words` where the layout asks for it.  Together they
 * replace make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items
 * (common.cuh:1052-1147, style DEVICE) and make_fused_8x4_load_balance_layout_host
 * (main_gpu_csr_bitbsr_spmv.cu:387-475, style HYBRID).
 */
COVE_API cove_status cove_lb_layout_count(int32_t num_block_rows, const int32_t* block_row_ptr,
                                          int32_t chunk_blocks, int32_t split_threshold_blocks,
                                          int32_t style, int32_t* item_row_ptr,
                                          int64_t* num_items, void* stream);
COVE_API cove_status cove_lb_layout_fill(int32_t num_block_rows, const int32_t* block_row_ptr,
                                         const int32_t* block_row_val_ptr, const uint32_t* bitmap,
                                         const int32_t* item_row_ptr, int32_t chunk_blocks,
                                         int32_t split_threshold_blocks, int32_t style,
                                         uint64_t* words, void* items, void* stream);

/* ---- SpMV ----------------------------------------------------------- */

/*
 * y = A x on the dispatched route (x: cols, y: rows, both device, dtype T).
 * Replaces run_csr_bitbsr_fused_8x4_lb / _bfp8 / _dict / _bfp8_outlier
 * (main_gpu_csr_bitbsr_spmv.cu:636-712, :899-1029).  y needs no zero-fill:
 * every row is written.  Asynchronous on `stream`.
 */
COVE_API cove_status cove_spmv(const cove_plan* plan, const void* x, void* y, void* stream);

/*
 * Caller-owned streams of the fused hybrid operator (the argument lists of
 * run_csr_bitbsr_fused_8x4_lb / _bfp8 / _dict / _bfp8_outlier,
 * main_gpu_csr_bitbsr_spmv.cu:636-650, :899-915, :932-948, :984-1003).
 * All pointers are device pointers; the flag bit of the words is ignored.
 */
typedef struct {
    int32_t rows, cols, num_block_rows, dtype;
    int64_t kept_blocks, kept_nnz, residual_nnz;
    const int32_t* block_row_ptr;      /* kept BitBSR, nbr+1 (DeviceBitBsrMatrix::block_row_ptr) */
    const int32_t* block_row_val_ptr;  /* nbr+1 (DeviceBitBsrMatrix::block_row_val_ptr) */
    const uint64_t* words;             /* packed col/flag/bitmap per kept block */
    const int32_t* res_row_ptr;        /* rows+1 */
    const int32_t* res_col_idx;        /* residual nnz */
    int32_t long_row_tau;              /* residual rows longer than this use the chunks */
    int64_t num_chunks;
    const int32_t* chunk_row;
    const int32_t* chunk_pbegin;
    const int32_t* chunk_pcount;
} cove_hybrid_desc;

typedef struct {
    int32_t route;                 /* cove_route */
    const void* kept;              /* T / uint8 / uint16 codes / int8, per kept nnz */
    const void* res;               /* T / codes / uint16 bf16, per residual nnz */
    const uint16_t* block_scale;   /* bfp8: bf16 bits per kept block */
    const void* codebook;          /* dict: T values */
    int64_t codebook_size;
    int64_t num_outliers;          /* bfp8_outlier side list */
    const int32_t* outlier_rows;
    const int32_t* outlier_cols;
    const void* outlier_vals;
    const uint32_t* tile_code_words;  /* tile-code route: tile_bits words per kept block */
    int32_t tile_bits;                /* 1, 2, 4, 8 or 16 */
    double value_scale;               /* const_c: the constant; sign2: the scale (1 for +-1) */
    const uint32_t* sign_masks;       /* sign2: one word per kept block, bit = cell, set = + */
} cove_values_desc;
/* Routes 7-11 are BitBSR-only value codecs of the family runner: the
 * hybrid descriptor must carry no residual.  fp16: kept = uint16 bits per
 * nnz; bfp4: kept = (nnz + 1) / 2 bytes of nibbles, block_scale = bf16 bits
 * per kept block. */

/*
 * y = A x over caller-owned streams.  Replaces the four launchers of
 * main_gpu_csr_bitbsr_spmv.cu:636-1029; the caller need not zero y.
 * Asynchronous on `stream`.
 */
COVE_API cove_status cove_hybrid_spmv(const cove_hybrid_desc* a, const cove_values_desc* v,
                                      const void* x, void* y, void* stream);

/* Same on an explicit route (the plan must hold that route's streams). */
COVE_API cove_status cove_spmv_route(const cove_plan* plan, int32_t route, const void* x, void* y,
                            void* stream);

/*
 * End-to-end call with HOST x and y (pinned or pageable): copies x in,
 * runs the dispatched route, copies y out, synchronizes `stream`.  The
 * device staging buffers belong to the plan.
 */
COVE_API cove_status cove_spmv_host(cove_plan* plan, const void* x_host, void* y_host, void* stream);

/* Number of kernel launches one cove_spmv / cove_spmv_route call makes. */
COVE_API int32_t cove_spmv_launches(const cove_plan* plan, int32_t route);

/*
 * Global-norm relative error of `got` against `ref` on the device
 * (compare_vectors, spmv.hpp:73-89): out3 = {max_abs, max_rel, global_rel}
 * computed in T.  Synchronizes `stream`.
 */
COVE_API cove_status cove_compare_vectors(const void* ref, const void* got, int64_t n, int32_t dtype,
                                 double* out3, void* stream);

/* Canonical gate input x[i] = T((i % 17) - 8) * T(0.125) (spmv_harness.hpp:32-39). */
COVE_API cove_status cove_canonical_x(void* x, int64_t n, int32_t dtype, void* stream);

/* ---- MatrixMarket reader (matrix_market.hpp:327-382) ------------------- */

typedef enum { COVE_MM_REAL = 0, COVE_MM_INTEGER = 1, COVE_MM_COMPLEX = 2, COVE_MM_PATTERN = 3 } cove_mm_field;
typedef enum {
    COVE_MM_GENERAL = 0, COVE_MM_SYMMETRIC = 1, COVE_MM_SKEW_SYMMETRIC = 2, COVE_MM_HERMITIAN = 3
} cove_mm_symmetry;

/* A CSR matrix read from a coordinate MatrixMarket file; host arrays owned
 * by the library (release with cove_mm_free). */
typedef struct {
    int32_t rows, cols;
    int64_t nnz;                   /* after duplicate summation and zero dropping */
    int64_t* row_ptr;              /* rows + 1 */
    int32_t* col_idx;              /* nnz, ascending within each row */
    void* values;                  /* nnz of dtype */
    int32_t dtype;                 /* cove_dtype */
    int32_t field;                 /* cove_mm_field */
    int32_t symmetry;              /* cove_mm_symmetry */
    int64_t stored_entries;        /* entries declared in the file */
    int64_t expanded_entries;      /* after symmetric expansion */
    int64_t coalesced_duplicates;  /* expanded entries minus nnz */
} cove_mm_matrix;

/*
 * read_matrix_market_with_info<T> (matrix_market.hpp:327-382): banner check,
 * comments, 1-based indices, pattern = 1, symmetric / skew-symmetric
 * expansion, per-row column sort, duplicates summed (in file order), exact
 * zeros dropped, values parsed as double and cast to the dtype.  Errors
 * (bad header, index out of range, short file, complex/hermitian) return a
 * status with the reference's message in cove_last_error().
 */
COVE_API cove_status cove_mm_read(const char* path, int32_t dtype, cove_mm_matrix* out);
COVE_API void cove_mm_free(cove_mm_matrix* m);

/* ---- conjugate gradient (bench_cg_solve.cu:165-197) ------------------ */

typedef struct {
    int32_t iterations;
    double rs_initial;   /* r0 . r0 */
    double rs_final;     /* r . r after the last iteration */
    double ms_total;     /* device time of the iterations (CUDA events) */
    double ms_spmv;      /* device time of the SpMV kernels alone (sum) */
    int64_t launches;    /* kernel launches of this library in the call */
} cove_cg_result;

/*
 * Textbook fp64 CG, x0 = 0, r = p = b, `iters` iterations of
 * {Ap = A p; alpha = rs / (p.Ap); x += alpha p; r -= alpha Ap;
 *  rs' = r.r; beta = rs'/rs; p = r + beta p}.  alpha and beta stay on the
 * device.  Single GPU; b, x device vectors of length rows (rows == cols).
 * The work vectors (r, p, Ap: three n-vectors) are allocated by the first
 * solve on a plan and kept in the plan for the next ones (freed with it), so
 * solves on one plan must not overlap on the GPU.
 */
COVE_API cove_status cove_cg_solve(const cove_plan* plan, const void* b, void* x, int32_t iters,
                          cove_cg_result* result, void* stream);

/* ---- mixed-precision solvers (bench_cg_solve.cu:280-448) --------------- */

typedef struct {
    int32_t outer;          /* outer iterations run */
    int32_t inner_total;    /* inner CG iterations run, all outer steps */
    double final_relres;    /* ||b - A x|| / ||b|| with the exact (lossless) route */
    int32_t reached;        /* final_relres <= tol */
    double ms_total;        /* device time of the solve (CUDA events) */
} cove_ir_result;

/*
 * Iterative refinement (run_ir, bench_cg_solve.cu:280-351): x0 = 0; until
 * ||r|| / ||b|| < tol or max_outer steps: d = k_inner steps of CG on
 * A d = r with the plan's `inner_route` (stopping for good when p.Ap is not
 * positive), x += d, r = b - A x with the exact route (the lossless hybrid
 * if the plan keeps it, else its lossless dictionary route).  Single GPU;
 * fp64 plans; b, x device vectors of length rows (rows == cols).
 */
COVE_API cove_status cove_ir_solve(const cove_plan* plan, int32_t inner_route, const void* b, void* x,
                                   double tol, int32_t k_inner, int32_t max_outer,
                                   cove_ir_result* result, void* stream);

/*
 * Flexible preconditioned CG (run_fcg, bench_cg_solve.cu:355-448): one outer
 * CG on the exact route, preconditioned by z = (k_inner inner CG steps on
 * `inner_route`) r, Polak-Ribiere beta = max(0, (r'.z' - r'.z) / r.z).
 */
COVE_API cove_status cove_fcg_solve(const cove_plan* plan, int32_t inner_route, const void* b, void* x,
                                    double tol, int32_t k_inner, int32_t max_outer,
                                    cove_ir_result* result, void* stream);

/*
 * CG that allocates no device memory.  It has no counterpart in the
 * reference.
 *
 * For callers that cannot call cudaMalloc while they run: applications whose
 * device memory belongs to their own pool or arena allocator (HBM reserved
 * up front, so a library's cudaMalloc fails or bypasses their accounting),
 * and loops with a latency budget, where cudaMalloc/cudaFree may synchronize
 * the device and take unbounded time.  Build the plan at set-up; this call
 * then runs the same recurrence as cove_cg_solve (same x and rs values)
 * with its work vectors in one fixed device array of about 3 MiB, held by
 * every GPU on which the library's CG code is loaded until the process
 * exits.  It calls no cudaMalloc, cudaFree or other allocating routine.
 *
 * Limits and rules:
 *  - plan rows <= COVE_CG_NOALLOC_MAX_ROWS; a larger plan is rejected with
 *    COVE_ERR_INVALID_ARGUMENT and a message naming the limit;
 *  - the first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture begins.  After cudaDeviceReset the next call
 *    on that device looks the address up again (the array then lives in a
 *    new context, starting from zero);
 *  - all calls on one device share the array: calls that overlap on the GPU
 *    (other streams, other host threads) race and give wrong results;
 *  - synchronizes `stream`; result->ms_total and ms_spmv are 0 (no timing).
 */
#define COVE_CG_NOALLOC_MAX_ROWS 131072
COVE_API cove_status cove_cg_solve_noalloc(const cove_plan* plan, const void* b, void* x,
                                           int32_t iters, cove_cg_result* result, void* stream);

/* ---- multi-GPU row-block partition (one process per GPU) -------------- */

typedef struct cove_dist cove_dist;

/* Size of the opaque NCCL unique id blob rank 0 creates and broadcasts. */
COVE_API size_t cove_dist_id_bytes(void);
COVE_API cove_status cove_dist_make_id(void* id_out);

/*
 * Join the communicator.  `plans` holds this rank's local row block
 * [row_begin, row_end) as one or more plans of consecutive rows; each plan's
 * columns are window-local: window column j is global column
 * (window_begin + j), window = [window_begin, window_begin + window_len).
 * The halo is the part of the window outside [row_begin, row_end); it must
 * lie within the neighbouring ranks' row blocks.
 */
COVE_API cove_status cove_dist_create(int32_t rank, int32_t world, const void* nccl_id,
                             cove_plan* const* plans, int32_t num_plans,
                             int64_t global_rows, int64_t row_begin, int64_t row_end,
                             int64_t window_begin, int64_t window_len,
                             int32_t timeout_ms, cove_dist** out);
COVE_API cove_status cove_dist_destroy(cove_dist* d);

/*
 * Halo transfer plan of `rank` (host only, no communicator): blocks4 holds
 * every rank's {row_begin, row_end, window_begin, window_len}; writes up to
 * `cap` records {peer, send_offset, send_count, recv_offset, recv_count}
 * (offsets into this rank's window) and returns their number, or -1 when
 * the window outside the rank's rows is not covered exactly by other ranks'
 * rows.  cove_dist_create uses it after an allgather of the blocks.
 */
COVE_API int32_t cove_dist_halo_plan(int32_t rank, int32_t world, const int64_t* blocks4,
                                     int64_t* xfers5, int32_t cap);

/* Halo exchange of a window vector (device, window_len T) over NCCL. */
COVE_API cove_status cove_dist_halo(cove_dist* d, void* x_window, void* stream);

/* Distributed CG over the partition; b and x are the local row blocks.
 * result->ms_spmv times the distributed SpMV (halo exchange included).  The
 * work vectors are kept in the handle between solves (freed with it). */
COVE_API cove_status cove_dist_cg_solve(cove_dist* d, const void* b_local, void* x_local, int32_t iters,
                               cove_cg_result* result, void* stream);

/* The mixed-precision solvers on the partition (flexible = 0: iterative
 * refinement, 1: flexible CG); b and x are the local row blocks. */
COVE_API cove_status cove_dist_mp_solve(cove_dist* d, int32_t flexible, int32_t inner_route,
                                        const void* b_local, void* x_local, double tol, int32_t k_inner,
                                        int32_t max_outer, cove_ir_result* result, void* stream);

/* Distributed SpMV: y_local = A_local x_window after the halo exchange of
 * x_window.  The exchange runs on a second stream while the block rows that
 * read only the rank's own columns are computed; the others follow it. */
COVE_API cove_status cove_dist_spmv(cove_dist* d, void* x_window, void* y_local, void* stream);

/* Kernel launches of this library in one cove_dist_spmv (NCCL's excluded). */
COVE_API int32_t cove_dist_spmv_launches(const cove_dist* d);

#ifdef __cplusplus
}
#endif

#endif /* COVE_B200_H */
