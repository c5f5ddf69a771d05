/*
 * cove_synth.h -- seeded synthetic workloads (this library's own API; the
 * reference measures on SuiteSparse files instead, which are not present).
 *
 * All random draws come from one counter-based generator,
 *   u = splitmix64(splitmix64(splitmix64(seed) ^ stream) ^ index),
 *   uniform01 = (u >> 11) * 2^-53,
 * so a value depends only on (seed, stream, index) and any shard of a
 * matrix can be generated independently.  splitmix64 is Steele, Lea and
 * Flood's SplitMix64 finaliser (OOPSLA 2014).  Normal draws use the
 * Box-Muller transform on two uniforms (host libm; host generators only).
 *
 * CSR outputs are row-sorted with strictly increasing columns and no stored
 * zeros.  Two-call protocol: call with null outputs to get rows/nnz, then
 * with buffers of that size.
 */
#ifndef COVE_SYNTH_H
#define COVE_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#include "cove_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

COVE_API uint64_t cove_rng_u64(uint64_t seed, uint64_t stream, uint64_t index);
COVE_API double cove_rng_uniform01(uint64_t seed, uint64_t stream, uint64_t index);

/* 2D 5-point Laplacian on nx x ny, Dirichlet: diagonal 4, neighbours -1 (double). */
COVE_API int64_t cove_synth_lapl2d(int32_t nx, int32_t ny, int64_t* row_ptr, int32_t* col_idx,
                          double* values);

/* 3D 7-point Laplacian on nx x ny x nz, rows [row_begin, row_end), columns
 * shifted by -col_shift (window-local).  Diagonal 6, neighbours -1 (double). */
COVE_API int64_t cove_synth_lapl3d(int32_t nx, int32_t ny, int32_t nz, int64_t row_begin,
                          int64_t row_end, int64_t col_shift, int64_t* row_ptr,
                          int32_t* col_idx, double* values);

/* FEM-like 27-point stencil on nx x ny x nz nodes with `dof` unknowns per
 * node and dense dof x dof couplings: symmetric, off-diagonal 0.05 * N(0,1)
 * keyed by the (min, max) index pair, diagonal 1 + row sum of |off|. */
COVE_API int64_t cove_synth_fem27(int32_t nx, int32_t ny, int32_t nz, int32_t dof, uint64_t seed,
                         int64_t* row_ptr, int32_t* col_idx, double* values);
/* Rows [row_begin, row_end) of the same matrix, columns shifted by -col_shift. */
COVE_API int64_t cove_synth_fem27_rows(int32_t nx, int32_t ny, int32_t nz, int32_t dof, uint64_t seed,
                              int64_t row_begin, int64_t row_end, int64_t col_shift,
                              int64_t* row_ptr, int32_t* col_idx, double* values);

/* R-MAT graph: 2^scale rows, edge_factor * 2^scale edge draws with
 * quadrant probabilities (a, b, c, 1-a-b-c); float values U(0,1];
 * duplicates merged by summation in draw order (float). */
COVE_API int64_t cove_synth_rmat(int32_t scale, int32_t edge_factor, double a, double b, double c,
                        uint64_t seed, int64_t* row_ptr, int32_t* col_idx, float* values);

/* Random 8x4 block-sparse n x n: block present w.p. p_block, entry of a
 * present block w.p. p_entry; values bf16-representable in [-8, 8] (zero
 * redrawn); a fraction `outlier_fraction` of entries replaced by
 * +-U(1e5, 1e6) (double). */
COVE_API int64_t cove_synth_blocksparse(int32_t n, double p_block, double p_entry,
                               double outlier_fraction, uint64_t seed, int64_t* row_ptr,
                               int32_t* col_idx, double* values);

/* Rows [row_begin, row_end) of the same matrix (row_ptr relative, rows + 1
 * entries; global columns).  row_begin a multiple of 8, row_end a multiple
 * of 8 or n.  Returns nnz (-1 for a bad range); null row_ptr counts only. */
COVE_API int64_t cove_synth_blocksparse_rows(int32_t n, double p_block, double p_entry,
                                    double outlier_fraction, uint64_t seed, int64_t row_begin,
                                    int64_t row_end, int64_t* row_ptr, int32_t* col_idx,
                                    double* values);

/* Vectors.  kind 0: U[-1,1]; 1: U[0,1]; 2: N(0,1).  dtype 0 double, 1 float. */
COVE_API void cove_synth_vector(int32_t kind, uint64_t seed, uint64_t stream, int64_t n, int32_t dtype,
                       void* out);

/* Device generator of the 7-point Laplacian rows [row_begin, row_end) into
 * device buffers (int32 row_ptr relative to row_begin, window-local columns
 * shifted by -col_shift).  Returns the status; nnz through *nnz_out when
 * row_ptr is null (count only). */
COVE_API int cove_synth_lapl3d_device(int32_t nx, int32_t ny, int32_t nz, int64_t row_begin,
                             int64_t row_end, int64_t col_shift, int32_t* row_ptr,
                             int32_t* col_idx, double* values, int64_t* nnz_out, void* stream);

/* Device generator of the block-sparse rows [row_begin, row_end) (same
 * matrix and range rules as cove_synth_blocksparse_rows) into device
 * buffers: int32 row_ptr relative to row_begin, global columns.  Returns the
 * status (COVE_ERR_OVERFLOW above INT32_MAX entries); nnz through *nnz_out;
 * null row_ptr counts only. */
COVE_API int cove_synth_blocksparse_device(int32_t n, double p_block, double p_entry,
                                  double outlier_fraction, uint64_t seed, int64_t row_begin,
                                  int64_t row_end, int32_t* row_ptr, int32_t* col_idx,
                                  double* values, int64_t* nnz_out, void* stream);

/* Device U[-1,1] (kind 0) / U[0,1] (kind 1) vector of global indices
 * [begin, begin + n), double. */
COVE_API int cove_synth_vector_device(int32_t kind, uint64_t seed, uint64_t stream, int64_t begin,
                             int64_t n, double* out, void* cuda_stream);

#ifdef __cplusplus
}
#endif

#endif /* COVE_SYNTH_H */
