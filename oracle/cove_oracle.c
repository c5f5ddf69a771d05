/*
 * cove_oracle.c -- CPU oracle for the COVE SpMV hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is a plain-C restatement of the
 * reference's host algorithms (fanna1234/cove-spmv, `structural/`), written
 * so that the CUDA product path can be checked against it.  Only the test
 * suite, `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py`
 * load it, and only as the checker.  Nothing in the product library links,
 * calls or falls back to it.
 *
 * Parity pin: every function here is checked (tests/test_oracle_golden.py)
 * against the known-answer vectors of the reference's own tests
 * (structural/tests/test_structural.cpp, structural/tests/test_gpu_convert.cu,
 * structural/tests/test_gpu_csr_bitbsr_spmv_cli.sh) and against the
 * reference itself, compiled from its headers into oracle/_ref/ by
 * oracle/Makefile, on seeded random matrices (fixtures in tests/golden/).
 *
 * Offsets are int64 here (the reference uses int32 `Offset`,
 * structural/include/structural/types.hpp:7-8); for inputs below 2^31 the
 * results are identical.  Values are handled as raw bytes of `esz` bytes
 * (8 = double, 4 = float) wherever the reference only moves them.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define OC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* value helpers                                                             */
/* ------------------------------------------------------------------------ */

static double load_as_double(const unsigned char* base, int64_t i, int esz) {
    if (esz == 8) {
        double v;
        memcpy(&v, base + i * 8, 8);
        return v;
    }
    float f;
    memcpy(&f, base + i * 4, 4);
    return (double)f;
}

/* `value == T{}` in the element type (convert.hpp:45,55,130). */
static int value_is_zero(const unsigned char* base, int64_t i, int esz) {
    if (esz == 8) {
        double v;
        memcpy(&v, base + i * 8, 8);
        return v == 0.0;
    }
    float f;
    memcpy(&f, base + i * 4, 4);
    return f == 0.0f;
}

static uint64_t value_key(const unsigned char* base, int64_t i, int esz) {
    /* raw-bit key, zero-extended for float (main_gpu_csr_bitbsr_spmv.cu:1226-1230) */
    uint64_t k = 0;
    memcpy(&k, base + i * esz, (size_t)esz);
    return k;
}

static int popcount32(uint32_t w) { return __builtin_popcount(w); }

static int64_t ceil_div64(int64_t v, int64_t d) { return (v + d - 1) / d; }

/* ------------------------------------------------------------------------ */
/* BitBSR container                                                          */
/* ------------------------------------------------------------------------ */

typedef struct oc_bitbsr {
    int32_t rows, cols, block_rows, block_cols;
    int32_t num_block_rows, num_block_cols, words_per_block;
    int32_t esz;
    int64_t num_blocks, nnz;
    int64_t* block_row_ptr;  /* num_block_rows + 1 */
    int32_t* block_col_idx;  /* num_blocks */
    uint32_t* bitmap_words;  /* num_blocks * words_per_block */
    int64_t* block_val_ptr;  /* num_blocks + 1 */
    unsigned char* values;   /* nnz * esz */
} oc_bitbsr;

OC_EXPORT void oc_bitbsr_free(oc_bitbsr* m) {
    if (!m) return;
    free(m->block_row_ptr);
    free(m->block_col_idx);
    free(m->bitmap_words);
    free(m->block_val_ptr);
    free(m->values);
    free(m);
}

static void set_err(char* err, int errlen, const char* msg) {
    if (err && errlen > 0) {
        snprintf(err, (size_t)errlen, "%s", msg);
    }
}

static int cmp_i32(const void* a, const void* b) {
    const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

/* CSR validation, csr.hpp:21-49. */
static int csr_validate(int32_t rows, int32_t cols, const int64_t* row_ptr,
                        const int32_t* col_idx, int64_t nnz, char* err, int errlen) {
    if (rows < 0 || cols < 0) {
        set_err(err, errlen, "CSR dimensions must be non-negative");
        return 0;
    }
    if (row_ptr[0] != 0) {
        set_err(err, errlen, "CSR row_ptr must start at zero");
        return 0;
    }
    for (int32_t r = 0; r < rows; ++r) {
        if (row_ptr[r] > row_ptr[r + 1]) {
            set_err(err, errlen, "CSR row_ptr must be monotonic");
            return 0;
        }
    }
    if (row_ptr[rows] != nnz) {
        set_err(err, errlen, "CSR row_ptr.back must equal nnz");
        return 0;
    }
    for (int64_t p = 0; p < nnz; ++p) {
        if (col_idx[p] < 0 || col_idx[p] >= cols) {
            set_err(err, errlen, "CSR column index out of range");
            return 0;
        }
    }
    return 1;
}

/*
 * CSR -> BitBSR with any block shape.  Restates convert_to_bitbsr
 * (structural/include/structural/convert.hpp:13-165):
 *   - stored zeros are skipped (:45, :55, :130);
 *   - per block row, block columns are the sorted distinct col/bc (:51-80);
 *   - each block's values are written in CSR traversal order (row, then CSR
 *     position) into the block's value range (:116-153);
 *   - a second entry on the same bit is an error (:147-149);
 *   - bit = local_row * bc + local_col, word = bit / 32 (:136-146).
 */
OC_EXPORT oc_bitbsr* oc_convert_to_bitbsr(int32_t rows, int32_t cols, const int64_t* row_ptr,
                                          const int32_t* col_idx, const void* values_v,
                                          int32_t esz, int32_t br, int32_t bc, char* err,
                                          int32_t errlen) {
    const unsigned char* values = (const unsigned char*)values_v;
    const int64_t nnz_in = row_ptr[rows];
    if (!csr_validate(rows, cols, row_ptr, col_idx, nnz_in, err, errlen)) return NULL;
    if (br <= 0 || bc <= 0) {
        set_err(err, errlen, "BitBSR block sizes must be positive");
        return NULL;
    }
    oc_bitbsr* out = (oc_bitbsr*)calloc(1, sizeof(oc_bitbsr));
    out->rows = rows;
    out->cols = cols;
    out->block_rows = br;
    out->block_cols = bc;
    out->num_block_rows = (int32_t)ceil_div64(rows, br);
    out->num_block_cols = (int32_t)ceil_div64(cols, bc);
    out->words_per_block = (int32_t)ceil_div64((int64_t)br * bc, 32);
    out->esz = esz;
    const int32_t nbr = out->num_block_rows;
    const int32_t wpb = out->words_per_block;

    /* pass 1: distinct block columns per block row and nnz per block row */
    int64_t* blocks_prefix = (int64_t*)calloc((size_t)nbr + 1, sizeof(int64_t));
    int64_t* nnz_prefix = (int64_t*)calloc((size_t)nbr + 1, sizeof(int64_t));
    int32_t** active = (int32_t**)calloc((size_t)nbr + 1, sizeof(int32_t*));
    int64_t* active_n = (int64_t*)calloc((size_t)nbr + 1, sizeof(int64_t));
    for (int32_t b = 0; b < nbr; ++b) {
        const int32_t r0 = b * br;
        const int32_t r1 = (r0 + br < rows) ? r0 + br : rows;
        int64_t cnt = 0;
        for (int32_t r = r0; r < r1; ++r)
            for (int64_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p)
                if (!value_is_zero(values, p, esz)) ++cnt;
        int32_t* seen = (int32_t*)malloc((size_t)(cnt > 0 ? cnt : 1) * sizeof(int32_t));
        int64_t k = 0;
        for (int32_t r = r0; r < r1; ++r)
            for (int64_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p)
                if (!value_is_zero(values, p, esz)) seen[k++] = col_idx[p] / bc;
        qsort(seen, (size_t)cnt, sizeof(int32_t), cmp_i32);
        int64_t nd = 0;
        for (int64_t i = 0; i < cnt; ++i)
            if (i == 0 || seen[i] != seen[i - 1]) seen[nd++] = seen[i];
        active[b] = seen;
        active_n[b] = nd;
        blocks_prefix[b + 1] = nd;
        nnz_prefix[b + 1] = cnt;
    }
    for (int32_t b = 0; b < nbr; ++b) {
        blocks_prefix[b + 1] += blocks_prefix[b];
        nnz_prefix[b + 1] += nnz_prefix[b];
    }
    const int64_t nblocks = blocks_prefix[nbr];
    const int64_t nnz = nnz_prefix[nbr];
    out->num_blocks = nblocks;
    out->nnz = nnz;
    out->block_row_ptr = blocks_prefix;
    out->block_col_idx = (int32_t*)malloc((size_t)(nblocks > 0 ? nblocks : 1) * 4);
    out->bitmap_words = (uint32_t*)calloc((size_t)(nblocks * wpb > 0 ? nblocks * wpb : 1), 4);
    out->block_val_ptr = (int64_t*)calloc((size_t)nblocks + 1, sizeof(int64_t));
    out->values = (unsigned char*)malloc((size_t)(nnz > 0 ? nnz : 1) * (size_t)esz);

    /* block_val_ptr from per-block counts; counts need a second walk */
    int64_t* block_counts = (int64_t*)calloc((size_t)(nblocks > 0 ? nblocks : 1), sizeof(int64_t));
    for (int32_t b = 0; b < nbr; ++b) {
        const int32_t r0 = b * br;
        const int32_t r1 = (r0 + br < rows) ? r0 + br : rows;
        const int64_t first = blocks_prefix[b];
        for (int64_t i = 0; i < active_n[b]; ++i) out->block_col_idx[first + i] = active[b][i];
        for (int32_t r = r0; r < r1; ++r) {
            for (int64_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
                if (value_is_zero(values, p, esz)) continue;
                const int32_t bcol = col_idx[p] / bc;
                /* lower_bound over the sorted distinct list */
                int64_t lo = 0, hi = active_n[b];
                while (lo < hi) {
                    const int64_t mid = (lo + hi) / 2;
                    if (active[b][mid] < bcol) lo = mid + 1; else hi = mid;
                }
                block_counts[first + lo] += 1;
            }
        }
    }
    for (int64_t i = 0; i < nblocks; ++i)
        out->block_val_ptr[i + 1] = out->block_val_ptr[i] + block_counts[i];

    int ok = 1;
    int64_t* write_pos = block_counts; /* reuse */
    for (int64_t i = 0; i < nblocks; ++i) write_pos[i] = out->block_val_ptr[i];
    for (int32_t b = 0; b < nbr && ok; ++b) {
        const int32_t r0 = b * br;
        const int32_t r1 = (r0 + br < rows) ? r0 + br : rows;
        const int64_t first = blocks_prefix[b];
        for (int32_t r = r0; r < r1 && ok; ++r) {
            const int32_t local_row = r - r0;
            for (int64_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
                if (value_is_zero(values, p, esz)) continue;
                const int32_t col = col_idx[p];
                const int32_t bcol = col / bc;
                const int32_t local_col = col % bc;
                const int32_t bit = local_row * bc + local_col;
                int64_t lo = 0, hi = active_n[b];
                while (lo < hi) {
                    const int64_t mid = (lo + hi) / 2;
                    if (active[b][mid] < bcol) lo = mid + 1; else hi = mid;
                }
                const int64_t blk = first + lo;
                uint32_t* w = &out->bitmap_words[blk * wpb + bit / 32];
                const uint32_t mask = 1u << (bit % 32);
                if (*w & mask) {
                    set_err(err, errlen, "duplicate CSR entry maps to the same BitBSR bit");
                    ok = 0;
                    break;
                }
                *w |= mask;
                memcpy(out->values + write_pos[blk] * esz, values + p * esz, (size_t)esz);
                write_pos[blk] += 1;
            }
        }
    }
    for (int32_t b = 0; b < nbr; ++b) free(active[b]);
    free(active);
    free(active_n);
    free(nnz_prefix);
    free(block_counts);
    if (!ok) {
        oc_bitbsr_free(out);
        return NULL;
    }
    return out;
}

/* ------------------------------------------------------------------------ */
/* CSR + BitBSR split                                                        */
/* ------------------------------------------------------------------------ */

typedef struct oc_split {
    oc_bitbsr* kept;
    int32_t rows, cols, esz;
    int64_t* res_row_ptr;     /* rows + 1 */
    int32_t* res_col_idx;     /* residual_nnz */
    unsigned char* res_values;
    int64_t kept_blocks, residual_blocks, kept_nnz, residual_nnz;
    int64_t cost_skipped_blocks, cost_skipped_nnz;
} oc_split;

OC_EXPORT void oc_split_free(oc_split* s) {
    if (!s) return;
    oc_bitbsr_free(s->kept);
    free(s->res_row_ptr);
    free(s->res_col_idx);
    free(s->res_values);
    free(s);
}

/*
 * CsrBitBsrSplitCostModel::should_move_to_residual
 * (csr_bitbsr_split.hpp:66-73): csr_cost < bitmap_cost, both affine in nnz.
 * Evaluated with plain double arithmetic; this file is built with
 * -ffp-contract=off so no fused multiply-add changes the comparison.
 */
OC_EXPORT int oc_cost_model_moves(double bitmap_block, double bitmap_nnz, double csr_block,
                                  double csr_nnz, int64_t block_nnz) {
    const double bitmap_cost = bitmap_block + bitmap_nnz * (double)block_nnz;
    const double csr_cost = csr_block + csr_nnz * (double)block_nnz;
    return csr_cost < bitmap_cost;
}

/*
 * convert_bitbsr_to_csr_bitbsr_split_if (csr_bitbsr_split.hpp:405-471) with
 * the cost-gated predicate (:481-490) when use_cost != 0, or the plain
 * threshold predicate (:473-479) when use_cost == 0.
 *   - a block moves to the residual iff nnz <= threshold && predicate(nnz) (:437);
 *   - blocks with nnz <= threshold that stay count as cost-skipped (:443-446);
 *   - residual rows are filled block by block (ascending block column), each
 *     block bit by bit (ctz order), so a residual row is column-sorted
 *     (:358-384, :452-467).
 * Only words_per_block == 1 shapes (br*bc <= 32) are handled here, which
 * covers every shape the reference's tests use for the split.
 */
OC_EXPORT oc_split* oc_split_bitbsr(const oc_bitbsr* full, int32_t threshold, int32_t use_cost,
                                    double c_bitmap_block, double c_bitmap_nnz,
                                    double c_csr_block, double c_csr_nnz, char* err,
                                    int32_t errlen) {
    if (threshold < 0) {
        set_err(err, errlen, "CSR+BitBSR residual threshold must be non-negative");
        return NULL;
    }
    if (c_bitmap_block < 0 || c_bitmap_nnz < 0 || c_csr_block < 0 || c_csr_nnz < 0) {
        set_err(err, errlen, "CSR+BitBSR split cost model must be non-negative");
        return NULL;
    }
    if (full->words_per_block != 1) {
        set_err(err, errlen, "oracle split handles one bitmap word per block");
        return NULL;
    }
    const int esz = full->esz;
    oc_split* s = (oc_split*)calloc(1, sizeof(oc_split));
    s->rows = full->rows;
    s->cols = full->cols;
    s->esz = esz;
    oc_bitbsr* k = (oc_bitbsr*)calloc(1, sizeof(oc_bitbsr));
    *k = *full;
    k->block_row_ptr = (int64_t*)calloc((size_t)full->num_block_rows + 1, sizeof(int64_t));
    k->block_col_idx = (int32_t*)malloc((size_t)(full->num_blocks > 0 ? full->num_blocks : 1) * 4);
    k->bitmap_words = (uint32_t*)malloc((size_t)(full->num_blocks > 0 ? full->num_blocks : 1) * 4);
    k->block_val_ptr = (int64_t*)calloc((size_t)full->num_blocks + 1, sizeof(int64_t));
    k->values = (unsigned char*)malloc((size_t)(full->nnz > 0 ? full->nnz : 1) * (size_t)esz);
    s->kept = k;

    int64_t* res_count = (int64_t*)calloc((size_t)full->rows + 1, sizeof(int64_t));
    unsigned char* moved = (unsigned char*)calloc((size_t)(full->num_blocks > 0 ? full->num_blocks : 1), 1);
    const int32_t br_sz = full->block_rows, bc_sz = full->block_cols;

    int64_t kb = 0, kn = 0;
    for (int32_t b = 0; b < full->num_block_rows; ++b) {
        k->block_row_ptr[b] = kb;
        for (int64_t blk = full->block_row_ptr[b]; blk < full->block_row_ptr[b + 1]; ++blk) {
            const int64_t bn = full->block_val_ptr[blk + 1] - full->block_val_ptr[blk];
            const int pred = use_cost ? oc_cost_model_moves(c_bitmap_block, c_bitmap_nnz,
                                                            c_csr_block, c_csr_nnz, bn)
                                      : 1;
            if (bn <= threshold && pred) {
                moved[blk] = 1;
                s->residual_blocks += 1;
                s->residual_nnz += bn;
                uint32_t w = full->bitmap_words[blk];
                while (w) {
                    const int bit = __builtin_ctz(w);
                    const int32_t row = b * br_sz + bit / bc_sz;
                    const int32_t col = full->block_col_idx[blk] * bc_sz + bit % bc_sz;
                    if (row < full->rows && col < full->cols) res_count[row] += 1;
                    w &= w - 1;
                }
                continue;
            }
            if (bn <= threshold) {
                s->cost_skipped_blocks += 1;
                s->cost_skipped_nnz += bn;
            }
            k->block_col_idx[kb] = full->block_col_idx[blk];
            k->bitmap_words[kb] = full->bitmap_words[blk];
            memcpy(k->values + kn * esz, full->values + full->block_val_ptr[blk] * esz,
                   (size_t)(bn * esz));
            kn += bn;
            kb += 1;
            k->block_val_ptr[kb] = kn;
        }
        k->block_row_ptr[b + 1] = kb;
    }
    k->num_blocks = kb;
    k->nnz = kn;
    s->kept_blocks = kb;
    s->kept_nnz = kn;

    s->res_row_ptr = (int64_t*)calloc((size_t)full->rows + 1, sizeof(int64_t));
    for (int32_t r = 0; r < full->rows; ++r) s->res_row_ptr[r + 1] = s->res_row_ptr[r] + res_count[r];
    const int64_t rn = s->res_row_ptr[full->rows];
    s->res_col_idx = (int32_t*)malloc((size_t)(rn > 0 ? rn : 1) * 4);
    s->res_values = (unsigned char*)malloc((size_t)(rn > 0 ? rn : 1) * (size_t)esz);
    int64_t* fill = res_count;
    for (int32_t r = 0; r < full->rows; ++r) fill[r] = s->res_row_ptr[r];
    for (int32_t b = 0; b < full->num_block_rows; ++b) {
        for (int64_t blk = full->block_row_ptr[b]; blk < full->block_row_ptr[b + 1]; ++blk) {
            if (!moved[blk]) continue;
            uint32_t w = full->bitmap_words[blk];
            int64_t rank = 0;
            while (w) {
                const int bit = __builtin_ctz(w);
                const int32_t row = b * br_sz + bit / bc_sz;
                const int32_t col = full->block_col_idx[blk] * bc_sz + bit % bc_sz;
                if (row < full->rows && col < full->cols) {
                    const int64_t dst = fill[row]++;
                    s->res_col_idx[dst] = col;
                    memcpy(s->res_values + dst * esz,
                           full->values + (full->block_val_ptr[blk] + rank) * esz, (size_t)esz);
                }
                ++rank;
                w &= w - 1;
            }
        }
    }
    free(res_count);
    free(moved);
    return s;
}

/* ------------------------------------------------------------------------ */
/* load-balance layout and packed block words                                */
/* ------------------------------------------------------------------------ */

/* pack_col_bitmap (bitbsr_spmv_8x4_common.cuh:95-104) */
static uint64_t pack_col_bitmap(uint32_t col, uint32_t bitmap, int flag) {
    const uint32_t cf = (col & 0x7fffffffu) | (flag ? 0x80000000u : 0u);
    return ((uint64_t)bitmap << 32) | (uint64_t)cf;
}

/*
 * Work items + packed words.
 * style 0 = hybrid host layout, make_fused_8x4_load_balance_layout_host
 *   (structural/src/main_gpu_csr_bitbsr_spmv.cu:387-475): an empty block
 *   row emits one item with block_count 0 (:429-437); a block row with more
 *   than split_threshold blocks is cut into chunk_blocks pieces and the flag
 *   bit is set on every piece's first block (:439-458).
 * style 1 = device layout, count/fill_bitbsr_8x4_load_balance_work_items
 *   (bitbsr_spmv_8x4_common.cuh:199-267): empty block rows emit no item; the
 *   flag is set iff the block row produced more than one piece.
 * items_out holds 4 uint32 per item (br, block_begin, block_count,
 * value_begin), common.cuh:15-22.  Returns the item count.
 */
OC_EXPORT int64_t oc_lb_layout(const oc_bitbsr* m, int32_t chunk_blocks,
                               int32_t split_threshold_blocks, int32_t style,
                               uint64_t* words_out, uint32_t* items_out,
                               int64_t* item_row_ptr_out) {
    for (int64_t b = 0; b < m->num_blocks; ++b)
        words_out[b] = pack_col_bitmap((uint32_t)m->block_col_idx[b], m->bitmap_words[b], 0);
    int64_t n = 0;
    for (int32_t br = 0; br < m->num_block_rows; ++br) {
        item_row_ptr_out[br] = n;
        const int64_t rs = m->block_row_ptr[br], re = m->block_row_ptr[br + 1];
        const int64_t cnt = re - rs;
        const int64_t vb = m->block_val_ptr[rs];
        if (cnt == 0) {
            if (style == 0) {
                uint32_t* it = items_out + 4 * n;
                it[0] = (uint32_t)br;
                it[1] = (uint32_t)rs;
                it[2] = 0;
                it[3] = (uint32_t)vb;
                ++n;
            }
            continue;
        }
        int atomic;
        int64_t eff;
        if (style == 0) {
            atomic = cnt > split_threshold_blocks;
            eff = atomic ? chunk_blocks : cnt;
        } else {
            const int64_t pieces = cnt <= split_threshold_blocks ? 1 : ceil_div64(cnt, chunk_blocks);
            atomic = pieces > 1;
            eff = atomic ? chunk_blocks : cnt;
        }
        int64_t blk = rs, vp = vb;
        while (blk < re) {
            const int64_t c = (eff < re - blk) ? eff : re - blk;
            uint32_t* it = items_out + 4 * n;
            it[0] = (uint32_t)br;
            it[1] = (uint32_t)blk;
            it[2] = (uint32_t)c;
            it[3] = (uint32_t)vp;
            ++n;
            if (atomic) words_out[blk] |= (uint64_t)0x80000000u;
            for (int64_t i = 0; i < c; ++i) vp += popcount32(m->bitmap_words[blk + i]);
            blk += c;
        }
    }
    item_row_ptr_out[m->num_block_rows] = n;
    return n;
}

/*
 * Long residual-row chunks (main_gpu_csr_bitbsr_spmv.cu:1155-1184): every
 * residual row longer than tau is cut into chunk_nnz (1024) pieces
 * {row, pbegin, pcount}.  With row_out == NULL only the count is returned.
 */
OC_EXPORT int64_t oc_long_chunks(int32_t rows, const int64_t* res_row_ptr, int32_t tau,
                                 int32_t chunk_nnz, int32_t* row_out, int64_t* pbegin_out,
                                 int32_t* pcount_out, int64_t* long_rows_out) {
    int64_t n = 0, nl = 0;
    if (tau <= 0) {
        if (long_rows_out) *long_rows_out = 0;
        return 0;
    }
    for (int32_t r = 0; r < rows; ++r) {
        const int64_t len = res_row_ptr[r + 1] - res_row_ptr[r];
        if (len > tau) {
            ++nl;
            for (int64_t off = 0; off < len; off += chunk_nnz) {
                if (row_out) {
                    row_out[n] = r;
                    pbegin_out[n] = res_row_ptr[r] + off;
                    pcount_out[n] = (int32_t)((len - off) < chunk_nnz ? (len - off) : chunk_nnz);
                }
                ++n;
            }
        }
    }
    if (long_rows_out) *long_rows_out = nl;
    return n;
}

/* ------------------------------------------------------------------------ */
/* value codecs                                                              */
/* ------------------------------------------------------------------------ */

static uint32_t f2u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
static float u2f(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* float_to_bf16_bits, value_compression.hpp:105-109 (round to nearest even) */
OC_EXPORT uint16_t oc_float_to_bf16_bits(float v) {
    const uint32_t bits = f2u(v);
    const uint32_t lsb = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7fffu + lsb) >> 16);
}

OC_EXPORT float oc_bf16_bits_to_float(uint16_t b) { return u2f((uint32_t)b << 16); }

/* std::lround: nearest integer, halves away from zero. */
static long lround_ref(double q) { return lround(q); }

/* one BFP8 block: scale = float(max|v| / 127) (1.0f if zero) -> bf16 RNE;
 * q = clamp(lround(v / decoded_scale), -127, 127).  gpu_value_codecs.cuh:294-315 */
static void bfp8_block(const oc_bitbsr* m, int64_t blk, const unsigned char* skip,
                       int8_t* q_out, uint16_t* scale_out) {
    const int64_t b0 = m->block_val_ptr[blk], b1 = m->block_val_ptr[blk + 1];
    double mx = 0.0;
    for (int64_t k = b0; k < b1; ++k) {
        if (skip && skip[k]) continue;
        const double a = fabs(load_as_double(m->values, k, m->esz));
        if (a > mx) mx = a;
    }
    float scale = (float)(mx / 127.0);
    if (scale == 0.0f) scale = 1.0f;
    const uint16_t sb = oc_float_to_bf16_bits(scale);
    scale_out[blk] = sb;
    const float dec = oc_bf16_bits_to_float(sb);
    for (int64_t k = b0; k < b1; ++k) {
        if (skip && skip[k]) {
            q_out[k] = 0;
            continue;
        }
        long q = lround_ref(load_as_double(m->values, k, m->esz) / (double)dec);
        if (q > 127) q = 127;
        if (q < -127) q = -127;
        q_out[k] = (int8_t)q;
    }
}

/* build_bfp8_blkscale_value_codec, gpu_value_codecs.cuh:287-317 */
OC_EXPORT void oc_bfp8_encode(const oc_bitbsr* m, int8_t* q_out, uint16_t* scale_out) {
    for (int64_t blk = 0; blk < m->num_blocks; ++blk) bfp8_block(m, blk, NULL, q_out, scale_out);
}

static int cmp_f64(const void* a, const void* b) {
    const double x = *(const double*)a, y = *(const double*)b;
    return (x > y) - (x < y);
}

/*
 * build_bfp8_outlier_blkscale_value_codec (gpu_value_codecs.cuh:360-461):
 *   threshold = the idx-th smallest |v| (nth_element), idx = size_t((1-P)*nnz)
 *   clamped to nnz-1 (:384-390); outlier iff |v| > threshold (:391-395);
 *   per-block scale over non-outliers, outlier mantissa 0 (:400-428);
 *   side list (row, col, value) in block-row / block / bit order (:434-458).
 * The order statistic is taken here by a full sort, which yields the same
 * value nth_element places at idx.  Output arrays have capacity nnz.
 * Returns the outlier count; *threshold_out receives the threshold.
 */
OC_EXPORT int64_t oc_bfp8_outlier_encode(const oc_bitbsr* m, double outlier_fraction,
                                         int8_t* q_out, uint16_t* scale_out, int32_t* orow,
                                         int32_t* ocol, void* oval_v, double* threshold_out) {
    const int64_t nnz = m->nnz;
    unsigned char* is_out = (unsigned char*)calloc((size_t)(nnz > 0 ? nnz : 1), 1);
    double thr = 0.0;
    if (outlier_fraction > 0.0 && nnz > 0) {
        double* a = (double*)malloc((size_t)nnz * sizeof(double));
        for (int64_t k = 0; k < nnz; ++k) a[k] = fabs(load_as_double(m->values, k, m->esz));
        double* s = (double*)malloc((size_t)nnz * sizeof(double));
        memcpy(s, a, (size_t)nnz * sizeof(double));
        size_t idx = (size_t)((1.0 - outlier_fraction) * (double)nnz);
        if (idx >= (size_t)nnz) idx = (size_t)nnz - 1;
        qsort(s, (size_t)nnz, sizeof(double), cmp_f64);
        thr = s[idx];
        for (int64_t k = 0; k < nnz; ++k)
            if (a[k] > thr) is_out[k] = 1;
        free(a);
        free(s);
    }
    if (threshold_out) *threshold_out = thr;
    for (int64_t blk = 0; blk < m->num_blocks; ++blk) bfp8_block(m, blk, is_out, q_out, scale_out);
    unsigned char* oval = (unsigned char*)oval_v;
    int64_t n = 0;
    for (int32_t br = 0; br < m->num_block_rows; ++br) {
        for (int64_t blk = m->block_row_ptr[br]; blk < m->block_row_ptr[br + 1]; ++blk) {
            const uint32_t bm = m->bitmap_words[blk];
            const int64_t base = m->block_val_ptr[blk];
            for (int bit = 0; bit < 32; ++bit) {
                if (!(bm & (1u << bit))) continue;
                const int64_t k = base + popcount32(bm & ((1u << bit) - 1u));
                if (!is_out[k]) continue;
                orow[n] = br * m->block_rows + bit / m->block_cols;
                ocol[n] = m->block_col_idx[blk] * m->block_cols + bit % m->block_cols;
                memcpy(oval + n * m->esz, m->values + k * m->esz, (size_t)m->esz);
                ++n;
            }
        }
    }
    free(is_out);
    return n;
}

/*
 * Residual bf16 transform (main_gpu_csr_bitbsr_spmv.cu:1302-1306,
 * :1334-1338): u = bits(float(v)); bf16 = (u + 0x8000) >> 16, i.e. round
 * half up on the magnitude, no tie-to-even.
 */
OC_EXPORT void oc_bf16_half_up(const void* vals, int64_t n, int32_t esz, uint16_t* out) {
    const unsigned char* v = (const unsigned char*)vals;
    for (int64_t i = 0; i < n; ++i) {
        const float f = (float)load_as_double(v, i, esz);
        out[i] = (uint16_t)((f2u(f) + 0x8000u) >> 16);
    }
}

/*
 * Exact-value interning for the joint dict arm
 * (main_gpu_csr_bitbsr_spmv.cu:1224-1258): kept values first, then residual
 * values, keyed by raw bits, codebook in first-occurrence order.  Returns
 * the number of distinct values.  Codes are written only while the count is
 * <= cap (cap >= 65536 gives every code the joint arm can use); beyond it the
 * function still counts but leaves codes undefined.
 */
typedef struct {
    uint64_t* keys;
    int32_t* ids;
    unsigned char* used;
    uint64_t mask;
} oc_hash;

static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

OC_EXPORT int64_t oc_dict_intern(const void* kept_v, int64_t nk, const void* res_v, int64_t nr,
                                 int32_t esz, void* codebook_out, int32_t* kept_codes,
                                 int32_t* res_codes, int64_t cap) {
    uint64_t size = 1;
    while (size < 2 * (uint64_t)(nk + nr + 1)) size <<= 1;
    oc_hash h;
    h.keys = (uint64_t*)malloc(size * 8);
    h.ids = (int32_t*)malloc(size * 4);
    h.used = (unsigned char*)calloc(size, 1);
    h.mask = size - 1;
    int64_t uniq = 0;
    unsigned char* cb = (unsigned char*)codebook_out;
    for (int pass = 0; pass < 2; ++pass) {
        const unsigned char* v = (const unsigned char*)(pass == 0 ? kept_v : res_v);
        const int64_t n = pass == 0 ? nk : nr;
        int32_t* codes = pass == 0 ? kept_codes : res_codes;
        for (int64_t i = 0; i < n; ++i) {
            const uint64_t key = value_key(v, i, esz);
            uint64_t slot = mix64(key) & h.mask;
            while (h.used[slot] && h.keys[slot] != key) slot = (slot + 1) & h.mask;
            if (!h.used[slot]) {
                h.used[slot] = 1;
                h.keys[slot] = key;
                h.ids[slot] = (int32_t)uniq;
                if (uniq < cap) memcpy(cb + uniq * esz, v + i * esz, (size_t)esz);
                ++uniq;
            }
            if (uniq <= cap && codes) codes[i] = h.ids[slot];
        }
    }
    free(h.keys);
    free(h.ids);
    free(h.used);
    return uniq;
}

/* ------------------------------------------------------------------------ */
/* SpMV and error metrics                                                    */
/* ------------------------------------------------------------------------ */

/* spmv_csr (spmv.hpp:12-29), serial row loop, sum in T */
OC_EXPORT void oc_spmv_csr(int32_t rows, const int64_t* row_ptr, const int32_t* col_idx,
                           const void* vals_v, const void* x_v, void* y_v, int32_t esz) {
    if (esz == 8) {
        const double* v = (const double*)vals_v;
        const double* x = (const double*)x_v;
        double* y = (double*)y_v;
        for (int32_t r = 0; r < rows; ++r) {
            double s = 0.0;
            for (int64_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) s += v[p] * x[col_idx[p]];
            y[r] = s;
        }
    } else {
        const float* v = (const float*)vals_v;
        const float* x = (const float*)x_v;
        float* y = (float*)y_v;
        for (int32_t r = 0; r < rows; ++r) {
            float s = 0.0f;
            for (int64_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) s += v[p] * x[col_idx[p]];
            y[r] = s;
        }
    }
}

/* compare_vectors (spmv.hpp:73-89), in T: out = {max_abs, max_rel, global_rel} */
OC_EXPORT void oc_compare_vectors(const void* ref_v, const void* got_v, int64_t n, int32_t esz,
                                  double* out3) {
    if (esz == 8) {
        const double* ref = (const double*)ref_v;
        const double* got = (const double*)got_v;
        double ma = 0, mr = 0, mref = 0;
        for (int64_t i = 0; i < n; ++i) {
            const double ae = fabs(ref[i] - got[i]);
            const double den = fabs(ref[i]) > 1e-30 ? fabs(ref[i]) : 1e-30;
            if (ae > ma) ma = ae;
            if (ae / den > mr) mr = ae / den;
            if (fabs(ref[i]) > mref) mref = fabs(ref[i]);
        }
        out3[0] = ma;
        out3[1] = mr;
        out3[2] = ma / (mref > 1e-30 ? mref : 1e-30);
    } else {
        const float* ref = (const float*)ref_v;
        const float* got = (const float*)got_v;
        const float tiny = (float)1e-30;
        float ma = 0, mr = 0, mref = 0;
        for (int64_t i = 0; i < n; ++i) {
            const float ae = fabsf(ref[i] - got[i]);
            const float den = fabsf(ref[i]) > tiny ? fabsf(ref[i]) : tiny;
            if (ae > ma) ma = ae;
            if (ae / den > mr) mr = ae / den;
            if (fabsf(ref[i]) > mref) mref = fabsf(ref[i]);
        }
        out3[0] = ma;
        out3[1] = mr;
        out3[2] = ma / (mref > tiny ? mref : tiny);
    }
}

/* make_input_vector (spmv_harness.hpp:32-39): x[i] = T((i % 17) - 8) * T(0.125) */
OC_EXPORT void oc_canonical_x(int64_t n, int32_t esz, void* out) {
    for (int64_t i = 0; i < n; ++i) {
        if (esz == 8) {
            ((double*)out)[i] = (double)((i % 17) - 8) * 0.125;
        } else {
            ((float*)out)[i] = (float)((i % 17) - 8) * 0.125f;
        }
    }
}

/*
 * Joint-route output with the decoded values of a lossy arm, as the joint
 * kernel computes it (main_gpu_csr_bitbsr_spmv.cu:726-736, 795-860,
 * 967-979): kept value = float(int8) * bf16(scale[block]); residual value =
 * bf16 -> float; products use float(x); the bulk sum is float, cast to T;
 * outliers are then added exactly in T.  Summation here runs in row order
 * (kept blocks then residual), which the GPU does not promise; callers
 * compare with a tolerance.
 */
OC_EXPORT void oc_joint_bfp8_spmv(const oc_bitbsr* kept, const int8_t* q, const uint16_t* scale,
                                  const int64_t* res_row_ptr, const int32_t* res_col,
                                  const uint16_t* res_bf16, int64_t num_out, const int32_t* orow,
                                  const int32_t* ocol, const void* oval_v, const void* x_v,
                                  void* y_v) {
    const int esz = kept->esz;
    const unsigned char* x = (const unsigned char*)x_v;
    float* acc = (float*)calloc((size_t)kept->rows + 1, sizeof(float));
    for (int32_t br = 0; br < kept->num_block_rows; ++br) {
        for (int64_t blk = kept->block_row_ptr[br]; blk < kept->block_row_ptr[br + 1]; ++blk) {
            const uint32_t bm = kept->bitmap_words[blk];
            const int64_t base = kept->block_val_ptr[blk];
            const float sc = oc_bf16_bits_to_float(scale[blk]);
            for (int bit = 0; bit < 32; ++bit) {
                if (!(bm & (1u << bit))) continue;
                const int64_t k = base + popcount32(bm & ((1u << bit) - 1u));
                const int32_t row = br * 8 + bit / 4;
                const int32_t col = kept->block_col_idx[blk] * 4 + bit % 4;
                if (row >= kept->rows || col >= kept->cols) continue;
                const float v = (float)q[k] * sc;
                acc[row] += v * (float)load_as_double(x, col, esz);
            }
        }
    }
    for (int32_t r = 0; r < kept->rows; ++r) {
        for (int64_t p = res_row_ptr[r]; p < res_row_ptr[r + 1]; ++p) {
            acc[r] += oc_bf16_bits_to_float(res_bf16[p]) * (float)load_as_double(x, res_col[p], esz);
        }
    }
    const unsigned char* oval = (const unsigned char*)oval_v;
    if (esz == 8) {
        double* y = (double*)y_v;
        for (int32_t r = 0; r < kept->rows; ++r) y[r] = (double)acc[r];
        for (int64_t i = 0; i < num_out; ++i)
            y[orow[i]] += load_as_double(oval, i, 8) * load_as_double(x, ocol[i], 8);
    } else {
        float* y = (float*)y_v;
        for (int32_t r = 0; r < kept->rows; ++r) y[r] = acc[r];
        for (int64_t i = 0; i < num_out; ++i) {
            float ov, xv;
            memcpy(&ov, oval + i * 4, 4);
            memcpy(&xv, x + (int64_t)ocol[i] * 4, 4);
            y[orow[i]] += ov * xv;
        }
    }
    free(acc);
}
