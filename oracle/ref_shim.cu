// ref_shim.cu -- C entry points over the reference's own host code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file against the
// reference's headers where they lie (include path into the read-only
// reference checkout) and writes the result to oracle/_ref/libcove_ref.so.
// No reference source is copied: this file only calls the reference's
// template functions and flattens their results into plain buffers so the
// tests can compare them with the plain-C oracle and with the CUDA product.
//
// Functions called (reference paths under structural/include/structural/):
//   convert_to_bitbsr                          convert.hpp:13-165
//   convert_bitbsr_to_csr_bitbsr_split{,_cost_gated}  csr_bitbsr_split.hpp:473-490
//   storage_stats                              csr_bitbsr_split.hpp:545-597
//   spmv_csr (OpenMP, the CPU baseline)        spmv.hpp:12-29
//   compare_vectors                            spmv.hpp:73-89
//   make_input_vector                          spmv_harness.hpp:32-39
//   build_bfp8_blkscale_value_codec            gpu_value_codecs.cuh:287-317
//   build_bfp8_outlier_blkscale_value_codec    gpu_value_codecs.cuh:360-461
//   float_to_bf16_bits                         value_compression.hpp:105-109
//   read_matrix_market_with_info               matrix_market.hpp:327-382
#include "structural/convert.hpp"
#include "structural/csr.hpp"
#include "structural/csr_bitbsr_split.hpp"
#include "structural/gpu_value_codecs.cuh"
#include "structural/matrix_market.hpp"
#include "structural/spmv.hpp"
#include "structural/spmv_harness.hpp"
#include "structural/value_compression.hpp"

#include <omp.h>

#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <vector>

#define REF_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_err;

template <typename T>
structural::CsrMatrix<T> make_csr(int32_t rows, int32_t cols, const int32_t* row_ptr,
                                  const int32_t* col_idx, const void* values) {
    structural::CsrMatrix<T> csr;
    csr.rows = rows;
    csr.cols = cols;
    csr.row_ptr.assign(row_ptr, row_ptr + rows + 1);
    const int32_t nnz = row_ptr[rows];
    csr.col_idx.assign(col_idx, col_idx + nnz);
    const T* v = static_cast<const T*>(values);
    csr.values.assign(v, v + nnz);
    return csr;
}

// Handle that owns a split result (kept BitBSR + residual CSR) of either type.
struct RefSplit {
    int esz = 8;
    structural::BitBsrMatrix<double> full_d, kept_d;
    structural::BitBsrMatrix<float> full_f, kept_f;
    structural::CsrMatrix<double> res_d;
    structural::CsrMatrix<float> res_f;
    int64_t counters[8] = {};
    long long stats_bits[4] = {};
};

template <typename T>
void fill_split(RefSplit& h, const structural::BitBsrMatrix<T>& full,
                const structural::CsrBitBsrSplitMatrix<T>& split,
                structural::BitBsrMatrix<T>& full_out, structural::BitBsrMatrix<T>& kept_out,
                structural::CsrMatrix<T>& res_out) {
    full_out = full;
    kept_out = split.bitbsr;
    res_out = split.residual;
    h.counters[0] = full.num_blocks();
    h.counters[1] = split.kept_blocks;
    h.counters[2] = split.residual_blocks;
    h.counters[3] = split.cost_skipped_blocks;
    h.counters[4] = split.kept_nnz;
    h.counters[5] = split.residual_nnz;
    h.counters[6] = split.cost_skipped_nnz;
    const auto stats = structural::storage_stats(full, split);
    h.stats_bits[0] = stats.full_bitbsr_position_bits;
    h.stats_bits[1] = stats.kept_bitbsr_position_bits;
    h.stats_bits[2] = stats.residual_csr_position_bits;
    h.stats_bits[3] = stats.split_position_bits;
}

template <typename T>
RefSplit* build_split(int32_t rows, int32_t cols, const int32_t* row_ptr, const int32_t* col_idx,
                      const void* values, int32_t br, int32_t bc, int32_t threshold,
                      int32_t use_cost, const double* cost4) {
    auto csr = make_csr<T>(rows, cols, row_ptr, col_idx, values);
    const auto full = structural::convert_to_bitbsr(csr, br, bc);
    structural::CsrBitBsrSplitMatrix<T> split;
    if (use_cost) {
        structural::CsrBitBsrSplitCostModel cm;
        cm.bitmap_block_cost = cost4[0];
        cm.bitmap_nnz_cost = cost4[1];
        cm.csr_block_cost = cost4[2];
        cm.csr_nnz_cost = cost4[3];
        split = structural::convert_bitbsr_to_csr_bitbsr_split_cost_gated(full, threshold, cm);
    } else {
        split = structural::convert_bitbsr_to_csr_bitbsr_split(full, threshold);
    }
    auto* h = new RefSplit();
    h->esz = sizeof(T);
    if constexpr (sizeof(T) == 8) {
        fill_split(*h, full, split, h->full_d, h->kept_d, h->res_d);
    } else {
        fill_split(*h, full, split, h->full_f, h->kept_f, h->res_f);
    }
    return h;
}

template <typename T>
void copy_bitbsr(const structural::BitBsrMatrix<T>& m, int64_t* sizes, int32_t* block_row_ptr,
                 int32_t* block_col_idx, uint32_t* bitmap, int32_t* block_val_ptr, void* values) {
    sizes[0] = m.num_block_rows;
    sizes[1] = m.num_blocks();
    sizes[2] = m.nnz();
    sizes[3] = m.words_per_block;
    if (block_row_ptr) std::memcpy(block_row_ptr, m.block_row_ptr.data(), m.block_row_ptr.size() * 4);
    if (block_col_idx) std::memcpy(block_col_idx, m.block_col_idx.data(), m.block_col_idx.size() * 4);
    if (bitmap) std::memcpy(bitmap, m.bitmap_words.data(), m.bitmap_words.size() * 4);
    if (block_val_ptr) std::memcpy(block_val_ptr, m.block_val_ptr.data(), m.block_val_ptr.size() * 4);
    if (values) std::memcpy(values, m.values.data(), m.values.size() * sizeof(T));
}

template <typename T>
void copy_csr(const structural::CsrMatrix<T>& m, int64_t* sizes, int32_t* row_ptr, int32_t* col,
              void* values) {
    sizes[0] = m.rows;
    sizes[1] = m.nnz();
    if (row_ptr) std::memcpy(row_ptr, m.row_ptr.data(), m.row_ptr.size() * 4);
    if (col) std::memcpy(col, m.col_idx.data(), m.col_idx.size() * 4);
    if (values) std::memcpy(values, m.values.data(), m.values.size() * sizeof(T));
}

}  // namespace

REF_EXPORT const char* ref_last_error() { return g_err.c_str(); }

// Build CSR -> full BitBSR (br x bc) -> split.  Returns NULL on a reference
// exception (message in ref_last_error()).
REF_EXPORT void* ref_split_build(int32_t rows, int32_t cols, const int32_t* row_ptr,
                                 const int32_t* col_idx, const void* values, int32_t esz,
                                 int32_t br, int32_t bc, int32_t threshold, int32_t use_cost,
                                 const double* cost4) {
    try {
        if (esz == 8) {
            return build_split<double>(rows, cols, row_ptr, col_idx, values, br, bc, threshold,
                                       use_cost, cost4);
        }
        return build_split<float>(rows, cols, row_ptr, col_idx, values, br, bc, threshold,
                                  use_cost, cost4);
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

REF_EXPORT void ref_split_free(void* h) { delete static_cast<RefSplit*>(h); }

// counters: full_blocks, kept_blocks, residual_blocks, cost_skipped_blocks,
// kept_nnz, residual_nnz, cost_skipped_nnz; bits: full, kept, residual, split
REF_EXPORT void ref_split_counters(void* hv, int64_t* counters7, long long* bits4) {
    auto* h = static_cast<RefSplit*>(hv);
    std::memcpy(counters7, h->counters, 7 * sizeof(int64_t));
    std::memcpy(bits4, h->stats_bits, 4 * sizeof(long long));
}

// which: 0 = full BitBSR, 1 = kept BitBSR.  Call with NULL arrays to get sizes.
REF_EXPORT void ref_split_bitbsr(void* hv, int32_t which, int64_t* sizes4, int32_t* block_row_ptr,
                                 int32_t* block_col_idx, uint32_t* bitmap,
                                 int32_t* block_val_ptr, void* values) {
    auto* h = static_cast<RefSplit*>(hv);
    if (h->esz == 8) {
        copy_bitbsr(which == 0 ? h->full_d : h->kept_d, sizes4, block_row_ptr, block_col_idx,
                    bitmap, block_val_ptr, values);
    } else {
        copy_bitbsr(which == 0 ? h->full_f : h->kept_f, sizes4, block_row_ptr, block_col_idx,
                    bitmap, block_val_ptr, values);
    }
}

REF_EXPORT void ref_split_residual(void* hv, int64_t* sizes2, int32_t* row_ptr, int32_t* col,
                                   void* values) {
    auto* h = static_cast<RefSplit*>(hv);
    if (h->esz == 8) {
        copy_csr(h->res_d, sizes2, row_ptr, col, values);
    } else {
        copy_csr(h->res_f, sizes2, row_ptr, col, values);
    }
}

// BFP8 codecs over the kept BitBSR of a split handle (which = 1) or the full
// one (which = 0).  outlier_fraction < 0 selects plain BFP8.  Outlier arrays
// need capacity nnz.  Returns the outlier count (0 for plain BFP8).
REF_EXPORT int64_t ref_bfp8(void* hv, int32_t which, double outlier_fraction, int8_t* q,
                            uint16_t* scale, int32_t* orow, int32_t* ocol, void* oval) {
    auto* h = static_cast<RefSplit*>(hv);
    auto run = [&](const auto& m) -> int64_t {
        using T = typename std::decay_t<decltype(m.values)>::value_type;
        if (outlier_fraction < 0.0) {
            const auto c = structural::build_bfp8_blkscale_value_codec(m);
            std::memcpy(q, c.int8_values.data(), c.int8_values.size());
            std::memcpy(scale, c.block_scale_bf16.data(), c.block_scale_bf16.size() * 2);
            return 0;
        }
        const auto c = structural::build_bfp8_outlier_blkscale_value_codec(m, outlier_fraction);
        std::memcpy(q, c.int8_values.data(), c.int8_values.size());
        std::memcpy(scale, c.block_scale_bf16.data(), c.block_scale_bf16.size() * 2);
        std::memcpy(orow, c.outlier_rows.data(), c.outlier_rows.size() * 4);
        std::memcpy(ocol, c.outlier_cols.data(), c.outlier_cols.size() * 4);
        std::memcpy(oval, c.outlier_vals.data(), c.outlier_vals.size() * sizeof(T));
        return c.num_outliers;
    };
    try {
        if (h->esz == 8) return run(which == 0 ? h->full_d : h->kept_d);
        return run(which == 0 ? h->full_f : h->kept_f);
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

REF_EXPORT uint16_t ref_float_to_bf16_bits(float v) { return structural::float_to_bf16_bits(v); }

// The reference CPU SpMV (OpenMP over rows, schedule(static)).  Returns the
// steady-clock milliseconds of the call, as time_call measures it.
REF_EXPORT double ref_spmv_csr(int32_t rows, int32_t cols, const int32_t* row_ptr,
                               const int32_t* col_idx, const void* values, int32_t esz,
                               const void* x, void* y) {
    try {
        if (esz == 8) {
            auto csr = make_csr<double>(rows, cols, row_ptr, col_idx, values);
            std::vector<double> xv(static_cast<const double*>(x),
                                   static_cast<const double*>(x) + cols);
            double ms = 0.0;
            const auto out = structural::time_call([&] { return structural::spmv_csr(csr, xv); }, ms);
            std::memcpy(y, out.data(), out.size() * 8);
            return ms;
        }
        auto csr = make_csr<float>(rows, cols, row_ptr, col_idx, values);
        std::vector<float> xv(static_cast<const float*>(x), static_cast<const float*>(x) + cols);
        double ms = 0.0;
        const auto out = structural::time_call([&] { return structural::spmv_csr(csr, xv); }, ms);
        std::memcpy(y, out.data(), out.size() * 4);
        return ms;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1.0;
    }
}

// Resident-CSR variant for timing: the matrix is copied into the reference's
// container once; ref_csr_spmv_timed then runs spmv_csr `reps` times and
// returns the minimum steady-clock milliseconds.
struct RefCsrHandle {
    int esz = 8;
    structural::CsrMatrix<double> d;
    structural::CsrMatrix<float> f;
    std::vector<double> xd;
    std::vector<float> xf;
};

REF_EXPORT void* ref_csr_create(int32_t rows, int32_t cols, const int32_t* row_ptr,
                                const int32_t* col_idx, const void* values, int32_t esz,
                                const void* x) {
    auto* h = new RefCsrHandle();
    h->esz = esz;
    if (esz == 8) {
        h->d = make_csr<double>(rows, cols, row_ptr, col_idx, values);
        h->xd.assign(static_cast<const double*>(x), static_cast<const double*>(x) + cols);
    } else {
        h->f = make_csr<float>(rows, cols, row_ptr, col_idx, values);
        h->xf.assign(static_cast<const float*>(x), static_cast<const float*>(x) + cols);
    }
    return h;
}

REF_EXPORT void ref_csr_free(void* h) { delete static_cast<RefCsrHandle*>(h); }

REF_EXPORT double ref_csr_spmv_timed(void* hv, int32_t reps, void* y_out) {
    auto* h = static_cast<RefCsrHandle*>(hv);
    double best = 1e300;
    for (int i = 0; i < reps; ++i) {
        double ms = 0.0;
        if (h->esz == 8) {
            const auto y = structural::time_call([&] { return structural::spmv_csr(h->d, h->xd); }, ms);
            if (y_out && i == reps - 1) std::memcpy(y_out, y.data(), y.size() * 8);
        } else {
            const auto y = structural::time_call([&] { return structural::spmv_csr(h->f, h->xf); }, ms);
            if (y_out && i == reps - 1) std::memcpy(y_out, y.data(), y.size() * 4);
        }
        best = ms < best ? ms : best;
    }
    return best;
}

REF_EXPORT int32_t ref_omp_max_threads() { return omp_get_max_threads(); }

// Thread count of the reference's OpenMP loops from here on (a launcher may
// have set OMP_NUM_THREADS=1 in the environment).
REF_EXPORT void ref_omp_set_threads(int32_t n) { omp_set_num_threads(n > 0 ? n : 1); }

REF_EXPORT void ref_compare_vectors(const void* ref, const void* got, int64_t n, int32_t esz,
                                    double* out3) {
    if (esz == 8) {
        std::vector<double> a(static_cast<const double*>(ref), static_cast<const double*>(ref) + n);
        std::vector<double> b(static_cast<const double*>(got), static_cast<const double*>(got) + n);
        const auto s = structural::compare_vectors(a, b);
        out3[0] = s.max_abs;
        out3[1] = s.max_rel;
        out3[2] = s.global_rel;
    } else {
        std::vector<float> a(static_cast<const float*>(ref), static_cast<const float*>(ref) + n);
        std::vector<float> b(static_cast<const float*>(got), static_cast<const float*>(got) + n);
        const auto s = structural::compare_vectors(a, b);
        out3[0] = s.max_abs;
        out3[1] = s.max_rel;
        out3[2] = s.global_rel;
    }
}

REF_EXPORT void ref_canonical_x(int32_t n, int32_t esz, void* out) {
    if (esz == 8) {
        const auto x = structural::make_input_vector<double>(n);
        std::memcpy(out, x.data(), x.size() * 8);
    } else {
        const auto x = structural::make_input_vector<float>(n);
        std::memcpy(out, x.data(), x.size() * 4);
    }
}

// read_matrix_market_with_info<T> on a file.  Call with row_ptr == nullptr
// for the sizes: returns nnz (or -1 with ref_last_error() set); shape2 =
// {rows, cols}, field_sym2 = {field, symmetry} as the reference's enums,
// counts3 = {stored, expanded, coalesced duplicates}.
REF_EXPORT int64_t ref_mm_read(const char* path, int32_t esz, int32_t* shape2, int32_t* field_sym2,
                               int64_t* counts3, int32_t* row_ptr, int32_t* col, void* values) {
    try {
        auto copy = [&](const auto& r) {
            shape2[0] = r.matrix.rows;
            shape2[1] = r.matrix.cols;
            field_sym2[0] = static_cast<int32_t>(r.info.field);
            field_sym2[1] = static_cast<int32_t>(r.info.symmetry);
            counts3[0] = r.stored_entries;
            counts3[1] = r.expanded_entries;
            counts3[2] = r.coalesced_duplicates;
            if (row_ptr) {
                std::memcpy(row_ptr, r.matrix.row_ptr.data(), r.matrix.row_ptr.size() * 4);
                std::memcpy(col, r.matrix.col_idx.data(), r.matrix.col_idx.size() * 4);
                std::memcpy(values, r.matrix.values.data(),
                            r.matrix.values.size() * sizeof(r.matrix.values[0]));
            }
            return static_cast<int64_t>(r.matrix.nnz());
        };
        if (esz == 8) return copy(structural::read_matrix_market_with_info<double>(path));
        return copy(structural::read_matrix_market_with_info<float>(path));
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
