// csr_bitbsr_split.hpp -- the CSR+BitBSR split of the structural:: API
// (structural/include/structural/csr_bitbsr_split.hpp:15-74, 405-511), same
// types, names, parameters and messages:
//   CsrBitBsrSplitMatrix, CsrBitBsrSplitCostModel
//   convert_bitbsr_to_csr_bitbsr_split_if(full, threshold, should_move)
//   convert_bitbsr_to_csr_bitbsr_split(full, threshold)
//   convert_bitbsr_to_csr_bitbsr_split_cost_gated(full, threshold, model)
//   convert_to_csr_bitbsr_split(csr, block_rows, block_cols, threshold)
//   convert_to_csr_bitbsr_split_cost_gated(csr, block_rows, block_cols, threshold, model)
// A block of population p moves to the CSR residual iff p <= threshold and
// should_move(p).  The predicate depends on p alone, so it is tabulated on
// the host for p = 0..32 and the split itself runs in the device plan build
// (COVE_SPLIT_MASK); kept blocks keep their order, residual rows list their
// entries by block then bit, as in the reference.  8x4 blocks only.
#pragma once

#include "structural/convert.hpp"
#include "structural/csr_bitbsr_hybrid.cuh"

#include <stdexcept>

namespace structural {

template <typename T>
struct CsrBitBsrSplitMatrix {
    BitBsrMatrix<T> bitbsr;
    CsrMatrix<T> residual;
    Index block_rows = 0;
    Index block_cols = 0;
    Index residual_threshold = 0;
    Offset kept_blocks = 0;
    Offset residual_blocks = 0;
    Offset kept_nnz = 0;
    Offset residual_nnz = 0;
    Offset cost_skipped_blocks = 0;
    Offset cost_skipped_nnz = 0;

    void validate() const {
        if (block_rows <= 0 || block_cols <= 0 || residual_threshold < 0)
            throw std::runtime_error("CSR+BitBSR split metadata is invalid");
        bitbsr.validate();
        residual.validate();
        if (bitbsr.rows != residual.rows || bitbsr.cols != residual.cols)
            throw std::runtime_error("CSR+BitBSR split dimensions differ");
        if (bitbsr.block_rows != block_rows || bitbsr.block_cols != block_cols)
            throw std::runtime_error("CSR+BitBSR split block size metadata differs");
        if (kept_blocks != bitbsr.num_blocks()) throw std::runtime_error("CSR+BitBSR split kept block count differs");
        if (kept_nnz != bitbsr.nnz()) throw std::runtime_error("CSR+BitBSR split kept nnz differs");
        if (residual_nnz != residual.nnz()) throw std::runtime_error("CSR+BitBSR split residual nnz differs");
    }
};

struct CsrBitBsrSplitCostModel {
    double bitmap_block_cost = 10.0;
    double bitmap_nnz_cost = 0.0;
    double csr_block_cost = 0.0;
    double csr_nnz_cost = 1.0;

    void validate() const {
        if (bitmap_block_cost < 0.0 || bitmap_nnz_cost < 0.0 || csr_block_cost < 0.0 || csr_nnz_cost < 0.0)
            throw std::runtime_error("CSR+BitBSR split cost model must be non-negative");
    }

    bool should_move_to_residual(Offset block_nnz) const {
        validate();
        const double n = static_cast<double>(block_nnz);
        return csr_block_cost + csr_nnz_cost * n < bitmap_block_cost + bitmap_nnz_cost * n;
    }
};

namespace split_detail {

// The CSR rows of an 8x4 host BitBSR, columns ascending.
template <typename T>
CsrMatrix<T> bitbsr_rows(const BitBsrMatrix<T>& b) {
    CsrMatrix<T> a;
    a.rows = b.rows;
    a.cols = b.cols;
    a.row_ptr.assign(static_cast<size_t>(b.rows) + 1, 0);
    a.col_idx.reserve(b.values.size());
    a.values.reserve(b.values.size());
    for (Index r = 0; r < b.rows; ++r) {
        const Index br = r / 8, lr = r % 8;
        for (Offset k = b.block_row_ptr[br]; k < b.block_row_ptr[br + 1]; ++k) {
            const BitmapWord bm = b.bitmap_words[k];
            for (int c = 0; c < 4; ++c) {
                const int bit = lr * 4 + c;
                if (!(bm >> bit & 1u)) continue;
                a.col_idx.push_back(b.block_col_idx[k] * 4 + c);
                a.values.push_back(b.values[b.block_val_ptr[k] + popcount_word(bm & ((1u << bit) - 1u))]);
            }
        }
        a.row_ptr[r + 1] = static_cast<Offset>(a.values.size());
    }
    return a;
}

// Split of `csr` on the device with blocks of population p moved iff
// p <= threshold and bit p of `mask` is set.
template <typename T>
CsrBitBsrSplitMatrix<T> split_on_device(const CsrMatrix<T>& csr, Index threshold, unsigned long long mask) {
    cove_plan_opts o;
    cove_plan_opts_default(&o);
    o.split_policy = COVE_SPLIT_MASK;
    o.move_mask = mask;
    o.residual_threshold = threshold;
    o.value_codec = COVE_CODEC_ORIGINAL;
    o.gate_enable = 0;
    o.keep_lossless = 1;
    const cove::Plan<T> plan(csr, &o);
    const cove_plan_info& in = plan.info();
    CsrBitBsrSplitMatrix<T> out;
    out.block_rows = 8;
    out.block_cols = 4;
    out.residual_threshold = threshold;
    auto& k = out.bitbsr;
    k.rows = csr.rows;
    k.cols = csr.cols;
    k.block_rows = 8;
    k.block_cols = 4;
    k.num_block_rows = ceil_div(csr.rows, 8);
    k.num_block_cols = ceil_div(csr.cols, 4);
    k.words_per_block = 1;
    k.block_row_ptr = plan.template stream<Offset>(COVE_STREAM_KEPT_BLOCK_ROW_PTR);
    k.block_col_idx = plan.template stream<Index>(COVE_STREAM_KEPT_BLOCK_COL_IDX);
    k.bitmap_words = plan.template stream<BitmapWord>(COVE_STREAM_KEPT_BITMAP);
    k.block_val_ptr = plan.template stream<Offset>(COVE_STREAM_KEPT_BLOCK_VAL_PTR);
    k.values = plan.template stream<T>(COVE_STREAM_KEPT_VALUES);
    auto& res = out.residual;
    res.rows = csr.rows;
    res.cols = csr.cols;
    res.row_ptr = plan.template stream<Offset>(COVE_STREAM_RES_ROW_PTR);
    res.col_idx = plan.template stream<Index>(COVE_STREAM_RES_COL_IDX);
    res.values = plan.template stream<T>(COVE_STREAM_RES_VALUES);
    out.kept_blocks = static_cast<Offset>(in.kept_blocks);
    out.residual_blocks = static_cast<Offset>(in.residual_blocks);
    out.kept_nnz = static_cast<Offset>(in.kept_nnz);
    out.residual_nnz = static_cast<Offset>(in.residual_nnz);
    out.cost_skipped_blocks = static_cast<Offset>(in.cost_skipped_blocks);
    out.cost_skipped_nnz = static_cast<Offset>(in.cost_skipped_nnz);
    out.validate();
    return out;
}

template <typename F>
unsigned long long tabulate(F&& should_move) {
    unsigned long long m = 0;
    for (Offset p = 0; p <= 32; ++p)
        if (should_move(p)) m |= 1ULL << p;
    return m;
}

}  // namespace split_detail

template <typename T, typename ShouldMoveToResidual>
CsrBitBsrSplitMatrix<T> convert_bitbsr_to_csr_bitbsr_split_if(const BitBsrMatrix<T>& full, Index residual_threshold,
                                                              ShouldMoveToResidual should_move_to_residual) {
    full.validate();
    if (residual_threshold < 0) throw std::runtime_error("CSR+BitBSR residual threshold must be non-negative");
    if (full.block_rows != 8 || full.block_cols != 4 || full.words_per_block != 1)
        throw std::runtime_error("this build splits 8x4 BitBSR blocks only");
    return split_detail::split_on_device(split_detail::bitbsr_rows(full), residual_threshold,
                                         split_detail::tabulate(should_move_to_residual));
}

template <typename T>
CsrBitBsrSplitMatrix<T> convert_bitbsr_to_csr_bitbsr_split(const BitBsrMatrix<T>& full, Index residual_threshold) {
    return convert_bitbsr_to_csr_bitbsr_split_if(full, residual_threshold, [](Offset) { return true; });
}

template <typename T>
CsrBitBsrSplitMatrix<T> convert_bitbsr_to_csr_bitbsr_split_cost_gated(const BitBsrMatrix<T>& full,
                                                                      Index residual_threshold,
                                                                      const CsrBitBsrSplitCostModel& cost_model) {
    cost_model.validate();
    return convert_bitbsr_to_csr_bitbsr_split_if(
        full, residual_threshold, [&](Offset p) { return cost_model.should_move_to_residual(p); });
}

// From CSR directly: one device plan build (conversion and split together).
template <typename T>
CsrBitBsrSplitMatrix<T> convert_to_csr_bitbsr_split(const CsrMatrix<T>& csr, Index block_rows, Index block_cols,
                                                    Index residual_threshold) {
    if (block_rows <= 0 || block_cols <= 0) throw std::runtime_error("BitBSR block sizes must be positive");
    if (block_rows != 8 || block_cols != 4) throw std::runtime_error("this build converts to 8x4 BitBSR blocks only");
    if (residual_threshold < 0) throw std::runtime_error("CSR+BitBSR residual threshold must be non-negative");
    return split_detail::split_on_device(csr, residual_threshold, split_detail::tabulate([](Offset) { return true; }));
}

template <typename T>
CsrBitBsrSplitMatrix<T> convert_to_csr_bitbsr_split_cost_gated(const CsrMatrix<T>& csr, Index block_rows,
                                                               Index block_cols, Index residual_threshold,
                                                               const CsrBitBsrSplitCostModel& cost_model) {
    cost_model.validate();
    if (block_rows <= 0 || block_cols <= 0) throw std::runtime_error("BitBSR block sizes must be positive");
    if (block_rows != 8 || block_cols != 4) throw std::runtime_error("this build converts to 8x4 BitBSR blocks only");
    if (residual_threshold < 0) throw std::runtime_error("CSR+BitBSR residual threshold must be non-negative");
    return split_detail::split_on_device(
        csr, residual_threshold,
        split_detail::tabulate([&](Offset p) { return cost_model.should_move_to_residual(p); }));
}

}  // namespace structural
