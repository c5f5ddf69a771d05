// cove_convert.cuh -- device-resident streams of a plan and the builders.
#pragma once

#include "cove_internal.cuh"

namespace cove {

// Un-split BitBSR 8x4 (DeviceBitBsrMatrix, gpu_convert.cuh:251-351).
struct FullBitBsr {
    int32_t rows = 0, cols = 0, nbr = 0;
    int64_t num_blocks = 0, nnz = 0;
    DevBuf block_row_ptr;      // int32 nbr+1
    DevBuf block_row_val_ptr;  // int32 nbr+1
    DevBuf block_col_idx;      // int32 blocks
    DevBuf bitmap;             // uint32 blocks
    DevBuf values;             // T nnz
};

// CSR + BitBSR split (CsrBitBsrSplitMatrix, csr_bitbsr_split.hpp:15-51).
struct SplitParts {
    int64_t kept_blocks = 0, kept_nnz = 0, residual_blocks = 0, residual_nnz = 0;
    int64_t cost_skipped_blocks = 0, cost_skipped_nnz = 0;
    DevBuf kept_block_row_ptr;      // int32 nbr+1
    DevBuf kept_block_row_val_ptr;  // int32 nbr+1
    DevBuf kept_block_val_ptr;      // int32 kept_blocks+1
    DevBuf kept_col;                // int32
    DevBuf kept_bitmap;             // uint32
    DevBuf kept_values;             // T
    DevBuf res_row_ptr;             // int32 rows+1
    DevBuf res_col;                 // int32
    DevBuf res_values;              // T
};

// Packed words + work items (BitBsrLoadBalanceLayout8x4, common.cuh:24-29).
struct Layout {
    int chunk_blocks = 0, split_threshold_blocks = 0;
    int64_t num_items = 0;
    DevBuf words;         // uint64 kept_blocks
    DevBuf items;         // WorkItem
    DevBuf item_row_ptr;  // int32 nbr+1
};

// Long residual-row chunks (main_gpu_csr_bitbsr_spmv.cu:1155-1184).
struct Chunks {
    int tau = 0;
    int64_t num_chunks = 0, long_rows = 0;
    DevBuf row, pbegin, pcount;  // int32 each
};

// Throws on invalid CSR; returns whether every row's columns are
// non-decreasing with stored zeros included (the converter may then cut
// long block rows into column-range pieces).
template <typename T>
bool validate_csr(const cove_csr_desc& d, cudaStream_t s);
// caller-buffer steps (the reference's step-by-step device API); `split`
// is validate_csr's answer
template <typename T>
void bitbsr_count(const cove_csr_desc& d, bool split, int32_t* brp, int32_t* brvp, int64_t* num_blocks,
                  int64_t* nnz, cudaStream_t s);
template <typename T>
void bitbsr_fill(const cove_csr_desc& d, bool split, int32_t* col, uint32_t* bitmap, T* values,
                 cudaStream_t s);
void pack_words(int64_t nb, const int32_t* col, const uint32_t* bitmap, uint64_t* words,
                cudaStream_t s);
int64_t lb_count(int32_t nbr, const int32_t* brp, int chunk, int split, int style,
                 int32_t* item_rp, cudaStream_t s);
void lb_fill(int32_t nbr, const int32_t* brp, const int32_t* brvp, const uint32_t* bitmap,
             const int32_t* item_rp, int chunk, int split, int style, uint64_t* words,
             WorkItem* items, cudaStream_t s);
template <typename T>
void build_full_bitbsr(const cove_csr_desc& d, bool split, FullBitBsr& out, cudaStream_t s);
unsigned long long move_mask_for(const cove_plan_opts& o);
template <typename T>
void build_split(const FullBitBsr& f, const cove_plan_opts& o, SplitParts& out, cudaStream_t s);
void build_layout(const SplitParts& sp, int32_t nbr, const cove_plan_opts& o, Layout& out,
                  cudaStream_t s);
void build_chunks(const int32_t* res_rp, int32_t rows, int tau, int chunk_nnz, Chunks& out,
                  cudaStream_t s);

}  // namespace cove
