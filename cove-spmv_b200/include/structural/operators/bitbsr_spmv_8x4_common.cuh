// bitbsr_spmv_8x4_common.cuh -- structural:: 8x4 layout types and builders
// over the B200 library.  Same names and layouts as the reference's
// structural/include/structural/operators/bitbsr_spmv_8x4_common.cuh
// (BitBsrWorkItem8x4 :15-22, BitBsrLoadBalanceLayout8x4 :24-29, the packed
// word helpers :95-117, make_bitbsr_8x4_col_bitmap_packed :1024-1050 and
// make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items :1137-1160).
#pragma once

#include "structural/gpu_convert.cuh"

#include <cstdint>

namespace structural {

struct BitBsrWorkItem8x4 {
    std::uint32_t br = 0;
    std::uint32_t block_begin = 0;
    std::uint32_t block_count = 0;
    std::uint32_t value_begin = 0;
};
static_assert(sizeof(BitBsrWorkItem8x4) == 16, "8x4 work item must stay 16 bytes");

struct BitBsrLoadBalanceLayout8x4 {
    int chunk_blocks = 0;
    int split_threshold_blocks = 0;
    thrust::device_vector<Offset> work_item_row_ptr;
    thrust::device_vector<BitBsrWorkItem8x4> work_items;
};

namespace gpu_detail {

constexpr int kSpmv8x4BlockRows = 8;
constexpr int kSpmv8x4BlockCols = 4;
constexpr std::uint32_t kSpmv8x4PackedFlagMask = 0x80000000U;
constexpr std::uint64_t kSpmv8x4PackedFlagBit = std::uint64_t{1} << 31;
constexpr std::uint64_t kSpmv8x4PackedAbsColMask = 0x7fffffffULL;

// word = bitmap << 32 | flag << 31 | (col & 0x7fffffff)
__host__ __device__ inline std::uint64_t pack_col_bitmap(std::uint32_t col, BitmapWord bitmap,
                                                         bool flag = false) {
    return (static_cast<std::uint64_t>(bitmap) << 32) | (col & kSpmv8x4PackedAbsColMask) |
           (flag ? kSpmv8x4PackedFlagBit : 0ULL);
}
__host__ __device__ inline std::uint32_t unpack_abs_col(std::uint64_t meta) {
    return static_cast<std::uint32_t>(meta & kSpmv8x4PackedAbsColMask);
}
__host__ __device__ inline bool unpack_col_bitmap_flag(std::uint64_t meta) {
    return (meta & kSpmv8x4PackedFlagBit) != 0ULL;
}
__host__ __device__ inline BitmapWord unpack_bitmap(std::uint64_t meta) {
    return static_cast<BitmapWord>(meta >> 32);
}

template <typename T>
void validate_bitbsr_8x4_shape(const DeviceBitBsrMatrix<T>& m) {
    m.validate_shape();
    if (m.block_rows != kSpmv8x4BlockRows || m.block_cols != kSpmv8x4BlockCols || m.words_per_block != 1) {
        throw std::runtime_error("GPU BitBSR 8x4 operator requires 8x4 blocks with one bitmap word");
    }
}

}  // namespace gpu_detail

template <typename T>
void make_bitbsr_8x4_col_bitmap_packed(const DeviceBitBsrMatrix<T>& bitbsr,
                                       thrust::device_vector<std::uint64_t>& packed_meta,
                                       float* device_ms = nullptr) {
    gpu_detail::validate_bitbsr_8x4_shape(bitbsr);
    packed_meta.resize(bitbsr.num_blocks);
    if (bitbsr.num_blocks == 0) {
        if (device_ms) *device_ms = 0.0f;
        return;
    }
    gpu_detail::CudaEventTimer timer(device_ms);
    cove_check(cove_pack_words(bitbsr.num_blocks, gpu_detail::raw(bitbsr.block_col_idx),
                               gpu_detail::raw(bitbsr.bitmap_words), gpu_detail::raw(packed_meta), nullptr));
    gpu_detail::finish(timer, device_ms);
}

namespace gpu_detail {

template <typename T>
void build_work_items(const DeviceBitBsrMatrix<T>& bitbsr, BitBsrLoadBalanceLayout8x4& layout,
                      int chunk_blocks, int split_threshold_blocks, int style,
                      thrust::device_vector<std::uint64_t>* packed_meta, float* device_ms) {
    validate_bitbsr_8x4_shape(bitbsr);
    if (chunk_blocks <= 0) throw std::runtime_error("GPU BitBSR load-balance chunk_blocks must be positive");
    if (split_threshold_blocks <= 0) {
        throw std::runtime_error("GPU BitBSR load-balance split_threshold_blocks must be positive");
    }
    thrust::device_vector<std::uint64_t> scratch;
    thrust::device_vector<std::uint64_t>& words = packed_meta ? *packed_meta : scratch;
    if (static_cast<Offset>(words.size()) != bitbsr.num_blocks) {
        if (packed_meta) throw std::runtime_error("GPU BitBSR col_bitmap_packed layout size mismatch");
        words.resize(bitbsr.num_blocks);
    }
    layout.chunk_blocks = chunk_blocks;
    layout.split_threshold_blocks = split_threshold_blocks;
    layout.work_item_row_ptr.assign(static_cast<size_t>(bitbsr.num_block_rows) + 1, 0);
    layout.work_items.clear();
    CudaEventTimer timer(device_ms);
    // flags are recomputed from scratch: clear them by repacking the words
    cove_check(cove_pack_words(bitbsr.num_blocks, raw(bitbsr.block_col_idx), raw(bitbsr.bitmap_words),
                               raw(words), nullptr));
    int64_t items = 0;
    cove_check(cove_lb_layout_count(bitbsr.num_block_rows, raw(bitbsr.block_row_ptr), chunk_blocks,
                                    split_threshold_blocks, style, raw(layout.work_item_row_ptr),
                                    &items, nullptr));
    layout.work_items.resize(static_cast<size_t>(items));
    cove_check(cove_lb_layout_fill(bitbsr.num_block_rows, raw(bitbsr.block_row_ptr),
                                   raw(bitbsr.block_row_val_ptr), raw(bitbsr.bitmap_words),
                                   raw(layout.work_item_row_ptr), chunk_blocks, split_threshold_blocks,
                                   style, raw(words), raw(layout.work_items), nullptr));
    finish(timer, device_ms);
}

}  // namespace gpu_detail

// Device layout: flag iff a block row is cut into more than one piece.
template <typename T>
void make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(
    const DeviceBitBsrMatrix<T>& bitbsr, BitBsrLoadBalanceLayout8x4& layout, int chunk_blocks,
    int split_threshold_blocks, thrust::device_vector<std::uint64_t>& packed_meta,
    float* device_ms = nullptr) {
    gpu_detail::build_work_items(bitbsr, layout, chunk_blocks, split_threshold_blocks, COVE_LB_DEVICE,
                                 &packed_meta, device_ms);
}

template <typename T>
void make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(
    const DeviceBitBsrMatrix<T>& bitbsr, BitBsrLoadBalanceLayout8x4& layout, int chunk_blocks,
    thrust::device_vector<std::uint64_t>& packed_meta, float* device_ms = nullptr) {
    make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(bitbsr, layout, chunk_blocks, chunk_blocks,
                                                            packed_meta, device_ms);
}

template <typename T>
void make_bitbsr_8x4_load_balance_work_items(const DeviceBitBsrMatrix<T>& bitbsr,
                                             BitBsrLoadBalanceLayout8x4& layout, int chunk_blocks,
                                             int split_threshold_blocks, float* device_ms = nullptr) {
    gpu_detail::build_work_items(bitbsr, layout, chunk_blocks, split_threshold_blocks, COVE_LB_DEVICE,
                                 nullptr, device_ms);
}

}  // namespace structural
