// bitbsr_spmv_8x4_dispatch.cuh -- structural:: BitBSR-only operator plan and
// dispatch over the B200 library: the enums (reference
// structural/include/structural/operators/bitbsr_spmv_8x4_dispatch.cuh:12-39),
// BitBsrSpmvPlan8x4 (:83-109) and run_bitbsr_spmv_once (:315-334).
//
// Every value codec of the enum is served by one route of cove_hybrid_spmv:
// Raw; ImplicitOne and ConstC (a constant); Sign2 and Sign2Scale (sign
// masks); the tile-code codecs Dict2, Unique4, Unique16, Dict256U8,
// Dict65536U16, K256U8 and GlobalLogKmeans16..128 (codes + codebook); Fp16
// and Bf16 (16-bit values per nnz); Bfp8, Bfp8Outlier and Bfp4 (block scale).
// The payloads are the plan fields the reference's builders fill.
#pragma once

#include "structural/operators/bitbsr_spmv_8x4_common.cuh"

namespace structural {

enum class BitBsrSpmvLayoutKind8x4 { ColBitmap64, ColBitmap64FlagLb, CusparseCsr };

enum class BitBsrValueCodecKind8x4 {
    Raw,
    ImplicitOne,
    ConstC,
    Sign2,
    Sign2Scale,
    Dict2,
    Unique4,
    Unique16,
    Dict256U8,
    Dict65536U16,
    Fp16,
    Bf16,
    Bfp8,
    Bfp8Outlier,
    Bfp4,
    K256U8,
    GlobalLogKmeans16,
    GlobalLogKmeans32,
    GlobalLogKmeans64,
    GlobalLogKmeans128,
};

inline bool bitbsr_spmv_8x4_uses_load_balance(BitBsrSpmvLayoutKind8x4 layout) {
    return layout == BitBsrSpmvLayoutKind8x4::ColBitmap64FlagLb;
}

inline bool bitbsr_spmv_8x4_is_non_raw_value_codec(BitBsrValueCodecKind8x4 c) {
    return c != BitBsrValueCodecKind8x4::Raw;
}

inline bool bitbsr_spmv_8x4_is_controlled_lossy_value_codec(BitBsrValueCodecKind8x4 c) {
    switch (c) {
        case BitBsrValueCodecKind8x4::Fp16:
        case BitBsrValueCodecKind8x4::Bf16:
        case BitBsrValueCodecKind8x4::Bfp8:
        case BitBsrValueCodecKind8x4::Bfp8Outlier:
        case BitBsrValueCodecKind8x4::Bfp4:
        case BitBsrValueCodecKind8x4::K256U8:
        case BitBsrValueCodecKind8x4::GlobalLogKmeans16:
        case BitBsrValueCodecKind8x4::GlobalLogKmeans32:
        case BitBsrValueCodecKind8x4::GlobalLogKmeans64:
        case BitBsrValueCodecKind8x4::GlobalLogKmeans128:
            return true;
        default:
            return false;
    }
}

template <typename T>
struct BitBsrSpmvPlan8x4 {
    BitBsrSpmvLayoutKind8x4 layout = BitBsrSpmvLayoutKind8x4::ColBitmap64FlagLb;
    BitBsrValueCodecKind8x4 value_codec = BitBsrValueCodecKind8x4::Raw;
    T value_scale = T{1};
    thrust::device_vector<std::uint32_t> tile_code_words;
    thrust::device_vector<std::uint32_t> sign_masks;
    thrust::device_vector<T> value_codebook;
    thrust::device_vector<signed char> int8_values;
    thrust::device_vector<std::uint16_t> block_scale_bf16;
    thrust::device_vector<std::uint8_t> packed_int4;
    thrust::device_vector<std::uint16_t> values16;
    thrust::device_vector<std::int32_t> outlier_rows;
    thrust::device_vector<std::int32_t> outlier_cols;
    thrust::device_vector<T> outlier_vals;
    thrust::device_vector<std::uint64_t> packed_col_bitmap_meta;
    BitBsrLoadBalanceLayout8x4 load_balance;
};

namespace gpu_detail {

template <typename T>
cove_hybrid_desc bitbsr_only_desc(const DeviceBitBsrMatrix<T>& device,
                                  const thrust::device_vector<std::uint64_t>& words) {
    cove_hybrid_desc a{};
    a.rows = device.rows;
    a.cols = device.cols;
    a.num_block_rows = device.num_block_rows;
    a.dtype = cove_dtype_of<T>();
    a.kept_blocks = device.num_blocks;
    a.kept_nnz = device.nnz;
    a.residual_nnz = 0;
    a.block_row_ptr = raw(device.block_row_ptr);
    a.block_row_val_ptr = raw(device.block_row_val_ptr);
    a.words = raw(words);
    a.res_row_ptr = nullptr;  // BitBSR only
    return a;
}

inline int tile_bits_of(BitBsrValueCodecKind8x4 c) {
    using K = BitBsrValueCodecKind8x4;
    switch (c) {
        case K::Dict2: return 1;
        case K::Unique4: return 2;
        case K::Unique16: return 4;
        case K::Dict256U8: return 8;
        case K::Dict65536U16: return 16;
        case K::K256U8:
        case K::GlobalLogKmeans16:
        case K::GlobalLogKmeans32:
        case K::GlobalLogKmeans64:
        case K::GlobalLogKmeans128: return 8;  // tile256 codes (bitbsr_spmv_8x4_lossy.cuh:59-105)
        default: return 0;
    }
}

}  // namespace gpu_detail

template <typename T>
void run_bitbsr_spmv_once(const DeviceBitBsrMatrix<T>& device, const BitBsrSpmvPlan8x4<T>& plan,
                          const thrust::device_vector<T>& d_x, thrust::device_vector<T>& d_y,
                          float* iter_ms = nullptr) {
    gpu_detail::validate_bitbsr_8x4_shape(device);
    if (plan.layout == BitBsrSpmvLayoutKind8x4::CusparseCsr) {
        throw std::runtime_error("internal error: unsupported BitBSR layout dispatch");
    }
    if (static_cast<Index>(d_x.size()) != device.cols) {
        throw std::runtime_error("GPU BitBSR SpMV input vector size mismatch");
    }
    if (static_cast<Offset>(plan.packed_col_bitmap_meta.size()) != device.num_blocks) {
        throw std::runtime_error("GPU BitBSR col_bitmap_packed layout size mismatch");
    }
    d_y.resize(device.rows);
    cove_hybrid_desc a = gpu_detail::bitbsr_only_desc(device, plan.packed_col_bitmap_meta);
    cove_values_desc v{};
    using K = BitBsrValueCodecKind8x4;
    switch (plan.value_codec) {
        case K::Raw:
            v.route = COVE_ROUTE_HYBRID;
            v.kept = gpu_detail::raw(device.values);
            break;
        case K::ImplicitOne:
            v.route = COVE_ROUTE_IMPLICIT_ONE;
            break;
        case K::ConstC:
            v.route = COVE_ROUTE_CONST_C;
            v.value_scale = static_cast<double>(plan.value_scale);
            break;
        case K::Sign2:
        case K::Sign2Scale:
            v.route = COVE_ROUTE_SIGN2;
            v.value_scale = plan.value_codec == K::Sign2 ? 1.0 : static_cast<double>(plan.value_scale);
            v.sign_masks = gpu_detail::raw(plan.sign_masks);
            if (static_cast<Offset>(plan.sign_masks.size()) != device.num_blocks) {
                throw std::runtime_error("GPU BitBSR sign tile mask count mismatch");
            }
            break;
        case K::Fp16:
            v.route = COVE_ROUTE_FP16_NNZ;
            v.kept = gpu_detail::raw(plan.values16);
            if (static_cast<Offset>(plan.values16.size()) != device.nnz) {
                throw std::runtime_error("GPU BitBSR round16 nnz value count mismatch");
            }
            break;
        case K::Bfp4:
            v.route = COVE_ROUTE_BFP4;
            v.kept = gpu_detail::raw(plan.packed_int4);
            v.block_scale = gpu_detail::raw(plan.block_scale_bf16);
            if (static_cast<Offset>(plan.packed_int4.size()) != (device.nnz + 1) / 2 ||
                static_cast<Offset>(plan.block_scale_bf16.size()) != device.num_blocks) {
                throw std::runtime_error("GPU BitBSR bfp4 payload size mismatch");
            }
            break;
        case K::Dict2:
        case K::Unique4:
        case K::Unique16:
        case K::Dict256U8:
        case K::Dict65536U16:
        case K::K256U8:
        case K::GlobalLogKmeans16:
        case K::GlobalLogKmeans32:
        case K::GlobalLogKmeans64:
        case K::GlobalLogKmeans128:
            v.route = COVE_ROUTE_TILE_CODE;
            v.tile_bits = gpu_detail::tile_bits_of(plan.value_codec);
            v.tile_code_words = gpu_detail::raw(plan.tile_code_words);
            v.codebook = gpu_detail::raw(plan.value_codebook);
            v.codebook_size = static_cast<int64_t>(plan.value_codebook.size());
            if (plan.tile_code_words.size() != static_cast<size_t>(device.num_blocks) * v.tile_bits) {
                throw std::runtime_error("GPU BitBSR tile code word count mismatch");
            }
            break;
        case K::Bf16:
            v.route = COVE_ROUTE_BF16_NNZ;
            v.kept = gpu_detail::raw(plan.values16);
            break;
        case K::Bfp8:
        case K::Bfp8Outlier:
            v.route = plan.value_codec == K::Bfp8 ? COVE_ROUTE_BFP8 : COVE_ROUTE_BFP8_OUTLIER;
            v.kept = gpu_detail::raw(plan.int8_values);
            v.block_scale = gpu_detail::raw(plan.block_scale_bf16);
            v.num_outliers = static_cast<int64_t>(plan.outlier_vals.size());
            v.outlier_rows = gpu_detail::raw(plan.outlier_rows);
            v.outlier_cols = gpu_detail::raw(plan.outlier_cols);
            v.outlier_vals = gpu_detail::raw(plan.outlier_vals);
            break;
        default:
            throw std::runtime_error("unsupported value codec for the B200 BitBSR operator");
    }
    gpu_detail::CudaEventTimer timer(iter_ms);
    cove_check(cove_hybrid_spmv(&a, &v, gpu_detail::raw(d_x), gpu_detail::raw(d_y), nullptr));
    gpu_detail::finish(timer, iter_ms);
}

}  // namespace structural
