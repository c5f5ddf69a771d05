// structural/operators/bitbsr_spmv_8x4.cuh -- the operator umbrella header
// (structural/include/structural/operators/bitbsr_spmv_8x4.cuh) with the
// per-codec load-balanced device wrappers that callers such as the CG bench
// (bench_cg_solve.cu:567-582) use directly:
//   spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_device
//       (bitbsr_spmv_8x4_raw.cuh:227-270)
//   spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_round16_nnz_device
//       (bitbsr_spmv_8x4_common.cuh:1418-1460)
//   spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_bfp8_blkscale_device
//       (:1512-1560)
//   spmv_bitbsr_gpu_8x4_bfp8_outlier_flag_load_balance_device (:1566-1620)
// Same parameters, size checks and messages; y is resized to rows and every
// row written (no zero-fill needed); synchronous unless device_ms is given,
// then timed with a CUDA event pair.  Each is one cove_hybrid_spmv call on
// the BitBSR-only route of its codec; the library sizes its own work split,
// so the load-balance layout is only checked, as the reference checks it.
#pragma once

#include "structural/operators/bitbsr_spmv_8x4_common.cuh"
#include "structural/operators/bitbsr_spmv_8x4_dispatch.cuh"

#include <string>

namespace structural {

namespace gpu_detail {

template <typename T>
void check_flag_lb_inputs(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint64_t>& packed_meta,
                          const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<T>& x) {
    validate_bitbsr_8x4_shape(m);
    if (static_cast<Index>(x.size()) != m.cols) throw std::runtime_error("GPU BitBSR SpMV input vector size mismatch");
    if (static_cast<Offset>(packed_meta.size()) != m.num_blocks)
        throw std::runtime_error("GPU BitBSR col_bitmap_packed layout size mismatch");
    if (static_cast<Index>(layout.work_item_row_ptr.size()) != m.num_block_rows + 1)
        throw std::runtime_error("GPU BitBSR load-balance work_item_row_ptr size mismatch");
}

template <typename T>
void check_bfp8_payload(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<signed char>& int8_values,
                        const thrust::device_vector<std::uint16_t>& block_scale_bf16, const char* name) {
    if (static_cast<Offset>(int8_values.size()) != m.nnz)
        throw std::runtime_error(std::string("GPU BitBSR ") + name + " int8 value size mismatch");
    if (static_cast<Offset>(block_scale_bf16.size()) != m.num_blocks)
        throw std::runtime_error(std::string("GPU BitBSR ") + name + " per-block scale size mismatch");
}

template <typename T>
void run_bitbsr_route(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint64_t>& packed_meta,
                      const cove_values_desc& v, const thrust::device_vector<T>& x, thrust::device_vector<T>& y,
                      float* device_ms) {
    y.resize(static_cast<size_t>(m.rows));
    const cove_hybrid_desc a = bitbsr_only_desc(m, packed_meta);
    CudaEventTimer timer(device_ms);
    cove_check(cove_hybrid_spmv(&a, &v, raw(x), raw(y), nullptr));
    finish(timer, device_ms);
}

}  // namespace gpu_detail

// y = A x with the raw T values (the lossless route).
template <typename T>
void spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<T>& x, thrust::device_vector<T>& y,
    float* device_ms = nullptr) {
    gpu_detail::check_flag_lb_inputs(bitbsr, packed_meta, layout, x);
    cove_values_desc v{};
    v.route = COVE_ROUTE_HYBRID;
    v.kept = gpu_detail::raw(bitbsr.values);
    gpu_detail::run_bitbsr_route(bitbsr, packed_meta, v, x, y, device_ms);
}

template <typename T>
thrust::device_vector<T> spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<T>& x, float* device_ms = nullptr) {
    thrust::device_vector<T> y;
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_device(bitbsr, packed_meta, layout, x, y, device_ms);
    return y;
}

// y = A x with one 16-bit value per nonzero: bf16 if Bf16, else fp16.
template <bool Bf16, typename T>
void spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_round16_nnz_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<std::uint16_t>& values16,
    const char* codec_name, const thrust::device_vector<T>& x, thrust::device_vector<T>& y,
    float* device_ms = nullptr) {
    gpu_detail::check_flag_lb_inputs(bitbsr, packed_meta, layout, x);
    if (static_cast<Offset>(values16.size()) != bitbsr.nnz)
        throw std::runtime_error(std::string("GPU BitBSR ") + codec_name + " per-nnz value size mismatch");
    cove_values_desc v{};
    v.route = Bf16 ? COVE_ROUTE_BF16_NNZ : COVE_ROUTE_FP16_NNZ;
    v.kept = gpu_detail::raw(values16);
    gpu_detail::run_bitbsr_route(bitbsr, packed_meta, v, x, y, device_ms);
}

// y = A x with int8 mantissas times a bf16 scale per block.
template <typename T>
void spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_bfp8_blkscale_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<signed char>& int8_values,
    const thrust::device_vector<std::uint16_t>& block_scale_bf16, const thrust::device_vector<T>& x,
    thrust::device_vector<T>& y, float* device_ms = nullptr) {
    gpu_detail::check_flag_lb_inputs(bitbsr, packed_meta, layout, x);
    gpu_detail::check_bfp8_payload(bitbsr, int8_values, block_scale_bf16, "bfp8_blkscale");
    cove_values_desc v{};
    v.route = COVE_ROUTE_BFP8;
    v.kept = gpu_detail::raw(int8_values);
    v.block_scale = gpu_detail::raw(block_scale_bf16);
    gpu_detail::run_bitbsr_route(bitbsr, packed_meta, v, x, y, device_ms);
}

// BFP8 bulk plus the exact side list of outliers (row, col, value), one
// event interval around both when timed.
template <typename T>
void spmv_bitbsr_gpu_8x4_bfp8_outlier_flag_load_balance_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<signed char>& int8_values,
    const thrust::device_vector<std::uint16_t>& block_scale_bf16, const thrust::device_vector<std::int32_t>& outlier_rows,
    const thrust::device_vector<std::int32_t>& outlier_cols, const thrust::device_vector<T>& outlier_vals,
    const thrust::device_vector<T>& x, thrust::device_vector<T>& y, float* device_ms = nullptr) {
    gpu_detail::check_flag_lb_inputs(bitbsr, packed_meta, layout, x);
    gpu_detail::check_bfp8_payload(bitbsr, int8_values, block_scale_bf16, "bfp8_outlier_blkscale");
    if (outlier_rows.size() != outlier_cols.size() || outlier_rows.size() != outlier_vals.size())
        throw std::runtime_error("GPU BitBSR bfp8_outlier side-list size mismatch");
    cove_values_desc v{};
    v.route = COVE_ROUTE_BFP8_OUTLIER;
    v.kept = gpu_detail::raw(int8_values);
    v.block_scale = gpu_detail::raw(block_scale_bf16);
    v.num_outliers = static_cast<int64_t>(outlier_vals.size());
    v.outlier_rows = gpu_detail::raw(outlier_rows);
    v.outlier_cols = gpu_detail::raw(outlier_cols);
    v.outlier_vals = gpu_detail::raw(outlier_vals);
    gpu_detail::run_bitbsr_route(bitbsr, packed_meta, v, x, y, device_ms);
}

// ---- the other per-codec operators (bitbsr_spmv_8x4_{raw,lossless,lossy}.cuh) ----
//
// Each codec has a load-balanced form (`..._flag_load_balance_<codec>`, with
// the layout argument, checked as above) and a plain form (no layout); both
// run the same route.  `..._device` takes device x and y; the form without
// the suffix takes a host x and returns a host y.

namespace gpu_detail {

template <typename T>
void check_plain_inputs(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint64_t>& packed_meta,
                        const thrust::device_vector<T>& x) {
    validate_bitbsr_8x4_shape(m);
    if (static_cast<Index>(x.size()) != m.cols) throw std::runtime_error("GPU BitBSR SpMV input vector size mismatch");
    if (static_cast<Offset>(packed_meta.size()) != m.num_blocks)
        throw std::runtime_error("GPU BitBSR col_bitmap_packed layout size mismatch");
}

// Checks (with the layout when given) and runs one route.
template <typename T>
void run_codec(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint64_t>& packed_meta,
               const BitBsrLoadBalanceLayout8x4* layout, const cove_values_desc& v, const thrust::device_vector<T>& x,
               thrust::device_vector<T>& y, float* device_ms) {
    if (layout) check_flag_lb_inputs(m, packed_meta, *layout, x);
    else check_plain_inputs(m, packed_meta, x);
    run_bitbsr_route(m, packed_meta, v, x, y, device_ms);
}

template <typename T>
cove_values_desc sign_desc(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint32_t>& masks,
                           double scale) {
    if (static_cast<Offset>(masks.size()) != m.num_blocks)
        throw std::runtime_error("GPU BitBSR sign tile mask count mismatch");
    cove_values_desc v{};
    v.route = COVE_ROUTE_SIGN2;
    v.value_scale = scale;
    v.sign_masks = raw(masks);
    return v;
}

// Codes of `bits` bits per cell into a codebook of at most max_codebook
// entries (validate_tile_code_value_codec, common.cuh:942-964).
template <typename T>
cove_values_desc tile_desc(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint32_t>& words,
                           const thrust::device_vector<T>& codebook, int bits, int max_codebook, const char* name) {
    if (words.size() != static_cast<size_t>(m.num_blocks) * bits)
        throw std::runtime_error(std::string("GPU BitBSR ") + name + " tile code word size mismatch");
    if (codebook.size() > static_cast<size_t>(max_codebook))
        throw std::runtime_error(std::string("GPU BitBSR ") + name + " codebook is too large");
    if (m.nnz > 0 && codebook.empty())
        throw std::runtime_error(std::string("GPU BitBSR ") + name + " codebook is empty");
    cove_values_desc v{};
    v.route = COVE_ROUTE_TILE_CODE;
    v.tile_bits = bits;
    v.tile_code_words = raw(words);
    v.codebook = raw(codebook);
    v.codebook_size = static_cast<int64_t>(codebook.size());
    return v;
}

template <typename T, typename F>
std::vector<T> on_host(const std::vector<T>& x, F&& device_call) {
    const thrust::device_vector<T> dx(x.begin(), x.end());
    thrust::device_vector<T> dy;
    device_call(dx, dy);
    std::vector<T> y(dy.size());
    thrust::copy(dy.begin(), dy.end(), y.begin());
    return y;
}

}  // namespace gpu_detail

// raw values, plain form and the host forms
template <typename T>
void spmv_bitbsr_gpu_8x4_col_bitmap_packed_device(const DeviceBitBsrMatrix<T>& bitbsr,
                                                  const thrust::device_vector<std::uint64_t>& packed_meta,
                                                  const thrust::device_vector<T>& x, thrust::device_vector<T>& y,
                                                  float* device_ms = nullptr) {
    cove_values_desc v{};
    v.route = COVE_ROUTE_HYBRID;
    v.kept = gpu_detail::raw(bitbsr.values);
    gpu_detail::run_codec(bitbsr, packed_meta, nullptr, v, x, y, device_ms);
}

template <typename T>
thrust::device_vector<T> spmv_bitbsr_gpu_8x4_col_bitmap_packed_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const thrust::device_vector<T>& x, float* device_ms = nullptr) {
    thrust::device_vector<T> y;
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_device(bitbsr, packed_meta, x, y, device_ms);
    return y;
}

template <typename T>
std::vector<T> spmv_bitbsr_gpu_8x4_col_bitmap_packed(const DeviceBitBsrMatrix<T>& bitbsr,
                                                     const thrust::device_vector<std::uint64_t>& packed_meta,
                                                     const std::vector<T>& x, float* device_ms = nullptr) {
    return gpu_detail::on_host(x, [&](const thrust::device_vector<T>& dx, thrust::device_vector<T>& dy) {
        spmv_bitbsr_gpu_8x4_col_bitmap_packed_device(bitbsr, packed_meta, dx, dy, device_ms);
    });
}

template <typename T>
std::vector<T> spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const std::vector<T>& x, float* device_ms = nullptr) {
    return gpu_detail::on_host(x, [&](const thrust::device_vector<T>& dx, thrust::device_vector<T>& dy) {
        spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_device(bitbsr, packed_meta, layout, dx, dy, device_ms);
    });
}

// The named forms of one codec: NAME_device / NAME (host) in the plain and
// the load-balanced variants.  PARAMS are the codec's payload parameters,
// ARGS the same names, DESC the cove_values_desc built from them.
#define COVE_SHIM_CODEC_OPERATORS(NAME, PARAMS, ARGS, DESC)                                                        \
    template <typename T>                                                                                          \
    void spmv_bitbsr_gpu_8x4_col_bitmap_packed_##NAME##_device(                                                    \
        const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta PARAMS,       \
        const thrust::device_vector<T>& x, thrust::device_vector<T>& y, float* device_ms = nullptr) {             \
        gpu_detail::run_codec(bitbsr, packed_meta, nullptr, DESC, x, y, device_ms);                               \
    }                                                                                                              \
    template <typename T>                                                                                          \
    std::vector<T> spmv_bitbsr_gpu_8x4_col_bitmap_packed_##NAME(                                                   \
        const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta PARAMS,       \
        const std::vector<T>& x, float* device_ms = nullptr) {                                                    \
        return gpu_detail::on_host(x, [&](const thrust::device_vector<T>& dx, thrust::device_vector<T>& dy) {     \
            spmv_bitbsr_gpu_8x4_col_bitmap_packed_##NAME##_device(bitbsr, packed_meta ARGS, dx, dy, device_ms);   \
        });                                                                                                        \
    }                                                                                                              \
    template <typename T>                                                                                          \
    void spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_##NAME##_device(                                  \
        const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,              \
        const BitBsrLoadBalanceLayout8x4& layout PARAMS, const thrust::device_vector<T>& x,                        \
        thrust::device_vector<T>& y, float* device_ms = nullptr) {                                                \
        gpu_detail::run_codec(bitbsr, packed_meta, &layout, DESC, x, y, device_ms);                               \
    }                                                                                                              \
    template <typename T>                                                                                          \
    std::vector<T> spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_##NAME(                                 \
        const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,              \
        const BitBsrLoadBalanceLayout8x4& layout PARAMS, const std::vector<T>& x, float* device_ms = nullptr) {    \
        return gpu_detail::on_host(x, [&](const thrust::device_vector<T>& dx, thrust::device_vector<T>& dy) {     \
            spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_##NAME##_device(bitbsr, packed_meta, layout    \
                                                                                        ARGS, dx, dy, device_ms); \
        });                                                                                                        \
    }

#define COVE_SHIM_COMMA ,
#define COVE_SHIM_TILE_PARAMS \
    COVE_SHIM_COMMA const thrust::device_vector<std::uint32_t>& tile_code_words COVE_SHIM_COMMA \
        const thrust::device_vector<T>& codebook
#define COVE_SHIM_TILE_ARGS COVE_SHIM_COMMA tile_code_words COVE_SHIM_COMMA codebook

namespace gpu_detail {
inline cove_values_desc route_only(int route) {
    cove_values_desc v{};
    v.route = route;
    return v;
}
template <typename T>
cove_values_desc nnz16_desc(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint16_t>& values16,
                            bool bf16, const char* name) {
    if (static_cast<Offset>(values16.size()) != m.nnz)
        throw std::runtime_error(std::string("GPU BitBSR ") + name + " per-nnz value size mismatch");
    cove_values_desc v{};
    v.route = bf16 ? COVE_ROUTE_BF16_NNZ : COVE_ROUTE_FP16_NNZ;
    v.kept = raw(values16);
    return v;
}
template <typename T>
cove_values_desc bfp4_desc(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint8_t>& packed_int4,
                           const thrust::device_vector<std::uint16_t>& block_scale_bf16) {
    if (static_cast<Offset>(packed_int4.size()) != (m.nnz + 1) / 2)
        throw std::runtime_error("GPU BitBSR bfp4_blkscale int4 value size mismatch");
    if (static_cast<Offset>(block_scale_bf16.size()) != m.num_blocks)
        throw std::runtime_error("GPU BitBSR bfp4_blkscale per-block scale size mismatch");
    cove_values_desc v{};
    v.route = COVE_ROUTE_BFP4;
    v.kept = raw(packed_int4);
    v.block_scale = raw(block_scale_bf16);
    return v;
}
inline cove_values_desc constant(double c) {
    cove_values_desc v{};
    v.route = COVE_ROUTE_CONST_C;
    v.value_scale = c;
    return v;
}
}  // namespace gpu_detail

// every value 1 / every value C (bitbsr_spmv_8x4_lossless.cuh)
COVE_SHIM_CODEC_OPERATORS(implicit_one, , , gpu_detail::route_only(COVE_ROUTE_IMPLICIT_ONE))
COVE_SHIM_CODEC_OPERATORS(const_c, COVE_SHIM_COMMA T value, COVE_SHIM_COMMA value,
                          gpu_detail::constant(static_cast<double>(value)))
// +-1 and +-C by a sign mask per block
COVE_SHIM_CODEC_OPERATORS(sign_tile32, COVE_SHIM_COMMA const thrust::device_vector<std::uint32_t>& sign_masks,
                          COVE_SHIM_COMMA sign_masks, gpu_detail::sign_desc(bitbsr, sign_masks, 1.0))
COVE_SHIM_CODEC_OPERATORS(sign2_scale_tile32,
                          COVE_SHIM_COMMA const thrust::device_vector<std::uint32_t>& sign_masks COVE_SHIM_COMMA T scale,
                          COVE_SHIM_COMMA sign_masks COVE_SHIM_COMMA scale,
                          gpu_detail::sign_desc(bitbsr, sign_masks, static_cast<double>(scale)))
// per-cell codes into a codebook: 1, 2, 4, 8, 16 bits
COVE_SHIM_CODEC_OPERATORS(dict2_tile32, COVE_SHIM_TILE_PARAMS, COVE_SHIM_TILE_ARGS,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, 1, 2, "dict2_tile32"))
COVE_SHIM_CODEC_OPERATORS(unique4_tile64, COVE_SHIM_TILE_PARAMS, COVE_SHIM_TILE_ARGS,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, 2, 4, "unique4_tile64"))
COVE_SHIM_CODEC_OPERATORS(unique16_tile128, COVE_SHIM_TILE_PARAMS, COVE_SHIM_TILE_ARGS,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, 4, 16, "unique16_tile128"))
COVE_SHIM_CODEC_OPERATORS(dict256_tile256, COVE_SHIM_TILE_PARAMS, COVE_SHIM_TILE_ARGS,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, 8, 256, "dict256_tile256"))
COVE_SHIM_CODEC_OPERATORS(k256_tile256, COVE_SHIM_TILE_PARAMS, COVE_SHIM_TILE_ARGS,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, 8, 256, "k256_tile256"))
COVE_SHIM_CODEC_OPERATORS(logkmeans_tile256, COVE_SHIM_TILE_PARAMS, COVE_SHIM_TILE_ARGS,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, 8, 256, "logkmeans_tile256"))
COVE_SHIM_CODEC_OPERATORS(dict65536_tile512, COVE_SHIM_TILE_PARAMS, COVE_SHIM_TILE_ARGS,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, 16, 65536, "dict65536_tile512"))

// 16-bit values per nonzero (bitbsr_spmv_8x4_lossy.cuh:35-58, 132-158)
COVE_SHIM_CODEC_OPERATORS(fp16_nnz, COVE_SHIM_COMMA const thrust::device_vector<std::uint16_t>& values16,
                          COVE_SHIM_COMMA values16, gpu_detail::nnz16_desc(bitbsr, values16, false, "fp16_nnz"))
COVE_SHIM_CODEC_OPERATORS(bf16_nnz, COVE_SHIM_COMMA const thrust::device_vector<std::uint16_t>& values16,
                          COVE_SHIM_COMMA values16, gpu_detail::nnz16_desc(bitbsr, values16, true, "bf16_nnz"))
// packed signed 4-bit mantissas times a bf16 scale per block
COVE_SHIM_CODEC_OPERATORS(bfp4_blkscale,
                          COVE_SHIM_COMMA const thrust::device_vector<std::uint8_t>& packed_int4 COVE_SHIM_COMMA
                              const thrust::device_vector<std::uint16_t>& block_scale_bf16,
                          COVE_SHIM_COMMA packed_int4 COVE_SHIM_COMMA block_scale_bf16,
                          gpu_detail::bfp4_desc(bitbsr, packed_int4, block_scale_bf16))

#undef COVE_SHIM_TILE_ARGS

template <bool Bf16, typename T>
void spmv_bitbsr_gpu_8x4_col_bitmap_packed_round16_nnz_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const thrust::device_vector<std::uint16_t>& values16, const char* codec_name, const thrust::device_vector<T>& x,
    thrust::device_vector<T>& y, float* device_ms = nullptr) {
    gpu_detail::run_codec(bitbsr, packed_meta, nullptr, gpu_detail::nnz16_desc(bitbsr, values16, Bf16, codec_name), x, y,
                          device_ms);
}

template <typename T>
void spmv_bitbsr_gpu_8x4_col_bitmap_packed_bfp8_blkscale_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const thrust::device_vector<signed char>& int8_values, const thrust::device_vector<std::uint16_t>& block_scale_bf16,
    const thrust::device_vector<T>& x, thrust::device_vector<T>& y, float* device_ms = nullptr) {
    gpu_detail::check_bfp8_payload(bitbsr, int8_values, block_scale_bf16, "bfp8_blkscale");
    cove_values_desc v{};
    v.route = COVE_ROUTE_BFP8;
    v.kept = gpu_detail::raw(int8_values);
    v.block_scale = gpu_detail::raw(block_scale_bf16);
    gpu_detail::run_codec(bitbsr, packed_meta, nullptr, v, x, y, device_ms);
}

// Codes of BitsPerCode (1, 2, 4, 8 or 16) bits per cell (common.cuh:1180-1300).
template <int BitsPerCode, typename T>
void spmv_bitbsr_gpu_8x4_col_bitmap_packed_code_tile_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const thrust::device_vector<std::uint32_t>& tile_code_words, const thrust::device_vector<T>& codebook,
    int max_codebook_size, const char* codec_name, const thrust::device_vector<T>& x, thrust::device_vector<T>& y,
    float* device_ms = nullptr) {
    static_assert(BitsPerCode == 1 || BitsPerCode == 2 || BitsPerCode == 4 || BitsPerCode == 8 || BitsPerCode == 16,
                  "tile codes are 1, 2, 4, 8 or 16 bits");
    gpu_detail::run_codec(bitbsr, packed_meta, nullptr,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, BitsPerCode, max_codebook_size,
                                                codec_name),
                          x, y, device_ms);
}

template <int BitsPerCode, typename T>
void spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_code_tile_device(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<std::uint32_t>& tile_code_words,
    const thrust::device_vector<T>& codebook, int max_codebook_size, const char* codec_name,
    const thrust::device_vector<T>& x, thrust::device_vector<T>& y, float* device_ms = nullptr) {
    static_assert(BitsPerCode == 1 || BitsPerCode == 2 || BitsPerCode == 4 || BitsPerCode == 8 || BitsPerCode == 16,
                  "tile codes are 1, 2, 4, 8 or 16 bits");
    gpu_detail::run_codec(bitbsr, packed_meta, &layout,
                          gpu_detail::tile_desc(bitbsr, tile_code_words, codebook, BitsPerCode, max_codebook_size,
                                                codec_name),
                          x, y, device_ms);
}
#undef COVE_SHIM_TILE_PARAMS
#undef COVE_SHIM_COMMA
#undef COVE_SHIM_CODEC_OPERATORS

}  // namespace structural
