// Instantiates every per-codec operator wrapper of structural/gpu_spmv.cuh for
// fp64 and fp32 (compiled by tests/test_shim_wrappers.py, never run): the
// parameter lists stay callable the way the reference's callers call them.
#include "structural/gpu_spmv.cuh"
using namespace structural;
template <typename T> void all(const DeviceBitBsrMatrix<T>& m, const thrust::device_vector<std::uint64_t>& w,
                               const BitBsrLoadBalanceLayout8x4& l, const thrust::device_vector<T>& x,
                               thrust::device_vector<T>& y, const std::vector<T>& hx) {
    thrust::device_vector<std::uint32_t> u32; thrust::device_vector<std::uint16_t> u16; thrust::device_vector<std::uint8_t> u8;
    thrust::device_vector<signed char> i8; thrust::device_vector<T> cb;
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_device(m, w, x, y);
    (void)spmv_bitbsr_gpu_8x4_col_bitmap_packed(m, w, hx);
    (void)spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance(m, w, l, hx);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_implicit_one_device(m, w, x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_implicit_one_device(m, w, l, x, y);
    (void)spmv_bitbsr_gpu_8x4_col_bitmap_packed_const_c(m, w, T(2), hx);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_sign2_scale_tile32_device(m, w, l, u32, T(2), x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_dict65536_tile512_device(m, w, u32, cb, x, y);
    (void)spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_logkmeans_tile256(m, w, l, u32, cb, hx);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_fp16_nnz_device(m, w, u16, x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_bf16_nnz_device(m, w, l, u16, x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_round16_nnz_device<true>(m, w, u16, "bf16_nnz", x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_bfp4_blkscale_device(m, w, u8, u16, x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_bfp4_blkscale_device(m, w, l, u8, u16, x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_bfp8_blkscale_device(m, w, i8, u16, x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_code_tile_device<4>(m, w, u32, cb, 16, "unique16_tile128", x, y);
    spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_code_tile_device<16>(m, w, l, u32, cb, 65536, "dict65536_tile512", x, y);
}
template void all<double>(const DeviceBitBsrMatrix<double>&, const thrust::device_vector<std::uint64_t>&, const BitBsrLoadBalanceLayout8x4&, const thrust::device_vector<double>&, thrust::device_vector<double>&, const std::vector<double>&);
template void all<float>(const DeviceBitBsrMatrix<float>&, const thrust::device_vector<std::uint64_t>&, const BitBsrLoadBalanceLayout8x4&, const thrust::device_vector<float>&, thrust::device_vector<float>&, const std::vector<float>&);
