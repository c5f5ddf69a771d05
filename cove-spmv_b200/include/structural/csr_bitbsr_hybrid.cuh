// csr_bitbsr_hybrid.cuh -- the hybrid / joint CSR+BitBSR operator of the
// reference's structural/src/main_gpu_csr_bitbsr_spmv.cu, promoted to a
// header with the launchers' own parameter lists:
//   make_fused_8x4_load_balance_layout_host   :387-475 (host BitBSR in,
//                                              device layout out; built here
//                                              by the sm_100a layout kernels)
//   run_csr_bitbsr_fused_8x4_lb               :636-712  (lossless)
//   run_csr_bitbsr_fused_8x4_lb_bfp8          :899-930
//   run_csr_bitbsr_fused_8x4_lb_dict<T,IdxT>  :932-963
//   run_csr_bitbsr_fused_8x4_lb_bfp8_outlier  :984-1029
// plus a RAII wrapper of the full device pipeline (cove::Plan).
//
// Differences a caller can see: y need not be zeroed (every row is written
// once), and the dict arm accumulates in T rather than fp32.
#pragma once

#include "structural/operators/bitbsr_spmv_8x4_dispatch.cuh"

#include <cstdint>

namespace structural {

template <typename T>
void make_fused_8x4_load_balance_layout_host(const BitBsrMatrix<T>& bitbsr,
                                             BitBsrLoadBalanceLayout8x4& layout,
                                             thrust::device_vector<std::uint64_t>& packed_meta,
                                             int chunk_blocks, int split_threshold_blocks,
                                             float* device_ms = nullptr) {
    bitbsr.validate();
    if (bitbsr.block_rows != 8 || bitbsr.block_cols != 4 || bitbsr.words_per_block != 1) {
        throw std::runtime_error("fused CSR+BitBSR GPU probe currently supports only 8x4 blocks");
    }
    if (chunk_blocks <= 0 || split_threshold_blocks <= 0) {
        throw std::runtime_error("fused CSR+BitBSR load-balance parameters must be positive");
    }
    const DeviceBitBsrMatrix<T> dev = copy_bitbsr_to_device(bitbsr);
    packed_meta.resize(dev.num_blocks);
    layout.chunk_blocks = chunk_blocks;
    layout.split_threshold_blocks = split_threshold_blocks;
    layout.work_item_row_ptr.assign(static_cast<size_t>(dev.num_block_rows) + 1, 0);
    using gpu_detail::raw;
    cove_check(cove_pack_words(dev.num_blocks, raw(dev.block_col_idx), raw(dev.bitmap_words),
                               raw(packed_meta), nullptr));
    int64_t items = 0;
    cove_check(cove_lb_layout_count(dev.num_block_rows, raw(dev.block_row_ptr), chunk_blocks,
                                    split_threshold_blocks, COVE_LB_HYBRID, raw(layout.work_item_row_ptr),
                                    &items, nullptr));
    layout.work_items.resize(static_cast<size_t>(items));
    cove_check(cove_lb_layout_fill(dev.num_block_rows, raw(dev.block_row_ptr), raw(dev.block_row_val_ptr),
                                   raw(dev.bitmap_words), raw(layout.work_item_row_ptr), chunk_blocks,
                                   split_threshold_blocks, COVE_LB_HYBRID, raw(packed_meta),
                                   raw(layout.work_items), nullptr));
    cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize()", __FILE__, __LINE__);
    if (device_ms) *device_ms = 0.0f;
}

namespace gpu_detail {

template <typename T>
cove_hybrid_desc hybrid_desc(const DeviceBitBsrMatrix<T>& bitbsr,
                             const thrust::device_vector<std::uint64_t>& packed_meta,
                             const BitBsrLoadBalanceLayout8x4& layout,
                             const thrust::device_vector<Offset>& residual_row_ptr,
                             const thrust::device_vector<Index>& residual_col_idx, int long_row_tau,
                             const thrust::device_vector<Index>& long_chunk_row,
                             const thrust::device_vector<Offset>& long_chunk_pbegin,
                             const thrust::device_vector<Index>& long_chunk_pcount,
                             const thrust::device_vector<T>& x, const thrust::device_vector<T>& y) {
    validate_bitbsr_8x4_shape(bitbsr);
    if (static_cast<Offset>(packed_meta.size()) != bitbsr.num_blocks) {
        throw std::runtime_error("fused CSR+BitBSR packed metadata size mismatch");
    }
    if (static_cast<Index>(layout.work_item_row_ptr.size()) != bitbsr.num_block_rows + 1) {
        throw std::runtime_error("fused CSR+BitBSR work_item_row_ptr size mismatch");
    }
    if (static_cast<Index>(y.size()) != bitbsr.rows) throw std::runtime_error("fused CSR+BitBSR output vector size mismatch");
    if (static_cast<Index>(x.size()) != bitbsr.cols) throw std::runtime_error("fused CSR+BitBSR input vector size mismatch");
    if (static_cast<Index>(residual_row_ptr.size()) != bitbsr.rows + 1) {
        throw std::runtime_error("fused CSR+BitBSR residual row_ptr size mismatch");
    }
    cove_hybrid_desc a{};
    a.rows = bitbsr.rows;
    a.cols = bitbsr.cols;
    a.num_block_rows = bitbsr.num_block_rows;
    a.dtype = cove_dtype_of<T>();
    a.kept_blocks = bitbsr.num_blocks;
    a.kept_nnz = bitbsr.nnz;
    a.residual_nnz = static_cast<int64_t>(residual_col_idx.size());
    a.block_row_ptr = raw(bitbsr.block_row_ptr);
    a.block_row_val_ptr = raw(bitbsr.block_row_val_ptr);
    a.words = raw(packed_meta);
    a.res_row_ptr = raw(residual_row_ptr);
    a.res_col_idx = raw(residual_col_idx);
    a.long_row_tau = long_row_tau;
    a.num_chunks = static_cast<int64_t>(long_chunk_row.size());
    a.chunk_row = raw(long_chunk_row);
    a.chunk_pbegin = raw(long_chunk_pbegin);
    a.chunk_pcount = raw(long_chunk_pcount);
    return a;
}

template <typename T>
void run_hybrid(const cove_hybrid_desc& a, const cove_values_desc& v, const thrust::device_vector<T>& x,
                thrust::device_vector<T>& y, float* iter_ms) {
    CudaEventTimer timer(iter_ms);
    cove_check(cove_hybrid_spmv(&a, &v, raw(x), raw(y), nullptr));
    finish(timer, iter_ms);
}

}  // namespace gpu_detail

template <typename T>
void run_csr_bitbsr_fused_8x4_lb(const DeviceBitBsrMatrix<T>& bitbsr,
                                 const thrust::device_vector<std::uint64_t>& packed_meta,
                                 const BitBsrLoadBalanceLayout8x4& layout,
                                 const thrust::device_vector<Offset>& residual_row_ptr,
                                 const thrust::device_vector<Index>& residual_col_idx,
                                 const thrust::device_vector<T>& residual_values, int long_row_tau,
                                 const thrust::device_vector<Index>& long_chunk_row,
                                 const thrust::device_vector<Offset>& long_chunk_pbegin,
                                 const thrust::device_vector<Index>& long_chunk_pcount,
                                 const thrust::device_vector<T>& x, thrust::device_vector<T>& y,
                                 float* iter_ms = nullptr) {
    const cove_hybrid_desc a = gpu_detail::hybrid_desc(bitbsr, packed_meta, layout, residual_row_ptr,
                                                       residual_col_idx, long_row_tau, long_chunk_row,
                                                       long_chunk_pbegin, long_chunk_pcount, x, y);
    cove_values_desc v{};
    v.route = COVE_ROUTE_HYBRID;
    v.kept = gpu_detail::raw(bitbsr.values);
    v.res = gpu_detail::raw(residual_values);
    gpu_detail::run_hybrid(a, v, x, y, iter_ms);
}

template <typename T>
void run_csr_bitbsr_fused_8x4_lb_bfp8(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<Offset>& residual_row_ptr,
    const thrust::device_vector<Index>& residual_col_idx, const thrust::device_vector<signed char>& blk_int8,
    const thrust::device_vector<std::uint16_t>& blk_scale_bf16,
    const thrust::device_vector<std::uint16_t>& residual_bf16, int long_row_tau,
    const thrust::device_vector<Index>& long_chunk_row, const thrust::device_vector<Offset>& long_chunk_pbegin,
    const thrust::device_vector<Index>& long_chunk_pcount, const thrust::device_vector<T>& x,
    thrust::device_vector<T>& y, float* iter_ms = nullptr) {
    const cove_hybrid_desc a = gpu_detail::hybrid_desc(bitbsr, packed_meta, layout, residual_row_ptr,
                                                       residual_col_idx, long_row_tau, long_chunk_row,
                                                       long_chunk_pbegin, long_chunk_pcount, x, y);
    cove_values_desc v{};
    v.route = COVE_ROUTE_BFP8;
    v.kept = gpu_detail::raw(blk_int8);
    v.block_scale = gpu_detail::raw(blk_scale_bf16);
    v.res = gpu_detail::raw(residual_bf16);
    gpu_detail::run_hybrid(a, v, x, y, iter_ms);
}

template <typename T, typename IdxT>
void run_csr_bitbsr_fused_8x4_lb_dict(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<Offset>& residual_row_ptr,
    const thrust::device_vector<Index>& residual_col_idx, const thrust::device_vector<IdxT>& blk_idx,
    const thrust::device_vector<T>& codebook, const thrust::device_vector<IdxT>& residual_idx,
    int long_row_tau, const thrust::device_vector<Index>& long_chunk_row,
    const thrust::device_vector<Offset>& long_chunk_pbegin,
    const thrust::device_vector<Index>& long_chunk_pcount, const thrust::device_vector<T>& x,
    thrust::device_vector<T>& y, float* iter_ms = nullptr) {
    static_assert(std::is_same_v<IdxT, std::uint8_t> || std::is_same_v<IdxT, std::uint16_t>,
                  "dictionary indices are uint8 or uint16");
    const cove_hybrid_desc a = gpu_detail::hybrid_desc(bitbsr, packed_meta, layout, residual_row_ptr,
                                                       residual_col_idx, long_row_tau, long_chunk_row,
                                                       long_chunk_pbegin, long_chunk_pcount, x, y);
    cove_values_desc v{};
    v.route = sizeof(IdxT) == 1 ? COVE_ROUTE_DICT_U8 : COVE_ROUTE_DICT_U16;
    v.kept = gpu_detail::raw(blk_idx);
    v.res = gpu_detail::raw(residual_idx);
    v.codebook = gpu_detail::raw(codebook);
    v.codebook_size = static_cast<int64_t>(codebook.size());
    gpu_detail::run_hybrid(a, v, x, y, iter_ms);
}

template <typename T>
void run_csr_bitbsr_fused_8x4_lb_bfp8_outlier(
    const DeviceBitBsrMatrix<T>& bitbsr, const thrust::device_vector<std::uint64_t>& packed_meta,
    const BitBsrLoadBalanceLayout8x4& layout, const thrust::device_vector<Offset>& residual_row_ptr,
    const thrust::device_vector<Index>& residual_col_idx, const thrust::device_vector<signed char>& blk_int8,
    const thrust::device_vector<std::uint16_t>& blk_scale_bf16,
    const thrust::device_vector<std::uint16_t>& residual_bf16,
    const thrust::device_vector<std::int32_t>& outlier_rows,
    const thrust::device_vector<std::int32_t>& outlier_cols, const thrust::device_vector<T>& outlier_vals,
    int long_row_tau, const thrust::device_vector<Index>& long_chunk_row,
    const thrust::device_vector<Offset>& long_chunk_pbegin,
    const thrust::device_vector<Index>& long_chunk_pcount, const thrust::device_vector<T>& x,
    thrust::device_vector<T>& y, float* iter_ms = nullptr) {
    const cove_hybrid_desc a = gpu_detail::hybrid_desc(bitbsr, packed_meta, layout, residual_row_ptr,
                                                       residual_col_idx, long_row_tau, long_chunk_row,
                                                       long_chunk_pbegin, long_chunk_pcount, x, y);
    cove_values_desc v{};
    v.route = COVE_ROUTE_BFP8_OUTLIER;
    v.kept = gpu_detail::raw(blk_int8);
    v.block_scale = gpu_detail::raw(blk_scale_bf16);
    v.res = gpu_detail::raw(residual_bf16);
    v.num_outliers = static_cast<int64_t>(outlier_vals.size());
    v.outlier_rows = gpu_detail::raw(outlier_rows);
    v.outlier_cols = gpu_detail::raw(outlier_cols);
    v.outlier_vals = gpu_detail::raw(outlier_vals);
    gpu_detail::run_hybrid(a, v, x, y, iter_ms);
}

namespace cove {

// RAII handle of the whole device pipeline (converter, split, layout, value
// codecs, gate and fall-back) for a host CSR.
template <typename T>
class Plan {
   public:
    explicit Plan(const CsrMatrix<T>& csr, const cove_plan_opts* opts = nullptr) {
        csr.validate();
        rp_ = csr.row_ptr;
        ci_ = csr.col_idx;
        v_ = csr.values;
        cove_csr_desc d{};
        d.rows = csr.rows;
        d.cols = csr.cols;
        d.nnz = csr.nnz();
        d.row_ptr = gpu_detail::raw(rp_);
        d.col_idx = gpu_detail::raw(ci_);
        d.values = gpu_detail::raw(v_);
        d.dtype = cove_dtype_of<T>();
        d.row_ptr_i32 = 1;
        cove_check(cove_plan_build(&d, opts, nullptr, &plan_));
        rp_.clear();
        ci_.clear();
        v_.clear();
        rp_.shrink_to_fit();
        ci_.shrink_to_fit();
        v_.shrink_to_fit();
        cove_check(cove_plan_get_info(plan_, &info_));
    }
    Plan(const Plan&) = delete;
    Plan& operator=(const Plan&) = delete;
    ~Plan() { cove_plan_destroy(plan_); }

    const cove_plan_info& info() const { return info_; }
    cove_plan* handle() const { return plan_; }

    // One of the plan's device streams (cove_stream_id) copied to the host
    // as V elements; an absent stream is an error.
    template <typename V>
    std::vector<V> stream(int which) const {
        size_t bytes = 0;
        cove_check(cove_plan_stream(plan_, which, nullptr, 0, &bytes, nullptr));
        if (bytes % sizeof(V) != 0) throw std::runtime_error("plan stream size is not a whole number of elements");
        std::vector<V> out(bytes / sizeof(V));
        if (bytes) cove_check(cove_plan_stream(plan_, which, out.data(), bytes, &bytes, nullptr));
        return out;
    }

    // y = A x on the dispatched route (or `route`), synchronous like the
    // reference wrappers; iter_ms as in their CudaEventTimer.
    void spmv(const thrust::device_vector<T>& x, thrust::device_vector<T>& y, int route = -1,
              float* iter_ms = nullptr) const {
        y.resize(info_.rows);
        gpu_detail::CudaEventTimer timer(iter_ms);
        if (route < 0) {
            cove_check(cove_spmv(plan_, gpu_detail::raw(x), gpu_detail::raw(y), nullptr));
        } else {
            cove_check(cove_spmv_route(plan_, route, gpu_detail::raw(x), gpu_detail::raw(y), nullptr));
        }
        gpu_detail::finish(timer, iter_ms);
    }

   private:
    cove_plan* plan_ = nullptr;
    cove_plan_info info_{};
    thrust::device_vector<Offset> rp_;
    thrust::device_vector<Index> ci_;
    thrust::device_vector<T> v_;
};

}  // namespace cove

}  // namespace structural
