// gpu_convert.cuh -- structural:: device BitBSR API over the B200 library.
//
// Same types and entry points as the reference's
// structural/include/structural/gpu_convert.cuh (DeviceBitBsrMatrix :251-351,
// copy_bitbsr_to_device :353-386, GpuBitBsrWorkspace :388-404,
// convert_to_bitbsr_gpu_warp_direct_8x4_device :495-512), implemented on the
// C ABI of libcove_b200.so (include/cove_b200.h).  Errors are thrown as
// std::runtime_error, as in the reference.
#pragma once

#include "cove_b200.h"
#include "structural/bitbsr.hpp"
#include "structural/csr.hpp"

#include <cuda_runtime.h>
#include <thrust/copy.h>
#include <thrust/device_vector.h>
#include <thrust/fill.h>

#include <sstream>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

namespace structural {

inline void cuda_check(cudaError_t status, const char* expr, const char* file, int line) {
    if (status != cudaSuccess) {
        std::ostringstream oss;
        oss << file << ':' << line << ": CUDA call failed: " << expr << ": "
            << cudaGetErrorString(status);
        throw std::runtime_error(oss.str());
    }
}

// Throws std::runtime_error with the library's message on a failing status.
inline void cove_check(cove_status status) {
    if (status != COVE_OK) throw std::runtime_error(cove_last_error());
}

template <typename T>
constexpr int32_t cove_dtype_of() {
    static_assert(std::is_same_v<T, double> || std::is_same_v<T, float>,
                  "structural operators support float and double");
    return std::is_same_v<T, double> ? COVE_F64 : COVE_F32;
}

namespace gpu_detail {

constexpr int kWarpDirectBlockRows = 8;
constexpr int kWarpDirect8x4BlockCols = 4;

// CUDA-event timer on the default stream (reference: gpu_convert.cuh:38-77).
class CudaEventTimer {
   public:
    explicit CudaEventTimer(float* elapsed_ms) : elapsed_ms_(elapsed_ms) {
        if (!elapsed_ms_) return;
        *elapsed_ms_ = 0.0f;
        cuda_check(cudaEventCreate(&start_), "cudaEventCreate", __FILE__, __LINE__);
        cuda_check(cudaEventCreate(&stop_), "cudaEventCreate", __FILE__, __LINE__);
        cuda_check(cudaEventRecord(start_), "cudaEventRecord", __FILE__, __LINE__);
    }
    CudaEventTimer(const CudaEventTimer&) = delete;
    CudaEventTimer& operator=(const CudaEventTimer&) = delete;
    ~CudaEventTimer() {
        if (start_) cudaEventDestroy(start_);
        if (stop_) cudaEventDestroy(stop_);
    }
    void stop() {
        if (!elapsed_ms_ || stopped_) return;
        cuda_check(cudaEventRecord(stop_), "cudaEventRecord", __FILE__, __LINE__);
        cuda_check(cudaEventSynchronize(stop_), "cudaEventSynchronize", __FILE__, __LINE__);
        cuda_check(cudaEventElapsedTime(elapsed_ms_, start_, stop_), "cudaEventElapsedTime",
                   __FILE__, __LINE__);
        stopped_ = true;
    }

   private:
    float* elapsed_ms_ = nullptr;
    cudaEvent_t start_ = nullptr;
    cudaEvent_t stop_ = nullptr;
    bool stopped_ = false;
};

template <typename V>
const V* raw(const thrust::device_vector<V>& v) {
    return v.empty() ? nullptr : thrust::raw_pointer_cast(v.data());
}
template <typename V>
V* raw(thrust::device_vector<V>& v) {
    return v.empty() ? nullptr : thrust::raw_pointer_cast(v.data());
}

// Finishes a synchronous call the way the reference's wrappers do: the
// timer if one was asked for, else a device synchronize.
inline void finish(CudaEventTimer& timer, float* ms) {
    if (ms) {
        timer.stop();
    } else {
        cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize()", __FILE__, __LINE__);
    }
}

}  // namespace gpu_detail

template <typename T>
struct DeviceBitBsrMatrix {
    Index rows = 0;
    Index cols = 0;
    Index block_rows = 0;
    Index block_cols = 0;
    Index num_block_rows = 0;
    Index num_block_cols = 0;
    Index words_per_block = 0;
    Offset num_blocks = 0;
    Offset nnz = 0;

    thrust::device_vector<Offset> block_row_ptr;
    thrust::device_vector<Offset> block_row_val_ptr;
    thrust::device_vector<Index> block_col_idx;
    thrust::device_vector<BitmapWord> bitmap_words;
    thrust::device_vector<T> values;

    void validate_shape() const {
        if (rows < 0 || cols < 0 || block_rows <= 0 || block_cols <= 0) {
            throw std::runtime_error("DeviceBitBSR dimensions or block sizes are invalid");
        }
        if (num_block_rows != ceil_div(rows, block_rows) || num_block_cols != ceil_div(cols, block_cols)) {
            throw std::runtime_error("DeviceBitBSR block-grid dimensions are inconsistent");
        }
        if (static_cast<Index>(block_row_ptr.size()) != num_block_rows + 1 ||
            static_cast<Index>(block_row_val_ptr.size()) != num_block_rows + 1) {
            throw std::runtime_error("DeviceBitBSR block-row pointer size is invalid");
        }
        if (static_cast<Offset>(block_col_idx.size()) != num_blocks ||
            bitmap_words.size() != static_cast<size_t>(num_blocks) * words_per_block ||
            static_cast<Offset>(values.size()) != nnz) {
            throw std::runtime_error("DeviceBitBSR stream sizes are invalid");
        }
    }

    // Host copy with block_val_ptr rebuilt from the bitmaps.
    BitBsrMatrix<T> to_host() const {
        validate_shape();
        BitBsrMatrix<T> out;
        out.rows = rows;
        out.cols = cols;
        out.block_rows = block_rows;
        out.block_cols = block_cols;
        out.num_block_rows = num_block_rows;
        out.num_block_cols = num_block_cols;
        out.words_per_block = words_per_block;
        out.block_row_ptr.resize(block_row_ptr.size());
        out.block_col_idx.resize(block_col_idx.size());
        out.bitmap_words.resize(bitmap_words.size());
        out.values.resize(values.size());
        thrust::copy(block_row_ptr.begin(), block_row_ptr.end(), out.block_row_ptr.begin());
        thrust::copy(block_col_idx.begin(), block_col_idx.end(), out.block_col_idx.begin());
        thrust::copy(bitmap_words.begin(), bitmap_words.end(), out.bitmap_words.begin());
        thrust::copy(values.begin(), values.end(), out.values.begin());
        out.block_val_ptr.assign(static_cast<size_t>(num_blocks) + 1, 0);
        for (Offset b = 0; b < num_blocks; ++b) {
            Offset bits = 0;
            for (Index w = 0; w < words_per_block; ++w) bits += popcount_word(out.bitmap_words[b * words_per_block + w]);
            out.block_val_ptr[b + 1] = out.block_val_ptr[b] + bits;
        }
        out.validate();
        return out;
    }
};

template <typename T>
void copy_bitbsr_to_device(const BitBsrMatrix<T>& host, DeviceBitBsrMatrix<T>& out) {
    host.validate();
    out.rows = host.rows;
    out.cols = host.cols;
    out.block_rows = host.block_rows;
    out.block_cols = host.block_cols;
    out.num_block_rows = host.num_block_rows;
    out.num_block_cols = host.num_block_cols;
    out.words_per_block = host.words_per_block;
    out.num_blocks = host.num_blocks();
    out.nnz = host.nnz();
    std::vector<Offset> brvp(static_cast<size_t>(host.num_block_rows) + 1);
    for (Index br = 0; br <= host.num_block_rows; ++br) brvp[br] = host.block_val_ptr[host.block_row_ptr[br]];
    out.block_row_ptr = host.block_row_ptr;
    out.block_row_val_ptr = brvp;
    out.block_col_idx = host.block_col_idx;
    out.bitmap_words = host.bitmap_words;
    out.values = host.values;
    out.validate_shape();
}

template <typename T>
DeviceBitBsrMatrix<T> copy_bitbsr_to_device(const BitBsrMatrix<T>& host) {
    DeviceBitBsrMatrix<T> out;
    copy_bitbsr_to_device(host, out);
    return out;
}

template <typename T>
struct GpuBitBsrWorkspace {
    thrust::device_vector<Offset> row_ptr;
    thrust::device_vector<Index> col_idx;
    thrust::device_vector<T> values;

    void upload_csr(const CsrMatrix<T>& csr) {
        row_ptr = csr.row_ptr;
        col_idx = csr.col_idx;
        values = csr.values;
    }
};

// CSR -> BitBSR 8x4 on the device (sm_100a converter; stored zeros dropped).
template <typename T>
void convert_to_bitbsr_gpu_warp_direct_8x4_device(const CsrMatrix<T>& csr,
                                                  GpuBitBsrWorkspace<T>& workspace,
                                                  DeviceBitBsrMatrix<T>& out,
                                                  float* device_ms = nullptr) {
    csr.validate();
    workspace.upload_csr(csr);
    out.rows = csr.rows;
    out.cols = csr.cols;
    out.block_rows = gpu_detail::kWarpDirectBlockRows;
    out.block_cols = gpu_detail::kWarpDirect8x4BlockCols;
    out.num_block_rows = ceil_div(csr.rows, out.block_rows);
    out.num_block_cols = ceil_div(csr.cols, out.block_cols);
    out.words_per_block = 1;
    out.block_row_ptr.assign(static_cast<size_t>(out.num_block_rows) + 1, 0);
    out.block_row_val_ptr.assign(static_cast<size_t>(out.num_block_rows) + 1, 0);
    cove_csr_desc d{};
    d.rows = csr.rows;
    d.cols = csr.cols;
    d.nnz = csr.nnz();
    d.row_ptr = gpu_detail::raw(workspace.row_ptr);
    d.col_idx = gpu_detail::raw(workspace.col_idx);
    d.values = gpu_detail::raw(workspace.values);
    d.dtype = cove_dtype_of<T>();
    d.row_ptr_i32 = 1;
    gpu_detail::CudaEventTimer timer(device_ms);
    int64_t nb = 0, nnz = 0;
    cove_check(cove_bitbsr8x4_count(&d, gpu_detail::raw(out.block_row_ptr),
                                    gpu_detail::raw(out.block_row_val_ptr), &nb, &nnz, nullptr));
    out.num_blocks = static_cast<Offset>(nb);
    out.nnz = static_cast<Offset>(nnz);
    out.block_col_idx.resize(out.num_blocks);
    out.bitmap_words.resize(out.num_blocks);
    out.values.resize(out.nnz);
    cove_check(cove_bitbsr8x4_fill(&d, gpu_detail::raw(out.block_row_ptr),
                                   gpu_detail::raw(out.block_row_val_ptr),
                                   gpu_detail::raw(out.block_col_idx), gpu_detail::raw(out.bitmap_words),
                                   gpu_detail::raw(out.values), nullptr));
    gpu_detail::finish(timer, device_ms);
    out.validate_shape();
}

template <typename T>
DeviceBitBsrMatrix<T> convert_to_bitbsr_gpu_warp_direct_8x4_device(const CsrMatrix<T>& csr,
                                                                   GpuBitBsrWorkspace<T>& workspace,
                                                                   float* device_ms = nullptr) {
    DeviceBitBsrMatrix<T> out;
    convert_to_bitbsr_gpu_warp_direct_8x4_device(csr, workspace, out, device_ms);
    return out;
}

}  // namespace structural
