// cove_internal.cuh -- shared host/device pieces of the B200 COVE library.
#pragma once

#include "cove_b200.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace cove {

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------

struct Error {
    cove_status status;
    std::string message;
};

void set_last_error(const std::string& msg);

#define COVE_THROW(st, msg) throw ::cove::Error{(st), (msg)}

inline void cuda_ok(cudaError_t e, const char* expr, const char* file, int line) {
    if (e != cudaSuccess) {
        std::string m = std::string(file) + ":" + std::to_string(line) +
                        ": CUDA call failed: " + expr + ": " + cudaGetErrorString(e);
        if (e == cudaErrorMemoryAllocation) COVE_THROW(COVE_ERR_OUT_OF_MEMORY, m);
        COVE_THROW(COVE_ERR_CUDA, m);
    }
}
#define CUDA_OK(expr) ::cove::cuda_ok((expr), #expr, __FILE__, __LINE__)
#define CUDA_LAUNCH_OK() ::cove::cuda_ok(cudaGetLastError(), "kernel launch", __FILE__, __LINE__)

// Runs fn, converting exceptions to a status and the thread's last error.
template <typename F>
cove_status guarded(F&& fn) {
    try {
        fn();
        set_last_error("");
        return COVE_OK;
    } catch (const Error& e) {
        set_last_error(e.message);
        return e.status;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return COVE_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return COVE_ERR_INVALID_ARGUMENT;
    }
}

// ---------------------------------------------------------------------------
// device buffer (owning)
// ---------------------------------------------------------------------------

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) {
            release();
            p = o.p;
            bytes = o.bytes;
            o.p = nullptr;
            o.bytes = 0;
        }
        return *this;
    }
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    // Every buffer carries kTailSlack readable bytes past its logical end, so
    // 16-byte-rounded bulk copies of a stream's last range stay in bounds.
    static constexpr size_t kTailSlack = 64;
    void alloc(size_t n) {
        release();
        CUDA_OK(cudaMalloc(&p, n + kTailSlack));
        bytes = n;
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

template <typename T>
inline void alloc_n(DevBuf& b, int64_t n) { b.alloc(static_cast<size_t>(n) * sizeof(T)); }

// ---------------------------------------------------------------------------
// constants of the 8x4 format
// ---------------------------------------------------------------------------

constexpr int kBlockRows = 8;
constexpr int kBlockCols = 4;
constexpr uint64_t kFlagBit = uint64_t{1} << 31;       // common.cuh:57-58
constexpr uint64_t kColMask = 0x7fffffffULL;             // common.cuh:59
constexpr int kLongChunkNnz = 1024;                      // main_gpu_csr_bitbsr_spmv.cu:1160

struct WorkItem {  // BitBsrWorkItem8x4, common.cuh:15-22
    uint32_t br, block_begin, block_count, value_begin;
};
static_assert(sizeof(WorkItem) == 16, "work item is 16 bytes");

__host__ __device__ inline uint64_t pack_word(uint32_t col, uint32_t bitmap, bool flag) {
    return (static_cast<uint64_t>(bitmap) << 32) | (static_cast<uint64_t>(col) & kColMask) |
           (flag ? kFlagBit : 0ULL);
}

inline int grid_for(int64_t n, int per) { return static_cast<int>((n + per - 1) / per); }

// ---------------------------------------------------------------------------
// scans (scan.cu)
// ---------------------------------------------------------------------------

// out[0] = 0, out[i+1] = out[i] + in[i]; out has n+1 entries.  Returns the
// total (synchronizes the stream).  TIn in {int32, int64}; TOut in {int32, int64}.
template <typename TIn, typename TOut>
int64_t exclusive_scan_total(const TIn* in, TOut* out, int64_t n, cudaStream_t s);

// Device-side: grid-wide max of |a-b| and of |a| (T) for compare_vectors.
template <typename T>
void compare_reduce(const T* ref, const T* got, int64_t n, double* out3, cudaStream_t s);

}  // namespace cove
