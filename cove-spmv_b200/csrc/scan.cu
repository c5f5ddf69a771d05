// scan.cu -- offset scans and vector-compare reductions used while building plans.
//
// Three-pass exclusive scan: tile sums, one-CTA scan of the tile sums, tile
// scan plus offset.  Plan building is not on the timed SpMV path; the scans
// turn per-row / per-block counts into the reference's offset streams.
#include "cove_internal.cuh"

#include <cmath>

namespace cove {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename V>
__device__ V block_exclusive_sum(V v, V* total) {
    __shared__ V warp_sums[kScanThreads / 32];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    V incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const V t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        V w = lane < kScanThreads / 32 ? warp_sums[lane] : V(0);
        V wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const V t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < kScanThreads / 32) warp_sums[lane] = wi - w;
        if (lane == kScanThreads / 32 - 1) *total = wi;
    }
    __syncthreads();
    const V out = incl - v + warp_sums[warp];
    __syncthreads();
    return out;
}

template <typename TIn>
__global__ void tile_sum_kernel(const TIn* __restrict__ in, int64_t n, int64_t* __restrict__ sums) {
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
    int64_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + static_cast<int64_t>(k) * kScanThreads + threadIdx.x;
        if (i < n) s += static_cast<int64_t>(in[i]);
    }
    __shared__ int64_t tot;
    (void)block_exclusive_sum<int64_t>(s, &tot);
    if (threadIdx.x == 0) sums[blockIdx.x] = tot;
}

// One CTA: exclusive scan of `sums` in place, total into sums[m].
__global__ void scan_tile_sums_kernel(int64_t* __restrict__ sums, int64_t m) {
    __shared__ int64_t tot;
    int64_t carry = 0;
    for (int64_t base = 0; base < m; base += kScanThreads) {
        const int64_t i = base + threadIdx.x;
        const int64_t v = i < m ? sums[i] : 0;
        const int64_t ex = block_exclusive_sum<int64_t>(v, &tot);
        if (i < m) sums[i] = ex + carry;
        carry += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) sums[m] = carry;
}

template <typename TIn, typename TOut>
__global__ void tile_scan_kernel(const TIn* __restrict__ in, int64_t n,
                                 const int64_t* __restrict__ offsets, TOut* __restrict__ out) {
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
    // each thread owns kScanItems consecutive elements
    int64_t v[kScanItems];
    int64_t local = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
        v[k] = i < n ? static_cast<int64_t>(in[i]) : 0;
        local += v[k];
    }
    __shared__ int64_t tot;
    int64_t run = block_exclusive_sum<int64_t>(local, &tot) + offsets[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
        run += v[k];
        if (i < n) out[i + 1] = static_cast<TOut>(run);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) out[0] = TOut(0);
}

template <typename T>
__global__ void compare_kernel(const T* __restrict__ ref, const T* __restrict__ got, int64_t n,
                               unsigned long long* __restrict__ acc3) {
    double ma = 0.0, mr = 0.0, mref = 0.0;
    const T tiny = static_cast<T>(1e-30);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const T r = ref[i];
        const T ae = r - got[i] < T(0) ? got[i] - r : r - got[i];
        const T ar = r < T(0) ? -r : r;
        const T den = ar > tiny ? ar : tiny;
        const T rel = ae / den;
        // std::max(acc, v) keeps acc when v is NaN (spmv.hpp:82-85)
        if (static_cast<double>(ae) > ma) ma = static_cast<double>(ae);
        if (static_cast<double>(rel) > mr) mr = static_cast<double>(rel);
        if (static_cast<double>(ar) > mref) mref = static_cast<double>(ar);
    }
    for (int o = 16; o > 0; o >>= 1) {
        ma = fmax(ma, __shfl_down_sync(0xffffffffu, ma, o));
        mr = fmax(mr, __shfl_down_sync(0xffffffffu, mr, o));
        mref = fmax(mref, __shfl_down_sync(0xffffffffu, mref, o));
    }
    if ((threadIdx.x & 31) == 0) {
        // non-negative doubles order like their bit patterns
        atomicMax(&acc3[0], static_cast<unsigned long long>(__double_as_longlong(ma)));
        atomicMax(&acc3[1], static_cast<unsigned long long>(__double_as_longlong(mr)));
        atomicMax(&acc3[2], static_cast<unsigned long long>(__double_as_longlong(mref)));
    }
}

}  // namespace

template <typename TIn, typename TOut>
int64_t exclusive_scan_total(const TIn* in, TOut* out, int64_t n, cudaStream_t s) {
    const int64_t tiles = n > 0 ? (n + kScanTile - 1) / kScanTile : 0;
    DevBuf sums;
    sums.alloc(static_cast<size_t>(tiles + 1) * sizeof(int64_t));
    if (tiles > 0) {
        tile_sum_kernel<TIn><<<static_cast<unsigned>(tiles), kScanThreads, 0, s>>>(
            in, n, sums.as<int64_t>());
        CUDA_LAUNCH_OK();
    }
    scan_tile_sums_kernel<<<1, kScanThreads, 0, s>>>(sums.as<int64_t>(), tiles);
    CUDA_LAUNCH_OK();
    if (tiles > 0) {
        tile_scan_kernel<TIn, TOut><<<static_cast<unsigned>(tiles), kScanThreads, 0, s>>>(
            in, n, sums.as<int64_t>(), out);
        CUDA_LAUNCH_OK();
    } else {
        CUDA_OK(cudaMemsetAsync(out, 0, sizeof(TOut), s));
    }
    int64_t total = 0;
    CUDA_OK(cudaMemcpyAsync(&total, sums.as<int64_t>() + tiles, sizeof(int64_t),
                            cudaMemcpyDeviceToHost, s));
    CUDA_OK(cudaStreamSynchronize(s));
    return total;
}

template int64_t exclusive_scan_total<int32_t, int32_t>(const int32_t*, int32_t*, int64_t, cudaStream_t);
template int64_t exclusive_scan_total<int32_t, int64_t>(const int32_t*, int64_t*, int64_t, cudaStream_t);
template int64_t exclusive_scan_total<int64_t, int64_t>(const int64_t*, int64_t*, int64_t, cudaStream_t);
template int64_t exclusive_scan_total<uint8_t, int32_t>(const uint8_t*, int32_t*, int64_t, cudaStream_t);

template <typename T>
void compare_reduce(const T* ref, const T* got, int64_t n, double* out3, cudaStream_t s) {
    DevBuf acc;
    acc.alloc(3 * sizeof(unsigned long long));
    CUDA_OK(cudaMemsetAsync(acc.p, 0, 3 * sizeof(unsigned long long), s));
    if (n > 0) {
        const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
        compare_kernel<T><<<grid, 256, 0, s>>>(ref, got, n, acc.as<unsigned long long>());
        CUDA_LAUNCH_OK();
    }
    unsigned long long h[3];
    CUDA_OK(cudaMemcpyAsync(h, acc.p, sizeof(h), cudaMemcpyDeviceToHost, s));
    CUDA_OK(cudaStreamSynchronize(s));
    double ma, mr, mref;
    std::memcpy(&ma, &h[0], 8);
    std::memcpy(&mr, &h[1], 8);
    std::memcpy(&mref, &h[2], 8);
    // global_rel = max_abs / max(max|ref|, 1e-30), computed in T (spmv.hpp:87)
    const T tiny = static_cast<T>(1e-30);
    const T den = static_cast<T>(mref) > tiny ? static_cast<T>(mref) : tiny;
    out3[0] = ma;
    out3[1] = mr;
    out3[2] = static_cast<double>(static_cast<T>(ma) / den);
}

template void compare_reduce<double>(const double*, const double*, int64_t, double*, cudaStream_t);
template void compare_reduce<float>(const float*, const float*, int64_t, double*, cudaStream_t);

}  // namespace cove
