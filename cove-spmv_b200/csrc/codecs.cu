// codecs.cu -- device encoders of the joint value streams.
//
//   BFP8 (int8 x per-block bf16 scale)   gpu_value_codecs.cuh:287-317
//   BFP8 + global outliers               gpu_value_codecs.cuh:360-461
//   bf16 residual (round half up)        main_gpu_csr_bitbsr_spmv.cu:1302-1306
//   exact dictionary (first occurrence)  main_gpu_csr_bitbsr_spmv.cu:1224-1258
//
// Each encoder reproduces the reference's host encoder byte for byte.  The
// outlier threshold -- the idx-th smallest |v| that the reference takes with
// std::nth_element -- is found by an 8-pass radix select over the bit
// patterns of |v| (non-negative doubles order like their bits).  The
// dictionary is built with a bounded open-addressing table in device memory
// that records each distinct value's first index; the codebook order is the
// order of those first indices.
#include "cove_codecs.cuh"

#include <algorithm>
#include <climits>
#include <cmath>

namespace cove {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float v) {
    // float_to_bf16_bits, value_compression.hpp:105-109
    const uint32_t bits = __float_as_uint(v);
    const uint32_t lsb = (bits >> 16) & 1u;
    return static_cast<uint16_t>((bits + 0x7fffu + lsb) >> 16);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// std::lround as glibc on x86-64 computes it: nearest integer with halves
// away from zero; NaN and out-of-range give LONG_MIN.
__device__ __forceinline__ long long lround_host(double q) {
    if (!(fabs(q) < 9.2e18)) return LLONG_MIN;
    double t = trunc(q);
    const double f = q - t;  // exact
    if (f >= 0.5) t += 1.0;
    if (f <= -0.5) t -= 1.0;
    return static_cast<long long>(t);
}

template <typename T>
__global__ void bfp8_kernel(int64_t nb, const int32_t* __restrict__ bvp,
                            const T* __restrict__ vals, const uint8_t* __restrict__ is_out,
                            int8_t* __restrict__ q, uint16_t* __restrict__ scale) {
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    const int k0 = bvp[b], k1 = bvp[b + 1];
    double mx = 0.0;
    for (int k = k0; k < k1; ++k) {
        if (is_out && is_out[k]) continue;
        const double a = fabs(static_cast<double>(vals[k]));
        if (a > mx) mx = a;
    }
    float sc = __double2float_rn(__ddiv_rn(mx, 127.0));
    if (sc == 0.0f) sc = 1.0f;
    const uint16_t sb = f32_to_bf16_rne(sc);
    scale[b] = sb;
    const double dec = static_cast<double>(bf16_to_f32(sb));
    for (int k = k0; k < k1; ++k) {
        if (is_out && is_out[k]) {
            q[k] = 0;
            continue;
        }
        long long l = lround_host(__ddiv_rn(static_cast<double>(vals[k]), dec));
        l = l > 127 ? 127 : (l < -127 ? -127 : l);
        q[k] = static_cast<int8_t>(l);
    }
}

template <typename T>
__device__ __forceinline__ uint64_t abs_key(T v) {
    return static_cast<uint64_t>(__double_as_longlong(fabs(static_cast<double>(v))));
}

template <typename T>
__global__ void radix_hist_kernel(int64_t n, const T* __restrict__ vals, uint64_t prefix,
                                  uint64_t mask, int shift,
                                  unsigned long long* __restrict__ hist) {
    __shared__ unsigned int sh[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sh[i] = 0;
    __syncthreads();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint64_t key = abs_key(vals[i]);
        if ((key & mask) == prefix) atomicAdd(&sh[(key >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        if (sh[i]) atomicAdd(&hist[i], static_cast<unsigned long long>(sh[i]));
    }
}

template <typename T>
__global__ void outlier_flag_kernel(int64_t n, const T* __restrict__ vals, double thr,
                                    uint8_t* __restrict__ flag) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) flag[i] = fabs(static_cast<double>(vals[i])) > thr ? 1 : 0;
}

template <typename T>
__global__ void outlier_list_kernel(int64_t nb, int32_t nbr, const int32_t* __restrict__ brp,
                                    const int32_t* __restrict__ bvp,
                                    const int32_t* __restrict__ col,
                                    const uint32_t* __restrict__ bitmap,
                                    const T* __restrict__ vals, const uint8_t* __restrict__ flag,
                                    const int32_t* __restrict__ pos, int32_t* __restrict__ orow,
                                    int32_t* __restrict__ ocol, T* __restrict__ oval) {
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    // block row of block b: last br with brp[br] <= b
    int lo = 0, hi = nbr;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (brp[mid] <= b) lo = mid; else hi = mid - 1;
    }
    const int br = lo;
    const uint32_t bm = bitmap[b];
    int k = bvp[b];
    for (int bit = 0; bit < 32; ++bit) {
        if (!(bm & (1u << bit))) continue;
        if (flag[k]) {
            const int p = pos[k];
            orow[p] = br * kBlockRows + bit / kBlockCols;
            ocol[p] = col[b] * kBlockCols + bit % kBlockCols;
            oval[p] = vals[k];
        }
        ++k;
    }
}

template <typename T>
__global__ void bf16_half_up_kernel(int64_t n, const T* __restrict__ v, uint16_t* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) {
        const uint32_t u = __float_as_uint(static_cast<float>(v[i]));
        out[i] = static_cast<uint16_t>((u + 0x8000u) >> 16);
    }
}

// ---- exact dictionary ------------------------------------------------------

constexpr int kTableLog2 = 18;
constexpr uint64_t kTableSize = uint64_t{1} << kTableLog2;
constexpr uint32_t kDictLimit = 65536;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

template <typename T>
__device__ __forceinline__ uint64_t value_key(T v) {
    if constexpr (sizeof(T) == 8) {
        return static_cast<uint64_t>(__double_as_longlong(v));
    } else {
        return static_cast<uint64_t>(__float_as_uint(v));
    }
}

template <typename T>
__global__ void dict_insert_kernel(int64_t nk, int64_t n, const T* __restrict__ kept,
                                   const T* __restrict__ res,
                                   unsigned long long* __restrict__ keys,
                                   unsigned int* __restrict__ first,
                                   unsigned int* __restrict__ count,
                                   volatile int* __restrict__ overflow) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool valid = i < n && !*overflow;
    const uint64_t key = valid ? value_key(i < nk ? kept[i] : res[i - nk]) : 0ULL;
    // Matrices with few distinct values would funnel every thread into the
    // same slots: lanes holding equal keys elect their lowest lane, which
    // also holds the group's smallest index, and only it touches the table.
    const unsigned act = __ballot_sync(0xffffffffu, valid);
    if (!valid) return;
    const unsigned peers = __match_any_sync(act, static_cast<unsigned long long>(key));
    if (static_cast<int>(threadIdx.x & 31) != __ffs(peers) - 1) return;
    const unsigned int idx = static_cast<unsigned int>(i);
    uint64_t h = mix64(key) & (kTableSize - 1);
    for (uint64_t probe = 0; probe < kTableSize; ++probe) {
        const unsigned long long cur = keys[h];
        if (cur == key) {
            if (first[h] > idx) atomicMin(&first[h], idx);  // a stale read only costs an atomic
            return;
        }
        if (cur == 0ULL) {
            // past the limit the answer is "too many values": stop claiming slots,
            // or the threads in flight would fill the table and probe all of it
            if (*overflow) return;
            const unsigned long long prev = atomicCAS(&keys[h], 0ULL, static_cast<unsigned long long>(key));
            if (prev == 0ULL) {
                const unsigned int c = atomicAdd(count, 1u);
                if (c >= kDictLimit) *overflow = 1;
                atomicMin(&first[h], idx);
                return;
            }
            if (prev == key) {
                if (first[h] > idx) atomicMin(&first[h], idx);
                return;
            }
        }
        if ((probe & 63) == 63 && *overflow) return;
        h = (h + 1) & (kTableSize - 1);
    }
    *overflow = 1;
}

__global__ void dict_compact_kernel(const unsigned long long* __restrict__ keys,
                                    const unsigned int* __restrict__ first,
                                    unsigned int* __restrict__ n_out,
                                    unsigned long long* __restrict__ out_keys,
                                    unsigned int* __restrict__ out_first,
                                    unsigned int* __restrict__ out_slot) {
    const uint64_t s = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (s >= kTableSize || keys[s] == 0ULL) return;
    const unsigned int o = atomicAdd(n_out, 1u);
    out_keys[o] = keys[s];
    out_first[o] = first[s];
    out_slot[o] = static_cast<unsigned int>(s);
}

__global__ void dict_slot_code_kernel(int64_t n, const unsigned int* __restrict__ slot,
                                      const unsigned int* __restrict__ code,
                                      unsigned int* __restrict__ code_of_slot) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) code_of_slot[slot[i]] = code[i];
}

template <typename T, typename IdxT>
__global__ void dict_encode_kernel(int64_t n, const T* __restrict__ v,
                                   const unsigned long long* __restrict__ keys,
                                   const unsigned int* __restrict__ code_of_slot,
                                   IdxT* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t key = value_key(v[i]);
    uint64_t h = mix64(key) & (kTableSize - 1);
    for (uint64_t probe = 0; probe < kTableSize; ++probe) {
        if (keys[h] == key) {
            out[i] = static_cast<IdxT>(code_of_slot[h]);
            return;
        }
        h = (h + 1) & (kTableSize - 1);
    }
}

}  // namespace

template <typename T>
void encode_bfp8(const SplitParts& sp, const uint8_t* is_out, DevBuf& q, DevBuf& scale,
                 cudaStream_t s) {
    alloc_n<int8_t>(q, sp.kept_nnz);
    alloc_n<uint16_t>(scale, sp.kept_blocks);
    if (sp.kept_blocks == 0) return;
    bfp8_kernel<T><<<grid_for(sp.kept_blocks, kThreads), kThreads, 0, s>>>(
        sp.kept_blocks, sp.kept_block_val_ptr.as<int32_t>(), sp.kept_values.as<T>(), is_out,
        q.as<int8_t>(), scale.as<uint16_t>());
    CUDA_LAUNCH_OK();
}

template <typename T>
double select_abs_order_statistic(const T* vals, int64_t n, int64_t idx, cudaStream_t s) {
    DevBuf hist;
    alloc_n<unsigned long long>(hist, 256);
    uint64_t prefix = 0, mask = 0;
    int64_t k = idx;
    const int grid = static_cast<int>(std::min<int64_t>(grid_for(n, kThreads), 148 * 8));
    for (int shift = 56; shift >= 0; shift -= 8) {
        CUDA_OK(cudaMemsetAsync(hist.p, 0, 256 * sizeof(unsigned long long), s));
        radix_hist_kernel<T><<<grid, kThreads, 0, s>>>(n, vals, prefix, mask, shift,
                                                       hist.as<unsigned long long>());
        CUDA_LAUNCH_OK();
        unsigned long long h[256];
        CUDA_OK(cudaMemcpyAsync(h, hist.p, sizeof(h), cudaMemcpyDeviceToHost, s));
        CUDA_OK(cudaStreamSynchronize(s));
        int digit = 0;
        for (; digit < 256; ++digit) {
            if (k < static_cast<int64_t>(h[digit])) break;
            k -= static_cast<int64_t>(h[digit]);
        }
        if (digit == 256) COVE_THROW(COVE_ERR_INVALID_INPUT, "order statistic out of range");
        prefix |= static_cast<uint64_t>(digit) << shift;
        mask |= uint64_t{0xFF} << shift;
    }
    double thr;
    std::memcpy(&thr, &prefix, sizeof(thr));
    return thr;
}

template <typename T>
void encode_bfp8_outlier(const SplitParts& sp, int32_t nbr, double fraction, DevBuf& q,
                         DevBuf& scale, DevBuf& orow, DevBuf& ocol, DevBuf& oval,
                         int64_t* num_out, double* threshold, cudaStream_t s) {
    const int64_t nnz = sp.kept_nnz;
    DevBuf flag;
    alloc_n<uint8_t>(flag, nnz);
    CUDA_OK(cudaMemsetAsync(flag.p, 0, flag.bytes, s));
    double thr = 0.0;
    if (fraction > 0.0 && nnz > 0) {
        // size_t((1.0 - P) * nnz), clamped (gpu_value_codecs.cuh:384-388)
        size_t idx = static_cast<size_t>((1.0 - fraction) * static_cast<double>(nnz));
        if (idx >= static_cast<size_t>(nnz)) idx = static_cast<size_t>(nnz) - 1;
        thr = select_abs_order_statistic<T>(sp.kept_values.as<T>(), nnz, static_cast<int64_t>(idx), s);
        outlier_flag_kernel<T><<<grid_for(nnz, kThreads), kThreads, 0, s>>>(
            nnz, sp.kept_values.as<T>(), thr, flag.as<uint8_t>());
        CUDA_LAUNCH_OK();
    }
    *threshold = thr;
    encode_bfp8<T>(sp, flag.as<uint8_t>(), q, scale, s);
    DevBuf pos;
    alloc_n<int32_t>(pos, nnz + 1);
    *num_out = exclusive_scan_total<uint8_t, int32_t>(flag.as<uint8_t>(), pos.as<int32_t>(), nnz, s);
    alloc_n<int32_t>(orow, *num_out);
    alloc_n<int32_t>(ocol, *num_out);
    alloc_n<T>(oval, *num_out);
    if (*num_out > 0 && sp.kept_blocks > 0) {
        outlier_list_kernel<T><<<grid_for(sp.kept_blocks, kThreads), kThreads, 0, s>>>(
            sp.kept_blocks, nbr, sp.kept_block_row_ptr.as<int32_t>(),
            sp.kept_block_val_ptr.as<int32_t>(), sp.kept_col.as<int32_t>(),
            sp.kept_bitmap.as<uint32_t>(), sp.kept_values.as<T>(), flag.as<uint8_t>(),
            pos.as<int32_t>(), orow.as<int32_t>(), ocol.as<int32_t>(), oval.as<T>());
        CUDA_LAUNCH_OK();
    }
}

template <typename T>
void encode_res_bf16(const SplitParts& sp, DevBuf& out, cudaStream_t s) {
    alloc_n<uint16_t>(out, sp.residual_nnz);
    if (sp.residual_nnz == 0) return;
    bf16_half_up_kernel<T><<<grid_for(sp.residual_nnz, kThreads), kThreads, 0, s>>>(
        sp.residual_nnz, sp.res_values.as<T>(), out.as<uint16_t>());
    CUDA_LAUNCH_OK();
}

template <typename T>
int64_t encode_dict(const SplitParts& sp, bool build_codes, DictStreams& out, cudaStream_t s) {
    const int64_t nk = sp.kept_nnz, nr = sp.residual_nnz, n = nk + nr;
    if (n > static_cast<int64_t>(UINT_MAX)) {
        COVE_THROW(COVE_ERR_OVERFLOW, "dictionary interning index exceeds 32 bits");
    }
    DevBuf keys, first, count, overflow;
    alloc_n<unsigned long long>(keys, kTableSize);
    alloc_n<unsigned int>(first, kTableSize);
    alloc_n<unsigned int>(count, 1);
    alloc_n<int>(overflow, 1);
    CUDA_OK(cudaMemsetAsync(keys.p, 0, kTableSize * 8, s));
    CUDA_OK(cudaMemsetAsync(first.p, 0xFF, kTableSize * 4, s));
    CUDA_OK(cudaMemsetAsync(count.p, 0, 4, s));
    CUDA_OK(cudaMemsetAsync(overflow.p, 0, 4, s));
    if (n > 0) {
        dict_insert_kernel<T><<<grid_for(n, kThreads), kThreads, 0, s>>>(
            nk, n, sp.kept_values.as<T>(), sp.res_values.as<T>(), keys.as<unsigned long long>(),
            first.as<unsigned int>(), count.as<unsigned int>(), overflow.as<int>());
        CUDA_LAUNCH_OK();
    }
    unsigned int hcount = 0;
    int hover = 0;
    CUDA_OK(cudaMemcpyAsync(&hcount, count.p, 4, cudaMemcpyDeviceToHost, s));
    CUDA_OK(cudaMemcpyAsync(&hover, overflow.p, 4, cudaMemcpyDeviceToHost, s));
    CUDA_OK(cudaStreamSynchronize(s));
    if (hover || hcount > kDictLimit) {
        out.uniq = -1;  // more than 65536 distinct values
        return -1;
    }
    out.uniq = hcount;
    if (!build_codes) return out.uniq;

    // codebook order = order of first occurrence
    DevBuf n_out, ok, of, os;
    alloc_n<unsigned int>(n_out, 1);
    alloc_n<unsigned long long>(ok, hcount);
    alloc_n<unsigned int>(of, hcount);
    alloc_n<unsigned int>(os, hcount);
    CUDA_OK(cudaMemsetAsync(n_out.p, 0, 4, s));
    dict_compact_kernel<<<grid_for(static_cast<int64_t>(kTableSize), kThreads), kThreads, 0, s>>>(
        keys.as<unsigned long long>(), first.as<unsigned int>(), n_out.as<unsigned int>(),
        ok.as<unsigned long long>(), of.as<unsigned int>(), os.as<unsigned int>());
    CUDA_LAUNCH_OK();
    std::vector<unsigned long long> hk(hcount);
    std::vector<unsigned int> hf(hcount), hs(hcount);
    if (hcount > 0) {
        CUDA_OK(cudaMemcpyAsync(hk.data(), ok.p, hcount * 8ULL, cudaMemcpyDeviceToHost, s));
        CUDA_OK(cudaMemcpyAsync(hf.data(), of.p, hcount * 4ULL, cudaMemcpyDeviceToHost, s));
        CUDA_OK(cudaMemcpyAsync(hs.data(), os.p, hcount * 4ULL, cudaMemcpyDeviceToHost, s));
    }
    CUDA_OK(cudaStreamSynchronize(s));
    std::vector<unsigned int> order(hcount);
    for (unsigned int i = 0; i < hcount; ++i) order[i] = i;
    std::sort(order.begin(), order.end(), [&](unsigned a, unsigned b) { return hf[a] < hf[b]; });
    std::vector<T> codebook(hcount);
    std::vector<unsigned int> slot(hcount), code(hcount);
    for (unsigned int c = 0; c < hcount; ++c) {
        const unsigned int e = order[c];
        const unsigned long long key = hk[e];
        std::memcpy(&codebook[c], &key, sizeof(T));
        slot[c] = hs[e];
        code[c] = c;
    }
    alloc_n<T>(out.codebook, hcount);
    DevBuf dslot, dcode, cos;
    alloc_n<unsigned int>(dslot, hcount);
    alloc_n<unsigned int>(dcode, hcount);
    alloc_n<unsigned int>(cos, kTableSize);
    if (hcount > 0) {
        CUDA_OK(cudaMemcpyAsync(out.codebook.p, codebook.data(), hcount * sizeof(T),
                                cudaMemcpyHostToDevice, s));
        CUDA_OK(cudaMemcpyAsync(dslot.p, slot.data(), hcount * 4ULL, cudaMemcpyHostToDevice, s));
        CUDA_OK(cudaMemcpyAsync(dcode.p, code.data(), hcount * 4ULL, cudaMemcpyHostToDevice, s));
        dict_slot_code_kernel<<<grid_for(hcount, kThreads), kThreads, 0, s>>>(
            hcount, dslot.as<unsigned int>(), dcode.as<unsigned int>(), cos.as<unsigned int>());
        CUDA_LAUNCH_OK();
    }
    out.bits = hcount <= 256 ? 8 : 16;
    const size_t isz = out.bits == 8 ? 1 : 2;
    out.kept_idx.alloc(static_cast<size_t>(nk) * isz);
    out.res_idx.alloc(static_cast<size_t>(nr) * isz);
    CUDA_OK(cudaMemsetAsync(out.kept_idx.p, 0, out.kept_idx.bytes, s));
    CUDA_OK(cudaMemsetAsync(out.res_idx.p, 0, out.res_idx.bytes, s));
    if (out.bits == 8) {
        if (nk > 0)
            dict_encode_kernel<T, uint8_t><<<grid_for(nk, kThreads), kThreads, 0, s>>>(
                nk, sp.kept_values.as<T>(), keys.as<unsigned long long>(), cos.as<unsigned int>(),
                out.kept_idx.as<uint8_t>());
        if (nr > 0)
            dict_encode_kernel<T, uint8_t><<<grid_for(nr, kThreads), kThreads, 0, s>>>(
                nr, sp.res_values.as<T>(), keys.as<unsigned long long>(), cos.as<unsigned int>(),
                out.res_idx.as<uint8_t>());
    } else {
        if (nk > 0)
            dict_encode_kernel<T, uint16_t><<<grid_for(nk, kThreads), kThreads, 0, s>>>(
                nk, sp.kept_values.as<T>(), keys.as<unsigned long long>(), cos.as<unsigned int>(),
                out.kept_idx.as<uint16_t>());
        if (nr > 0)
            dict_encode_kernel<T, uint16_t><<<grid_for(nr, kThreads), kThreads, 0, s>>>(
                nr, sp.res_values.as<T>(), keys.as<unsigned long long>(), cos.as<unsigned int>(),
                out.res_idx.as<uint16_t>());
    }
    CUDA_LAUNCH_OK();
    CUDA_OK(cudaStreamSynchronize(s));
    return out.uniq;
}

template void encode_bfp8<double>(const SplitParts&, const uint8_t*, DevBuf&, DevBuf&, cudaStream_t);
template void encode_bfp8<float>(const SplitParts&, const uint8_t*, DevBuf&, DevBuf&, cudaStream_t);
template void encode_bfp8_outlier<double>(const SplitParts&, int32_t, double, DevBuf&, DevBuf&, DevBuf&,
                                          DevBuf&, DevBuf&, int64_t*, double*, cudaStream_t);
template void encode_bfp8_outlier<float>(const SplitParts&, int32_t, double, DevBuf&, DevBuf&, DevBuf&,
                                         DevBuf&, DevBuf&, int64_t*, double*, cudaStream_t);
template void encode_res_bf16<double>(const SplitParts&, DevBuf&, cudaStream_t);
template void encode_res_bf16<float>(const SplitParts&, DevBuf&, cudaStream_t);
template int64_t encode_dict<double>(const SplitParts&, bool, DictStreams&, cudaStream_t);
template int64_t encode_dict<float>(const SplitParts&, bool, DictStreams&, cudaStream_t);

}  // namespace cove
