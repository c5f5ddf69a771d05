// spmv.cu -- fused load-balanced CSR+BitBSR SpMV for sm_100a.
//
// One launch computes y = A x over the kept 8x4 bit blocks and the CSR
// residual.  It replaces the reference's unified kernels
// (structural/src/main_gpu_csr_bitbsr_spmv.cu:517-634 lossless,
// :755-860 joint/quantized) and the outlier correction (:967-979).
//
// Work split (the plan picks one main-pass kernel from the matrix's shape):
//  - hybrid_main_kernel: one group of 8*SLOTS lanes owns one block row.  The
//    group loads G block words with one coalesced load, scans their
//    popcounts for the value bases and hands the blocks to the slots by
//    shuffle; lane (s, r) handles local row r of every SLOTS-th block: the
//    four cells of a row segment are contiguous in the value stream (bit
//    order is row-major) and the four x values are contiguous (two 16-byte
//    loads).  The SLOTS lanes of a row then stride its residual entries and
//    the slots are reduced with xor-shuffles.
//  - hybrid_row_kernel: a lane owns whole rows (two of them) for matrices
//    with few kept blocks per block row and short residual rows.
//  - bfp8_block_lane_kernel: a lane owns a block, for the BFP8 routes of
//    block-dense matrices.
//  - bfp8_segment_kernel: a lane owns a block, for the BFP8 routes of block
//    rows of many 32-block batches (next batch's words loaded ahead, cells
//    decoded a row segment at a time by byte permutes).
// Each row is stored once: no atomics, no zero-fill, deterministic.
//
// Block rows with more than `heavy_limit` kept blocks and residual rows
// longer than `long_tau` are finished by a second launch (one warp per
// piece / 1024-nnz chunk, atomicAdd into y), which also applies the exact
// BFP8 outlier side list.  Matrices without such rows need one launch.
//
// Accumulation: lossless routes accumulate in double; the BFP8 and bf16
// routes accumulate in fp32 with x cast to float, as the reference's joint
// kernel does (:795, :811).
#include "cove_spmv.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

namespace cove {
namespace {

constexpr int kThreads = 128;  // measured best for the main passes (64-512 tried)

// The kernels' dynamic shared memory (a shared codebook).  Decoders index it
// through this name, so the compiler emits shared-memory loads; a generic
// pointer to it would cost generic loads on every lookup.
extern __shared__ __align__(16) unsigned char g_smem[];

__device__ __forceinline__ float bf16_to_float(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// float(q) for |q| < 2^22 with an integer add and a float subtract instead of
// the int -> float conversion unit (its throughput bounds the BFP decoders):
// adding q to the bit pattern of 1.5 * 2^23 adds q to its value, exactly.
__device__ __forceinline__ float small_int_to_float(int q) {
    return __int_as_float(0x4B400000 + q) - 12582912.0f;
}

// The four x values of a block column, as the accumulator type.  With
// `vec` (x 16-byte aligned, cols a multiple of 4) they come from 16-byte
// read-only vector loads; otherwise only the cells present in `nib`.
template <typename Acc, typename T>
__device__ __forceinline__ void load_x4(const T* __restrict__ x, int64_t c4, bool vec,
                                        uint32_t nib, Acc* out) {
    if constexpr (sizeof(T) == 8) {
        if (vec) {
            const double2 a = __ldg(reinterpret_cast<const double2*>(x + c4));
            const double2 b = __ldg(reinterpret_cast<const double2*>(x + c4 + 2));
            out[0] = static_cast<Acc>(a.x);
            out[1] = static_cast<Acc>(a.y);
            out[2] = static_cast<Acc>(b.x);
            out[3] = static_cast<Acc>(b.y);
            return;
        }
    } else {
        if (vec) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(x + c4));
            out[0] = static_cast<Acc>(a.x);
            out[1] = static_cast<Acc>(a.y);
            out[2] = static_cast<Acc>(a.z);
            out[3] = static_cast<Acc>(a.w);
            return;
        }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) out[c] = (nib & (1u << c)) ? static_cast<Acc>(__ldg(x + c4 + c)) : Acc(0);
}

// The four fp64 x values of a block column as one 32-byte read-only load
// (x 32-byte aligned, cols a multiple of 4).
template <typename Acc, typename T>
__device__ __forceinline__ void load_x4_32(const T* __restrict__ x, int64_t c4, Acc* out) {
    static_assert(sizeof(T) == 8, "32-byte x loads are for fp64 x");
    double d0, d1, d2, d3;
    asm("ld.global.nc.v4.f64 {%0, %1, %2, %3}, [%4];"
        : "=d"(d0), "=d"(d1), "=d"(d2), "=d"(d3)
        : "l"(x + c4));
    out[0] = static_cast<Acc>(d0);
    out[1] = static_cast<Acc>(d1);
    out[2] = static_cast<Acc>(d2);
    out[3] = static_cast<Acc>(d3);
}

// Hint: start pulling [p, p + bytes) into L2 before the dependent loads ask
// for it.  The range is widened to 16-byte bounds; plan buffers are
// 256-byte aligned and carry tail slack, so it stays inside the allocation.
__device__ __forceinline__ void prefetch_l2(const void* p, int64_t bytes) {
    if (bytes <= 0) return;
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t lo = a & ~static_cast<uintptr_t>(15);
    const uintptr_t hi = (a + static_cast<uintptr_t>(bytes) + 15) & ~static_cast<uintptr_t>(15);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"(static_cast<uint32_t>(hi - lo))
                 : "memory");
}

// ---- value decoders ------------------------------------------------------------
// V: element type of the kept value stream; decode(raw, ctx, bit) turns a
// stored element into the accumulator type (ctx is per block, bit the cell).

// Lossless routes accumulate in double (fp32 matrices too: a long fp32 row
// summed in fp32 drifts by ~sqrt(len) ulps, above a 1e-6 normwise bound).
template <typename T>
struct RawDec {
    using Acc = double;
    using V = T;
    static constexpr bool kHasKept = true;
    const T* __restrict__ kept;
    const T* __restrict__ res;
    __device__ __forceinline__ void prepare(void*) {}
    __device__ __forceinline__ V load(int64_t p) const { return kept[p]; }
    __device__ __forceinline__ void prefetch_values(int64_t a, int64_t b) const {
        prefetch_l2(kept + a, (b - a) * static_cast<int64_t>(sizeof(V)));
    }
    __device__ __forceinline__ Acc block_ctx(int64_t) const { return Acc(1); }
    __device__ __forceinline__ Acc decode(V raw, Acc, int) const { return static_cast<Acc>(raw); }
    __device__ __forceinline__ Acc res_val(int64_t p) const { return static_cast<Acc>(res[p]); }
    __device__ __forceinline__ Acc xv(const T* __restrict__ x, int64_t c) const { return static_cast<Acc>(x[c]); }
};

template <typename T, typename IdxT, bool Smem>
struct DictDec {
    using Acc = double;
    using V = IdxT;
    static constexpr bool kHasKept = true;
    const IdxT* __restrict__ kept;
    const IdxT* __restrict__ res;
    const T* __restrict__ codebook;
    int64_t size;
    __device__ __forceinline__ void prepare(void*) {
        if constexpr (Smem) {
            T* s = reinterpret_cast<T*>(g_smem);
            for (int64_t i = threadIdx.x; i < size; i += blockDim.x) s[i] = codebook[i];
        }
    }
    // the codebook entry: from the shared copy (Smem) or global memory
    __device__ __forceinline__ T entry(uint32_t i) const {
        if constexpr (Smem) return reinterpret_cast<const T*>(g_smem)[i];
        return __ldg(codebook + i);
    }
    __device__ __forceinline__ V load(int64_t p) const { return kept[p]; }
    __device__ __forceinline__ void prefetch_values(int64_t a, int64_t b) const {
        prefetch_l2(kept + a, (b - a) * static_cast<int64_t>(sizeof(V)));
    }
    __device__ __forceinline__ Acc block_ctx(int64_t) const { return Acc(1); }
    __device__ __forceinline__ Acc decode(V raw, Acc, int) const { return static_cast<Acc>(entry(raw)); }
    __device__ __forceinline__ Acc res_val(int64_t p) const { return static_cast<Acc>(entry(res[p])); }
    __device__ __forceinline__ Acc xv(const T* __restrict__ x, int64_t c) const { return static_cast<Acc>(x[c]); }
};

template <typename T>
struct Bfp8Dec {
    using Acc = float;
    using V = int8_t;
    static constexpr bool kHasKept = true;
    const int8_t* __restrict__ kept;
    const uint16_t* __restrict__ res;
    const uint16_t* __restrict__ scale;
    __device__ __forceinline__ void prepare(void*) {}
    __device__ __forceinline__ V load(int64_t p) const { return kept[p]; }
    __device__ __forceinline__ void prefetch_values(int64_t a, int64_t b) const {
        prefetch_l2(kept + a, (b - a) * static_cast<int64_t>(sizeof(V)));
    }
    __device__ __forceinline__ float block_ctx(int64_t b) const { return bf16_to_float(scale[b]); }
    __device__ __forceinline__ float decode(V raw, float sc, int) const {
        return small_int_to_float(raw) * sc;
    }
    __device__ __forceinline__ float res_val(int64_t p) const { return bf16_to_float(res[p]); }
    __device__ __forceinline__ float xv(const T* __restrict__ x, int64_t c) const {
        return static_cast<float>(x[c]);
    }
};

// Family-runner exact dictionary with per-cell tile codes: Bits-bit code of
// cell `bit` in the block's tile words (common.cuh:62-93, 147-160), value =
// codebook[code], accumulated in double.  The block context is the block.
template <typename T, int Bits>
struct TileDec {
    using Acc = double;
    using V = uint8_t;  // no per-nnz kept stream
    static constexpr bool kHasKept = false;
    static constexpr int kWords = Bits;  // words_per_tile = Bits for 8x4 cells
    static constexpr int kPerWord = 32 / Bits;
    static constexpr uint32_t kMask = (1u << Bits) - 1u;
    const uint32_t* __restrict__ words;
    const T* __restrict__ codebook;
    const T* __restrict__ res;
    const uint8_t* kept = nullptr;
    __device__ __forceinline__ void prepare(void*) {}
    __device__ __forceinline__ V load(int64_t) const { return V{}; }
    __device__ __forceinline__ Acc block_ctx(int64_t b) const { return static_cast<Acc>(b); }
    __device__ __forceinline__ Acc decode(V, Acc blk, int bit) const {
        const int64_t b = static_cast<int64_t>(blk);
        const uint32_t w = __ldg(words + b * kWords + bit / kPerWord);
        return static_cast<Acc>(codebook[(w >> ((bit % kPerWord) * Bits)) & kMask]);
    }
    __device__ __forceinline__ Acc res_val(int64_t p) const { return static_cast<Acc>(res[p]); }
    __device__ __forceinline__ Acc xv(const T* __restrict__ x, int64_t c) const { return static_cast<Acc>(x[c]); }
};

// Per-nnz bf16 values (round16_nnz, common.cuh:632-687), fp32 accumulate.
template <typename T>
struct Bf16NnzDec {
    using Acc = float;
    using V = uint16_t;
    static constexpr bool kHasKept = true;
    const uint16_t* __restrict__ kept;
    const uint16_t* __restrict__ res;
    __device__ __forceinline__ void prepare(void*) {}
    __device__ __forceinline__ V load(int64_t p) const { return kept[p]; }
    __device__ __forceinline__ void prefetch_values(int64_t a, int64_t b) const {
        prefetch_l2(kept + a, (b - a) * static_cast<int64_t>(sizeof(V)));
    }
    __device__ __forceinline__ float block_ctx(int64_t) const { return 1.0f; }
    __device__ __forceinline__ float decode(V raw, float, int) const { return bf16_to_float(raw); }
    __device__ __forceinline__ float res_val(int64_t p) const { return bf16_to_float(res[p]); }
    __device__ __forceinline__ float xv(const T* __restrict__ x, int64_t c) const {
        return static_cast<float>(x[c]);
    }
};

// ---- family value codecs without a per-nnz value stream ---------------------------
// (BitBSR-only routes, as the reference's family runner; no residual)

// Every stored value is one constant: 1 (implicit_one) or C (const_c),
// lossless, T-exact accumulation (bitbsr_spmv_8x4_lossless.cuh).
template <typename T>
struct ConstDec {
    using Acc = double;
    using V = uint8_t;
    static constexpr bool kHasKept = false;
    double c;
    __device__ __forceinline__ void prepare(void*) {}
    __device__ __forceinline__ V load(int64_t) const { return V{}; }
    __device__ __forceinline__ Acc block_ctx(int64_t) const { return Acc(1); }
    __device__ __forceinline__ Acc decode(V, Acc, int) const { return c; }
    __device__ __forceinline__ Acc res_val(int64_t) const { return Acc(0); }
    __device__ __forceinline__ Acc xv(const T* __restrict__ x, int64_t col) const { return static_cast<Acc>(x[col]); }
};

// Sign masks, one 32-bit word per block: cell bit set -> +scale, clear ->
// -scale (decode_sign_tile32_value, common.cuh:119-125; sign2 has scale 1).
template <typename T>
struct SignDec {
    using Acc = double;
    using V = uint8_t;
    static constexpr bool kHasKept = false;
    const uint32_t* __restrict__ masks;
    double scale;
    __device__ __forceinline__ void prepare(void*) {}
    __device__ __forceinline__ V load(int64_t) const { return V{}; }
    __device__ __forceinline__ Acc block_ctx(int64_t b) const { return static_cast<Acc>(b); }
    __device__ __forceinline__ Acc decode(V, Acc blk, int bit) const {
        return ((__ldg(masks + static_cast<int64_t>(blk)) >> bit) & 1u) ? scale : -scale;
    }
    __device__ __forceinline__ Acc res_val(int64_t) const { return Acc(0); }
    __device__ __forceinline__ Acc xv(const T* __restrict__ x, int64_t col) const { return static_cast<Acc>(x[col]); }
};

// Per-nnz fp16 bits, fp32 accumulation (round16_nnz with fp16, common.cuh:626-687).
template <typename T>
struct Fp16NnzDec {
    using Acc = float;
    using V = uint16_t;
    static constexpr bool kHasKept = true;
    const uint16_t* __restrict__ kept;
    __device__ __forceinline__ void prepare(void*) {}
    __device__ __forceinline__ V load(int64_t p) const { return kept[p]; }
    __device__ __forceinline__ void prefetch_values(int64_t a, int64_t b) const {
        prefetch_l2(kept + a, (b - a) * 2);
    }
    __device__ __forceinline__ float block_ctx(int64_t) const { return 1.0f; }
    __device__ __forceinline__ float decode(V raw, float, int) const { return __half2float(__ushort_as_half(raw)); }
    __device__ __forceinline__ float res_val(int64_t) const { return 0.0f; }
    __device__ __forceinline__ float xv(const T* __restrict__ x, int64_t col) const {
        return static_cast<float>(x[col]);
    }
};

// BFP4: signed 4-bit mantissa (two's complement, [-7, 7]) at the nibble
// (p & 1) of byte p/2 of the linear nnz position p, times the block's bf16
// scale, fp32 accumulation (decode_bfp4_nibble, common.cuh:780-835).
template <typename T>
struct Bfp4Dec {
    using Acc = float;
    using V = int;
    static constexpr bool kHasKept = true;
    const uint8_t* __restrict__ packed;
    const uint16_t* __restrict__ scale;
    __device__ __forceinline__ void prepare(void*) {}
    __device__ __forceinline__ V load(int64_t p) const {
        const uint8_t byte = packed[p >> 1];
        const int nib = (p & 1) ? (byte >> 4) : (byte & 0xF);
        return (nib ^ 0x8) - 0x8;
    }
    __device__ __forceinline__ void prefetch_values(int64_t a, int64_t b) const {
        prefetch_l2(packed + (a >> 1), ((b + 1) >> 1) - (a >> 1));
    }
    __device__ __forceinline__ float block_ctx(int64_t b) const { return bf16_to_float(scale[b]); }
    __device__ __forceinline__ float decode(V raw, float sc, int) const { return small_int_to_float(raw) * sc; }
    __device__ __forceinline__ float res_val(int64_t) const { return 0.0f; }
    __device__ __forceinline__ float xv(const T* __restrict__ x, int64_t col) const {
        return static_cast<float>(x[col]);
    }
};

// ---- main pass -----------------------------------------------------------------

// XVEC: x is 16-byte aligned and cols % 4 == 0, so a block's four x values
// are two 16-byte loads (a compile-time choice: with a run-time flag both
// paths stay in the loop and the kernel measured 6 % slower on FEM; one
// 32-byte load instead: 0.131 -> 0.134-0.136 ms on FEM at 32-40 registers)
template <typename T, typename Dec, int SLOTS, bool XVEC>
__global__ void __launch_bounds__(kThreads)
hybrid_main_kernel(const KernelShape k, Dec dec, const T* __restrict__ x, T* __restrict__ y) {
    dec.prepare(g_smem);
    __syncthreads();  // a shared codebook is complete before any lane reads it
    using Acc = typename Dec::Acc;
    using V = typename Dec::V;
    constexpr int G = 8 * SLOTS;
    const int lane = threadIdx.x & 31;
    const int gl = lane & (G - 1);
    const int s = gl >> 3;
    const int r = gl & 7;
    const unsigned gmask = G == 32 ? 0xffffffffu : (((1u << G) - 1u) << (lane & ~(G - 1)));
    const int64_t br = k.br_begin + (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / G;
    if (br >= k.nbr) return;  // the whole group leaves together

    const int b0 = k.kept_brp[br];
    int b1 = k.kept_brp[br + 1];
    if (b1 - b0 > k.heavy_limit) b1 = b0 + k.heavy_limit;
    int vb = k.kept_brvp[br];
    const uint64_t* __restrict__ words = k.words;
    if constexpr (Dec::kHasKept) {
        if (k.l2_prefetch && gl == 0) {  // the block row's words and values, in bulk
            prefetch_l2(words + b0, static_cast<int64_t>(b1 - b0) * 8);
            dec.prefetch_values(vb, k.kept_brvp[br + 1]);
        }
    }
    const uint32_t lowmask = (1u << (4 * r)) - 1u;
    Acc sum = Acc(0);

    // Narrow groups (residual-heavy rows, few blocks) request the residual
    // rows' pointers and each lane's first two residual entries before the
    // block loop, so the residual's dependent loads (row_ptr -> col -> x)
    // overlap the blocks'.  Wide groups (block-dense rows) keep the registers
    // for the block loop and walk the residual afterwards.
    constexpr bool kPrefetch = SLOTS <= 2;
    int rq = 0, re = 0, col0 = 0, col1 = 0;
    Acc val0 = Acc(0), val1 = Acc(0);
    if constexpr (kPrefetch) {
        const int64_t row = br * kBlockRows + r;
        if (row < k.rows && k.res_rp != nullptr) {
            rq = k.res_rp[row] + s;
            re = k.res_rp[row + 1];
            if (k.long_tau > 0 && re - (rq - s) > k.long_tau) re = rq;  // finished by the overflow pass
        }
        if (rq < re) {
            col0 = __ldg(k.res_col + rq);
            val0 = dec.res_val(rq);
        }
        if (rq + SLOTS < re) {
            col1 = __ldg(k.res_col + rq + SLOTS);
            val1 = dec.res_val(rq + SLOTS);
        }
    }

    // One coalesced load brings G block words into the group; a group scan of
    // their popcounts gives every block's value base; the blocks are then
    // handed to the slots by shuffle, so consecutive steps are independent.
    for (int batch = b0; batch < b1; batch += G) {
        const int nblk = min(G, b1 - batch);
        const uint64_t wl = gl < nblk ? __ldg(words + batch + gl) : 0ULL;
        const int pcl = __popc(static_cast<uint32_t>(wl >> 32));
        int incl = pcl;
#pragma unroll
        for (int o = 1; o < G; o <<= 1) {
            const int t = __shfl_up_sync(gmask, incl, o, G);
            if (gl >= o) incl += t;
        }
        const int exl = incl - pcl;
        const int total = __shfl_sync(gmask, incl, G - 1, G);
#pragma unroll 4
        for (int j0 = 0; j0 < nblk; j0 += SLOTS) {
            const int j = j0 + s;
            const uint64_t w = __shfl_sync(gmask, wl, j, G);
            const int vblk = vb + __shfl_sync(gmask, exl, j, G);
            // lanes past the batch read a zero word: nib = 0, nothing loads
            const uint32_t bm = static_cast<uint32_t>(w >> 32);
            const uint32_t nib = (bm >> (4 * r)) & 0xFu;
            if (nib) {
                const int64_t c4 = static_cast<int64_t>(w & 0x7fffffffULL) * 4;
                const Acc ctx = dec.block_ctx(batch + j);
                int v0 = vblk + __popc(bm & lowmask);
                Acc xs[4];
                load_x4<Acc, T>(x, c4, XVEC, nib, xs);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (nib & (1u << c)) {
                        V raw{};
                        if constexpr (Dec::kHasKept) raw = dec.load(v0);
                        sum += dec.decode(raw, ctx, 4 * r + c) * xs[c];
                        ++v0;
                    }
                }
            }
        }
        vb += total;
    }

    const int64_t row = br * kBlockRows + r;
    const int32_t* __restrict__ rc = k.res_col;
    if constexpr (kPrefetch) {
        if (rq < re) sum += val0 * dec.xv(x, col0);
        if (rq + SLOTS < re) sum += val1 * dec.xv(x, col1);
#pragma unroll 4
        for (int q = rq + 2 * SLOTS; q < re; q += SLOTS) sum += dec.res_val(q) * dec.xv(x, rc[q]);
    } else if (row < k.rows && k.res_rp != nullptr) {
        const int rs = k.res_rp[row];
        const int re_ = k.res_rp[row + 1];
        if (!(k.long_tau > 0 && re_ - rs > k.long_tau)) {
#pragma unroll 4
            for (int q = rs + s; q < re_; q += SLOTS) sum += dec.res_val(q) * dec.xv(x, rc[q]);
        }
    }
    if constexpr (SLOTS > 1) sum += __shfl_xor_sync(gmask, sum, 8, G);
    if constexpr (SLOTS > 2) sum += __shfl_xor_sync(gmask, sum, 16, G);
    if (s == 0 && row < k.rows) y[row] = static_cast<T>(sum);
}

// ---- main pass, one lane per row (block rows with few blocks) ------------------
//
// For short rows (a few kept blocks per block row, a few residual entries
// per row) the group machinery above costs more instructions than the work
// itself.  Here a lane owns whole rows: it walks its row's nibble of each
// block of the row's block row in order (the 8 lanes of a block row read the
// same word, one transaction), then the row's residual entries.  Each lane
// carries kRowLanes rows, kThreads apart in the CTA's tile of kRowLanes *
// kThreads rows, and steps their loops together, so every step issues
// independent loads for both rows (one row per lane: 10-14 % slower on the
// 3D Laplacians; four: slower, 48 registers).  Same accumulation order per
// row as the one-slot group, so the results are identical.

constexpr int kRowLanes = 2;

template <typename T, typename Dec>
__global__ void __launch_bounds__(kThreads)
hybrid_row_kernel(const KernelShape k, Dec dec, const T* __restrict__ x, T* __restrict__ y) {
    dec.prepare(g_smem);
    __syncthreads();  // a shared codebook is complete before any lane reads it
    using Acc = typename Dec::Acc;
    using V = typename Dec::V;
    constexpr int R = kRowLanes;
    const int64_t brows = static_cast<int64_t>(k.nbr) * kBlockRows;
    const int64_t end = brows < k.rows ? brows : k.rows;
    const int64_t tile = static_cast<int64_t>(k.br_begin) * kBlockRows +
                         static_cast<int64_t>(blockIdx.x) * (R * kThreads) + threadIdx.x;
    const uint64_t* __restrict__ words = k.words;
    const int32_t* __restrict__ rc = k.res_col;
    int b0[R], b1[R], vb[R], q[R], qe[R];
    Acc sum[R];
    int nb = 0, nr = 0;
#pragma unroll
    for (int h = 0; h < R; ++h) {
        const int64_t row = tile + h * kThreads;
        sum[h] = Acc(0);
        b0[h] = b1[h] = vb[h] = q[h] = qe[h] = 0;
        if (row < end) {
            const int64_t br = row / kBlockRows;
            b0[h] = k.kept_brp[br];
            b1[h] = k.kept_brp[br + 1];
            if (b1[h] - b0[h] > k.heavy_limit) b1[h] = b0[h] + k.heavy_limit;
            vb[h] = k.kept_brvp[br];
            if (k.res_rp != nullptr) {
                q[h] = k.res_rp[row];
                qe[h] = k.res_rp[row + 1];
                if (k.long_tau > 0 && qe[h] - q[h] > k.long_tau) qe[h] = q[h];  // finished by the overflow pass
            }
        }
        nb = max(nb, b1[h] - b0[h]);
        nr = max(nr, qe[h] - q[h]);
    }
    for (int t = 0; t < nb; ++t) {
#pragma unroll
        for (int h = 0; h < R; ++h) {
            const int b = b0[h] + t;
            if (b < b1[h]) {
                const int r = static_cast<int>((tile + h * kThreads) & (kBlockRows - 1));
                const uint64_t w = __ldg(words + b);
                const uint32_t bm = static_cast<uint32_t>(w >> 32);
                const uint32_t nib = (bm >> (4 * r)) & 0xFu;
                if (nib) {
                    const int64_t c4 = static_cast<int64_t>(w & 0x7fffffffULL) * 4;
                    const Acc ctx = dec.block_ctx(b);
                    int v0 = vb[h] + __popc(bm & ((1u << (4 * r)) - 1u));
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (nib & (1u << c)) {
                            V raw{};
                            if constexpr (Dec::kHasKept) raw = dec.load(v0);
                            sum[h] += dec.decode(raw, ctx, 4 * r + c) * dec.xv(x, c4 + c);
                            ++v0;
                        }
                    }
                }
                vb[h] += __popc(bm);
            }
        }
    }
    for (int t = 0; t < nr; ++t) {
#pragma unroll
        for (int h = 0; h < R; ++h) {
            const int p = q[h] + t;
            if (p < qe[h]) sum[h] += dec.res_val(p) * dec.xv(x, rc[p]);
        }
    }
#pragma unroll
    for (int h = 0; h < R; ++h) {
        const int64_t row = tile + h * kThreads;
        if (row < end) y[row] = static_cast<T>(sum[h]);
    }
}

// ---- main pass for BFP8 on block-dense rows: one lane per block ----------------
//
// With many kept blocks per block row (FEM: 29) the group kernel spends most
// of its instructions on per-row-segment work that the eight lanes of a block
// repeat: the word, the value base, the scale, the four x values converted to
// fp32.  Here a warp owns a block row and a lane one block of each 32-block
// batch: the batch's int8 values (one contiguous run) are staged in shared
// memory with coalesced 16-byte loads, each lane decodes its block's present
// cells into eight fp32 row sums (decoded value times x, as the group kernel
// and the reference's joint kernel), the lanes (row, slot) add the residual
// entries of their row, and the eight rows are reduced across the warp in
// five exchange steps.  Staging reads up to 15 bytes past a batch's values,
// so it runs only on plan buffers (16-byte aligned, with tail slack).
// FEM forced to BFP8: 0.128 -> 0.096 ms; block-sparse 2^18: 0.147 -> 0.093 ms.

constexpr int kLaneWarps = kThreads / 32;
constexpr int kLaneStage = 32 * 32 + 32;  // one batch's values plus the alignment head

template <typename T, bool XVEC>
__global__ void __launch_bounds__(kThreads)
bfp8_block_lane_kernel(const KernelShape k, Bfp8Dec<T> dec, const T* __restrict__ x, T* __restrict__ y) {
    __shared__ __align__(16) int8_t stage[kLaneWarps][kLaneStage];
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const int br = k.br_begin + static_cast<int>(blockIdx.x) * kLaneWarps + wp;
    if (br >= k.nbr) return;  // the whole warp leaves together
    const int b0 = k.kept_brp[br];
    int b1 = k.kept_brp[br + 1];
    if (b1 - b0 > k.heavy_limit) b1 = b0 + k.heavy_limit;
    int vb = k.kept_brvp[br];
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    for (int batch = b0; batch < b1; batch += 32) {
        const int j = batch + lane;
        const uint64_t w = j < b1 ? __ldg(k.words + j) : 0ULL;
        const uint32_t bm = static_cast<uint32_t>(w >> 32);
        const int pc = __popc(bm);
        int incl = pc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        const int base = vb & ~15;
        const int nch = (vb + total - base + 15) >> 4;
        // (a plain load: the read-only form makes ptxas keep 16 more registers)
        for (int c = lane; c < nch; c += 32)
            reinterpret_cast<uint4*>(stage[wp])[c] = reinterpret_cast<const uint4*>(dec.kept + base)[c];
        __syncwarp();
        if (bm) {
            const float sc = dec.block_ctx(j);
            const int64_t c4 = static_cast<int64_t>(w & 0x7fffffffULL) * 4;
            float xq[4];
            if constexpr (XVEC) {
                load_x4<float, T>(x, c4, true, 0xFu, xq);
            } else {  // only the columns a present cell reads (the last block may pass cols)
                uint32_t cols = bm | (bm >> 16);
                cols |= cols >> 8;
                cols |= cols >> 4;
                load_x4<float, T>(x, c4, false, cols & 0xFu, xq);
            }
            int p = vb + incl - pc - base;
#pragma unroll
            for (int b = 0; b < 32; ++b) {
                if (bm & (1u << b)) {
                    acc[b >> 2] += dec.decode(stage[wp][p], sc, b) * xq[b & 3];
                    ++p;
                }
            }
        }
        vb += total;
        __syncwarp();  // every lane has read the batch before the next one is staged
    }
    {  // residual: lane (slot s, row r) strides row r's entries by 4
        const int r = lane & 7, s = lane >> 3;
        const int64_t row = static_cast<int64_t>(br) * kBlockRows + r;
        float rs = 0.0f;
        if (row < k.rows && k.res_rp != nullptr) {
            const int q0 = k.res_rp[row], q1 = k.res_rp[row + 1];
            if (!(k.long_tau > 0 && q1 - q0 > k.long_tau)) {
                for (int q = q0 + s; q < q1; q += 4) rs += dec.res_val(q) * dec.xv(x, k.res_col[q]);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i == r) acc[i] += rs;
    }
    // eight row sums over 32 lanes: halve the rows a lane keeps at each of
    // three exchanges (partner lane ^16, ^8, ^4), then sum the last two bits
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
    float a4[4], a2[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = h16 ? acc[i] : acc[i + 4];
        a4[i] = (h16 ? acc[i + 4] : acc[i]) + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = h8 ? a4[i] : a4[i + 2];
        a2[i] = (h8 ? a4[i + 2] : a4[i]) + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float a1 = (h4 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, h4 ? a2[0] : a2[1], 4);
    a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
    a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
    const int64_t row = static_cast<int64_t>(br) * kBlockRows + (h16 ? 4 : 0) + (h8 ? 2 : 0) + (h4 ? 1 : 0);
    if ((lane & 3) == 0 && row < k.rows) y[row] = static_cast<T>(a1);
}

// ---- main pass for BFP8 on long block-dense rows: a row segment per permute ----
//
// With many 32-block batches per block row (block-sparse 2^18: 131 kept
// blocks a block row) the lane kernel above waits on each batch's word load
// and decodes every cell with a shared byte load (bank-conflicted: the
// lanes' blocks lie about 19 bytes apart).  Here each lane also owns a block,
// but:
//  - the next batch's words are loaded while the current batch is decoded;
//  - a lane copies its block's int8 run (the 48 bytes from the 16-byte
//    boundary below it) into its own column of a transposed shared array
//    (word m of lane l at [m][l], so every shared access of the warp hits 32
//    distinct banks, whatever the offsets);
//  - a row segment (the <= 4 packed cells of one block row) is decoded from a
//    4-byte window: one byte permute puts the cells in column order (absent
//    columns read a zero code, selector from a 16-entry table), four
//    permutes build 2^23 + 128 + q as floats, and packed f32x2 adds and FMAs
//    remove the offset and multiply by the block's scaled x (scale * x is
//    formed once per block; two partial sums per row).
// Block-sparse 2^18: 0.092 -> 0.078 ms; FEM (one batch a block row) stays on
// the lane kernel (0.090 there, 0.104 here).  Reads up to 47 bytes past a
// block's first value, so it runs only on plan buffers (tail slack).

constexpr int kSegmentMinBlocks = 64;  // kept blocks per block row from which it runs
constexpr int kSegWords = 12;          // 48 staged bytes a lane

__device__ __forceinline__ uint64_t f32x2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float f32x2_sum(uint64_t v) {
    float a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
    return a + b;
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f32x2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// XM: 2 = the four x values as one 32-byte load (fp64 x 32-byte aligned,
// cols % 4 == 0), 1 = 16-byte loads (x_vec_ok), 0 = only the present columns
template <typename T, int XM>
__global__ void __launch_bounds__(kThreads)
bfp8_segment_kernel(const KernelShape k, Bfp8Dec<T> dec, const T* __restrict__ x, T* __restrict__ y) {
    __shared__ uint32_t cols[kLaneWarps][kSegWords][32];
    __shared__ uint32_t sel[16];  // nibble -> byte selector of the column-order permute
    if (threadIdx.x < 16) {
        uint32_t s = 0, n = 0;
        for (int c = 0; c < 4; ++c) {
            const bool on = (threadIdx.x >> c) & 1u;
            s |= (on ? n : 4u) << (4 * c);  // 4: a byte of the zero-code operand
            n += on ? 1u : 0u;
        }
        sel[threadIdx.x] = s;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const int br = k.br_begin + static_cast<int>(blockIdx.x) * kLaneWarps + wp;
    if (br >= k.nbr) return;  // the whole warp leaves together
    const int b0 = k.kept_brp[br];
    int b1 = k.kept_brp[br + 1];
    if (b1 - b0 > k.heavy_limit) b1 = b0 + k.heavy_limit;
    int vb = k.kept_brvp[br];
    uint64_t acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0ULL;
    const uint64_t moff = f32x2_pack(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    uint32_t* mine = &cols[wp][0][lane];
    uint64_t wnext = b0 + lane < b1 ? __ldg(k.words + b0 + lane) : 0ULL;
    for (int batch = b0; batch < b1; batch += 32) {
        const int j = batch + lane;
        const uint64_t w = wnext;
        wnext = j + 32 < b1 ? __ldg(k.words + j + 32) : 0ULL;
        const uint32_t bm = static_cast<uint32_t>(w >> 32);
        const int pc = __popc(bm);
        int incl = pc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        if (bm) {
            const int p = vb + incl - pc;  // the block's first value
            const int a16 = p & ~15;
            const uint4* src = reinterpret_cast<const uint4*>(dec.kept + a16);
            const uint4 c0 = __ldg(src), c1 = __ldg(src + 1);
            uint4 c2 = make_uint4(0u, 0u, 0u, 0u);
            if (p - a16 + pc > 32) c2 = __ldg(src + 2);
            mine[0 * 32] = c0.x; mine[1 * 32] = c0.y; mine[2 * 32] = c0.z; mine[3 * 32] = c0.w;
            mine[4 * 32] = c1.x; mine[5 * 32] = c1.y; mine[6 * 32] = c1.z; mine[7 * 32] = c1.w;
            mine[8 * 32] = c2.x; mine[9 * 32] = c2.y; mine[10 * 32] = c2.z; mine[11 * 32] = c2.w;
            const float sc = dec.block_ctx(j);
            const int64_t c4 = static_cast<int64_t>(w & 0x7fffffffULL) * 4;
            float xq[4];
            if constexpr (XM == 2) {
                load_x4_32<float, T>(x, c4, xq);
            } else if constexpr (XM == 1) {
                load_x4<float, T>(x, c4, true, 0xFu, xq);
            } else {  // only the columns a present cell reads (the last block may pass cols)
                uint32_t cm = bm | (bm >> 16);
                cm |= cm >> 8;
                cm |= cm >> 4;
                load_x4<float, T>(x, c4, false, cm & 0xFu, xq);
            }
            const uint64_t xs01 = f32x2_pack(sc * xq[0], sc * xq[1]);
            const uint64_t xs23 = f32x2_pack(sc * xq[2], sc * xq[3]);
            // bit position of the current segment's first cell in the staged
            // bytes: at most 8 * (15 + 28), so words m, m + 1 stay below 12
            uint32_t q8 = static_cast<uint32_t>(p - a16) * 8u;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const uint32_t nib = (bm >> (4 * r)) & 0xFu;
                const uint32_t m = q8 >> 5;
                const uint32_t lo = mine[m * 32], hi = mine[m * 32 + 32];
                const uint32_t win = __funnelshift_r(lo, hi, q8) ^ 0x80808080u;  // codes + 128
                const uint32_t cw = __byte_perm(win, 0x80808080u, sel[nib]);
                const float f0 = __uint_as_float(__byte_perm(cw, 0x4B000000u, 0x7440));
                const float f1 = __uint_as_float(__byte_perm(cw, 0x4B000000u, 0x7441));
                const float f2 = __uint_as_float(__byte_perm(cw, 0x4B000000u, 0x7442));
                const float f3 = __uint_as_float(__byte_perm(cw, 0x4B000000u, 0x7443));
                acc[r] = f32x2_fma(f32x2_add(f32x2_pack(f0, f1), moff), xs01, acc[r]);
                acc[r] = f32x2_fma(f32x2_add(f32x2_pack(f2, f3), moff), xs23, acc[r]);
                q8 += 8u * static_cast<uint32_t>(__popc(nib));
            }
        }
        vb += total;
    }
    float rsum[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) rsum[i] = f32x2_sum(acc[i]);
    {  // residual: lane (slot s, row r) strides row r's entries by 4
        const int r = lane & 7, s = lane >> 3;
        const int64_t row = static_cast<int64_t>(br) * kBlockRows + r;
        float rs = 0.0f;
        if (row < k.rows && k.res_rp != nullptr) {
            const int q0 = k.res_rp[row], q1 = k.res_rp[row + 1];
            if (!(k.long_tau > 0 && q1 - q0 > k.long_tau)) {
                for (int q = q0 + s; q < q1; q += 4) rs += dec.res_val(q) * dec.xv(x, k.res_col[q]);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i == r) rsum[i] += rs;
    }
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
    float a4[4], a2[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = h16 ? rsum[i] : rsum[i + 4];
        a4[i] = (h16 ? rsum[i + 4] : rsum[i]) + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = h8 ? a4[i] : a4[i + 2];
        a2[i] = (h8 ? a4[i + 2] : a4[i]) + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float a1 = (h4 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, h4 ? a2[0] : a2[1], 4);
    a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
    a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
    const int64_t row = static_cast<int64_t>(br) * kBlockRows + (h16 ? 4 : 0) + (h8 ? 2 : 0) + (h4 ? 1 : 0);
    if ((lane & 3) == 0 && row < k.rows) y[row] = static_cast<T>(a1);
}

template <typename Dec>
struct is_bfp8 : std::false_type {};
template <typename T>
struct is_bfp8<Bfp8Dec<T>> : std::true_type {};

// ---- overflow pass: heavy block-row pieces, long residual chunks, outliers ----

template <typename T, typename Dec>
__global__ void __launch_bounds__(kThreads)
hybrid_overflow_kernel(const KernelShape k, Dec dec, const T* __restrict__ x, T* __restrict__ y,
                       int heavy_ctas, int chunk_ctas, int64_t num_out,
                       const int32_t* __restrict__ orow, const int32_t* __restrict__ ocol,
                       const T* __restrict__ oval) {
    dec.prepare(g_smem);
    __syncthreads();
    using Acc = typename Dec::Acc;
    using V = typename Dec::V;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int cta = static_cast<int>(blockIdx.x);
    if (cta < heavy_ctas) {
        const int64_t t = static_cast<int64_t>(cta) * (kThreads / 32) + warp;
        if (t >= k.num_heavy) return;
        const int64_t br = k.heavy_br[t];
        const int b0 = k.heavy_b0[t], b1 = k.heavy_b1[t];
        const int s = lane >> 3, r = lane & 7;
        int vb = k.kept_bvp[b0];
        Acc sum = Acc(0);
        for (int base = b0; base < b1; base += 4) {
            const int b = base + s;
            const bool valid = b < b1;
            const uint64_t w = valid ? __ldg(k.words + b) : 0ULL;
            const uint32_t bm = static_cast<uint32_t>(w >> 32);
            const int bc = static_cast<int>(w & 0x7fffffffULL);
            const int pc = __popc(bm);
            int incl = pc;
            int tt = __shfl_up_sync(0xffffffffu, incl, 8);
            if (s >= 1) incl += tt;
            tt = __shfl_up_sync(0xffffffffu, incl, 16);
            if (s >= 2) incl += tt;
            const int total = __shfl_sync(0xffffffffu, incl, 31);
            const int vblk = vb + incl - pc;
            vb += total;
            const uint32_t nib = (bm >> (4 * r)) & 0xFu;
            if (nib) {
                const Acc ctx = dec.block_ctx(b);
                int v0 = vblk + __popc(bm & ((1u << (4 * r)) - 1u));
                const int64_t c4 = static_cast<int64_t>(bc) * 4;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (nib & (1u << c)) {
                        V raw{};
                        if constexpr (Dec::kHasKept) raw = dec.load(v0);
                        sum += dec.decode(raw, ctx, 4 * r + c) * dec.xv(x, c4 + c);
                        ++v0;
                    }
                }
            }
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 8);
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        const int64_t row = br * kBlockRows + r;
        if (s == 0 && row < k.rows) atomicAdd(&y[row], static_cast<T>(sum));
        return;
    }
    if (cta < heavy_ctas + chunk_ctas) {
        const int64_t c = static_cast<int64_t>(cta - heavy_ctas) * (kThreads / 32) + warp;
        if (c >= k.num_chunks) return;
        const int row = k.chunk_row[c];
        const int pb = k.chunk_pbegin[c];
        const int pn = k.chunk_pcount[c];
        Acc sum = Acc(0);
        // four independent column -> x chains in flight per lane
        constexpr int U = 4;
        int q = lane;
        for (; q + 32 * (U - 1) < pn; q += 32 * U) {
            int col[U];
            Acc val[U];
#pragma unroll
            for (int u = 0; u < U; ++u) col[u] = __ldg(k.res_col + pb + q + 32 * u);
#pragma unroll
            for (int u = 0; u < U; ++u) val[u] = dec.res_val(pb + q + 32 * u);
#pragma unroll
            for (int u = 0; u < U; ++u) sum += val[u] * dec.xv(x, col[u]);
        }
        for (; q < pn; q += 32) sum += dec.res_val(pb + q) * dec.xv(x, k.res_col[pb + q]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) atomicAdd(&y[row], static_cast<T>(sum));
        return;
    }
    // exact outlier correction in T (main_gpu_csr_bitbsr_spmv.cu:967-979)
    const int64_t i = static_cast<int64_t>(cta - heavy_ctas - chunk_ctas) * kThreads + threadIdx.x;
    if (i < num_out) atomicAdd(&y[orow[i]], oval[i] * x[ocol[i]]);
}

template <typename T>
void launch_segment(const KernelShape& k, const Bfp8Dec<T>& dec, const T* x, T* y, int grid, cudaStream_t s) {
    if constexpr (sizeof(T) == 8) {
        if (k.x_vec_ok && reinterpret_cast<uintptr_t>(x) % 32 == 0) {
            bfp8_segment_kernel<T, 2><<<grid, kThreads, 0, s>>>(k, dec, x, y);
            return;
        }
    }
    if (k.x_vec_ok) {
        bfp8_segment_kernel<T, 1><<<grid, kThreads, 0, s>>>(k, dec, x, y);
    } else {
        bfp8_segment_kernel<T, 0><<<grid, kThreads, 0, s>>>(k, dec, x, y);
    }
}

template <typename T, typename Dec, int SLOTS>
void launch_main(const KernelShape& k, const Dec& dec, int smem, const T* x, T* y, cudaStream_t s) {
    if constexpr (SLOTS == 0) {
        const int64_t rows = std::min<int64_t>(static_cast<int64_t>(k.nbr) * kBlockRows, k.rows) -
                             static_cast<int64_t>(k.br_begin) * kBlockRows;
        hybrid_row_kernel<T, Dec><<<grid_for(rows, kRowLanes * kThreads), kThreads, smem, s>>>(k, dec, x, y);
    } else if (SLOTS == 4 && is_bfp8<Dec>::value && k.l2_prefetch) {
        if constexpr (is_bfp8<Dec>::value) {
            const int grid = grid_for(static_cast<int64_t>(k.nbr) - k.br_begin, kLaneWarps);
            if (k.kb_avg >= kSegmentMinBlocks) {
                launch_segment<T>(k, dec, x, y, grid, s);
            } else if (k.x_vec_ok) {
                bfp8_block_lane_kernel<T, true><<<grid, kThreads, 0, s>>>(k, dec, x, y);
            } else {
                bfp8_block_lane_kernel<T, false><<<grid, kThreads, 0, s>>>(k, dec, x, y);
            }
        }
    } else {
        constexpr int G = 8 * SLOTS;
        const int grid = grid_for(static_cast<int64_t>(k.nbr) - k.br_begin, kThreads / G);
        if (k.x_vec_ok) {
            hybrid_main_kernel<T, Dec, SLOTS, true><<<grid, kThreads, smem, s>>>(k, dec, x, y);
        } else {
            hybrid_main_kernel<T, Dec, SLOTS, false><<<grid, kThreads, smem, s>>>(k, dec, x, y);
        }
    }
    CUDA_LAUNCH_OK();
}

template <typename T, typename Dec>
int launch_with(const KernelShape& k, Dec dec, size_t smem, const RouteValues& v, const void* xv,
                void* yv, cudaStream_t s) {
    const T* x = static_cast<const T*>(xv);
    T* y = static_cast<T*>(yv);
    int launches = 0;
    KernelShape kk = k;
    kk.x_vec_ok = (reinterpret_cast<uintptr_t>(xv) % 16 == 0) && (k.cols % 4 == 0);
    if (k.part != 2 && k.nbr > k.br_begin) {
        switch (k.slots) {
            case 0: launch_main<T, Dec, 0>(kk, dec, static_cast<int>(smem), x, y, s); break;
            case 1: launch_main<T, Dec, 1>(kk, dec, static_cast<int>(smem), x, y, s); break;
            case 2: launch_main<T, Dec, 2>(kk, dec, static_cast<int>(smem), x, y, s); break;
            default: launch_main<T, Dec, 4>(kk, dec, static_cast<int>(smem), x, y, s); break;
        }
        ++launches;
    }
    const int heavy_ctas = grid_for(k.num_heavy, kThreads / 32);
    const int chunk_ctas = grid_for(k.num_chunks, kThreads / 32);
    const int out_ctas = grid_for(v.num_outliers, kThreads);
    if (k.part != 1 && heavy_ctas + chunk_ctas + out_ctas > 0) {
        hybrid_overflow_kernel<T, Dec><<<heavy_ctas + chunk_ctas + out_ctas, kThreads, smem, s>>>(
            kk, dec, x, y, heavy_ctas, chunk_ctas, v.num_outliers, v.out_rows, v.out_cols,
            static_cast<const T*>(v.out_vals));
        CUDA_LAUNCH_OK();
        ++launches;
    }
    return launches;
}

template <typename T>
int launch_typed(const KernelShape& k, const RouteValues& v, const void* x, void* y,
                 cudaStream_t s) {
    switch (v.route) {
        case COVE_ROUTE_HYBRID: {
            RawDec<T> d{static_cast<const T*>(v.kept), static_cast<const T*>(v.res)};
            return launch_with<T>(k, d, 0, v, x, y, s);
        }
        case COVE_ROUTE_DICT_U8: {
            DictDec<T, uint8_t, true> d{static_cast<const uint8_t*>(v.kept),
                                        static_cast<const uint8_t*>(v.res),
                                        static_cast<const T*>(v.codebook), v.codebook_size};
            return launch_with<T>(k, d, static_cast<size_t>(v.codebook_size) * sizeof(T), v, x, y, s);
        }
        case COVE_ROUTE_DICT_U16: {
            DictDec<T, uint16_t, false> d{static_cast<const uint16_t*>(v.kept),
                                          static_cast<const uint16_t*>(v.res),
                                          static_cast<const T*>(v.codebook), v.codebook_size};
            return launch_with<T>(k, d, 0, v, x, y, s);
        }
        case COVE_ROUTE_BFP8:
        case COVE_ROUTE_BFP8_OUTLIER: {
            Bfp8Dec<T> d{static_cast<const int8_t*>(v.kept), static_cast<const uint16_t*>(v.res),
                         v.scale};
            return launch_with<T>(k, d, 0, v, x, y, s);
        }
        case COVE_ROUTE_TILE_CODE: {
            const auto* w = static_cast<const uint32_t*>(v.tile_words);
            const auto* cbk = static_cast<const T*>(v.codebook);
            const auto* res = static_cast<const T*>(v.res);
            switch (v.tile_bits) {
                case 1: return launch_with<T>(k, TileDec<T, 1>{w, cbk, res}, 0, v, x, y, s);
                case 2: return launch_with<T>(k, TileDec<T, 2>{w, cbk, res}, 0, v, x, y, s);
                case 4: return launch_with<T>(k, TileDec<T, 4>{w, cbk, res}, 0, v, x, y, s);
                case 8: return launch_with<T>(k, TileDec<T, 8>{w, cbk, res}, 0, v, x, y, s);
                case 16: return launch_with<T>(k, TileDec<T, 16>{w, cbk, res}, 0, v, x, y, s);
                default: COVE_THROW(COVE_ERR_UNSUPPORTED, "tile codes must have 1, 2, 4, 8 or 16 bits");
            }
        }
        case COVE_ROUTE_BF16_NNZ: {
            Bf16NnzDec<T> d{static_cast<const uint16_t*>(v.kept), static_cast<const uint16_t*>(v.res)};
            return launch_with<T>(k, d, 0, v, x, y, s);
        }
        case COVE_ROUTE_IMPLICIT_ONE:
            return launch_with<T>(k, ConstDec<T>{1.0}, 0, v, x, y, s);
        case COVE_ROUTE_CONST_C:
            return launch_with<T>(k, ConstDec<T>{v.value_scale}, 0, v, x, y, s);
        case COVE_ROUTE_SIGN2:
            return launch_with<T>(k, SignDec<T>{v.sign_masks, v.value_scale}, 0, v, x, y, s);
        case COVE_ROUTE_FP16_NNZ:
            return launch_with<T>(k, Fp16NnzDec<T>{static_cast<const uint16_t*>(v.kept)}, 0, v, x, y, s);
        case COVE_ROUTE_BFP4:
            return launch_with<T>(k, Bfp4Dec<T>{static_cast<const uint8_t*>(v.kept), v.scale}, 0, v, x, y, s);
        default:
            COVE_THROW(COVE_ERR_UNSUPPORTED, "unknown route");
    }
}

}  // namespace

int launch_hybrid_spmv(const KernelShape& k, const RouteValues& v, const void* x, void* y,
                       cudaStream_t s) {
    if (k.dtype == COVE_F64) return launch_typed<double>(k, v, x, y, s);
    return launch_typed<float>(k, v, x, y, s);
}

int hybrid_spmv_launch_count(const KernelShape& k, const RouteValues& v) {
    int n = k.nbr > 0 ? 1 : 0;
    if (k.num_heavy + k.num_chunks + v.num_outliers > 0) ++n;
    return n;
}

int choose_slots(int64_t nbr, int64_t kept_blocks, int64_t rows, int64_t residual_nnz,
                 const ResidualProfile* prof) {
    const double kb = nbr > 0 ? static_cast<double>(kept_blocks) / static_cast<double>(nbr) : 0.0;
    const double rr = rows > 0 ? static_cast<double>(residual_nnz) / static_cast<double>(rows) : 0.0;
    if (kb >= 8.0) return 4;
    if (prof == nullptr) {
        if (kb < 6.0 && rr < 6.0) return 0;
    } else if (kb < 6.0 && rows > 0) {
        // one lane per row: its light rows stay in the lanes, the longer rows go
        // to warp chunks, which pay only when those rows are long
        const int64_t heavy_nnz = residual_nnz - prof->light_nnz;
        const bool heavy_ok = heavy_nnz * 10 <= residual_nnz ||
                              heavy_nnz >= static_cast<int64_t>(kProfileHeavyAvg) * prof->heavy_rows;
        const double lr = static_cast<double>(prof->light_nnz) / static_cast<double>(rows);
        const bool diagonal = prof->diag_nnz * 2 >= prof->light_nnz;
        if (heavy_ok && (lr < 12.0 || (diagonal && lr < 24.0))) return 0;
    }
    if (rr >= 24.0) return 4;
    if (kb >= 1.5 || rr >= 2.5) return 2;
    return 1;
}

}  // namespace cove
