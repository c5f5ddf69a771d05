// convert.cu -- the 8x4 position converter on sm_100a.
//
// CSR -> full BitBSR 8x4 -> cost-gated CSR+BitBSR split -> packed block words,
// work items and long residual-row chunks.  Each stage is bit-exact with the
// reference's host pipeline:
//   convert_to_bitbsr                 structural/include/structural/convert.hpp:13-165
//   warp-direct GPU converter         structural/include/structural/gpu_convert.cuh:126-243
//   split (cost gate)                 structural/include/structural/csr_bitbsr_split.hpp:405-490
//   work items + packed words         structural/src/main_gpu_csr_bitbsr_spmv.cu:387-475
//                                     structural/include/structural/operators/bitbsr_spmv_8x4_common.cuh:95-117,199-267
//   long-row chunks                   structural/src/main_gpu_csr_bitbsr_spmv.cu:1155-1184
//
// Layout of the kernels: the converter runs one 8-lane group per block row
// (lane = row of the block row, four block rows per warp) and merges the
// eight sorted rows with __reduce_min_sync over the group, so all 32 lanes
// work.  The split runs one warp per block row with one lane per block; the
// eight per-row residual counts of a block are packed as 8-bit fields of a
// 64-bit word so one warp scan covers all eight rows.
#include "cove_convert.cuh"

#include <climits>

namespace cove {
namespace {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ bool is_zero(T v) { return v == T(0); }

__device__ __forceinline__ unsigned group_mask(int lane) { return 0xFFu << (lane & 24); }

// ---------------------------------------------------------------------------
// validation: monotonic row_ptr, columns in range, strictly increasing
// columns among the nonzero entries of each row.  Error bits: 1 row_ptr,
// 2 column range, 4 column order; the host reports them in that priority,
// the reference's order (csr.hpp:23-49 checks every row_ptr step, then every
// column's range; the converter then meets duplicates, convert.hpp:145-149).
// Bit 8 is no error: some row's columns decrease across a stored zero, so
// the converter may not binary-search rows for column ranges.
// ---------------------------------------------------------------------------

constexpr int kValidateLong = 256;  // longer rows are cut into units of kValidateSeg entries
constexpr int kValidateSeg = 2048;

template <typename T, typename RP>
__global__ void validate_csr_kernel(int32_t rows, int32_t cols, int64_t nnz, const RP* __restrict__ rp,
                                    const int32_t* __restrict__ ci, const T* __restrict__ v,
                                    int* __restrict__ err, int32_t* __restrict__ unit_row,
                                    int32_t* __restrict__ unit_seg, int64_t unit_cap,
                                    unsigned long long* __restrict__ n_units) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int64_t b = static_cast<int64_t>(rp[r]);
    const int64_t e = static_cast<int64_t>(rp[r + 1]);
    // rp[0] = 0 and rp[rows] = nnz are checked on the host, so an offset
    // outside [0, nnz] means row_ptr is not monotonic
    if (b > e || b < 0 || e > nnz) {
        atomicOr(err, 1);
        return;
    }
    if (e - b > kValidateLong) {
        // with monotonic offsets the units number at most
        // nnz / kValidateSeg + nnz / kValidateLong; more means another row
        // fails the check above
        const int64_t nseg = (e - b + kValidateSeg - 1) / kValidateSeg;
        const int64_t k0 = static_cast<int64_t>(atomicAdd(n_units, static_cast<unsigned long long>(nseg)));
        for (int64_t k = 0; k < nseg && k0 + k < unit_cap; ++k) {
            unit_row[k0 + k] = static_cast<int32_t>(r);
            unit_seg[k0 + k] = static_cast<int32_t>(k);
        }
        return;
    }
    int prev = -1;
    int prev_any = INT_MIN;
    int bits = 0;
    for (int64_t p = b; p < e; ++p) {
        const int c = ci[p];
        if (c < 0 || c >= cols) {
            bits |= 2;
            break;
        }
        if (c < prev_any) bits |= 8;
        prev_any = c;
        if (is_zero(v[p])) continue;
        if (c <= prev) bits |= 4;
        prev = c;
    }
    if (bits) atomicOr(err, bits);
}

// One warp per unit (kValidateSeg entries of a long row), a lane per entry:
// each entry is checked against the entry before it and, if nonzero, against
// the previous nonzero entry of the row (found by walking back over zeros;
// the walks of a row add up to at most its zero count).
template <typename T, typename RP>
__global__ void validate_long_rows_kernel(int32_t cols, const RP* __restrict__ rp,
                                          const int32_t* __restrict__ ci, const T* __restrict__ v,
                                          const int32_t* __restrict__ unit_row,
                                          const int32_t* __restrict__ unit_seg, int64_t unit_cap,
                                          const unsigned long long* __restrict__ n_units,
                                          int* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t nu = min(static_cast<int64_t>(*n_units), unit_cap);
    for (int64_t u = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; u < nu; u += nw) {
        const int32_t r = unit_row[u];
        const int64_t rb = static_cast<int64_t>(rp[r]);
        const int64_t re = static_cast<int64_t>(rp[r + 1]);
        const int64_t b = rb + static_cast<int64_t>(unit_seg[u]) * kValidateSeg;
        const int64_t e = b + kValidateSeg < re ? b + kValidateSeg : re;
        int bits = 0;
        for (int64_t p = b + lane; p < e; p += 32) {
            const int c = ci[p];
            if (c < 0 || c >= cols) bits |= 2;
            if (p > rb && c < ci[p - 1]) bits |= 8;
            if (!is_zero(v[p])) {
                int64_t q = p - 1;
                while (q >= rb && is_zero(v[q])) --q;
                if (q >= rb && c <= ci[q]) bits |= 4;
            }
        }
        bits = __reduce_or_sync(0xffffffffu, bits);
        if (lane == 0 && bits) atomicOr(err, bits);
    }
}

// ---------------------------------------------------------------------------
// full BitBSR: count and fill (one 8-lane group per block row)
// ---------------------------------------------------------------------------

template <typename T, typename RP>
struct RowCursor {
    int64_t pos, end;
    __device__ __forceinline__ void skip_zeros(const T* __restrict__ v) {
        while (pos < end && is_zero(v[pos])) ++pos;
    }
};

// Pieces: a block row with more than kPieceEntries CSR entries is cut into
// column ranges [c0, c1) on block boundaries, taken from its longest row at
// evenly spaced positions, and each piece is walked by its own 8-lane group
// (a single group over an R-MAT hub row would walk ~10^5 blocks serially).
// The ranges need every row's columns non-decreasing, stored zeros included;
// otherwise each block row is one piece.
constexpr int kPieceEntries = 1024;

template <typename RP>
__global__ void piece_count_kernel(int32_t rows, int32_t nbr, const RP* __restrict__ rp, int split,
                                   int32_t* __restrict__ np) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    const int64_t r0 = br * kBlockRows;
    const int64_t r1 = r0 + kBlockRows < rows ? r0 + kBlockRows : rows;
    const int64_t e = static_cast<int64_t>(rp[r1]) - static_cast<int64_t>(rp[r0]);
    np[br] = (split && e > kPieceEntries) ? static_cast<int32_t>((e + kPieceEntries - 1) / kPieceEntries) : 1;
}

template <typename RP>
__global__ void piece_bounds_kernel(int32_t rows, int32_t nbr, const RP* __restrict__ rp,
                                    const int32_t* __restrict__ ci, const int64_t* __restrict__ first,
                                    int32_t* __restrict__ pbr, int32_t* __restrict__ pc0,
                                    int32_t* __restrict__ pc1) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    const int64_t o = first[br];
    const int64_t n = first[br + 1] - o;
    if (n == 1) {
        pbr[o] = static_cast<int32_t>(br);
        pc0[o] = 0;
        pc1[o] = INT_MAX;
        return;
    }
    const int64_t r0 = br * kBlockRows;
    const int64_t r1 = r0 + kBlockRows < rows ? r0 + kBlockRows : rows;
    int64_t lb = 0, len = -1;
    for (int64_t r = r0; r < r1; ++r) {
        const int64_t b = static_cast<int64_t>(rp[r]);
        const int64_t l = static_cast<int64_t>(rp[r + 1]) - b;
        if (l > len) {
            len = l;
            lb = b;
        }
    }
    // n <= ceil(8 len / kPieceEntries) <= len, so every sampled position is in the row
    int32_t prev = 0;
    for (int64_t k = 0; k < n; ++k) {
        int32_t end = INT_MAX;
        if (k + 1 < n) {
            end = ci[lb + (k + 1) * len / n] & ~(kBlockCols - 1);
            if (end < prev) end = prev;
        }
        pbr[o + k] = static_cast<int32_t>(br);
        pc0[o + k] = prev;
        pc1[o + k] = end;
        prev = end;
    }
}

// First position in [lo, hi) whose column is >= c (columns non-decreasing).
__device__ __forceinline__ int64_t lower_bound_col(const int32_t* __restrict__ ci, int64_t lo, int64_t hi,
                                                   int32_t c) {
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (ci[mid] < c) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// This lane's CSR range inside piece j (its row of the piece's block row).
template <typename RP>
__device__ __forceinline__ void piece_row_range(int32_t rows, const RP* __restrict__ rp,
                                                const int32_t* __restrict__ ci, int32_t br, int32_t c0,
                                                int32_t c1, int l8, int64_t* b, int64_t* e) {
    const int64_t row = static_cast<int64_t>(br) * kBlockRows + l8;
    int64_t lo = 0, hi = 0;
    if (row < rows) {
        lo = static_cast<int64_t>(rp[row]);
        hi = static_cast<int64_t>(rp[row + 1]);
        if (c0 > 0) lo = lower_bound_col(ci, lo, hi, c0);
        if (c1 != INT_MAX) hi = lower_bound_col(ci, lo, hi, c1);
    }
    *b = lo;
    *e = hi;
}

template <typename T, typename RP>
__global__ void full_count_kernel(int32_t rows, int64_t npieces, const RP* __restrict__ rp,
                                  const int32_t* __restrict__ ci, const T* __restrict__ v,
                                  const int32_t* __restrict__ pbr, const int32_t* __restrict__ pc0,
                                  const int32_t* __restrict__ pc1,
                                  int32_t* __restrict__ block_counts,
                                  int32_t* __restrict__ nnz_counts) {
    const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t j = gt >> 3;
    const int lane = threadIdx.x & 31;
    const int l8 = lane & 7;
    const unsigned gm = group_mask(lane);
    if (j >= npieces) return;  // whole group leaves together
    int64_t b, e;
    piece_row_range(rows, rp, ci, pbr[j], pc0[j], pc1[j], l8, &b, &e);
    RowCursor<T, RP> cur{b, e};
    cur.skip_zeros(v);
    int nblocks = 0;
    int nnz = 0;
    while (true) {
        const int cand = cur.pos < cur.end ? (ci[cur.pos] >> 2) : INT_MAX;
        const int bc = __reduce_min_sync(gm, cand);
        if (bc == INT_MAX) break;
        ++nblocks;
        while (cur.pos < cur.end && (ci[cur.pos] >> 2) == bc) {
            ++nnz;
            ++cur.pos;
            cur.skip_zeros(v);
        }
    }
    const int total = __reduce_add_sync(gm, nnz);
    if (l8 == 0) {
        block_counts[j] = nblocks;
        nnz_counts[j] = total;
    }
}

template <typename T, typename RP>
__global__ void full_fill_kernel(int32_t rows, int64_t npieces, const RP* __restrict__ rp,
                                 const int32_t* __restrict__ ci, const T* __restrict__ v,
                                 const int32_t* __restrict__ pbr, const int32_t* __restrict__ pc0,
                                 const int32_t* __restrict__ pc1,
                                 const int32_t* __restrict__ piece_block_off,
                                 const int32_t* __restrict__ piece_val_off,
                                 int32_t* __restrict__ block_col_idx,
                                 uint32_t* __restrict__ bitmap, T* __restrict__ values) {
    const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t j = gt >> 3;
    const int lane = threadIdx.x & 31;
    const int l8 = lane & 7;
    const unsigned gm = group_mask(lane);
    if (j >= npieces) return;
    int64_t b, e;
    piece_row_range(rows, rp, ci, pbr[j], pc0[j], pc1[j], l8, &b, &e);
    RowCursor<T, RP> cur{b, e};
    cur.skip_zeros(v);
    int64_t block_id = piece_block_off[j];
    int64_t value_pos = piece_val_off[j];
    while (true) {
        const int cand = cur.pos < cur.end ? (ci[cur.pos] >> 2) : INT_MAX;
        const int bc = __reduce_min_sync(gm, cand);
        if (bc == INT_MAX) break;
        // this row's entries of block bc, in CSR order = bit order
        unsigned bits = 0;
        int cnt = 0;
        const int64_t start = cur.pos;
        while (cur.pos < cur.end && (ci[cur.pos] >> 2) == bc) {
            bits |= 1u << (l8 * kBlockCols + (ci[cur.pos] & 3));
            ++cnt;
            ++cur.pos;
            cur.skip_zeros(v);
        }
        // exclusive prefix of cnt over the 8 lanes of the group
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const int t = __shfl_up_sync(gm, incl, o, 8);
            if (l8 >= o) incl += t;
        }
        const int total = __shfl_sync(gm, incl, 7, 8);
        const unsigned bm = __reduce_or_sync(gm, bits);
        // copy values, skipping stored zeros
        int64_t dst = value_pos + (incl - cnt);
        for (int64_t p = start; p < cur.pos; ++p) {
            const T val = v[p];
            if (is_zero(val)) continue;
            values[dst++] = val;
        }
        if (l8 == 0) {
            block_col_idx[block_id] = bc;
            bitmap[block_id] = bm;
        }
        ++block_id;
        value_pos += total;
    }
}

// ---------------------------------------------------------------------------
// split: count and fill (one warp per block row, one lane per block)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint64_t nibble_counts(uint32_t bm) {
    uint64_t packed = 0;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        packed |= static_cast<uint64_t>(__popc((bm >> (4 * r)) & 0xFu)) << (8 * r);
    }
    return packed;
}

__device__ __forceinline__ uint64_t warp_incl_scan_u64(uint64_t v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

__device__ __forceinline__ int warp_incl_scan_i32(int v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Block rows with more than kSplitPiece blocks are split as pieces of
// kSplitPiece blocks, a warp each (an R-MAT hub block row holds ~10^5
// blocks: one warp would walk them serially); the others keep one warp per
// block row.  Both walk their blocks with the loops below.
constexpr int kSplitPiece = 2048;

struct SplitCounts {
    int kc = 0, kn = 0, rb = 0, sb = 0, sn = 0, fn = 0;
    int run = 0;  // lane r < 8: residual entries of row r
};

__device__ __forceinline__ SplitCounts split_count_range(int b0, int b1, int32_t threshold,
                                                         unsigned long long move_mask,
                                                         const uint32_t* __restrict__ bitmap, int lane) {
    SplitCounts c;
    for (int base = b0; base < b1; base += 32) {
        const int b = base + lane;
        const bool valid = b < b1;
        const uint32_t bm = valid ? bitmap[b] : 0u;
        const int bn = __popc(bm);
        const bool small = valid && bn <= threshold;
        const bool moved = small && ((move_mask >> bn) & 1ULL);
        const bool kept = valid && !moved;
        c.kc += __popc(__ballot_sync(0xffffffffu, kept));
        c.kn += __reduce_add_sync(0xffffffffu, kept ? bn : 0);
        c.rb += __popc(__ballot_sync(0xffffffffu, moved));
        c.sb += __popc(__ballot_sync(0xffffffffu, small && !moved));
        c.sn += __reduce_add_sync(0xffffffffu, (small && !moved) ? bn : 0);
        c.fn += __reduce_add_sync(0xffffffffu, bn);
        uint64_t packed = moved ? nibble_counts(bm) : 0ULL;
        packed = warp_incl_scan_u64(packed, lane);
        const uint64_t tot = __shfl_sync(0xffffffffu, packed, 31);
        c.run += static_cast<int>((tot >> (8 * (lane & 7))) & 0xFFu);
    }
    return c;
}

__global__ void split_count_kernel(int32_t rows, int32_t nbr, int32_t threshold,
                                   unsigned long long move_mask,
                                   const int32_t* __restrict__ brp,
                                   const uint32_t* __restrict__ bitmap,
                                   int32_t* __restrict__ kept_count,
                                   int32_t* __restrict__ kept_nnz,
                                   int32_t* __restrict__ res_count,
                                   int32_t* __restrict__ res_blocks,
                                   int32_t* __restrict__ skipped_blocks,
                                   int32_t* __restrict__ skipped_nnz) {
    const int64_t br = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (br >= nbr) return;
    const int b0 = brp[br], b1 = brp[br + 1];
    if (b1 - b0 > kSplitPiece) return;  // counted by pieces
    const SplitCounts c = split_count_range(b0, b1, threshold, move_mask, bitmap, lane);
    if (lane == 0) {
        kept_count[br] = c.kc;
        kept_nnz[br] = c.kn;
        res_blocks[br] = c.rb;
        skipped_blocks[br] = c.sb;
        skipped_nnz[br] = c.sn;
    }
    if (lane < 8) {
        const int64_t row = br * kBlockRows + lane;
        if (row < rows) res_count[row] = c.run;
    }
}

// Pieces of the heavy block rows: count them, then list (block row, block range).
__global__ void split_piece_count_kernel(int32_t nbr, const int32_t* __restrict__ brp, int32_t* __restrict__ np) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    const int n = brp[br + 1] - brp[br];
    np[br] = n > kSplitPiece ? (n + kSplitPiece - 1) / kSplitPiece : 0;
}

__global__ void split_piece_list_kernel(int32_t nbr, const int32_t* __restrict__ brp,
                                        const int64_t* __restrict__ first, int32_t* __restrict__ pbr,
                                        int32_t* __restrict__ pb0, int32_t* __restrict__ pb1) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    const int b0 = brp[br], b1 = brp[br + 1];
    int64_t o = first[br];
    for (int b = b0; o < first[br + 1]; b += kSplitPiece, ++o) {
        pbr[o] = static_cast<int32_t>(br);
        pb0[o] = b;
        pb1[o] = min(b + kSplitPiece, b1);
    }
}

// Per piece: kept blocks, kept nnz, full nnz, moved / skipped counts and the
// eight rows' residual counts (pcnt[p * 14 + ...]).
constexpr int kPieceFields = 14;

__global__ void split_piece_count_pass(int64_t npieces, int32_t threshold, unsigned long long move_mask,
                                       const int32_t* __restrict__ pb0, const int32_t* __restrict__ pb1,
                                       const uint32_t* __restrict__ bitmap, int32_t* __restrict__ pcnt) {
    const int64_t p = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (p >= npieces) return;
    const SplitCounts c = split_count_range(pb0[p], pb1[p], threshold, move_mask, bitmap, lane);
    int32_t* o = pcnt + p * kPieceFields;
    if (lane == 0) {
        o[0] = c.kc;
        o[1] = c.kn;
        o[2] = c.rb;
        o[3] = c.sb;
        o[4] = c.sn;
        o[5] = c.fn;
    }
    if (lane < 8) o[6 + lane] = c.run;
}

// A heavy block row's totals (into the per-block-row and per-row counts the
// scans read) and each piece's exclusive prefixes within its block row
// (pcnt fields 0, 1, 5 and 6..13 are replaced by their prefixes).
__global__ void split_piece_sum_kernel(int32_t rows, int32_t nbr, const int64_t* __restrict__ first,
                                       int32_t* __restrict__ pcnt, int32_t* __restrict__ kept_count,
                                       int32_t* __restrict__ kept_nnz, int32_t* __restrict__ res_count,
                                       int32_t* __restrict__ res_blocks, int32_t* __restrict__ skipped_blocks,
                                       int32_t* __restrict__ skipped_nnz) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    const int64_t p0 = first[br], p1 = first[br + 1];
    if (p0 == p1) return;
    int kc = 0, kn = 0, rb = 0, sb = 0, sn = 0, fn = 0;
    int run[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t p = p0; p < p1; ++p) {
        int32_t* o = pcnt + p * kPieceFields;
        const int c0 = o[0], c1 = o[1], c5 = o[5];
        o[0] = kc;
        o[1] = kn;
        o[5] = fn;
        kc += c0;
        kn += c1;
        fn += c5;
        rb += o[2];
        sb += o[3];
        sn += o[4];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int t = o[6 + r];
            o[6 + r] = run[r];
            run[r] += t;
        }
    }
    kept_count[br] = kc;
    kept_nnz[br] = kn;
    res_blocks[br] = rb;
    skipped_blocks[br] = sb;
    skipped_nnz[br] = sn;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int64_t row = br * kBlockRows + r;
        if (row < rows) res_count[row] = run[r];
    }
}

// Blocks [b0, b1) of block row br: kept blocks to kb / kv onward, moved
// blocks' entries to the rows' residual positions s_base[0..7] onward
// (shared, one set per warp; advanced here).  fv: the first value of b0.
template <typename T>
__device__ __forceinline__ void split_fill_range(int b0, int b1, int kb, int kv, int fv, int* s_base,
                                                 int32_t threshold, unsigned long long move_mask,
                                                 const int32_t* __restrict__ full_col,
                                                 const uint32_t* __restrict__ bitmap,
                                                 const T* __restrict__ full_values,
                                                 int32_t* __restrict__ kept_col,
                                                 uint32_t* __restrict__ kept_bitmap,
                                                 T* __restrict__ kept_values, int32_t* __restrict__ res_col,
                                                 T* __restrict__ res_values, int lane) {
    const unsigned lt = (1u << lane) - 1u;
    for (int base = b0; base < b1; base += 32) {
        const int b = base + lane;
        const bool valid = b < b1;
        const uint32_t bm = valid ? bitmap[b] : 0u;
        const int bn = __popc(bm);
        const bool moved = valid && bn <= threshold && ((move_mask >> bn) & 1ULL);
        const bool kept = valid && !moved;
        const unsigned kballot = __ballot_sync(0xffffffffu, kept);
        const int fv_incl = warp_incl_scan_i32(bn, lane);
        const int kv_incl = warp_incl_scan_i32(kept ? bn : 0, lane);
        const uint64_t packed = moved ? nibble_counts(bm) : 0ULL;
        const uint64_t p_incl = warp_incl_scan_u64(packed, lane);
        const uint64_t p_excl = p_incl - packed;
        const int my_fv = fv + fv_incl - bn;
        if (kept) {
            const int dst = kb + __popc(kballot & lt);
            kept_col[dst] = full_col[b];
            kept_bitmap[dst] = bm;
            const int vdst = kv + kv_incl - bn;
            for (int k = 0; k < bn; ++k) kept_values[vdst + k] = full_values[my_fv + k];
        } else if (moved) {
            const int bc = full_col[b];
            uint32_t rest = bm;
            int rank = 0;
            while (rest) {
                const int bit = __ffs(rest) - 1;
                const int r = bit >> 2;
                const int c = bit & 3;
                const uint32_t nib = (bm >> (4 * r)) & 0xFu;
                const int within = __popc(nib & ((1u << c) - 1u));
                const int dst = s_base[r] + static_cast<int>((p_excl >> (8 * r)) & 0xFFu) + within;
                res_col[dst] = bc * kBlockCols + c;
                res_values[dst] = full_values[my_fv + rank];
                ++rank;
                rest &= rest - 1u;
            }
        }
        const uint64_t tot = __shfl_sync(0xffffffffu, p_incl, 31);
        kb += __popc(kballot);
        kv += __shfl_sync(0xffffffffu, kv_incl, 31);
        fv += __shfl_sync(0xffffffffu, fv_incl, 31);
        __syncwarp();
        if (lane < 8) s_base[lane] += static_cast<int>((tot >> (8 * lane)) & 0xFFu);
        __syncwarp();
    }
}

template <typename T>
__global__ void split_fill_kernel(int32_t rows, int32_t nbr, int32_t threshold,
                                  unsigned long long move_mask,
                                  const int32_t* __restrict__ brp,
                                  const int32_t* __restrict__ brvp,
                                  const int32_t* __restrict__ full_col,
                                  const uint32_t* __restrict__ bitmap,
                                  const T* __restrict__ full_values,
                                  const int32_t* __restrict__ kept_brp,
                                  const int32_t* __restrict__ kept_brvp,
                                  const int32_t* __restrict__ res_rp,
                                  int32_t* __restrict__ kept_col,
                                  uint32_t* __restrict__ kept_bitmap,
                                  T* __restrict__ kept_values,
                                  int32_t* __restrict__ res_col,
                                  T* __restrict__ res_values) {
    __shared__ int s_base[kThreads / 32][8];
    const int64_t br = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    if (br >= nbr) return;
    const int b0 = brp[br], b1 = brp[br + 1];
    if (b1 - b0 > kSplitPiece) return;  // filled by pieces
    if (lane < 8) {
        const int64_t row = br * kBlockRows + lane;
        s_base[w][lane] = row < rows ? res_rp[row] : 0;
    }
    __syncwarp();
    split_fill_range<T>(b0, b1, kept_brp[br], kept_brvp[br], brvp[br], s_base[w], threshold, move_mask,
                        full_col, bitmap, full_values, kept_col, kept_bitmap, kept_values, res_col, res_values,
                        lane);
}

template <typename T>
__global__ void split_piece_fill_kernel(int32_t rows, int64_t npieces, int32_t threshold,
                                        unsigned long long move_mask, const int32_t* __restrict__ pbr,
                                        const int32_t* __restrict__ pb0, const int32_t* __restrict__ pb1,
                                        const int32_t* __restrict__ pcnt, const int32_t* __restrict__ brvp,
                                        const int32_t* __restrict__ full_col,
                                        const uint32_t* __restrict__ bitmap,
                                        const T* __restrict__ full_values,
                                        const int32_t* __restrict__ kept_brp,
                                        const int32_t* __restrict__ kept_brvp,
                                        const int32_t* __restrict__ res_rp, int32_t* __restrict__ kept_col,
                                        uint32_t* __restrict__ kept_bitmap, T* __restrict__ kept_values,
                                        int32_t* __restrict__ res_col, T* __restrict__ res_values) {
    __shared__ int s_base[kThreads / 32][8];
    const int64_t p = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    if (p >= npieces) return;
    const int32_t* o = pcnt + p * kPieceFields;
    const int64_t br = pbr[p];
    if (lane < 8) {
        const int64_t row = br * kBlockRows + lane;
        s_base[w][lane] = row < rows ? res_rp[row] + o[6 + lane] : 0;
    }
    __syncwarp();
    split_fill_range<T>(pb0[p], pb1[p], kept_brp[br] + o[0], kept_brvp[br] + o[1], brvp[br] + o[5], s_base[w],
                        threshold, move_mask, full_col, bitmap, full_values, kept_col, kept_bitmap, kept_values,
                        res_col, res_values, lane);
}

// ---------------------------------------------------------------------------
// block popcounts (block_val_ptr), packed words, work items, long chunks
// ---------------------------------------------------------------------------

__global__ void popc_kernel(int64_t n, const uint32_t* __restrict__ bitmap,
                            int32_t* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __popc(bitmap[i]);
}

__global__ void pack_words_kernel(int64_t n, const int32_t* __restrict__ col,
                                  const uint32_t* __restrict__ bitmap,
                                  uint64_t* __restrict__ words) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) words[i] = pack_word(static_cast<uint32_t>(col[i]), bitmap[i], false);
}

__device__ __forceinline__ void lb_shape(int count, int chunk, int split, int style,
                                         int* pieces, bool* atomic, int* eff) {
    if (count == 0) {
        *pieces = style == COVE_LB_HYBRID ? 1 : 0;
        *atomic = false;
        *eff = 0;
        return;
    }
    if (style == COVE_LB_HYBRID) {
        *atomic = count > split;
        *eff = *atomic ? chunk : count;
        *pieces = (count + *eff - 1) / *eff;
    } else {
        *pieces = count <= split ? 1 : (count + chunk - 1) / chunk;
        *atomic = *pieces > 1;
        *eff = *atomic ? chunk : count;
    }
}

__global__ void lb_count_kernel(int32_t nbr, const int32_t* __restrict__ kbrp, int chunk,
                                int split, int style, int32_t* __restrict__ out) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    int pieces, eff;
    bool atomic;
    lb_shape(kbrp[br + 1] - kbrp[br], chunk, split, style, &pieces, &atomic, &eff);
    out[br] = pieces;
}

__global__ void lb_fill_kernel(int32_t nbr, const int32_t* __restrict__ kbrp,
                               const int32_t* __restrict__ kbrvp,
                               const uint32_t* __restrict__ kbitmap,
                               const int32_t* __restrict__ item_rp, int chunk, int split,
                               int style, uint64_t* __restrict__ words,
                               WorkItem* __restrict__ items) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    const int rs = kbrp[br], re = kbrp[br + 1];
    int pieces, eff;
    bool atomic;
    lb_shape(re - rs, chunk, split, style, &pieces, &atomic, &eff);
    int out = item_rp[br];
    if (re == rs) {
        if (pieces == 1) items[out] = WorkItem{static_cast<uint32_t>(br), static_cast<uint32_t>(rs), 0u,
                                               static_cast<uint32_t>(kbrvp[br])};
        return;
    }
    int blk = rs;
    int vp = kbrvp[br];
    while (blk < re) {
        const int c = min(eff, re - blk);
        items[out++] = WorkItem{static_cast<uint32_t>(br), static_cast<uint32_t>(blk),
                                static_cast<uint32_t>(c), static_cast<uint32_t>(vp)};
        if (atomic) words[blk] |= kFlagBit;
        for (int i = 0; i < c; ++i) vp += __popc(kbitmap[blk + i]);
        blk += c;
    }
}

__global__ void chunk_count_kernel(int32_t rows, const int32_t* __restrict__ rp, int tau,
                                   int chunk_nnz, int32_t* __restrict__ out,
                                   int32_t* __restrict__ long_flag) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int len = rp[r + 1] - rp[r];
    const bool lg = tau > 0 && len > tau;
    out[r] = lg ? (len + chunk_nnz - 1) / chunk_nnz : 0;
    long_flag[r] = lg ? 1 : 0;
}

__global__ void chunk_fill_kernel(int32_t rows, const int32_t* __restrict__ rp, int tau,
                                  int chunk_nnz, const int64_t* __restrict__ crp,
                                  int32_t* __restrict__ crow, int32_t* __restrict__ cbegin,
                                  int32_t* __restrict__ ccount) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int b = rp[r];
    const int len = rp[r + 1] - b;
    if (!(tau > 0 && len > tau)) return;
    int64_t o = crp[r];
    for (int off = 0; off < len; off += chunk_nnz) {
        crow[o] = static_cast<int32_t>(r);
        cbegin[o] = b + off;
        ccount[o] = min(chunk_nnz, len - off);
        ++o;
    }
}

int32_t checked_i32(int64_t v, const char* what) {
    if (v > INT32_MAX) {
        COVE_THROW(COVE_ERR_OVERFLOW, std::string(what) + " exceeds int32 offsets (" +
                                          std::to_string(v) + ")");
    }
    return static_cast<int32_t>(v);
}

}  // namespace

// ---------------------------------------------------------------------------
// host drivers
// ---------------------------------------------------------------------------

template <typename T>
bool validate_csr(const cove_csr_desc& d, cudaStream_t s) {
    if (d.rows < 0 || d.cols < 0 || d.nnz < 0) {
        COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "CSR dimensions must be non-negative");
    }
    if (d.rows > 0 && d.row_ptr == nullptr) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "CSR row_ptr is null");
    if (d.nnz > 0 && (d.col_idx == nullptr || d.values == nullptr)) {
        COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "CSR col_idx/values are null");
    }
    // endpoints
    int64_t first = 0, last = 0;
    if (d.row_ptr_i32) {
        int32_t a = 0, b = 0;
        CUDA_OK(cudaMemcpyAsync(&a, d.row_ptr, 4, cudaMemcpyDeviceToHost, s));
        CUDA_OK(cudaMemcpyAsync(&b, static_cast<const int32_t*>(d.row_ptr) + d.rows, 4,
                                cudaMemcpyDeviceToHost, s));
        CUDA_OK(cudaStreamSynchronize(s));
        first = a;
        last = b;
    } else {
        CUDA_OK(cudaMemcpyAsync(&first, d.row_ptr, 8, cudaMemcpyDeviceToHost, s));
        CUDA_OK(cudaMemcpyAsync(&last, static_cast<const int64_t*>(d.row_ptr) + d.rows, 8,
                                cudaMemcpyDeviceToHost, s));
        CUDA_OK(cudaStreamSynchronize(s));
    }
    if (first != 0) COVE_THROW(COVE_ERR_INVALID_INPUT, "CSR row_ptr must start at zero");
    if (last != d.nnz) COVE_THROW(COVE_ERR_INVALID_INPUT, "CSR row_ptr.back must equal nnz");
    if (d.rows == 0) return true;
    DevBuf err, units, urow, useg;
    err.alloc(sizeof(int));
    alloc_n<unsigned long long>(units, 1);
    const int64_t unit_cap = d.nnz / kValidateSeg + d.nnz / kValidateLong + 1;
    alloc_n<int32_t>(urow, unit_cap);
    alloc_n<int32_t>(useg, unit_cap);
    CUDA_OK(cudaMemsetAsync(err.p, 0, sizeof(int), s));
    CUDA_OK(cudaMemsetAsync(units.p, 0, sizeof(unsigned long long), s));
    const T* v = static_cast<const T*>(d.values);
    const int long_grid = 148 * 8;
    if (d.row_ptr_i32) {
        const int32_t* rp = static_cast<const int32_t*>(d.row_ptr);
        validate_csr_kernel<T, int32_t><<<grid_for(d.rows, kThreads), kThreads, 0, s>>>(
            d.rows, d.cols, d.nnz, rp, d.col_idx, v, err.as<int>(), urow.as<int32_t>(), useg.as<int32_t>(),
            unit_cap, units.as<unsigned long long>());
        CUDA_LAUNCH_OK();
        validate_long_rows_kernel<T, int32_t><<<long_grid, kThreads, 0, s>>>(
            d.cols, rp, d.col_idx, v, urow.as<int32_t>(), useg.as<int32_t>(), unit_cap,
            units.as<unsigned long long>(), err.as<int>());
    } else {
        const int64_t* rp = static_cast<const int64_t*>(d.row_ptr);
        validate_csr_kernel<T, int64_t><<<grid_for(d.rows, kThreads), kThreads, 0, s>>>(
            d.rows, d.cols, d.nnz, rp, d.col_idx, v, err.as<int>(), urow.as<int32_t>(), useg.as<int32_t>(),
            unit_cap, units.as<unsigned long long>());
        CUDA_LAUNCH_OK();
        validate_long_rows_kernel<T, int64_t><<<long_grid, kThreads, 0, s>>>(
            d.cols, rp, d.col_idx, v, urow.as<int32_t>(), useg.as<int32_t>(), unit_cap,
            units.as<unsigned long long>(), err.as<int>());
    }
    CUDA_LAUNCH_OK();
    int h = 0;
    CUDA_OK(cudaMemcpyAsync(&h, err.p, sizeof(int), cudaMemcpyDeviceToHost, s));
    CUDA_OK(cudaStreamSynchronize(s));
    if (h & 1) COVE_THROW(COVE_ERR_INVALID_INPUT, "CSR row_ptr must be monotonic");
    if (h & 2) COVE_THROW(COVE_ERR_INVALID_INPUT, "CSR column index out of range");
    if (h & 4) {
        COVE_THROW(COVE_ERR_INVALID_INPUT,
                   "CSR columns must be strictly increasing within a row "
                   "(duplicate CSR entry maps to the same BitBSR bit)");
    }
    return (h & 8) == 0;
}

namespace {

__global__ void piece_rows_kernel(int32_t nbr, const int64_t* __restrict__ first,
                                  const int32_t* __restrict__ boff, const int32_t* __restrict__ voff,
                                  int32_t* __restrict__ brp, int32_t* __restrict__ brvp) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br > nbr) return;
    const int64_t j = first[br];
    brp[br] = boff[j];
    brvp[br] = voff[j];
}

// Pieces of the block rows with their block / nnz counts and offsets.
struct PieceCounts {
    int64_t n = 0, num_blocks = 0, nnz = 0;
    DevBuf first;       // int64 nbr+1: first piece of each block row
    DevBuf br, c0, c1;  // int32 n
    DevBuf boff, voff;  // int32 n+1: exclusive scans of the block / nnz counts
};

template <typename T, typename RP>
void count_pieces(const cove_csr_desc& d, const RP* rp, bool split, PieceCounts& p, cudaStream_t s) {
    const int32_t nbr = (d.rows + kBlockRows - 1) / kBlockRows;
    DevBuf np;
    alloc_n<int32_t>(np, nbr);
    alloc_n<int64_t>(p.first, nbr + 1);
    piece_count_kernel<RP><<<grid_for(nbr, kThreads), kThreads, 0, s>>>(d.rows, nbr, rp, split ? 1 : 0,
                                                                         np.as<int32_t>());
    CUDA_LAUNCH_OK();
    p.n = exclusive_scan_total<int32_t, int64_t>(np.as<int32_t>(), p.first.as<int64_t>(), nbr, s);
    alloc_n<int32_t>(p.br, p.n);
    alloc_n<int32_t>(p.c0, p.n);
    alloc_n<int32_t>(p.c1, p.n);
    piece_bounds_kernel<RP><<<grid_for(nbr, kThreads), kThreads, 0, s>>>(
        d.rows, nbr, rp, d.col_idx, p.first.as<int64_t>(), p.br.as<int32_t>(), p.c0.as<int32_t>(),
        p.c1.as<int32_t>());
    CUDA_LAUNCH_OK();
    DevBuf counts, nnzc;
    alloc_n<int32_t>(counts, p.n);
    alloc_n<int32_t>(nnzc, p.n);
    full_count_kernel<T, RP><<<grid_for(p.n * 8, kThreads), kThreads, 0, s>>>(
        d.rows, p.n, rp, d.col_idx, static_cast<const T*>(d.values), p.br.as<int32_t>(),
        p.c0.as<int32_t>(), p.c1.as<int32_t>(), counts.as<int32_t>(), nnzc.as<int32_t>());
    CUDA_LAUNCH_OK();
    alloc_n<int32_t>(p.boff, p.n + 1);
    alloc_n<int32_t>(p.voff, p.n + 1);
    // the scans carry int64 totals, so an int32 overflow is detected
    p.num_blocks = checked_i32(exclusive_scan_total<int32_t, int32_t>(counts.as<int32_t>(), p.boff.as<int32_t>(),
                                                                      p.n, s),
                               "BitBSR block count");
    p.nnz = checked_i32(exclusive_scan_total<int32_t, int32_t>(nnzc.as<int32_t>(), p.voff.as<int32_t>(), p.n, s),
                        "BitBSR nnz");
}

template <typename T>
void count_pieces(const cove_csr_desc& d, bool split, PieceCounts& p, cudaStream_t s) {
    if (d.row_ptr_i32) count_pieces<T, int32_t>(d, static_cast<const int32_t*>(d.row_ptr), split, p, s);
    else count_pieces<T, int64_t>(d, static_cast<const int64_t*>(d.row_ptr), split, p, s);
}

template <typename T>
void fill_pieces(const cove_csr_desc& d, const PieceCounts& p, int32_t* col, uint32_t* bitmap, T* values,
                 cudaStream_t s) {
    if (p.num_blocks == 0) return;
    const T* v = static_cast<const T*>(d.values);
    const int grid = grid_for(p.n * 8, kThreads);
    if (d.row_ptr_i32) {
        full_fill_kernel<T, int32_t><<<grid, kThreads, 0, s>>>(
            d.rows, p.n, static_cast<const int32_t*>(d.row_ptr), d.col_idx, v, p.br.as<int32_t>(),
            p.c0.as<int32_t>(), p.c1.as<int32_t>(), p.boff.as<int32_t>(), p.voff.as<int32_t>(), col, bitmap,
            values);
    } else {
        full_fill_kernel<T, int64_t><<<grid, kThreads, 0, s>>>(
            d.rows, p.n, static_cast<const int64_t*>(d.row_ptr), d.col_idx, v, p.br.as<int32_t>(),
            p.c0.as<int32_t>(), p.c1.as<int32_t>(), p.boff.as<int32_t>(), p.voff.as<int32_t>(), col, bitmap,
            values);
    }
    CUDA_LAUNCH_OK();
}

}  // namespace

template <typename T>
void bitbsr_count(const cove_csr_desc& d, bool split, int32_t* brp, int32_t* brvp, int64_t* num_blocks,
                  int64_t* nnz, cudaStream_t s) {
    const int32_t nbr = (d.rows + kBlockRows - 1) / kBlockRows;
    if (nbr == 0) {
        CUDA_OK(cudaMemsetAsync(brp, 0, sizeof(int32_t), s));
        CUDA_OK(cudaMemsetAsync(brvp, 0, sizeof(int32_t), s));
        *num_blocks = 0;
        *nnz = 0;
        return;
    }
    PieceCounts p;
    count_pieces<T>(d, split, p, s);
    piece_rows_kernel<<<grid_for(static_cast<int64_t>(nbr) + 1, kThreads), kThreads, 0, s>>>(
        nbr, p.first.as<int64_t>(), p.boff.as<int32_t>(), p.voff.as<int32_t>(), brp, brvp);
    CUDA_LAUNCH_OK();
    *num_blocks = p.num_blocks;
    *nnz = p.nnz;
}

template <typename T>
void bitbsr_fill(const cove_csr_desc& d, bool split, int32_t* col, uint32_t* bitmap, T* values,
                 cudaStream_t s) {
    const int32_t nbr = (d.rows + kBlockRows - 1) / kBlockRows;
    if (nbr == 0 || d.nnz == 0) return;
    PieceCounts p;  // the pieces' offsets are recounted: they are not the caller's per-block-row ones
    count_pieces<T>(d, split, p, s);
    fill_pieces<T>(d, p, col, bitmap, values, s);
}

template <typename T>
void build_full_bitbsr(const cove_csr_desc& d, bool split, FullBitBsr& out, cudaStream_t s) {
    out.rows = d.rows;
    out.cols = d.cols;
    out.nbr = (d.rows + kBlockRows - 1) / kBlockRows;
    alloc_n<int32_t>(out.block_row_ptr, out.nbr + 1);
    alloc_n<int32_t>(out.block_row_val_ptr, out.nbr + 1);
    if (out.nbr == 0) {
        CUDA_OK(cudaMemsetAsync(out.block_row_ptr.p, 0, sizeof(int32_t), s));
        CUDA_OK(cudaMemsetAsync(out.block_row_val_ptr.p, 0, sizeof(int32_t), s));
        out.num_blocks = 0;
        out.nnz = 0;
        return;
    }
    PieceCounts p;
    count_pieces<T>(d, split, p, s);
    piece_rows_kernel<<<grid_for(static_cast<int64_t>(out.nbr) + 1, kThreads), kThreads, 0, s>>>(
        out.nbr, p.first.as<int64_t>(), p.boff.as<int32_t>(), p.voff.as<int32_t>(),
        out.block_row_ptr.as<int32_t>(), out.block_row_val_ptr.as<int32_t>());
    CUDA_LAUNCH_OK();
    out.num_blocks = p.num_blocks;
    out.nnz = p.nnz;
    alloc_n<int32_t>(out.block_col_idx, out.num_blocks);
    alloc_n<uint32_t>(out.bitmap, out.num_blocks);
    alloc_n<T>(out.values, out.nnz);
    fill_pieces<T>(d, p, out.block_col_idx.as<int32_t>(), out.bitmap.as<uint32_t>(), out.values.as<T>(), s);
}

void pack_words(int64_t nb, const int32_t* col, const uint32_t* bitmap, uint64_t* words,
                cudaStream_t s) {
    if (nb <= 0) return;
    pack_words_kernel<<<grid_for(nb, kThreads), kThreads, 0, s>>>(nb, col, bitmap, words);
    CUDA_LAUNCH_OK();
}

int64_t lb_count(int32_t nbr, const int32_t* brp, int chunk, int split, int style,
                 int32_t* item_rp, cudaStream_t s) {
    DevBuf cnt;
    alloc_n<int32_t>(cnt, nbr);
    if (nbr > 0) {
        lb_count_kernel<<<grid_for(nbr, kThreads), kThreads, 0, s>>>(nbr, brp, chunk, split, style,
                                                                     cnt.as<int32_t>());
        CUDA_LAUNCH_OK();
    }
    return checked_i32(exclusive_scan_total<int32_t, int32_t>(cnt.as<int32_t>(), item_rp, nbr, s),
                       "work items");
}

void lb_fill(int32_t nbr, const int32_t* brp, const int32_t* brvp, const uint32_t* bitmap,
             const int32_t* item_rp, int chunk, int split, int style, uint64_t* words,
             WorkItem* items, cudaStream_t s) {
    if (nbr <= 0) return;
    lb_fill_kernel<<<grid_for(nbr, kThreads), kThreads, 0, s>>>(nbr, brp, brvp, bitmap, item_rp,
                                                                chunk, split, style, words, items);
    CUDA_LAUNCH_OK();
}

// CsrBitBsrSplitCostModel::should_move_to_residual (csr_bitbsr_split.hpp:66-73)
// tabulated for every block population 0..32 on the host, with plain double
// arithmetic, so the device applies exactly the reference's decisions; the
// mask policy hands over a caller's own table.
unsigned long long move_mask_for(const cove_plan_opts& o) {
    if (o.split_policy == COVE_SPLIT_MASK) return o.move_mask & ((1ULL << 33) - 1);
    unsigned long long m = 0;
    for (int bn = 0; bn <= 32; ++bn) {
        bool move = true;
        if (o.split_policy == COVE_SPLIT_COST_GATED) {
            volatile double nnz = static_cast<double>(bn);
            volatile double bitmap_cost = o.cost_bitmap_block + o.cost_bitmap_nnz * nnz;
            volatile double csr_cost = o.cost_csr_block + o.cost_csr_nnz * nnz;
            move = csr_cost < bitmap_cost;
        } else if (o.split_policy == COVE_SPLIT_NONE) {
            move = false;
        }
        if (move) m |= 1ULL << bn;
    }
    return m;
}

template <typename T>
void build_split(const FullBitBsr& f, const cove_plan_opts& o, SplitParts& out, cudaStream_t s) {
    const int32_t nbr = f.nbr;
    const int32_t rows = f.rows;
    const unsigned long long mm = move_mask_for(o);
    const int32_t thr = o.split_policy == COVE_SPLIT_NONE ? -1 : o.residual_threshold;
    DevBuf kc, kn, rc, rb, sb, sn;
    alloc_n<int32_t>(kc, nbr);
    alloc_n<int32_t>(kn, nbr);
    alloc_n<int32_t>(rb, nbr);
    alloc_n<int32_t>(sb, nbr);
    alloc_n<int32_t>(sn, nbr);
    alloc_n<int32_t>(rc, rows);
    CUDA_OK(cudaMemsetAsync(rc.p, 0, rc.bytes, s));
    const int grid = grid_for(static_cast<int64_t>(nbr) * 32, kThreads);
    if (nbr > 0) {
        split_count_kernel<<<grid, kThreads, 0, s>>>(
            rows, nbr, thr, mm, f.block_row_ptr.as<int32_t>(), f.bitmap.as<uint32_t>(),
            kc.as<int32_t>(), kn.as<int32_t>(), rc.as<int32_t>(), rb.as<int32_t>(),
            sb.as<int32_t>(), sn.as<int32_t>());
        CUDA_LAUNCH_OK();
    }
    // heavy block rows: pieces of kSplitPiece blocks
    DevBuf pbr, pb0, pb1, pcnt;
    int64_t npieces = 0;
    if (nbr > 0) {
        DevBuf np, first;
        alloc_n<int32_t>(np, nbr);
        alloc_n<int64_t>(first, nbr + 1);
        split_piece_count_kernel<<<grid_for(nbr, kThreads), kThreads, 0, s>>>(
            nbr, f.block_row_ptr.as<int32_t>(), np.as<int32_t>());
        CUDA_LAUNCH_OK();
        npieces = exclusive_scan_total<int32_t, int64_t>(np.as<int32_t>(), first.as<int64_t>(), nbr, s);
        if (npieces > 0) {
            alloc_n<int32_t>(pbr, npieces);
            alloc_n<int32_t>(pb0, npieces);
            alloc_n<int32_t>(pb1, npieces);
            alloc_n<int32_t>(pcnt, npieces * kPieceFields);
            split_piece_list_kernel<<<grid_for(nbr, kThreads), kThreads, 0, s>>>(
                nbr, f.block_row_ptr.as<int32_t>(), first.as<int64_t>(), pbr.as<int32_t>(), pb0.as<int32_t>(),
                pb1.as<int32_t>());
            CUDA_LAUNCH_OK();
            split_piece_count_pass<<<grid_for(npieces * 32, kThreads), kThreads, 0, s>>>(
                npieces, thr, mm, pb0.as<int32_t>(), pb1.as<int32_t>(), f.bitmap.as<uint32_t>(),
                pcnt.as<int32_t>());
            CUDA_LAUNCH_OK();
            split_piece_sum_kernel<<<grid_for(nbr, kThreads), kThreads, 0, s>>>(
                rows, nbr, first.as<int64_t>(), pcnt.as<int32_t>(), kc.as<int32_t>(), kn.as<int32_t>(),
                rc.as<int32_t>(), rb.as<int32_t>(), sb.as<int32_t>(), sn.as<int32_t>());
            CUDA_LAUNCH_OK();
        }
    }
    alloc_n<int32_t>(out.kept_block_row_ptr, nbr + 1);
    alloc_n<int32_t>(out.kept_block_row_val_ptr, nbr + 1);
    alloc_n<int32_t>(out.res_row_ptr, rows + 1);
    out.kept_blocks = exclusive_scan_total<int32_t, int32_t>(kc.as<int32_t>(),
                                                             out.kept_block_row_ptr.as<int32_t>(), nbr, s);
    out.kept_nnz = exclusive_scan_total<int32_t, int32_t>(kn.as<int32_t>(),
                                                          out.kept_block_row_val_ptr.as<int32_t>(), nbr, s);
    out.residual_nnz = checked_i32(
        exclusive_scan_total<int32_t, int32_t>(rc.as<int32_t>(), out.res_row_ptr.as<int32_t>(), rows, s),
        "residual nnz");
    {
        DevBuf tmp;
        alloc_n<int32_t>(tmp, nbr + 1);
        out.residual_blocks = exclusive_scan_total<int32_t, int32_t>(rb.as<int32_t>(), tmp.as<int32_t>(), nbr, s);
        out.cost_skipped_blocks = exclusive_scan_total<int32_t, int32_t>(sb.as<int32_t>(), tmp.as<int32_t>(), nbr, s);
        out.cost_skipped_nnz = exclusive_scan_total<int32_t, int32_t>(sn.as<int32_t>(), tmp.as<int32_t>(), nbr, s);
    }
    alloc_n<int32_t>(out.kept_col, out.kept_blocks);
    alloc_n<uint32_t>(out.kept_bitmap, out.kept_blocks);
    alloc_n<T>(out.kept_values, out.kept_nnz);
    alloc_n<int32_t>(out.res_col, out.residual_nnz);
    alloc_n<T>(out.res_values, out.residual_nnz);
    if (nbr > 0 && f.num_blocks > 0) {
        split_fill_kernel<T><<<grid, kThreads, 0, s>>>(
            rows, nbr, thr, mm, f.block_row_ptr.as<int32_t>(), f.block_row_val_ptr.as<int32_t>(),
            f.block_col_idx.as<int32_t>(), f.bitmap.as<uint32_t>(), f.values.as<T>(),
            out.kept_block_row_ptr.as<int32_t>(), out.kept_block_row_val_ptr.as<int32_t>(),
            out.res_row_ptr.as<int32_t>(), out.kept_col.as<int32_t>(),
            out.kept_bitmap.as<uint32_t>(), out.kept_values.as<T>(), out.res_col.as<int32_t>(),
            out.res_values.as<T>());
        CUDA_LAUNCH_OK();
        if (npieces > 0) {
            split_piece_fill_kernel<T><<<grid_for(npieces * 32, kThreads), kThreads, 0, s>>>(
                rows, npieces, thr, mm, pbr.as<int32_t>(), pb0.as<int32_t>(), pb1.as<int32_t>(),
                pcnt.as<int32_t>(), f.block_row_val_ptr.as<int32_t>(), f.block_col_idx.as<int32_t>(),
                f.bitmap.as<uint32_t>(), f.values.as<T>(), out.kept_block_row_ptr.as<int32_t>(),
                out.kept_block_row_val_ptr.as<int32_t>(), out.res_row_ptr.as<int32_t>(),
                out.kept_col.as<int32_t>(), out.kept_bitmap.as<uint32_t>(), out.kept_values.as<T>(),
                out.res_col.as<int32_t>(), out.res_values.as<T>());
            CUDA_LAUNCH_OK();
        }
    }
    // BitBsrMatrix::block_val_ptr of the kept part
    alloc_n<int32_t>(out.kept_block_val_ptr, out.kept_blocks + 1);
    {
        DevBuf pc;
        alloc_n<int32_t>(pc, out.kept_blocks);
        if (out.kept_blocks > 0) {
            popc_kernel<<<grid_for(out.kept_blocks, kThreads), kThreads, 0, s>>>(
                out.kept_blocks, out.kept_bitmap.as<uint32_t>(), pc.as<int32_t>());
            CUDA_LAUNCH_OK();
        }
        exclusive_scan_total<int32_t, int32_t>(pc.as<int32_t>(), out.kept_block_val_ptr.as<int32_t>(),
                                               out.kept_blocks, s);
    }
}

void build_layout(const SplitParts& sp, int32_t nbr, const cove_plan_opts& o, Layout& out,
                  cudaStream_t s) {
    const int chunk = o.lb_chunk_blocks;
    const int split = o.lb_split_threshold_blocks < 0 ? chunk : o.lb_split_threshold_blocks;
    if (chunk <= 0 || split <= 0) {
        COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "fused CSR+BitBSR load-balance parameters must be positive");
    }
    out.chunk_blocks = chunk;
    out.split_threshold_blocks = split;
    alloc_n<uint64_t>(out.words, sp.kept_blocks);
    if (sp.kept_blocks > 0) {
        pack_words_kernel<<<grid_for(sp.kept_blocks, kThreads), kThreads, 0, s>>>(
            sp.kept_blocks, sp.kept_col.as<int32_t>(), sp.kept_bitmap.as<uint32_t>(),
            out.words.as<uint64_t>());
        CUDA_LAUNCH_OK();
    }
    DevBuf cnt;
    alloc_n<int32_t>(cnt, nbr);
    alloc_n<int32_t>(out.item_row_ptr, nbr + 1);
    if (nbr > 0) {
        lb_count_kernel<<<grid_for(nbr, kThreads), kThreads, 0, s>>>(
            nbr, sp.kept_block_row_ptr.as<int32_t>(), chunk, split, o.lb_style, cnt.as<int32_t>());
        CUDA_LAUNCH_OK();
    }
    out.num_items = checked_i32(
        exclusive_scan_total<int32_t, int32_t>(cnt.as<int32_t>(), out.item_row_ptr.as<int32_t>(), nbr, s),
        "work items");
    alloc_n<WorkItem>(out.items, out.num_items);
    if (nbr > 0 && out.num_items > 0) {
        lb_fill_kernel<<<grid_for(nbr, kThreads), kThreads, 0, s>>>(
            nbr, sp.kept_block_row_ptr.as<int32_t>(), sp.kept_block_row_val_ptr.as<int32_t>(),
            sp.kept_bitmap.as<uint32_t>(), out.item_row_ptr.as<int32_t>(), chunk, split,
            o.lb_style, out.words.as<uint64_t>(), out.items.as<WorkItem>());
        CUDA_LAUNCH_OK();
    }
}

void build_chunks(const int32_t* res_rp, int32_t rows, int tau, int chunk_nnz, Chunks& out,
                  cudaStream_t s) {
    out.tau = tau;
    out.num_chunks = 0;
    out.long_rows = 0;
    if (tau <= 0 || rows == 0) return;
    DevBuf cnt, flag, crp;
    alloc_n<int32_t>(cnt, rows);
    alloc_n<int32_t>(flag, rows);
    alloc_n<int64_t>(crp, rows + 1);
    chunk_count_kernel<<<grid_for(rows, kThreads), kThreads, 0, s>>>(
        rows, res_rp, tau, chunk_nnz, cnt.as<int32_t>(), flag.as<int32_t>());
    CUDA_LAUNCH_OK();
    out.num_chunks = exclusive_scan_total<int32_t, int64_t>(cnt.as<int32_t>(), crp.as<int64_t>(), rows, s);
    {
        DevBuf tmp;
        alloc_n<int64_t>(tmp, rows + 1);
        out.long_rows = exclusive_scan_total<int32_t, int64_t>(flag.as<int32_t>(), tmp.as<int64_t>(), rows, s);
    }
    checked_i32(out.num_chunks, "long-row chunks");
    alloc_n<int32_t>(out.row, out.num_chunks);
    alloc_n<int32_t>(out.pbegin, out.num_chunks);
    alloc_n<int32_t>(out.pcount, out.num_chunks);
    if (out.num_chunks > 0) {
        chunk_fill_kernel<<<grid_for(rows, kThreads), kThreads, 0, s>>>(
            rows, res_rp, tau, chunk_nnz, crp.as<int64_t>(), out.row.as<int32_t>(),
            out.pbegin.as<int32_t>(), out.pcount.as<int32_t>());
        CUDA_LAUNCH_OK();
    }
}

template bool validate_csr<double>(const cove_csr_desc&, cudaStream_t);
template bool validate_csr<float>(const cove_csr_desc&, cudaStream_t);
template void build_full_bitbsr<double>(const cove_csr_desc&, bool, FullBitBsr&, cudaStream_t);
template void build_full_bitbsr<float>(const cove_csr_desc&, bool, FullBitBsr&, cudaStream_t);
template void bitbsr_count<double>(const cove_csr_desc&, bool, int32_t*, int32_t*, int64_t*, int64_t*, cudaStream_t);
template void bitbsr_count<float>(const cove_csr_desc&, bool, int32_t*, int32_t*, int64_t*, int64_t*, cudaStream_t);
template void bitbsr_fill<double>(const cove_csr_desc&, bool, int32_t*, uint32_t*, double*, cudaStream_t);
template void bitbsr_fill<float>(const cove_csr_desc&, bool, int32_t*, uint32_t*, float*, cudaStream_t);
template void build_split<double>(const FullBitBsr&, const cove_plan_opts&, SplitParts&, cudaStream_t);
template void build_split<float>(const FullBitBsr&, const cove_plan_opts&, SplitParts&, cudaStream_t);

}  // namespace cove
