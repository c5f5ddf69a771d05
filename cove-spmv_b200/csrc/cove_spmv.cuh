// cove_spmv.cuh -- launch interface of the fused hybrid SpMV kernels.
#pragma once

#include "cove_internal.cuh"

namespace cove {

// Value stream of one route, as raw device pointers.
struct RouteValues {
    int route = COVE_ROUTE_HYBRID;
    const void* kept = nullptr;        // T (hybrid), uint8/uint16 codes (dict), int8 (bfp8)
    const void* res = nullptr;         // T (hybrid), codes (dict), uint16 bf16 (bfp8)
    const uint16_t* scale = nullptr;   // bfp8 per-block bf16 scales
    const void* codebook = nullptr;    // dict codebook (T)
    int64_t codebook_size = 0;
    int64_t num_outliers = 0;          // bfp8 outlier side list
    const int32_t* out_rows = nullptr;
    const int32_t* out_cols = nullptr;
    const void* out_vals = nullptr;    // T
    const void* tile_words = nullptr;  // family tile codes: Bits u32 words per block
    int tile_bits = 0;
    double value_scale = 1.0;          // const_c constant, sign2 scale
    const uint32_t* sign_masks = nullptr;  // sign2: one word per kept block
};

// Position streams and the kernel's own work split.
struct KernelShape {
    int dtype = COVE_F64;
    int32_t rows = 0, cols = 0, nbr = 0;
    int32_t br_begin = 0;                 // the main pass covers block rows [br_begin, nbr)
    int part = 0;                         // 0: main + overflow pass, 1: main only, 2: overflow only
    const int32_t* kept_brp = nullptr;    // int32 nbr+1
    const int32_t* kept_brvp = nullptr;   // int32 nbr+1
    const int32_t* kept_bvp = nullptr;    // int32 kept blocks+1
    const uint64_t* words = nullptr;      // packed words (flag bit ignored)
    const int32_t* res_rp = nullptr;      // int32 rows+1
    const int32_t* res_col = nullptr;
    int slots = 4;                        // lanes per block row = 8 * slots; 0: one lane per row
    int heavy_limit = 0x7fffffff;         // blocks a block row handles in the main pass
    int long_tau = 0;                     // residual rows longer than this go to chunks
    bool x_vec_ok = false;                // set per launch: x 16-byte aligned, cols % 4 == 0
    bool l2_prefetch = false;             // plan buffers: aligned with tail slack, bulk L2 prefetch allowed
    int32_t kb_avg = 0;                   // kept blocks per block row (whole plan, rounded down)
    // overflow tasks (second launch)
    int64_t num_heavy = 0;
    const int32_t* heavy_br = nullptr;
    const int32_t* heavy_b0 = nullptr;
    const int32_t* heavy_b1 = nullptr;
    int64_t num_chunks = 0;
    const int32_t* chunk_row = nullptr;
    const int32_t* chunk_pbegin = nullptr;
    const int32_t* chunk_pcount = nullptr;
};

// y = A x for one route; returns the number of kernel launches made.
int launch_hybrid_spmv(const KernelShape& k, const RouteValues& v, const void* x, void* y,
                       cudaStream_t s);
int hybrid_spmv_launch_count(const KernelShape& k, const RouteValues& v);

// Residual rows as a lane-per-row launch would see them: entries of the rows
// of at most kProfileTau entries (`light_nnz`), those of them whose column
// lies 0-2 columns right of the same-position entry of the next row
// (`diag_nnz`: neighbouring lanes then read neighbouring x), and the number of
// longer rows (`heavy_rows`), which that launch hands to warp chunks.
constexpr int kProfileTau = 32;
constexpr int kProfileHeavyAvg = 128;  // mean heavy-row length at which warp chunks pay
struct ResidualProfile {
    int64_t light_nnz = 0, diag_nnz = 0, heavy_rows = 0;
};

// Choose lanes per block row from the average kept blocks per block row and
// residual entries per row; 0 selects the lane-per-row kernel.  With a
// profile, one lane per row is taken for few kept blocks when the light rows
// are short (or short-ish and diagonal) and the heavy rows, if they matter,
// are long; without one, only for short residual rows throughout.
int choose_slots(int64_t nbr, int64_t kept_blocks, int64_t rows, int64_t residual_nnz,
                 const ResidualProfile* prof = nullptr);

}  // namespace cove
