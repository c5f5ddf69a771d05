// plan.cu -- plan building (converter, split, layout, codecs, gate) and the C ABI.
//
// cove_plan_build runs the whole host pipeline of the reference's hybrid /
// joint operator on the device (structural/src/main_gpu_csr_bitbsr_spmv.cu:
// 1083-1184 position streams, :1222-1358 value menu, :1360-1376 gate) and
// applies the gate fall-back that structural/scripts/plot_eval_performance.py:
// 216-219 applies offline: a joint route that fails the gate dispatches the
// lossless hybrid instead.
#include "cove_plan.cuh"

#include <algorithm>
#include <cmath>
#include <cstdio>

namespace cove {

namespace {
thread_local std::string g_last_error;
constexpr int kThreads = 256;

__global__ void heavy_count_kernel(int32_t nbr, const int32_t* __restrict__ kbrp, int limit,
                                   int piece, int32_t* __restrict__ out) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    const int c = kbrp[br + 1] - kbrp[br];
    out[br] = c > limit ? (c - limit + piece - 1) / piece : 0;
}

// ResidualProfile counts (grid-stride over rows, warp sums, three atomics a warp).
__global__ void residual_profile_kernel(int32_t rows, const int32_t* __restrict__ rp,
                                        const int32_t* __restrict__ ci,
                                        unsigned long long* __restrict__ out) {
    unsigned long long light = 0, diag = 0, heavy = 0;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < rows; r += stride) {
        const int32_t b = rp[r], nb = rp[r + 1];
        const int32_t len = nb - b;
        if (len > kProfileTau) {
            ++heavy;
            continue;
        }
        light += static_cast<unsigned long long>(len);
        if (r + 1 < rows) {
            const int32_t m = min(len, rp[r + 2] - nb);
            for (int32_t k = 0; k < m; ++k) {
                const int32_t d = ci[nb + k] - ci[b + k];
                diag += (d >= 0 && d <= 2) ? 1ull : 0ull;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        light += __shfl_xor_sync(0xffffffffu, light, o);
        diag += __shfl_xor_sync(0xffffffffu, diag, o);
        heavy += __shfl_xor_sync(0xffffffffu, heavy, o);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(out, light);
        atomicAdd(out + 1, diag);
        atomicAdd(out + 2, heavy);
    }
}

ResidualProfile residual_profile(const SplitParts& sp, int32_t rows, cudaStream_t s) {
    ResidualProfile p;
    if (rows <= 0) return p;
    DevBuf acc;
    alloc_n<unsigned long long>(acc, 3);
    CUDA_OK(cudaMemsetAsync(acc.p, 0, 3 * sizeof(unsigned long long), s));
    const int grid = static_cast<int>(std::min<int64_t>(grid_for(rows, kThreads), 148 * 8));
    residual_profile_kernel<<<grid, kThreads, 0, s>>>(rows, sp.res_row_ptr.as<int32_t>(),
                                                      sp.res_col.as<int32_t>(),
                                                      acc.as<unsigned long long>());
    CUDA_LAUNCH_OK();
    unsigned long long h[3];
    CUDA_OK(cudaMemcpyAsync(h, acc.p, sizeof(h), cudaMemcpyDeviceToHost, s));
    CUDA_OK(cudaStreamSynchronize(s));
    p.light_nnz = static_cast<int64_t>(h[0]);
    p.diag_nnz = static_cast<int64_t>(h[1]);
    p.heavy_rows = static_cast<int64_t>(h[2]);
    return p;
}

__global__ void heavy_fill_kernel(int32_t nbr, const int32_t* __restrict__ kbrp, int limit,
                                  int piece, const int64_t* __restrict__ off,
                                  int32_t* __restrict__ hbr, int32_t* __restrict__ hb0,
                                  int32_t* __restrict__ hb1) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    const int b0 = kbrp[br], b1 = kbrp[br + 1];
    if (b1 - b0 <= limit) return;
    int64_t o = off[br];
    for (int b = b0 + limit; b < b1; b += piece) {
        hbr[o] = static_cast<int32_t>(br);
        hb0[o] = b;
        hb1[o] = min(b + piece, b1);
        ++o;
    }
}

template <typename T>
__global__ void canonical_x_kernel(int64_t n, T* __restrict__ x) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    // make_input_vector, spmv_harness.hpp:32-39
    if (i < n) x[i] = static_cast<T>(static_cast<int>(i % 17) - 8) * static_cast<T>(0.125);
}

// Lowest and highest column of x each block row reads: a kept block reads
// its four columns (clipped to cols), a residual row (column-sorted) its
// first to last entry.  {INT_MAX, -1} for a block row without nonzeros.
__global__ void block_row_col_bounds_kernel(int32_t nbr, int32_t rows, int32_t cols,
                                            const int32_t* __restrict__ kbrp,
                                            const uint64_t* __restrict__ words,
                                            const int32_t* __restrict__ rrp,
                                            const int32_t* __restrict__ rcol,
                                            int32_t* __restrict__ lo, int32_t* __restrict__ hi) {
    const int64_t br = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (br >= nbr) return;
    int mn = 0x7fffffff, mx = -1;
    for (int b = kbrp[br]; b < kbrp[br + 1]; ++b) {
        const int c4 = static_cast<int>(words[b] & 0x7fffffffULL) * 4;
        mn = min(mn, c4);
        mx = max(mx, min(c4 + 3, cols - 1));
    }
    if (rrp != nullptr) {
        const int64_t r1 = (br + 1) * kBlockRows < rows ? (br + 1) * kBlockRows : rows;
        for (int64_t r = br * kBlockRows; r < r1; ++r) {
            if (rrp[r + 1] > rrp[r]) {
                mn = min(mn, rcol[rrp[r]]);
                mx = max(mx, rcol[rrp[r + 1] - 1]);
            }
        }
    }
    lo[br] = mn;
    hi[br] = mx;
}

}  // namespace

void set_last_error(const std::string& msg) { g_last_error = msg; }

void block_row_col_bounds(const cove_plan* P, std::vector<int32_t>* lo, std::vector<int32_t>* hi) {
    lo->assign(static_cast<size_t>(P->nbr), 0);
    hi->assign(static_cast<size_t>(P->nbr), -1);
    if (P->nbr == 0) return;
    DevBuf dlo, dhi;
    alloc_n<int32_t>(dlo, P->nbr);
    alloc_n<int32_t>(dhi, P->nbr);
    const KernelShape k = P->shape();
    block_row_col_bounds_kernel<<<grid_for(P->nbr, kThreads), kThreads>>>(
        P->nbr, P->rows, P->cols, k.kept_brp, k.words, k.res_rp, k.res_col, dlo.as<int32_t>(),
        dhi.as<int32_t>());
    CUDA_LAUNCH_OK();
    CUDA_OK(cudaMemcpy(lo->data(), dlo.p, lo->size() * sizeof(int32_t), cudaMemcpyDeviceToHost));
    CUDA_OK(cudaMemcpy(hi->data(), dhi.p, hi->size() * sizeof(int32_t), cudaMemcpyDeviceToHost));
}

HostPipeline::~HostPipeline() {
    for (cudaEvent_t e : x_ready) cudaEventDestroy(e);
    for (cudaEvent_t e : y_ready) cudaEventDestroy(e);
    if (start) cudaEventDestroy(start);
    if (out_done) cudaEventDestroy(out_done);
    if (s_in) cudaStreamDestroy(s_in);
    if (s_out) cudaStreamDestroy(s_out);
    if (exec) cudaGraphExecDestroy(exec);
    if (s_cap) cudaStreamDestroy(s_cap);
}

namespace {

// Slices for a vector of n elements of esz bytes: about 2^kHostSliceShift
// bytes each, at most kHostMaxSlices; x boundaries on 32-element multiples.
constexpr int kHostSliceShift = 20;
constexpr int kHostMaxSlices = 8;
int slice_count(int64_t n, size_t esz) {
    const int64_t bytes = n * static_cast<int64_t>(esz);
    return static_cast<int>(std::max<int64_t>(
        1, std::min<int64_t>(kHostMaxSlices, bytes >> kHostSliceShift)));
}

std::unique_ptr<HostPipeline> build_host_pipeline(const cove_plan* P) {
    auto hp = std::make_unique<HostPipeline>();
    hp->kx = slice_count(P->cols, P->esz);
    hp->ky = std::min<int>(slice_count(P->rows, P->esz), std::max<int32_t>(P->nbr, 1));
    hp->x_cut.resize(hp->kx + 1);
    for (int i = 0; i <= hp->kx; ++i) {
        const int64_t c = (static_cast<int64_t>(P->cols) * i / hp->kx) & ~int64_t(31);
        hp->x_cut[i] = i == hp->kx ? P->cols : c;
    }
    hp->br_cut.resize(hp->ky + 1);
    for (int j = 0; j <= hp->ky; ++j)
        hp->br_cut[j] = static_cast<int32_t>(static_cast<int64_t>(P->nbr) * j / hp->ky);
    // the last x slice each block-row slice reads
    std::vector<int32_t> lo, mc;
    block_row_col_bounds(P, &lo, &mc);
    hp->need.assign(hp->ky, -1);
    int run = -1;
    for (int j = 0; j < hp->ky; ++j) {
        for (int32_t b = hp->br_cut[j]; b < hp->br_cut[j + 1]; ++b) run = std::max(run, mc[b]);
        if (run >= 0) {
            int i = 0;
            while (hp->x_cut[i + 1] <= run) ++i;
            hp->need[j] = i;
        }
    }
    CUDA_OK(cudaStreamCreateWithFlags(&hp->s_in, cudaStreamNonBlocking));
    CUDA_OK(cudaStreamCreateWithFlags(&hp->s_out, cudaStreamNonBlocking));
    CUDA_OK(cudaStreamCreateWithFlags(&hp->s_cap, cudaStreamNonBlocking));
    hp->x_ready.resize(hp->kx);
    hp->y_ready.resize(hp->ky);
    for (auto& e : hp->x_ready) CUDA_OK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (auto& e : hp->y_ready) CUDA_OK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    CUDA_OK(cudaEventCreateWithFlags(&hp->start, cudaEventDisableTiming));
    CUDA_OK(cudaEventCreateWithFlags(&hp->out_done, cudaEventDisableTiming));
    return hp;
}

bool is_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// x slices in on s_in; block-row slices of the main pass on s, each after the
// x slices it reads; y slices out on s_out as soon as their rows are final
// (after the overflow pass, when the plan has one).  Everything joins s.
void issue_sliced(const cove_plan* P, HostPipeline& hp, const void* x_host, void* y_host,
                  cudaStream_t s) {
    const KernelShape k = P->shape();
    const RouteValues rv = P->route_values(P->dispatched_route);
    auto* xs = static_cast<char*>(P->x_stage.p);
    auto* ys = static_cast<char*>(P->y_stage.p);
    const auto* xh = static_cast<const char*>(x_host);
    auto* yh = static_cast<char*>(y_host);
    const size_t esz = P->esz;
    CUDA_OK(cudaEventRecord(hp.start, s));
    CUDA_OK(cudaStreamWaitEvent(hp.s_in, hp.start, 0));
    CUDA_OK(cudaStreamWaitEvent(hp.s_out, hp.start, 0));
    for (int i = 0; i < hp.kx; ++i) {
        const int64_t c0 = hp.x_cut[i], c1 = hp.x_cut[i + 1];
        if (c1 > c0)
            CUDA_OK(cudaMemcpyAsync(xs + c0 * esz, xh + c0 * esz, static_cast<size_t>(c1 - c0) * esz,
                                    cudaMemcpyHostToDevice, hp.s_in));
        CUDA_OK(cudaEventRecord(hp.x_ready[i], hp.s_in));
    }
    const bool late_rows = hybrid_spmv_launch_count(k, rv) > 1;
    int waited = -1;
    for (int j = 0; j < hp.ky; ++j) {
        if (hp.need[j] > waited) {
            waited = hp.need[j];
            CUDA_OK(cudaStreamWaitEvent(s, hp.x_ready[waited], 0));
        }
        KernelShape kj = k;
        kj.part = 1;
        kj.br_begin = hp.br_cut[j];
        kj.nbr = hp.br_cut[j + 1];
        launch_hybrid_spmv(kj, rv, xs, ys, s);
        if (!late_rows) {
            const int64_t r0 = static_cast<int64_t>(hp.br_cut[j]) * kBlockRows;
            const int64_t r1 =
                std::min<int64_t>(static_cast<int64_t>(hp.br_cut[j + 1]) * kBlockRows, P->rows);
            CUDA_OK(cudaEventRecord(hp.y_ready[j], s));
            CUDA_OK(cudaStreamWaitEvent(hp.s_out, hp.y_ready[j], 0));
            if (r1 > r0)
                CUDA_OK(cudaMemcpyAsync(yh + r0 * esz, ys + r0 * esz, static_cast<size_t>(r1 - r0) * esz,
                                        cudaMemcpyDeviceToHost, hp.s_out));
        }
    }
    if (waited < hp.kx - 1) CUDA_OK(cudaStreamWaitEvent(s, hp.x_ready[hp.kx - 1], 0));
    if (late_rows) {
        KernelShape ko = k;
        ko.part = 2;
        launch_hybrid_spmv(ko, rv, xs, ys, s);
        CUDA_OK(cudaEventRecord(hp.y_ready[0], s));
        CUDA_OK(cudaStreamWaitEvent(hp.s_out, hp.y_ready[0], 0));
        CUDA_OK(cudaMemcpyAsync(yh, ys, static_cast<size_t>(P->rows) * esz, cudaMemcpyDeviceToHost,
                                hp.s_out));
    }
    CUDA_OK(cudaEventRecord(hp.out_done, hp.s_out));
    CUDA_OK(cudaStreamWaitEvent(s, hp.out_done, 0));
}

}  // namespace

}  // namespace cove

using namespace cove;

cove::KernelShape cove_plan::shape() const {
    KernelShape k;
    k.dtype = dtype;
    k.rows = rows;
    k.cols = cols;
    k.nbr = nbr;
    k.kept_brp = sp.kept_block_row_ptr.as<int32_t>();
    k.kept_brvp = sp.kept_block_row_val_ptr.as<int32_t>();
    k.kept_bvp = sp.kept_block_val_ptr.as<int32_t>();
    k.words = lay.words.as<uint64_t>();
    k.res_rp = sp.res_row_ptr.as<int32_t>();
    k.res_col = sp.res_col.as<int32_t>();
    k.slots = slots;
    k.l2_prefetch = true;  // DevBuf: cudaMalloc alignment and kTailSlack
    k.kb_avg = nbr > 0 ? static_cast<int32_t>(sp.kept_blocks / nbr) : 0;
    k.heavy_limit = heavy_limit;
    k.long_tau = long_tau;
    k.num_heavy = num_heavy;
    k.heavy_br = heavy_br.as<int32_t>();
    k.heavy_b0 = heavy_b0.as<int32_t>();
    k.heavy_b1 = heavy_b1.as<int32_t>();
    const Chunks& c = kchunks_alias ? chunks : kchunks;
    k.num_chunks = long_tau > 0 ? c.num_chunks : 0;
    k.chunk_row = c.row.as<int32_t>();
    k.chunk_pbegin = c.pbegin.as<int32_t>();
    k.chunk_pcount = c.pcount.as<int32_t>();
    return k;
}

bool cove_plan::has_route(int route) const {
    switch (route) {
        case COVE_ROUTE_HYBRID: return has_lossless;
        case COVE_ROUTE_DICT_U8: return has_dict && dict.bits == 8;
        case COVE_ROUTE_DICT_U16: return has_dict && dict.bits == 16;
        case COVE_ROUTE_BFP8: return has_bfp8 && !has_outlier;
        case COVE_ROUTE_BFP8_OUTLIER: return has_bfp8 && has_outlier;
        default: return false;
    }
}

cove::RouteValues cove_plan::route_values(int route) const {
    RouteValues v;
    v.route = route;
    switch (route) {
        case COVE_ROUTE_HYBRID:
            v.kept = sp.kept_values.p;
            v.res = sp.res_values.p;
            break;
        case COVE_ROUTE_DICT_U8:
        case COVE_ROUTE_DICT_U16:
            v.kept = dict.kept_idx.p;
            v.res = dict.res_idx.p;
            v.codebook = dict.codebook.p;
            v.codebook_size = dict.uniq;
            break;
        case COVE_ROUTE_BFP8:
        case COVE_ROUTE_BFP8_OUTLIER:
            v.kept = bfp8_q.p;
            v.res = res_bf16.p;
            v.scale = bfp8_scale.as<uint16_t>();
            if (route == COVE_ROUTE_BFP8_OUTLIER) {
                v.num_outliers = num_out;
                v.out_rows = out_rows.as<int32_t>();
                v.out_cols = out_cols.as<int32_t>();
                v.out_vals = out_vals.p;
            }
            break;
    }
    return v;
}

namespace {

template <typename T>
void build_plan_typed(cove_plan* P, const cove_csr_desc& d, cudaStream_t s) {
    const cove_plan_opts& o = P->opts;
    const bool split = validate_csr<T>(d, s);
    build_full_bitbsr<T>(d, split, P->full, s);
    P->nnz = P->full.nnz;
    P->nbr = P->full.nbr;
    build_split<T>(P->full, o, P->sp, s);
    // only the counts of the full BitBSR are needed past the split; its
    // arrays go before the codecs allocate theirs
    P->has_full = o.keep_full_bitbsr != 0;
    if (!P->has_full) {
        P->full.block_col_idx.release();
        P->full.bitmap.release();
        P->full.values.release();
        P->full.block_row_ptr.release();
        P->full.block_row_val_ptr.release();
    }
    build_layout(P->sp, P->nbr, o, P->lay, s);
    build_chunks(P->sp.res_row_ptr.as<int32_t>(), P->rows, o.long_row_split, kLongChunkNnz,
                 P->chunks, s);

    // kernel work split
    const ResidualProfile prof = residual_profile(P->sp, P->rows, s);
    P->slots = choose_slots(P->nbr, P->sp.kept_blocks, P->rows, P->sp.residual_nnz, &prof);
    const double avg_blocks = P->nbr > 0 ? static_cast<double>(P->sp.kept_blocks) / P->nbr : 0.0;
    // a block row's blocks beyond the limit go to 256-block overflow pieces;
    // a lane-per-row launch walks blocks serially, so its limit is lower
    P->heavy_limit = static_cast<int>(
        std::max(P->slots == 0 ? 32.0 : 256.0, 8.0 * std::ceil(avg_blocks)));
    const int piece = 256;
    {
        DevBuf cnt, off;
        alloc_n<int32_t>(cnt, P->nbr);
        alloc_n<int64_t>(off, P->nbr + 1);
        if (P->nbr > 0) {
            heavy_count_kernel<<<grid_for(P->nbr, kThreads), kThreads, 0, s>>>(
                P->nbr, P->sp.kept_block_row_ptr.as<int32_t>(), P->heavy_limit, piece,
                cnt.as<int32_t>());
            CUDA_LAUNCH_OK();
        }
        P->num_heavy = exclusive_scan_total<int32_t, int64_t>(cnt.as<int32_t>(), off.as<int64_t>(), P->nbr, s);
        alloc_n<int32_t>(P->heavy_br, P->num_heavy);
        alloc_n<int32_t>(P->heavy_b0, P->num_heavy);
        alloc_n<int32_t>(P->heavy_b1, P->num_heavy);
        if (P->num_heavy > 0) {
            heavy_fill_kernel<<<grid_for(P->nbr, kThreads), kThreads, 0, s>>>(
                P->nbr, P->sp.kept_block_row_ptr.as<int32_t>(), P->heavy_limit, piece,
                off.as<int64_t>(), P->heavy_br.as<int32_t>(), P->heavy_b0.as<int32_t>(),
                P->heavy_b1.as<int32_t>());
            CUDA_LAUNCH_OK();
        }
    }
    // residual rows longer than 64 entries per lane (32 for one lane per row)
    // go to 1024-nnz warp chunks
    P->long_tau = P->slots == 0 ? 32 : 64 * P->slots;
    if (o.long_row_split > 0 && o.long_row_split == P->long_tau) {
        P->kchunks_alias = true;
    } else {
        build_chunks(P->sp.res_row_ptr.as<int32_t>(), P->rows, P->long_tau, kLongChunkNnz,
                     P->kchunks, s);
    }

    // joint value menu (main_gpu_csr_bitbsr_spmv.cu:1222-1358)
    int chosen = o.value_codec;
    if (chosen == COVE_CODEC_AUTO || chosen == COVE_CODEC_DICT) {
        const int64_t uniq = encode_dict<T>(P->sp, false, P->dict, s);
        P->uniq = uniq;  // -1: above 65536
        const bool small = uniq >= 0 && uniq <= 256;
        const bool fits = uniq >= 0 && uniq <= 65536;
        if (chosen == COVE_CODEC_AUTO) chosen = small ? COVE_CODEC_DICT : COVE_CODEC_BFP8;
        if (chosen == COVE_CODEC_DICT && !fits) chosen = COVE_CODEC_BFP8;
    }
    switch (chosen) {
        case COVE_CODEC_ORIGINAL:
            P->joint_route = COVE_ROUTE_HYBRID;
            break;
        case COVE_CODEC_DICT:
            encode_dict<T>(P->sp, true, P->dict, s);
            P->has_dict = true;
            P->joint_route = P->dict.bits == 8 ? COVE_ROUTE_DICT_U8 : COVE_ROUTE_DICT_U16;
            break;
        case COVE_CODEC_BFP8:
            encode_bfp8<T>(P->sp, nullptr, P->bfp8_q, P->bfp8_scale, s);
            encode_res_bf16<T>(P->sp, P->res_bf16, s);
            P->has_bfp8 = true;
            P->joint_route = COVE_ROUTE_BFP8;
            break;
        case COVE_CODEC_BFP8_OUTLIER:
            encode_bfp8_outlier<T>(P->sp, P->nbr, o.outlier_fraction, P->bfp8_q, P->bfp8_scale,
                                   P->out_rows, P->out_cols, P->out_vals, &P->num_out,
                                   &P->outlier_threshold, s);
            encode_res_bf16<T>(P->sp, P->res_bf16, s);
            P->has_bfp8 = true;
            P->has_outlier = true;
            P->joint_route = COVE_ROUTE_BFP8_OUTLIER;
            break;
        default:
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "unknown value codec");
    }

    // gate: global_rel of the joint route against the lossless route on the
    // canonical x (spmv_harness.hpp:32-39), pass iff 0 <= rel <= tolerance
    P->dispatched_route = P->joint_route;
    if (P->joint_route != COVE_ROUTE_HYBRID && o.gate_enable) {
        DevBuf x, y0, y1;
        alloc_n<T>(x, P->cols);
        alloc_n<T>(y0, P->rows);
        alloc_n<T>(y1, P->rows);
        if (P->cols > 0) {
            canonical_x_kernel<T><<<grid_for(P->cols, kThreads), kThreads, 0, s>>>(P->cols, x.as<T>());
            CUDA_LAUNCH_OK();
        }
        const KernelShape k = P->shape();
        launch_hybrid_spmv(k, P->route_values(COVE_ROUTE_HYBRID), x.p, y0.p, s);
        launch_hybrid_spmv(k, P->route_values(P->joint_route), x.p, y1.p, s);
        double out3[3];
        compare_reduce<T>(y0.as<T>(), y1.as<T>(), P->rows, out3, s);
        P->joint_rel = out3[2];
        P->gate_evaluated = true;
        P->gate_pass = P->joint_rel >= 0.0 && P->joint_rel <= o.gate_tolerance;
        if (!P->gate_pass) P->dispatched_route = COVE_ROUTE_HYBRID;
    }
    if (!o.keep_lossless && P->dispatched_route != COVE_ROUTE_HYBRID) {
        P->sp.kept_values.release();
        P->sp.res_values.release();
        P->has_lossless = false;
    }
    CUDA_OK(cudaStreamSynchronize(s));
}

int64_t route_bytes(const cove_plan* P, int route) {
    if (!P->has_route(route)) return 0;
    const int64_t s = static_cast<int64_t>(P->esz);
    const int64_t kb = P->sp.kept_blocks, kn = P->sp.kept_nnz, rn = P->sp.residual_nnz;
    // position streams the fused kernel reads once per SpMV
    int64_t b = 8 * kb + 2 * 4 * (static_cast<int64_t>(P->nbr) + 1) +
                4 * (static_cast<int64_t>(P->rows) + 1) + 4 * rn;
    b += s * P->cols + s * P->rows;  // x read once, y written once
    switch (route) {
        case COVE_ROUTE_HYBRID: b += s * (kn + rn); break;
        case COVE_ROUTE_DICT_U8: b += (kn + rn) + s * P->dict.uniq; break;
        case COVE_ROUTE_DICT_U16: b += 2 * (kn + rn) + s * P->dict.uniq; break;
        case COVE_ROUTE_BFP8: b += kn + 2 * kb + 2 * rn; break;
        case COVE_ROUTE_BFP8_OUTLIER: b += kn + 2 * kb + 2 * rn + (8 + s) * P->num_out; break;
    }
    const Chunks& c = P->kchunks_alias ? P->chunks : P->kchunks;
    if (P->long_tau > 0) b += 12 * c.num_chunks;
    b += 12 * P->num_heavy;
    return b;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================

extern "C" {

const char* cove_last_error(void) { return cove::g_last_error.c_str(); }

const char* cove_status_string(cove_status s) {
    switch (s) {
        case COVE_OK: return "ok";
        case COVE_ERR_INVALID_ARGUMENT: return "invalid argument";
        case COVE_ERR_INVALID_INPUT: return "invalid input matrix";
        case COVE_ERR_OVERFLOW: return "int32 offset overflow";
        case COVE_ERR_CUDA: return "CUDA error";
        case COVE_ERR_OUT_OF_MEMORY: return "out of memory";
        case COVE_ERR_UNSUPPORTED: return "unsupported";
        case COVE_ERR_NCCL: return "NCCL error";
        case COVE_ERR_TIMEOUT: return "timeout";
    }
    return "unknown status";
}

const char* cove_version(void) { return "cove-b200 0.2.0 (sm_100a)"; }

void cove_plan_opts_default(cove_plan_opts* o) {
    if (!o) return;
    std::memset(o, 0, sizeof(*o));
    o->residual_threshold = 32;
    o->split_policy = COVE_SPLIT_COST_GATED;
    o->cost_bitmap_block = 10.0;
    o->cost_bitmap_nnz = 0.0;
    o->cost_csr_block = 0.0;
    o->cost_csr_nnz = 1.0;
    o->lb_chunk_blocks = 32;
    o->lb_split_threshold_blocks = -1;
    o->lb_style = COVE_LB_HYBRID;
    o->long_row_split = 0;
    o->value_codec = COVE_CODEC_ORIGINAL;
    o->outlier_fraction = 0.005;
    o->gate_tolerance = 1e-2;
    o->gate_enable = 1;
    o->keep_full_bitbsr = 0;
    o->keep_lossless = 1;
}

cove_status cove_plan_build(const cove_csr_desc* csr, const cove_plan_opts* opts, void* stream,
                            cove_plan** out) {
    return guarded([&] {
        if (!csr || !out) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        *out = nullptr;
        cove_plan_opts o;
        if (opts) o = *opts; else cove_plan_opts_default(&o);
        if (o.residual_threshold < 0) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "residual-threshold must be non-negative");
        }
        if (o.cost_bitmap_block < 0 || o.cost_bitmap_nnz < 0 || o.cost_csr_block < 0 ||
            o.cost_csr_nnz < 0) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "CSR+BitBSR split cost model must be non-negative");
        }
        if (o.lb_chunk_blocks <= 0) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "lb-chunk-blocks must be positive");
        if (o.lb_split_threshold_blocks == 0) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "lb-split-threshold-blocks must be positive");
        }
        if (o.long_row_split < 0) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "long-row-split must be non-negative");
        if (o.split_policy < 0 || o.split_policy > 3 || o.lb_style < 0 || o.lb_style > 1 ||
            o.value_codec < 0 || o.value_codec > 4) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "unknown option value");
        }
        if (csr->dtype != COVE_F64 && csr->dtype != COVE_F32) {
            COVE_THROW(COVE_ERR_UNSUPPORTED, "dtype must be float64 or float32");
        }
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        auto* P = new cove_plan();
        P->opts = o;
        P->dtype = csr->dtype;
        P->esz = csr->dtype == COVE_F64 ? 8 : 4;
        P->rows = csr->rows;
        P->cols = csr->cols;
        try {
            if (csr->dtype == COVE_F64) build_plan_typed<double>(P, *csr, s);
            else build_plan_typed<float>(P, *csr, s);
        } catch (...) {
            delete P;
            throw;
        }
        *out = P;
    });
}

cove_status cove_plan_destroy(cove_plan* plan) {
    return guarded([&] { delete plan; });
}

const char* cove_route_name(int32_t route) {
    switch (route) {
        case COVE_ROUTE_HYBRID: return "original";
        case COVE_ROUTE_DICT_U8: return "dict_u8_lossless";
        case COVE_ROUTE_DICT_U16: return "dict_u16_lossless";
        case COVE_ROUTE_BFP8: return "bfp8_blocks+bf16_residual";
        case COVE_ROUTE_BFP8_OUTLIER: return "bfp8_outlier_blocks+bf16_residual";
        case COVE_ROUTE_TILE_CODE: return "tile_code";
        case COVE_ROUTE_BF16_NNZ: return "bf16_nnz";
        case COVE_ROUTE_IMPLICIT_ONE: return "implicit_one";
        case COVE_ROUTE_CONST_C: return "const_c";
        case COVE_ROUTE_SIGN2: return "sign2";
        case COVE_ROUTE_FP16_NNZ: return "fp16_nnz";
        case COVE_ROUTE_BFP4: return "bfp4";
    }
    return "unknown";
}

cove_status cove_plan_get_info(const cove_plan* P, cove_plan_info* info) {
    return guarded([&] {
        if (!P || !info) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        std::memset(info, 0, sizeof(*info));
        info->rows = P->rows;
        info->cols = P->cols;
        info->dtype = P->dtype;
        info->nnz = P->nnz;
        info->full_blocks = P->full.num_blocks;
        info->kept_blocks = P->sp.kept_blocks;
        info->residual_blocks = P->sp.residual_blocks;
        info->cost_skipped_blocks = P->sp.cost_skipped_blocks;
        info->kept_nnz = P->sp.kept_nnz;
        info->residual_nnz = P->sp.residual_nnz;
        info->cost_skipped_nnz = P->sp.cost_skipped_nnz;
        info->work_items = P->lay.num_items;
        info->long_rows = P->chunks.long_rows;
        info->long_row_chunks = P->chunks.num_chunks;
        info->num_outliers = P->num_out;
        info->value_cardinality = P->uniq;
        // storage_stats (csr_bitbsr_split.hpp:559-573), 32 bits per entry
        const int64_t nbr1 = static_cast<int64_t>(P->nbr) + 1;
        info->full_bitbsr_position_bits = nbr1 * 32 + P->full.num_blocks * 32 * 2 +
                                          (P->full.num_blocks + 1) * 32;
        info->kept_bitbsr_position_bits = nbr1 * 32 + P->sp.kept_blocks * 32 * 2 +
                                          (P->sp.kept_blocks + 1) * 32;
        info->residual_csr_position_bits = (static_cast<int64_t>(P->rows) + 1) * 32 +
                                           P->sp.residual_nnz * 32;
        info->split_position_bits = info->kept_bitbsr_position_bits + info->residual_csr_position_bits;
        info->requested_codec = P->opts.value_codec;
        info->joint_route = P->joint_route;
        info->dispatched_route = P->dispatched_route;
        info->gate_evaluated = P->gate_evaluated ? 1 : 0;
        info->gate_pass = P->gate_pass ? 1 : 0;
        info->joint_rel_err = P->gate_evaluated ? P->joint_rel : -1.0;
        // joint_bytes_per_nnz (main_gpu_csr_bitbsr_spmv.cu:1261-1263, 1322-1325, 1354-1356)
        const double total = static_cast<double>(P->nnz);
        const double kn = static_cast<double>(P->sp.kept_nnz), rn = static_cast<double>(P->sp.residual_nnz);
        double bpn = 0.0;
        switch (P->joint_route) {
            case COVE_ROUTE_DICT_U8:
            case COVE_ROUTE_DICT_U16: {
                const double idx_b = P->dict.uniq <= 256 ? 1.0 : 2.0;
                bpn = (idx_b * (kn + rn) + 8.0 * static_cast<double>(P->dict.uniq)) / total;
                break;
            }
            case COVE_ROUTE_BFP8:
                bpn = (kn + 2.0 * static_cast<double>(P->sp.kept_blocks) + 2.0 * rn) / total;
                break;
            case COVE_ROUTE_BFP8_OUTLIER:
                bpn = (kn + 2.0 * static_cast<double>(P->sp.kept_blocks) + 2.0 * rn +
                       16.0 * static_cast<double>(P->num_out)) / total;
                break;
            default:
                bpn = static_cast<double>(P->esz);
        }
        info->joint_bytes_per_nnz = total > 0 ? bpn : 0.0;
        info->outlier_threshold = P->outlier_threshold;
        for (int r = 0; r < 5; ++r) info->algorithmic_bytes[r] = route_bytes(P, r);
        info->kernel_slots = P->slots;
        info->kernel_overflow_tasks = static_cast<int32_t>(
            P->num_heavy + (P->long_tau > 0 ? (P->kchunks_alias ? P->chunks : P->kchunks).num_chunks : 0));
    });
}

cove_status cove_plan_stream(const cove_plan* P, int32_t which, void* dst, size_t capacity,
                             size_t* bytes, void* stream) {
    return guarded([&] {
        if (!P) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null plan");
        const void* src = nullptr;
        size_t n = 0;
        const int64_t nbr1 = static_cast<int64_t>(P->nbr) + 1;
        const size_t dict_isz = P->dict.bits == 16 ? 2 : 1;
        auto need_full = [&] {
            if (!P->has_full) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan was built without keep_full_bitbsr");
        };
        switch (which) {
            case COVE_STREAM_FULL_BLOCK_ROW_PTR: need_full(); src = P->full.block_row_ptr.p; n = nbr1 * 4; break;
            case COVE_STREAM_FULL_BLOCK_COL_IDX: need_full(); src = P->full.block_col_idx.p; n = P->full.num_blocks * 4; break;
            case COVE_STREAM_FULL_BITMAP: need_full(); src = P->full.bitmap.p; n = P->full.num_blocks * 4; break;
            case COVE_STREAM_FULL_VALUES: need_full(); src = P->full.values.p; n = P->full.nnz * P->esz; break;
            case COVE_STREAM_FULL_BLOCK_ROW_VAL_PTR: need_full(); src = P->full.block_row_val_ptr.p; n = nbr1 * 4; break;
            case COVE_STREAM_KEPT_BLOCK_ROW_PTR: src = P->sp.kept_block_row_ptr.p; n = nbr1 * 4; break;
            case COVE_STREAM_KEPT_BLOCK_COL_IDX: src = P->sp.kept_col.p; n = P->sp.kept_blocks * 4; break;
            case COVE_STREAM_KEPT_BITMAP: src = P->sp.kept_bitmap.p; n = P->sp.kept_blocks * 4; break;
            case COVE_STREAM_KEPT_VALUES:
                if (!P->has_lossless) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "raw values were released");
                src = P->sp.kept_values.p; n = P->sp.kept_nnz * P->esz; break;
            case COVE_STREAM_KEPT_BLOCK_VAL_PTR: src = P->sp.kept_block_val_ptr.p; n = (P->sp.kept_blocks + 1) * 4; break;
            case COVE_STREAM_KEPT_BLOCK_ROW_VAL_PTR: src = P->sp.kept_block_row_val_ptr.p; n = nbr1 * 4; break;
            case COVE_STREAM_RES_ROW_PTR: src = P->sp.res_row_ptr.p; n = (static_cast<int64_t>(P->rows) + 1) * 4; break;
            case COVE_STREAM_RES_COL_IDX: src = P->sp.res_col.p; n = P->sp.residual_nnz * 4; break;
            case COVE_STREAM_RES_VALUES:
                if (!P->has_lossless) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "raw values were released");
                src = P->sp.res_values.p; n = P->sp.residual_nnz * P->esz; break;
            case COVE_STREAM_WORDS: src = P->lay.words.p; n = P->sp.kept_blocks * 8; break;
            case COVE_STREAM_WORK_ITEMS: src = P->lay.items.p; n = P->lay.num_items * 16; break;
            case COVE_STREAM_WORK_ITEM_ROW_PTR: src = P->lay.item_row_ptr.p; n = nbr1 * 4; break;
            case COVE_STREAM_CHUNK_ROW: src = P->chunks.row.p; n = P->chunks.num_chunks * 4; break;
            case COVE_STREAM_CHUNK_PBEGIN: src = P->chunks.pbegin.p; n = P->chunks.num_chunks * 4; break;
            case COVE_STREAM_CHUNK_PCOUNT: src = P->chunks.pcount.p; n = P->chunks.num_chunks * 4; break;
            case COVE_STREAM_DICT_CODEBOOK:
                if (!P->has_dict) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no dictionary");
                src = P->dict.codebook.p; n = P->dict.uniq * P->esz; break;
            case COVE_STREAM_DICT_KEPT_IDX:
                if (!P->has_dict) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no dictionary");
                src = P->dict.kept_idx.p; n = P->sp.kept_nnz * dict_isz; break;
            case COVE_STREAM_DICT_RES_IDX:
                if (!P->has_dict) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no dictionary");
                src = P->dict.res_idx.p; n = P->sp.residual_nnz * dict_isz; break;
            case COVE_STREAM_BFP8_INT8:
                if (!P->has_bfp8) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no bfp8 stream");
                src = P->bfp8_q.p; n = P->sp.kept_nnz; break;
            case COVE_STREAM_BFP8_SCALE:
                if (!P->has_bfp8) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no bfp8 stream");
                src = P->bfp8_scale.p; n = P->sp.kept_blocks * 2; break;
            case COVE_STREAM_RES_BF16:
                if (!P->has_bfp8) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no bf16 residual");
                src = P->res_bf16.p; n = P->sp.residual_nnz * 2; break;
            case COVE_STREAM_OUTLIER_ROWS:
                if (!P->has_outlier) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no outliers");
                src = P->out_rows.p; n = P->num_out * 4; break;
            case COVE_STREAM_OUTLIER_COLS:
                if (!P->has_outlier) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no outliers");
                src = P->out_cols.p; n = P->num_out * 4; break;
            case COVE_STREAM_OUTLIER_VALS:
                if (!P->has_outlier) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan has no outliers");
                src = P->out_vals.p; n = P->num_out * P->esz; break;
            default:
                COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "unknown stream id");
        }
        if (bytes) *bytes = n;
        if (!dst) return;
        if (capacity < n) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "destination capacity too small");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (n > 0) CUDA_OK(cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, s));
        CUDA_OK(cudaStreamSynchronize(s));
    });
}

cove_status cove_spmv_route(const cove_plan* P, int32_t route, const void* x, void* y,
                            void* stream) {
    return guarded([&] {
        if (!P) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null plan");
        if (!P->has_route(route)) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan does not hold that route");
        if ((P->cols > 0 && !x) || (P->rows > 0 && !y)) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null vector");
        launch_hybrid_spmv(P->shape(), P->route_values(route), x, y, static_cast<cudaStream_t>(stream));
    });
}

cove_status cove_bitbsr8x4_count(const cove_csr_desc* csr, int32_t* brp, int32_t* brvp,
                                 int64_t* num_blocks, int64_t* nnz, void* stream) {
    return guarded([&] {
        if (!csr || !brp || !brvp || !num_blocks || !nnz) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (csr->dtype == COVE_F64) {
            bitbsr_count<double>(*csr, validate_csr<double>(*csr, s), brp, brvp, num_blocks, nnz, s);
        } else if (csr->dtype == COVE_F32) {
            bitbsr_count<float>(*csr, validate_csr<float>(*csr, s), brp, brvp, num_blocks, nnz, s);
        } else {
            COVE_THROW(COVE_ERR_UNSUPPORTED, "dtype must be float64 or float32");
        }
    });
}

cove_status cove_bitbsr8x4_fill(const cove_csr_desc* csr, const int32_t* brp, const int32_t* brvp,
                                int32_t* col, uint32_t* bitmap, void* values, void* stream) {
    return guarded([&] {
        if (!csr || !brp || !brvp) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        if (csr->nnz > 0 && (!col || !bitmap || !values)) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null output");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        // the fill re-validates: it walks the CSR on its own and needs the
        // column-order answer for its pieces
        if (csr->dtype == COVE_F64) {
            bitbsr_fill<double>(*csr, validate_csr<double>(*csr, s), col, bitmap, static_cast<double*>(values), s);
        } else if (csr->dtype == COVE_F32) {
            bitbsr_fill<float>(*csr, validate_csr<float>(*csr, s), col, bitmap, static_cast<float*>(values), s);
        } else {
            COVE_THROW(COVE_ERR_UNSUPPORTED, "dtype must be float64 or float32");
        }
    });
}

cove_status cove_pack_words(int64_t nb, const int32_t* col, const uint32_t* bitmap, uint64_t* words,
                            void* stream) {
    return guarded([&] {
        if (nb < 0 || (nb > 0 && (!col || !bitmap || !words))) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "bad argument");
        pack_words(nb, col, bitmap, words, static_cast<cudaStream_t>(stream));
    });
}

cove_status cove_lb_layout_count(int32_t nbr, const int32_t* brp, int32_t chunk, int32_t split,
                                 int32_t style, int32_t* item_rp, int64_t* num_items, void* stream) {
    return guarded([&] {
        if (chunk <= 0) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "GPU BitBSR load-balance chunk_blocks must be positive");
        if (split < 0) split = chunk;
        if (split == 0) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "GPU BitBSR load-balance split_threshold_blocks must be positive");
        if (style != COVE_LB_HYBRID && style != COVE_LB_DEVICE) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "unknown layout style");
        if (nbr < 0 || !brp || !item_rp || !num_items) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "bad argument");
        *num_items = lb_count(nbr, brp, chunk, split, style, item_rp, static_cast<cudaStream_t>(stream));
    });
}

cove_status cove_lb_layout_fill(int32_t nbr, const int32_t* brp, const int32_t* brvp,
                                const uint32_t* bitmap, const int32_t* item_rp, int32_t chunk,
                                int32_t split, int32_t style, uint64_t* words, void* items,
                                void* stream) {
    return guarded([&] {
        if (chunk <= 0) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "GPU BitBSR load-balance chunk_blocks must be positive");
        if (split < 0) split = chunk;
        if (split == 0) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "GPU BitBSR load-balance split_threshold_blocks must be positive");
        if (nbr < 0 || !brp || !brvp || !item_rp) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "bad argument");
        lb_fill(nbr, brp, brvp, bitmap, item_rp, chunk, split, style, words,
                static_cast<WorkItem*>(items), static_cast<cudaStream_t>(stream));
    });
}

cove_status cove_hybrid_spmv(const cove_hybrid_desc* a, const cove_values_desc* v, const void* x,
                             void* y, void* stream) {
    return guarded([&] {
        if (!a || !v) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null descriptor");
        if (a->rows < 0 || a->cols < 0 || a->num_block_rows != (a->rows + kBlockRows - 1) / kBlockRows) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "fused CSR+BitBSR shape mismatch");
        }
        if (a->dtype != COVE_F64 && a->dtype != COVE_F32) COVE_THROW(COVE_ERR_UNSUPPORTED, "dtype");
        if (v->route < COVE_ROUTE_HYBRID || v->route > COVE_ROUTE_BFP4) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "unknown route");
        }
        const bool bitbsr_only = v->route >= COVE_ROUTE_IMPLICIT_ONE;
        if (bitbsr_only && (a->residual_nnz > 0 || a->num_chunks > 0)) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT,
                       std::string(cove_route_name(v->route)) + " is a BitBSR-only value codec: no residual");
        }
        if (v->route == COVE_ROUTE_SIGN2 && a->kept_blocks > 0 && !v->sign_masks) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "sign2 route needs sign_masks");
        }
        if ((v->route == COVE_ROUTE_FP16_NNZ || v->route == COVE_ROUTE_BFP4) && a->kept_nnz > 0 && !v->kept) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "per-nnz value stream missing");
        }
        if (v->route == COVE_ROUTE_BFP4 && a->kept_blocks > 0 && !v->block_scale) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "bfp4 route needs block_scale");
        }
        if (a->rows > 0 && (!a->block_row_ptr || !a->block_row_val_ptr || !y)) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null stream");
        }
        if (a->num_chunks > 0 && (!a->chunk_row || !a->chunk_pbegin || !a->chunk_pcount)) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null long-row chunk stream");
        }
        KernelShape k;
        k.dtype = a->dtype;
        k.rows = a->rows;
        k.cols = a->cols;
        k.nbr = a->num_block_rows;
        k.kept_brp = a->block_row_ptr;
        k.kept_brvp = a->block_row_val_ptr;
        k.words = a->words;
        k.res_rp = bitbsr_only ? nullptr : a->res_row_ptr;
        k.res_col = bitbsr_only ? nullptr : a->res_col_idx;
        // the caller's layout has no heavy-row split: keep the group kernel
        k.slots = std::max(1, choose_slots(a->num_block_rows, a->kept_blocks, a->rows, a->residual_nnz));
        k.long_tau = a->num_chunks > 0 ? a->long_row_tau : 0;
        k.num_chunks = a->num_chunks > 0 ? a->num_chunks : 0;
        k.chunk_row = a->chunk_row;
        k.chunk_pbegin = a->chunk_pbegin;
        k.chunk_pcount = a->chunk_pcount;
        RouteValues rv;
        rv.route = v->route;
        rv.kept = v->kept;
        rv.res = v->res;
        rv.scale = v->block_scale;
        rv.codebook = v->codebook;
        rv.codebook_size = v->codebook_size;
        if (v->route == COVE_ROUTE_BFP8_OUTLIER) {
            rv.num_outliers = v->num_outliers;
            rv.out_rows = v->outlier_rows;
            rv.out_cols = v->outlier_cols;
            rv.out_vals = v->outlier_vals;
        }
        rv.tile_words = v->tile_code_words;
        rv.tile_bits = v->tile_bits;
        rv.value_scale = v->value_scale;
        rv.sign_masks = v->sign_masks;
        if (v->route == COVE_ROUTE_TILE_CODE && !v->tile_code_words) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "tile-code route needs tile_code_words");
        }
        if (v->route == COVE_ROUTE_DICT_U8 && v->codebook_size > 256) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "u8 dictionary holds at most 256 values");
        }
        launch_hybrid_spmv(k, rv, x, y, static_cast<cudaStream_t>(stream));
    });
}

cove_status cove_spmv(const cove_plan* P, const void* x, void* y, void* stream) {
    if (!P) {
        cove::set_last_error("null plan");
        return COVE_ERR_INVALID_ARGUMENT;
    }
    return cove_spmv_route(P, P->dispatched_route, x, y, stream);
}

cove_status cove_spmv_host(cove_plan* P, const void* x_host, void* y_host, void* stream) {
    return guarded([&] {
        if (!P || !x_host || !y_host) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (!P->x_stage.p) P->x_stage.alloc(static_cast<size_t>(P->cols) * P->esz);
        if (!P->y_stage.p) P->y_stage.alloc(static_cast<size_t>(P->rows) * P->esz);
        if (!P->pipe) P->pipe = build_host_pipeline(P);
        HostPipeline& hp = *P->pipe;
        const bool overlap = (hp.kx > 1 || hp.ky > 1) && is_pinned(x_host) && is_pinned(y_host);
        if (!overlap) {  // pageable buffers: copies are host-synchronous anyway
            CUDA_OK(cudaMemcpyAsync(P->x_stage.p, x_host, static_cast<size_t>(P->cols) * P->esz,
                                    cudaMemcpyHostToDevice, s));
            launch_hybrid_spmv(P->shape(), P->route_values(P->dispatched_route), P->x_stage.p,
                               P->y_stage.p, s);
            CUDA_OK(cudaMemcpyAsync(y_host, P->y_stage.p, static_cast<size_t>(P->rows) * P->esz,
                                    cudaMemcpyDeviceToHost, s));
            CUDA_OK(cudaStreamSynchronize(s));
            return;
        }
        // The sliced sequence is a few dozen API calls; it is captured once per
        // pair of host buffers and replayed as one graph launch.
        if (!(hp.exec && hp.graph_x == x_host && hp.graph_y == y_host)) {
            if (hp.exec) cudaGraphExecDestroy(hp.exec);
            hp.exec = nullptr;
            cudaGraph_t g = nullptr;
            CUDA_OK(cudaStreamBeginCapture(hp.s_cap, cudaStreamCaptureModeThreadLocal));
            try {
                issue_sliced(P, hp, x_host, y_host, hp.s_cap);
            } catch (...) {
                cudaStreamEndCapture(hp.s_cap, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            CUDA_OK(cudaStreamEndCapture(hp.s_cap, &g));
            const cudaError_t ie = cudaGraphInstantiate(&hp.exec, g, 0);
            cudaGraphDestroy(g);
            CUDA_OK(ie);
            hp.graph_x = x_host;
            hp.graph_y = y_host;
        }
        CUDA_OK(cudaGraphLaunch(hp.exec, s));
        CUDA_OK(cudaStreamSynchronize(s));
    });
}

int32_t cove_spmv_launches(const cove_plan* P, int32_t route) {
    if (!P || !P->has_route(route)) return -1;
    return hybrid_spmv_launch_count(P->shape(), P->route_values(route));
}

cove_status cove_compare_vectors(const void* ref, const void* got, int64_t n, int32_t dtype,
                                 double* out3, void* stream) {
    return guarded([&] {
        if (!out3 || (n > 0 && (!ref || !got))) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (dtype == COVE_F64) {
            compare_reduce<double>(static_cast<const double*>(ref), static_cast<const double*>(got), n, out3, s);
        } else {
            compare_reduce<float>(static_cast<const float*>(ref), static_cast<const float*>(got), n, out3, s);
        }
    });
}

cove_status cove_canonical_x(void* x, int64_t n, int32_t dtype, void* stream) {
    return guarded([&] {
        if (n > 0 && !x) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null vector");
        if (n == 0) return;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (dtype == COVE_F64) {
            canonical_x_kernel<double><<<grid_for(n, kThreads), kThreads, 0, s>>>(n, static_cast<double*>(x));
        } else {
            canonical_x_kernel<float><<<grid_for(n, kThreads), kThreads, 0, s>>>(n, static_cast<float*>(x));
        }
        CUDA_LAUNCH_OK();
    });
}

}  // extern "C"
