// cove_plan.cuh -- the plan object behind the C ABI.
#pragma once

#include "cove_codecs.cuh"
#include "cove_spmv.cuh"

#include <memory>

namespace cove {

// Copy/compute overlap of cove_spmv_host: x arrives in kx slices on one
// copy stream; the main pass runs in ky block-row slices, each as soon as
// the x slices up to its highest column have landed; each y slice leaves on
// a second copy stream as soon as its rows are final.  Built on first use;
// the sequence is replayed as a CUDA graph while the host buffers stay the same.
struct HostPipeline {
    int kx = 0, ky = 0;
    std::vector<int64_t> x_cut;   // kx+1 element offsets into x
    std::vector<int32_t> br_cut;  // ky+1 block-row offsets
    std::vector<int> need;        // per block-row slice: last x slice it reads (-1: none)
    cudaStream_t s_in = nullptr, s_out = nullptr;
    std::vector<cudaEvent_t> x_ready, y_ready;
    cudaEvent_t start = nullptr, out_done = nullptr;
    // the sequence captured as a graph for one pair of host buffers
    cudaStream_t s_cap = nullptr;
    cudaGraphExec_t exec = nullptr;
    const void* graph_x = nullptr;
    const void* graph_y = nullptr;
    ~HostPipeline();
};

// Per block row, the lowest and highest column of x the SpMV reads
// ({INT_MAX, -1} for an empty block row); synchronous.
void block_row_col_bounds(const cove_plan* P, std::vector<int32_t>* lo, std::vector<int32_t>* hi);

}  // namespace cove

namespace cove {
// Work vectors of a CG solve (r, the p window, Ap, dot partials, scalars),
// allocated by the first solve and reused while the sizes stay the same.
struct CgWorkspace {
    DevBuf r, pw, ap, partial, scal;
    int64_t n = -1, wl = -1;
};
}  // namespace cove

struct cove_plan {
    cove_plan_opts opts{};
    int dtype = COVE_F64;
    size_t esz = 8;
    int32_t rows = 0, cols = 0, nbr = 0;
    int64_t nnz = 0;

    cove::FullBitBsr full;
    bool has_full = false;
    cove::SplitParts sp;
    cove::Layout lay;
    cove::Chunks chunks;      // reference long-row chunk stream (tau from opts)
    cove::Chunks kchunks;     // the kernel's own long-row chunks
    bool kchunks_alias = false;

    // kernel work split
    int slots = 4;
    int heavy_limit = 0x7fffffff;
    int long_tau = 0;
    int64_t num_heavy = 0;
    cove::DevBuf heavy_br, heavy_b0, heavy_b1;

    // joint value streams
    bool has_lossless = true;
    cove::DictStreams dict;
    bool has_dict = false;
    cove::DevBuf bfp8_q, bfp8_scale, res_bf16;
    bool has_bfp8 = false;
    cove::DevBuf out_rows, out_cols, out_vals;
    int64_t num_out = 0;
    double outlier_threshold = 0.0;
    bool has_outlier = false;

    int64_t uniq = 0;
    int joint_route = COVE_ROUTE_HYBRID;
    int dispatched_route = COVE_ROUTE_HYBRID;
    bool gate_evaluated = false;
    bool gate_pass = false;
    double joint_rel = -1.0;

    // host-call staging of x and y (cove_spmv_host)
    cove::DevBuf x_stage, y_stage;
    // CG work vectors, kept between solves on this plan (cove_cg_solve)
    mutable cove::CgWorkspace cg_ws;
    std::unique_ptr<cove::HostPipeline> pipe;

    cove::KernelShape shape() const;
    cove::RouteValues route_values(int route) const;
    bool has_route(int route) const;
};
