// cove_plan.cuh -- the plan object behind the C ABI.
#pragma once

#include "cove_codecs.cuh"
#include "cove_spmv.cuh"

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

    // staging for cove_spmv_host
    cove::DevBuf x_stage, y_stage;
    cove::DevBuf err;  // int, set by a kernel whose bounded wait gave up

    cove::KernelShape shape() const;
    cove::RouteValues route_values(int route) const;
    bool has_route(int route) const;
};
