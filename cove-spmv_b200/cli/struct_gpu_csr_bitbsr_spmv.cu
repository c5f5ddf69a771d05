// struct_gpu_csr_bitbsr_spmv -- command-line driver of the hybrid / joint
// CSR+BitBSR SpMV with the reference CLI's options and key: value report
// (structural/src/main_gpu_csr_bitbsr_spmv.cu:30-150 options, :1186-1476
// report), so the reference's sweep scripts (run_joint_sweep.py, the family
// sweep's parse_key_values) can drive this build unchanged.
//
// Built: --mode fused_lb with the CSR residual (the hot path; the reference's
// CLI accepts only the CSR residual too).  Its --mode two_pass is not part
// of this library: it is refused once the matrix is read, where the
// reference would start it.  Option checks and messages are the
// reference's, in its order.  The cuSPARSE CSR baseline is the cusparse_csr
// layout of struct_gpu_spmv.
// Everything runs through the C ABI (cove_b200.h): the plan
// is built on the GPU, x is the reference's canonical input vector, y is
// timed with CUDA events, and --verify-cpu compares against a CPU CSR SpMV.
#include "cove_b200.h"
#include "structural/matrix_market.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <iomanip>
#include <iostream>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

struct Options {
    std::string matrix_path;
    std::string precision = "double";
    std::string mode = "fused_lb";
    std::string split_policy = "cost_gated";
    std::string residual_format = "csr";
    double cost_bitmap_block = 10.0, cost_bitmap_nnz = 0.0, cost_csr_block = 0.0, cost_csr_nnz = 1.0;
    int block_rows = 8, block_cols = 4;
    int residual_threshold = 32;
    int long_row_split = 0;
    int lb_chunk_blocks = 32;
    int lb_split_threshold_blocks = -1;
    std::string cusparse_alg = "default";
    int warmup = 5;
    int iterations = 20;
    bool verify_cpu = false;
    std::string operator_label = "hybrid_fused_lb";
    std::string value_codec = "original";
};

void usage(const char* argv0) {
    // the reference's text (--value-codec is accepted too, as there)
    std::cerr << "usage: " << argv0 << " MATRIX.mtx [--precision float|double] [--mode fused_lb|two_pass]"
              << " [--split-policy threshold|cost_gated] [--residual-format csr] [--br 8] [--bc 4]"
              << " [--residual-threshold N] [--long-row-split N]"
              << " [--cost-bitmap-block X] [--cost-bitmap-nnz X] [--cost-csr-block X] [--cost-csr-nnz X]"
              << " [--lb-chunk-blocks N] [--lb-split-threshold-blocks N]"
              << " [--cusparse-alg default|csr_alg1|csr_alg2] [--operator-label NAME]"
              << " [--warmup N] [--iters N] [--verify-cpu]\n";
}

int to_int(const std::string& s) { return std::stoi(s); }
double to_double(const std::string& s) { return std::stod(s); }

// The joint codecs (:1222-1223); any other --value-codec runs the lossless
// hybrid alone, as the reference does.
bool joint_codec(const std::string& c) { return c == "auto" || c == "dict" || c == "bfp8" || c == "bfp8_outlier"; }

Options parse_options(int argc, char** argv) {
    Options o;
    if (argc < 2) {
        usage(argv[0]);
        std::exit(2);
    }
    o.matrix_path = argv[1];
    if (o.matrix_path == "--help" || o.matrix_path == "-h") {
        usage(argv[0]);
        std::exit(0);
    }
    for (int i = 2; i < argc; ++i) {
        const std::string a = argv[i];
        const bool has = i + 1 < argc;
        auto val = [&]() { return std::string(argv[++i]); };
        // values checked as they are read, with the reference's aliases and
        // messages (main_gpu_csr_bitbsr_spmv.cu:85-106, 128-141)
        if (a == "--precision" && has) {
            o.precision = val();
            if (o.precision != "float" && o.precision != "double")
                throw std::runtime_error("precision must be float or double");
        } else if (a == "--mode" && has) {
            o.mode = val();
            if (o.mode == "fused") o.mode = "fused_lb";
            if (o.mode != "fused_lb" && o.mode != "two_pass") throw std::runtime_error("mode must be fused_lb or two_pass");
        } else if (a == "--split-policy" && has) {
            o.split_policy = val();
            if (o.split_policy == "cost" || o.split_policy == "auto") o.split_policy = "cost_gated";
            if (o.split_policy != "threshold" && o.split_policy != "cost_gated")
                throw std::runtime_error("split-policy must be threshold or cost_gated");
        } else if (a == "--residual-format" && has) {
            o.residual_format = val();
            if (o.residual_format != "csr") throw std::runtime_error("residual-format must be csr");
        }
        else if (a == "--br" && has) o.block_rows = to_int(val());
        else if (a == "--bc" && has) o.block_cols = to_int(val());
        else if ((a == "--residual-threshold" || a == "--threshold") && has) o.residual_threshold = to_int(val());
        else if (a == "--value-codec" && has) o.value_codec = val();
        else if (a == "--long-row-split" && has) o.long_row_split = to_int(val());
        else if (a == "--cost-bitmap-block" && has) o.cost_bitmap_block = to_double(val());
        else if (a == "--cost-bitmap-nnz" && has) o.cost_bitmap_nnz = to_double(val());
        else if (a == "--cost-csr-block" && has) o.cost_csr_block = to_double(val());
        else if (a == "--cost-csr-nnz" && has) o.cost_csr_nnz = to_double(val());
        else if ((a == "--lb-chunk-blocks" || a == "--chunk-blocks") && has) o.lb_chunk_blocks = to_int(val());
        else if ((a == "--lb-split-threshold-blocks" || a == "--split-threshold-blocks" ||
                  a == "--lb-split-threshold") && has) o.lb_split_threshold_blocks = to_int(val());
        else if (a == "--cusparse-alg" && has) {
            o.cusparse_alg = val();
            if (o.cusparse_alg == "alg1") o.cusparse_alg = "csr_alg1";
            if (o.cusparse_alg == "alg2") o.cusparse_alg = "csr_alg2";
            if (o.cusparse_alg != "default" && o.cusparse_alg != "csr_alg1" && o.cusparse_alg != "csr_alg2")
                throw std::runtime_error("cusparse-alg must be default, csr_alg1, or csr_alg2");
        }
        else if (a == "--operator-label" && has) o.operator_label = val();
        else if (a == "--warmup" && has) o.warmup = to_int(val());
        else if ((a == "--iters" || a == "--iterations") && has) o.iterations = to_int(val());
        else if (a == "--verify-cpu") o.verify_cpu = true;
        else if (a == "--help" || a == "-h") {
            usage(argv[0]);
            std::exit(0);
        } else {
            throw std::runtime_error("unknown or incomplete argument: " + a);
        }
    }
    // the reference's checks, in its order (main_gpu_csr_bitbsr_spmv.cu:158-184)
    if (o.block_rows != 8 || o.block_cols != 4)
        throw std::runtime_error("CSR+BitBSR GPU probe currently supports only 8x4 blocks");
    if (o.residual_threshold < 0) throw std::runtime_error("residual-threshold must be non-negative");
    if (o.cost_bitmap_block < 0 || o.cost_bitmap_nnz < 0 || o.cost_csr_block < 0 || o.cost_csr_nnz < 0)
        throw std::runtime_error("CSR+BitBSR split cost model must be non-negative");
    if (o.warmup < 0 || o.iterations <= 0)
        throw std::runtime_error("warmup must be non-negative and iterations must be positive");
    if (o.lb_chunk_blocks <= 0) throw std::runtime_error("lb-chunk-blocks must be positive");
    if (o.lb_split_threshold_blocks < 0) o.lb_split_threshold_blocks = o.lb_chunk_blocks;
    if (o.lb_split_threshold_blocks <= 0) throw std::runtime_error("lb-split-threshold-blocks must be positive");
    return o;
}

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void cove_ok(cove_status s) {
    if (s != COVE_OK) throw std::runtime_error(cove_last_error());
}

double host_ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

template <typename T>
struct DeviceArray {
    T* p = nullptr;
    explicit DeviceArray(size_t n) { cuda_ok(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)), "cudaMalloc"); }
    ~DeviceArray() { cudaFree(p); }
    DeviceArray(const DeviceArray&) = delete;
    DeviceArray& operator=(const DeviceArray&) = delete;
};

// y = A x in T, row by row (the reference's spmv_csr arithmetic).
template <typename T>
std::vector<T> cpu_spmv(const structural::CsrMatrix<T>& a, const std::vector<T>& x) {
    std::vector<T> y(static_cast<size_t>(a.rows));
#pragma omp parallel for schedule(static)
    for (int r = 0; r < a.rows; ++r) {
        T s = T(0);
        for (int p = a.row_ptr[r]; p < a.row_ptr[r + 1]; ++p) s += a.values[p] * x[a.col_idx[p]];
        y[static_cast<size_t>(r)] = s;
    }
    return y;
}

// Times `reps` launches of one route; returns {min, sum} in milliseconds.
std::pair<float, double> time_route(cove_plan* plan, int32_t route, const void* x, void* y, int warmup,
                                    int reps) {
    for (int i = 0; i < warmup; ++i) cove_ok(cove_spmv_route(plan, route, x, y, nullptr));
    cudaEvent_t a, b;
    cuda_ok(cudaEventCreate(&a), "cudaEventCreate");
    cuda_ok(cudaEventCreate(&b), "cudaEventCreate");
    float mn = std::numeric_limits<float>::max();
    double sum = 0.0;
    for (int i = 0; i < reps; ++i) {
        cuda_ok(cudaEventRecord(a, nullptr), "cudaEventRecord");
        cove_ok(cove_spmv_route(plan, route, x, y, nullptr));
        cuda_ok(cudaEventRecord(b, nullptr), "cudaEventRecord");
        cuda_ok(cudaEventSynchronize(b), "cudaEventSynchronize");
        float ms = 0.0f;
        cuda_ok(cudaEventElapsedTime(&ms, a, b), "cudaEventElapsedTime");
        mn = std::min(mn, ms);
        sum += ms;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return {mn, sum};
}

template <typename T>
int run(const Options& o) {
    const auto t_load = std::chrono::steady_clock::now();
    const auto loaded = structural::read_matrix_market_with_info<T>(o.matrix_path);
    const double load_ms = host_ms_since(t_load);
    if (o.mode == "two_pass") throw std::runtime_error("mode two_pass is not part of this build (fused_lb only)");
    const auto& A = loaded.matrix;

    const auto t_ctx = std::chrono::steady_clock::now();
    cuda_ok(cudaFree(nullptr), "CUDA context");
    const double cuda_context_ms = host_ms_since(t_ctx);

    const auto t_up = std::chrono::steady_clock::now();
    const size_t nnz = A.values.size();
    DeviceArray<int32_t> d_rp(A.row_ptr.size()), d_ci(nnz);
    DeviceArray<T> d_v(nnz), d_x(static_cast<size_t>(A.cols)), d_y(static_cast<size_t>(A.rows));
    cuda_ok(cudaMemcpy(d_rp.p, A.row_ptr.data(), A.row_ptr.size() * 4, cudaMemcpyHostToDevice), "upload");
    if (nnz > 0) {
        cuda_ok(cudaMemcpy(d_ci.p, A.col_idx.data(), nnz * 4, cudaMemcpyHostToDevice), "upload");
        cuda_ok(cudaMemcpy(d_v.p, A.values.data(), nnz * sizeof(T), cudaMemcpyHostToDevice), "upload");
    }
    const double upload_ms = host_ms_since(t_up);
    const int32_t dtype = sizeof(T) == 8 ? COVE_F64 : COVE_F32;

    cove_csr_desc d{};
    d.rows = A.rows;
    d.cols = A.cols;
    d.nnz = static_cast<int64_t>(nnz);
    d.row_ptr = d_rp.p;
    d.col_idx = d_ci.p;
    d.values = d_v.p;
    d.dtype = dtype;
    d.row_ptr_i32 = 1;
    cove_plan_opts po;
    cove_plan_opts_default(&po);
    po.residual_threshold = o.residual_threshold;
    po.split_policy = o.split_policy == "threshold" ? COVE_SPLIT_THRESHOLD : COVE_SPLIT_COST_GATED;
    po.cost_bitmap_block = o.cost_bitmap_block;
    po.cost_bitmap_nnz = o.cost_bitmap_nnz;
    po.cost_csr_block = o.cost_csr_block;
    po.cost_csr_nnz = o.cost_csr_nnz;
    po.lb_chunk_blocks = o.lb_chunk_blocks;
    po.lb_split_threshold_blocks = o.lb_split_threshold_blocks;
    po.lb_style = COVE_LB_HYBRID;
    po.long_row_split = std::max(0, o.long_row_split);  // <= 0: no long-row chunks, as :1159
    po.value_codec = o.value_codec == "auto" ? COVE_CODEC_AUTO
                     : o.value_codec == "dict" ? COVE_CODEC_DICT
                     : o.value_codec == "bfp8" ? COVE_CODEC_BFP8
                     : o.value_codec == "bfp8_outlier" ? COVE_CODEC_BFP8_OUTLIER
                     : COVE_CODEC_ORIGINAL;
    po.gate_enable = 0;      // the report carries the joint error; dispatch is the caller's
    po.keep_lossless = 1;    // the hybrid fp64 route is timed beside the joint one
    cove_plan* plan = nullptr;
    const auto t_plan = std::chrono::steady_clock::now();
    cove_ok(cove_plan_build(&d, &po, nullptr, &plan));
    cuda_ok(cudaDeviceSynchronize(), "plan build");
    const double plan_ms = host_ms_since(t_plan);
    struct PlanGuard {
        cove_plan* p;
        ~PlanGuard() { cove_plan_destroy(p); }
    } guard{plan};
    cove_plan_info info{};
    cove_ok(cove_plan_get_info(plan, &info));

    // x = make_input_vector (spmv_harness.hpp:32-39), on the device and the host
    cove_ok(cove_canonical_x(d_x.p, A.cols, dtype, nullptr));
    std::vector<T> x(static_cast<size_t>(A.cols));
    cuda_ok(cudaMemcpy(x.data(), d_x.p, x.size() * sizeof(T), cudaMemcpyDeviceToHost), "download");

    const auto [fused_min_ms, fused_sum_ms] =
        time_route(plan, COVE_ROUTE_HYBRID, d_x.p, d_y.p, o.warmup, o.iterations);

    std::vector<T> y0;
    double cpu_spmv_ms = 0.0;
    DeviceArray<T> d_y0(static_cast<size_t>(A.rows));
    if (o.verify_cpu) {
        const auto t_cpu = std::chrono::steady_clock::now();
        y0 = cpu_spmv(A, x);
        cpu_spmv_ms = host_ms_since(t_cpu);
        cuda_ok(cudaMemcpy(d_y0.p, y0.data(), y0.size() * sizeof(T), cudaMemcpyHostToDevice), "upload");
    }
    auto compare = [&](const T* got) {
        double e[3] = {0.0, 0.0, 0.0};
        cove_ok(cove_compare_vectors(d_y0.p, got, A.rows, dtype, e, nullptr));
        return std::vector<double>{e[0], e[1], e[2]};
    };
    bool verified = true;
    std::vector<double> err{0.0, 0.0, 0.0};
    if (o.verify_cpu) {
        err = compare(d_y.p);  // d_y holds the last hybrid result
        const double abs_tol = sizeof(T) == 4 ? 1e-2 : 1e-8;
        const double rel_tol = sizeof(T) == 4 ? 1e-4 : 1e-10;
        verified = err[0] <= abs_tol || err[1] <= rel_tol;
    }

    if (joint_codec(o.value_codec)) {
        const auto [joint_min_ms, joint_sum_ms] =
            time_route(plan, info.joint_route, d_x.p, d_y.p, o.warmup, o.iterations);
        (void)joint_sum_ms;
        double jrel = -1.0;
        if (o.verify_cpu) jrel = compare(d_y.p)[2];
        const bool counted = o.value_codec == "auto" || o.value_codec == "dict";
        std::cout << "joint_value_codec: " << cove_route_name(info.joint_route) << "\n";
        std::cout << "joint_requested_codec: " << o.value_codec << "\n";
        std::cout << "joint_value_cardinality: " << (counted ? info.value_cardinality : 0) << "\n";
        std::cout << "joint_min_ms: " << joint_min_ms << "\n";
        std::cout << "joint_hybrid_fp64_min_ms: " << fused_min_ms << "\n";
        std::cout << "joint_speedup_vs_hybrid_fp64: "
                  << (joint_min_ms > 0.0f ? fused_min_ms / joint_min_ms : -1.0) << "\n";
        std::cout << "joint_bytes_per_nnz: " << info.joint_bytes_per_nnz << "\n";
        std::cout << "joint_rel_err: " << jrel << "\n";
        std::cout << "joint_verify_pass_1e-2: " << ((jrel >= 0.0 && jrel <= 1e-2) ? 1 : 0) << "\n";
    }

    const double full_bits = static_cast<double>(info.full_bitbsr_position_bits);
    const double split_bits = static_cast<double>(info.split_position_bits);
    const double res_bits = static_cast<double>(info.residual_csr_position_bits);
    const double kn = static_cast<double>(info.kept_nnz + info.residual_nnz);
    std::cout << "matrix: " << o.matrix_path << "\n";
    std::cout << "matrix_market_field: " << structural::to_string(loaded.info.field) << "\n";
    std::cout << "matrix_market_symmetry: " << structural::to_string(loaded.info.symmetry) << "\n";
    std::cout << "precision: " << o.precision << "\n";
    std::cout << "shape: " << A.rows << " x " << A.cols << "\n";
    std::cout << "nnz: " << nnz << "\n";
    std::cout << "block: " << o.block_rows << " x " << o.block_cols << "\n";
    std::cout << "spmv_layout: csr_bitbsr_split\n";
    std::cout << "spmv_effective_layout: csr_bitbsr_fused_lb\n";
    std::cout << "residual_format: csr\n";
    std::cout << "residual_threshold: " << o.residual_threshold << "\n";
    std::cout << "split_policy: " << o.split_policy << "\n";
    std::cout << "cost_model: bitmap_block=" << o.cost_bitmap_block << ", bitmap_nnz=" << o.cost_bitmap_nnz
              << ", csr_block=" << o.cost_csr_block << ", csr_nnz=" << o.cost_csr_nnz << "\n";
    std::cout << "cusparse_alg: none\n";
    std::cout << "cusparse_buffer_bytes: 0\n";
    std::cout << "load_balance_chunk_blocks: " << o.lb_chunk_blocks << "\n";
    std::cout << "load_balance_split_threshold_blocks: " << o.lb_split_threshold_blocks << "\n";
    std::cout << "gpu_work_items: " << info.work_items << "\n";
    std::cout << "gpu_output_residency: device\n";
    std::cout << "full_bitbsr_blocks: " << info.full_blocks << "\n";
    std::cout << "kept_blocks: " << info.kept_blocks << "\n";
    std::cout << "residual_blocks: " << info.residual_blocks << "\n";
    std::cout << "cost_skipped_blocks: " << info.cost_skipped_blocks << "\n";
    std::cout << "kept_nnz: " << info.kept_nnz << "\n";
    std::cout << "residual_nnz: " << info.residual_nnz << "\n";
    std::cout << "cost_skipped_nnz: " << info.cost_skipped_nnz << "\n";
    std::cout << "full_bitbsr_position_bits: " << info.full_bitbsr_position_bits << "\n";
    std::cout << "kept_bitbsr_position_bits: " << info.kept_bitbsr_position_bits << "\n";
    std::cout << "residual_csr_position_bits: " << info.residual_csr_position_bits << "\n";
    std::cout << "split_position_bits: " << info.split_position_bits << "\n";
    std::cout << std::fixed << std::setprecision(6);
    std::cout << "split_vs_full_bitbsr_ratio: " << (full_bits > 0 ? split_bits / full_bits : 0.0) << "\n";
    std::cout << "residual_block_ratio: "
              << (info.full_blocks > 0 ? static_cast<double>(info.residual_blocks) / info.full_blocks : 0.0) << "\n";
    std::cout << "residual_nnz_ratio: " << (kn > 0 ? info.residual_nnz / kn : 0.0) << "\n";
    std::cout << "residual_position_ratio_in_split: " << (split_bits > 0 ? res_bits / split_bits : 0.0) << "\n";
    std::cout << "residual_position_ratio_vs_full: " << (full_bits > 0 ? res_bits / full_bits : 0.0) << "\n";
    std::cout << std::defaultfloat;
    std::cout << "operator_name: " << o.operator_label << "\n";
    std::cout << "operator_family: structural_hybrid\n";
    std::cout << "operator_promotion_status: promoted\n";
    std::cout << "operator_runner: csr_bitbsr_fused_lb\n";
    std::cout << "status: ok\n";
    std::cout << "verify_gate: exact_abs_or_rel\n";
    std::cout << "value_codec: original\n";
    std::cout << "value_codec_effective: " << (sizeof(T) == 8 ? "raw_double" : "raw_float") << "\n";
    std::cout << "value_codec_exact: 1\n";
    std::cout << "value_codec_codebook_size: 0\n";
    std::cout << "value_codec_bytes_per_nnz: " << sizeof(T) << "\n";
    std::cout << "value_codec_payload_bytes: " << nnz * sizeof(T) << "\n";
    std::cout << "gpu_num_blocks: " << info.full_blocks << "\n";
    std::cout << std::fixed << std::setprecision(6);
    std::cout << "min_ms: " << fused_min_ms << "\n";
    std::cout << "avg_ms: " << fused_sum_ms / o.iterations << "\n";
    std::cout << std::setprecision(4);
    std::cout << "timing_ms: load=" << load_ms << ", cuda_context=" << cuda_context_ms
              << ", upload_host=" << upload_ms << ", plan_build_gpu=" << plan_ms
              << ", gpu_spmv_avg_event=" << fused_sum_ms / o.iterations
              << ", gpu_spmv_min_event=" << fused_min_ms
              << ", gpu_fused_avg_event=" << fused_sum_ms / o.iterations
              << ", gpu_fused_min_event=" << fused_min_ms
              << ", cpu_spmv=" << (o.verify_cpu ? cpu_spmv_ms : 0.0) << "\n";
    std::cout << std::defaultfloat;
    if (o.verify_cpu) {
        std::cout << "verify_cpu: " << (verified ? "PASS" : "FAIL") << ", max_abs=" << err[0]
                  << ", max_rel=" << err[1] << "\n";
    } else {
        std::cout << "verify_cpu: SKIP\n";
    }
    return verified ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        const Options o = parse_options(argc, argv);
        return o.precision == "float" ? run<float>(o) : run<double>(o);
    } catch (const std::exception& e) {
        std::cerr << "error: " << e.what() << "\n";
        return 1;
    }
}
