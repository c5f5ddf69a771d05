// struct_gpu_spmv -- command-line driver of the BitBSR-only family runner
// (run_bitbsr_spmv_once over every value codec) and of the cuSPARSE CSR
// baseline, with the reference CLI's options, operator contract and
// key: value report (structural/src/main_gpu_spmv.cu, options
// structural/include/structural/spmv_cli_options.hpp, operator naming
// spmv_operator_plan.hpp), so run_gpu_spmv_family_sweep.py can drive this
// build unchanged.  The BitBSR layouts run through the C++ shim
// (include/structural/*) over the library's C ABI; x is the reference's
// canonical input vector; every timed SpMV is a CUDA-event pair.
#include "structural/gpu_convert.cuh"
#include "structural/gpu_value_codecs.cuh"
#include "structural/matrix_market.hpp"
#include "structural/operators/bitbsr_spmv_8x4_dispatch.cuh"
#include "structural/spmv_cli_options.hpp"
#include "structural/spmv_operator_plan.hpp"

#include <cuda_runtime.h>
#include <cusparse.h>
#include <thrust/device_vector.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <iomanip>
#include <iostream>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace {

using structural::Index;
using structural::Offset;
using Layout = structural::BitBsrSpmvLayoutKind8x4;
using Codec = structural::BitBsrValueCodecKind8x4;

// ---- options: structural/spmv_cli_options.hpp ------------------------------------

using Options = structural::SpmvCliOptions;

// report name of each value codec (value_codec_effective), in the enum's order
const std::vector<std::pair<Codec, const char*>>& codec_names() {
    static const std::vector<std::pair<Codec, const char*>> t = {
        {Codec::Raw, "original"},          {Codec::ImplicitOne, "all_one"},
        {Codec::ConstC, "const_c"},        {Codec::Sign2, "sign2"},
        {Codec::Sign2Scale, "sign2_scale"}, {Codec::Dict2, "dict2"},
        {Codec::Unique4, "dict4"},         {Codec::Unique16, "dict16"},
        {Codec::Dict256U8, "dict256_u8"},  {Codec::Dict65536U16, "dict65536_u16"},
        {Codec::Fp16, "fp16"},             {Codec::Bf16, "bf16"},
        {Codec::Bfp8, "bfp8"},             {Codec::Bfp8Outlier, "bfp8_outlier"},
        {Codec::Bfp4, "bfp4"},             {Codec::K256U8, "codebook256_u8"},
        {Codec::GlobalLogKmeans16, "global_logkmeans16"}, {Codec::GlobalLogKmeans32, "global_logkmeans32"},
        {Codec::GlobalLogKmeans64, "global_logkmeans64"}, {Codec::GlobalLogKmeans128, "global_logkmeans128"}};
    return t;
}
const char* codec_name(Codec c) {
    for (const auto& [k, n] : codec_names())
        if (k == c) return n;
    return "unknown";
}

// ---- operator contract: structural/spmv_operator_plan.hpp --------------------------

using structural::SpmvOperatorSpec;

structural::LoadBalancePolicy requested_policy(const Options& o) {
    return o.lb_policy == "binary_implicit_one" ? structural::LoadBalancePolicy::BinaryImplicitOne
                                                : structural::LoadBalancePolicy::Manual;
}

bool lossy_gate(const SpmvOperatorSpec& s) { return s.verify_gate == structural::SpmvVerifyGate::SpmvMaxRel; }

// ---- shared pieces ------------------------------------------------------------------

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void cusparse_ok(cusparseStatus_t s, const char* what) {
    if (s != CUSPARSE_STATUS_SUCCESS) throw std::runtime_error(std::string("cuSPARSE ") + what + " failed");
}

template <typename F>
auto timed_host(F&& f, double& ms) {
    const auto t0 = std::chrono::steady_clock::now();
    auto r = f();
    ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return r;
}

template <typename T>
std::vector<T> canonical_x(Index n) {  // spmv_harness.hpp:32-39
    std::vector<T> x(static_cast<size_t>(n));
    for (Index i = 0; i < n; ++i) x[static_cast<size_t>(i)] = static_cast<T>(static_cast<int>(i % 17) - 8) * static_cast<T>(0.125);
    return x;
}

struct Verify {
    bool run = false, pass = true;
    double max_abs = 0, max_rel = 0, global_rel = 0, cpu_ms = 0;
};

// y0 = A x in T on the host (spmv_csr), compared with the device y by the
// library's compare (max_abs, max_rel, global_rel of spmv.hpp:73-89).
template <typename T>
Verify verify(const structural::CsrMatrix<T>& a, const std::vector<T>& x, const thrust::device_vector<T>& d_y,
              bool lossy_gate) {
    Verify v;
    v.run = true;
    std::vector<T> y0(static_cast<size_t>(a.rows));
    timed_host([&] {
#pragma omp parallel for schedule(static)
        for (Index r = 0; r < a.rows; ++r) {
            T s = T(0);
            for (Offset p = a.row_ptr[r]; p < a.row_ptr[r + 1]; ++p) s += a.values[p] * x[a.col_idx[p]];
            y0[static_cast<size_t>(r)] = s;
        }
        return 0;
    }, v.cpu_ms);
    thrust::device_vector<T> d_y0(y0.begin(), y0.end());
    double e[3] = {0, 0, 0};
    const cove_status st = cove_compare_vectors(thrust::raw_pointer_cast(d_y0.data()),
                                                thrust::raw_pointer_cast(d_y.data()), a.rows,
                                                sizeof(T) == 8 ? COVE_F64 : COVE_F32, e, nullptr);
    if (st != COVE_OK) throw std::runtime_error(cove_last_error());
    v.max_abs = e[0];
    v.max_rel = e[1];
    v.global_rel = e[2];
    if (lossy_gate) {
        v.pass = v.global_rel <= 1e-2;
    } else {
        const double abs_tol = sizeof(T) == 4 ? 1e-2 : 1e-9, rel_tol = sizeof(T) == 4 ? 1e-4 : 1e-10;
        v.pass = v.max_abs <= abs_tol || v.max_rel <= rel_tol;
    }
    return v;
}

template <typename T>
void print_matrix_header(const Options& o, const structural::MatrixMarketLoadResult<T>& m, const char* block) {
    std::cout << "report_schema: structural_spmv_cli_v3\n";
    std::cout << "matrix: " << o.matrix_path << "\n";
    std::cout << "matrix_market_field: " << structural::to_string(m.info.field) << "\n";
    std::cout << "matrix_market_symmetry: " << structural::to_string(m.info.symmetry) << "\n";
    std::cout << "precision: " << o.precision << "\n";
    std::cout << "shape: " << m.matrix.rows << " x " << m.matrix.cols << "\n";
    std::cout << "nnz: " << m.matrix.nnz() << "\n";
    std::cout << "block: " << block << "\n";
}

void print_contract(const SpmvOperatorSpec& s) {
    std::cout << "operator_name: " << s.operator_name << "\n";
    std::cout << "operator_family: " << structural::spmv_operator_family_name(s.family) << "\n";
    std::cout << "operator_promotion_status: " << structural::spmv_promotion_status_name(s.promotion_status) << "\n";
    std::cout << "operator_runner: " << structural::spmv_operator_runner_name(s.runner) << "\n";
}

void print_verify(const Verify& v) {
    if (!v.run) {
        std::cout << "verify_cpu: SKIP\n";
        return;
    }
    std::cout << std::defaultfloat;
    std::cout << "verify_cpu: " << (v.pass ? "PASS" : "FAIL") << ", max_abs=" << v.max_abs
              << ", max_rel=" << v.max_rel << "\n";
    std::cout << "spmv_output_rel_err: " << v.global_rel << "\n";
}

// Warm-up and timed launches of `once(iter_ms)`; returns {sum, min}.
template <typename F>
std::pair<double, float> time_loop(const Options& o, F&& once) {
    for (int i = 0; i < o.warmup; ++i) once(nullptr);
    double sum = 0.0;
    float mn = std::numeric_limits<float>::max();
    for (int i = 0; i < o.iterations; ++i) {
        float ms = 0.0f;
        once(&ms);
        sum += ms;
        mn = std::min(mn, ms);
    }
    return {sum, mn};
}

// ---- cuSPARSE CSR baseline ---------------------------------------------------------

template <typename T>
int run_cusparse(const Options& o, const SpmvOperatorSpec& spec) {
    if (o.value_codec != "original")
        throw std::runtime_error("compressed value codecs are only supported for BitBSR layouts");
    double load_ms = 0, ctx_ms = 0, upload_ms = 0, setup_ms = 0, pre_ms = 0;
    float pre_event_ms = 0.0f;
    const auto m = timed_host([&] { return structural::read_matrix_market_with_info<T>(o.matrix_path); }, load_ms);
    const auto& a = m.matrix;
    timed_host([&] { cuda_ok(cudaFree(nullptr), "CUDA context"); return 0; }, ctx_ms);
    const auto x = canonical_x<T>(a.cols);
    thrust::device_vector<Offset> d_rp;
    thrust::device_vector<Index> d_ci;
    thrust::device_vector<T> d_v, d_x, d_y;
    timed_host([&] {
        d_rp = a.row_ptr;
        d_ci = a.col_idx;
        d_v = a.values;
        d_x = x;
        d_y.assign(static_cast<size_t>(a.rows), T(0));
        return 0;
    }, upload_ms);
    const cudaDataType vt = sizeof(T) == 8 ? CUDA_R_64F : CUDA_R_32F;
    const cusparseSpMVAlg_t alg = o.cusparse_alg == "csr_alg1"   ? CUSPARSE_SPMV_CSR_ALG1
                                  : o.cusparse_alg == "csr_alg2" ? CUSPARSE_SPMV_CSR_ALG2
                                                                 : CUSPARSE_SPMV_ALG_DEFAULT;
    cusparseHandle_t h = nullptr;
    cusparseSpMatDescr_t ma = nullptr;
    cusparseDnVecDescr_t vx = nullptr, vy = nullptr;
    size_t buf_bytes = 0;
    const T alpha = T(1), beta = T(0);
    timed_host([&] {
        cusparse_ok(cusparseCreate(&h), "create");
        cusparse_ok(cusparseCreateCsr(&ma, a.rows, a.cols, a.nnz(), thrust::raw_pointer_cast(d_rp.data()),
                                      thrust::raw_pointer_cast(d_ci.data()), thrust::raw_pointer_cast(d_v.data()),
                                      CUSPARSE_INDEX_32I, CUSPARSE_INDEX_32I, CUSPARSE_INDEX_BASE_ZERO, vt),
                    "create CSR");
        cusparse_ok(cusparseCreateDnVec(&vx, a.cols, thrust::raw_pointer_cast(d_x.data()), vt), "create x");
        cusparse_ok(cusparseCreateDnVec(&vy, a.rows, thrust::raw_pointer_cast(d_y.data()), vt), "create y");
        cusparse_ok(cusparseSpMV_bufferSize(h, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, ma, vx, &beta, vy, vt, alg,
                                            &buf_bytes),
                    "buffer size");
        return 0;
    }, setup_ms);
    thrust::device_vector<std::uint8_t> buf(buf_bytes);
    void* bp = buf_bytes ? thrust::raw_pointer_cast(buf.data()) : nullptr;
    cudaEvent_t e0, e1;
    cuda_ok(cudaEventCreate(&e0), "event");
    cuda_ok(cudaEventCreate(&e1), "event");
    timed_host([&] {
#if defined(CUSPARSE_VERSION) && CUSPARSE_VERSION >= 12700
        cuda_ok(cudaEventRecord(e0), "event");
        cusparse_ok(cusparseSpMV_preprocess(h, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, ma, vx, &beta, vy, vt, alg, bp),
                    "preprocess");
        cuda_ok(cudaEventRecord(e1), "event");
        cuda_ok(cudaEventSynchronize(e1), "event");
        cuda_ok(cudaEventElapsedTime(&pre_event_ms, e0, e1), "event");
#endif
        return 0;
    }, pre_ms);
    const auto [sum_ms, min_ms] = time_loop(o, [&](float* ms) {
        if (ms) cuda_ok(cudaEventRecord(e0), "event");
        cusparse_ok(cusparseSpMV(h, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, ma, vx, &beta, vy, vt, alg, bp), "SpMV");
        if (ms) {
            cuda_ok(cudaEventRecord(e1), "event");
            cuda_ok(cudaEventSynchronize(e1), "event");
            cuda_ok(cudaEventElapsedTime(ms, e0, e1), "event");
        }
    });
    cuda_ok(cudaDeviceSynchronize(), "SpMV");
    Verify v;
    if (o.verify_cpu) v = verify(a, x, d_y, lossy_gate(spec));

    print_matrix_header(o, m, "csr");
    print_contract(spec);
    std::cout << "spmv_layout: " << o.layout << "\n";
    std::cout << "spmv_effective_layout: cusparse_csr\n";
    std::cout << "position_codec: csr\n";
    std::cout << "position_codec_exact: true\n";
    std::cout << "position_codec_payload_bytes: "
              << static_cast<size_t>(a.rows + 1) * sizeof(Offset) + static_cast<size_t>(a.nnz()) * sizeof(Index) << "\n";
    std::cout << "value_codec: original\n";
    std::cout << "value_codec_exact: true\n";
    std::cout << "value_codec_codebook_size: 0\n";
    std::cout << "value_codec_payload_bytes: " << static_cast<size_t>(a.nnz()) * sizeof(T) << "\n";
    std::cout << "value_codec_bytes_per_nnz: " << sizeof(T) << "\n";
    std::cout << "cusparse_alg: " << o.cusparse_alg << "\n";
    std::cout << "cusparse_buffer_bytes: " << buf_bytes << "\n";
    std::cout << "load_balance_policy: manual\n";
    std::cout << "load_balance_chunk_blocks: 0\n";
    std::cout << "load_balance_split_threshold_blocks: 0\n";
    std::cout << "gpu_work_items: 0\n";
    std::cout << "gpu_output_residency: device\n";
    std::cout << "gpu_num_blocks: 0\n";
    std::cout << "verify_gate: " << structural::spmv_verify_gate_name(spec.verify_gate) << "\n";
    std::cout << "timing_scope: cusparse_event_includes_beta_zero\n";
    std::cout << std::fixed << std::setprecision(4);
    std::cout << "timing_ms: load=" << load_ms << ", cuda_context=" << ctx_ms
              << ", gpu_convert_host=0.0000, gpu_convert_event=0.0000, csr_upload_host=" << upload_ms
              << ", cusparse_setup_host=" << setup_ms << ", cusparse_preprocess_host=" << pre_ms
              << ", cusparse_preprocess_event=" << pre_event_ms
              << ", col_bitmap_pack_host=0.0000, col_bitmap_pack_event=0.0000, load_balance_pack_host=0.0000"
              << ", load_balance_pack_event=0.0000, value_codec_pack_host=0.0000"
              << ", gpu_spmv_avg_event=" << (sum_ms / o.iterations) << ", gpu_spmv_min_event=" << min_ms
              << ", cpu_spmv=" << (o.verify_cpu ? v.cpu_ms : 0.0) << "\n";
    print_verify(v);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cusparseDestroyDnVec(vy);
    cusparseDestroyDnVec(vx);
    cusparseDestroySpMat(ma);
    cusparseDestroy(h);
    return v.pass ? 0 : 1;
}

// ---- BitBSR family runner ----------------------------------------------------------

struct Report {
    bool auto_selected = false;
    int auto_unique_count = 0;
    bool auto_unique_overflow = false;
    size_t auto_raw_bytes = 0, auto_candidate_bytes = 0;
    size_t position_bytes = 0;
    bool exact = false;
    int codebook_size = 0;
    size_t payload_bytes = 0;
    bool value_only_valid = false;
    size_t value_only_bytes = 0;
    long long num_outliers = 0;
};

struct Timing {
    double load = 0, ctx = 0, convert_host = 0, auto_host = 0, pack_host = 0, lb_host = 0, codec_host = 0;
    float convert_event = 0, auto_event = 0, pack_event = 0, lb_event = 0;
};

size_t candidate_bytes(const structural::DeviceExactValueHistogram& h, Codec c) {
    switch (c) {
        case Codec::ImplicitOne: return 0;
        case Codec::ConstC: return h.const_c_payload_bytes;
        case Codec::Sign2: return h.sign2_payload_bytes;
        case Codec::Sign2Scale: return h.sign2_scale_payload_bytes;
        case Codec::Dict2: return h.dict2_payload_bytes;
        case Codec::Unique4: return h.dict4_payload_bytes;
        case Codec::Unique16: return h.dict16_payload_bytes;
        case Codec::Dict256U8: return h.dict256_u8_payload_bytes;
        case Codec::Dict65536U16: return h.dict65536_u16_payload_bytes;
        default: return h.raw_payload_bytes;
    }
}

// The value payload of `codec` built on the host from the BitBSR values and
// loaded into the plan (main_gpu_spmv.cu:631-848 lists the same fields).
template <typename T>
void build_values(const structural::BitBsrMatrix<T>& b, Codec codec, structural::BitBsrSpmvPlan8x4<T>& plan,
                  Report& r) {
    using namespace structural;
    auto load_tile = [&](const auto& t) {
        plan.tile_code_words.assign(t.tile_code_words.begin(), t.tile_code_words.end());
        plan.value_codebook.assign(t.codebook.begin(), t.codebook.end());
    };
    r.exact = !bitbsr_spmv_8x4_is_controlled_lossy_value_codec(codec);
    switch (codec) {
        case Codec::ImplicitOne:
            for (const T v : b.values)
                if (v != T(1)) throw std::runtime_error("all_one value codec requires every stored value to be 1");
            r.codebook_size = 0;
            r.payload_bytes = 0;
            break;
        case Codec::ConstC:
            plan.value_scale = build_const_c_value(b);
            r.codebook_size = 1;
            r.payload_bytes = sizeof(T);
            break;
        case Codec::Sign2: {
            const auto m = build_sign2_tile32_masks(b);
            plan.sign_masks.assign(m.begin(), m.end());
            r.payload_bytes = m.size() * 4;
            break;
        }
        case Codec::Sign2Scale: {
            const auto c = build_sign2_scale_tile32_value_codec(b);
            plan.value_scale = c.scale;
            plan.sign_masks.assign(c.sign_masks.begin(), c.sign_masks.end());
            r.codebook_size = 1;
            r.payload_bytes = c.sign_masks.size() * 4 + sizeof(T);
            break;
        }
        case Codec::Dict2: { const auto c = build_dict2_tile32_value_codec(b); load_tile(c); r.codebook_size = static_cast<int>(c.codebook.size()); r.payload_bytes = c.payload_bytes(); break; }
        case Codec::Unique4: { const auto c = build_unique4_tile64_value_codec(b); load_tile(c); r.codebook_size = static_cast<int>(c.codebook.size()); r.payload_bytes = c.payload_bytes(); break; }
        case Codec::Unique16: { const auto c = build_unique16_tile128_value_codec(b); load_tile(c); r.codebook_size = static_cast<int>(c.codebook.size()); r.payload_bytes = c.payload_bytes(); break; }
        case Codec::Dict256U8: { const auto c = build_dict256_tile256_value_codec(b); load_tile(c); r.codebook_size = static_cast<int>(c.codebook.size()); r.payload_bytes = c.payload_bytes(); break; }
        case Codec::Dict65536U16: { const auto c = build_dict65536_tile512_value_codec(b); load_tile(c); r.codebook_size = static_cast<int>(c.codebook.size()); r.payload_bytes = c.payload_bytes(); break; }
        case Codec::Fp16:
        case Codec::Bf16: {
            const auto c = codec == Codec::Fp16
                               ? build_round16_nnz_value_codec(b, [](T v) { return float_to_fp16_bits(static_cast<float>(v)); })
                               : build_round16_nnz_value_codec(b, [](T v) { return float_to_bf16_bits(static_cast<float>(v)); });
            plan.values16.assign(c.values16.begin(), c.values16.end());
            r.payload_bytes = c.values16.size() * 2;
            break;
        }
        case Codec::Bfp8: {
            const auto c = build_bfp8_blkscale_value_codec(b);
            plan.int8_values.assign(c.int8_values.begin(), c.int8_values.end());
            plan.block_scale_bf16.assign(c.block_scale_bf16.begin(), c.block_scale_bf16.end());
            r.payload_bytes = c.int8_values.size() + c.block_scale_bf16.size() * 2;
            break;
        }
        case Codec::Bfp8Outlier: {
            const auto c = build_bfp8_outlier_blkscale_value_codec(b);
            plan.int8_values.assign(c.int8_values.begin(), c.int8_values.end());
            plan.block_scale_bf16.assign(c.block_scale_bf16.begin(), c.block_scale_bf16.end());
            plan.outlier_rows.assign(c.outlier_rows.begin(), c.outlier_rows.end());
            plan.outlier_cols.assign(c.outlier_cols.begin(), c.outlier_cols.end());
            plan.outlier_vals.assign(c.outlier_vals.begin(), c.outlier_vals.end());
            r.payload_bytes = c.payload_bytes();
            r.value_only_valid = true;
            r.value_only_bytes = c.value_only_payload_bytes();
            r.num_outliers = c.num_outliers;
            break;
        }
        case Codec::Bfp4: {
            const auto c = build_bfp4_blkscale_value_codec(b);
            plan.packed_int4.assign(c.packed_int4.begin(), c.packed_int4.end());
            plan.block_scale_bf16.assign(c.block_scale_bf16.begin(), c.block_scale_bf16.end());
            r.payload_bytes = c.packed_int4.size() + c.block_scale_bf16.size() * 2;
            break;
        }
        case Codec::K256U8: {
            const auto c = build_k256_tile256_build_result(b);
            load_tile(c.tile);
            r.exact = c.tile.exact;
            r.codebook_size = c.used_codebook_size;
            r.payload_bytes = c.tile.payload_bytes();
            break;
        }
        case Codec::GlobalLogKmeans16:
        case Codec::GlobalLogKmeans32:
        case Codec::GlobalLogKmeans64:
        case Codec::GlobalLogKmeans128: {
            const int k = codec == Codec::GlobalLogKmeans16   ? 16
                          : codec == Codec::GlobalLogKmeans32 ? 32
                          : codec == Codec::GlobalLogKmeans64 ? 64
                                                              : 128;
            const auto c = build_logkmeans_tile256_build_result(b, k);
            load_tile(c.tile);
            r.exact = false;
            r.codebook_size = c.used_codebook_size;
            r.payload_bytes = c.tile.payload_bytes();
            break;
        }
        case Codec::Raw:
            throw std::runtime_error("original value codec must use the original traversal runner");
    }
}

template <typename T>
int run(const Options& o) {
    const Layout layout = structural::spmv_layout_kind_from_name(o.layout);
    const bool auto_lossless = o.value_codec == "auto_lossless";
    if (auto_lossless && layout == Layout::CusparseCsr)
        throw std::runtime_error("auto_lossless value codec is only supported for BitBSR layouts");
    Codec codec = auto_lossless ? Codec::Raw : structural::spmv_value_codec_kind_from_name(o.value_codec);
    // before loading the matrix; auto_lossless re-derives it for the chosen codec
    SpmvOperatorSpec spec = structural::make_spmv_operator_spec(
        layout, codec, auto_lossless ? structural::LoadBalancePolicy::Manual : requested_policy(o), structural::spmv_has_manual_load_balance_override(o));
    if (layout == Layout::CusparseCsr) return run_cusparse<T>(o, spec);

    Timing tm;
    Report r;
    r.auto_selected = auto_lossless;
    const auto m = timed_host([&] { return structural::read_matrix_market_with_info<T>(o.matrix_path); }, tm.load);
    const auto& a = m.matrix;
    timed_host([&] { cuda_ok(cudaFree(nullptr), "CUDA context"); return 0; }, tm.ctx);
    structural::GpuBitBsrWorkspace<T> ws;
    structural::DeviceBitBsrMatrix<T> dev;
    timed_host([&] {
        structural::convert_to_bitbsr_gpu_warp_direct_8x4_device(a, ws, dev, &tm.convert_event);
        return 0;
    }, tm.convert_host);
    if (auto_lossless) {
        const auto h = timed_host([&] { return structural::build_device_exact_value_histogram(dev, &tm.auto_event); },
                                  tm.auto_host);
        codec = structural::cove::select_auto_lossless_value_codec(h);
        spec = structural::make_spmv_operator_spec(layout, codec, requested_policy(o), structural::spmv_has_manual_load_balance_override(o));
        r.auto_unique_count = h.unique_count;
        r.auto_unique_overflow = h.unique_overflow;
        r.auto_raw_bytes = h.raw_payload_bytes;
        r.auto_candidate_bytes = candidate_bytes(h, codec);
    }
    const auto x = canonical_x<T>(a.cols);
    thrust::device_vector<T> d_x(x.begin(), x.end()), d_y;
    // load-balance chunking: the requested policy unless chunk sizes were given
    int chunk = o.lb_chunk_blocks, split = o.lb_split_threshold_blocks;
    const bool binary_lb = structural::effective_requested_load_balance_policy(requested_policy(o), structural::spmv_has_manual_load_balance_override(o)) ==
                           structural::LoadBalancePolicy::BinaryImplicitOne;
    if (binary_lb) {  // the spec above already required flag_lb + all_one
        const auto p = structural::select_binary_implicit_one_load_balance_policy(dev.num_blocks, dev.rows);
        chunk = p.chunk_blocks;
        split = p.split_threshold_blocks;
    }

    structural::BitBsrSpmvPlan8x4<T> plan;
    plan.layout = layout;
    plan.value_codec = codec;
    if (codec == Codec::Raw) {
        r.exact = true;
        r.payload_bytes = static_cast<size_t>(dev.nnz) * sizeof(T);
    } else {
        timed_host([&] {
            build_values(dev.to_host(), codec, plan, r);
            return 0;
        }, tm.codec_host);
    }
    timed_host([&] {
        structural::make_bitbsr_8x4_col_bitmap_packed(dev, plan.packed_col_bitmap_meta, &tm.pack_event);
        return 0;
    }, tm.pack_host);
    r.position_bytes = plan.packed_col_bitmap_meta.size() * sizeof(std::uint64_t);
    if (layout == Layout::ColBitmap64FlagLb) {
        timed_host([&] {
            structural::make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(
                dev, plan.load_balance, chunk, split, plan.packed_col_bitmap_meta, &tm.lb_event);
            return 0;
        }, tm.lb_host);
    }
    const auto [sum_ms, min_ms] =
        time_loop(o, [&](float* ms) { structural::run_bitbsr_spmv_once(dev, plan, d_x, d_y, ms); });
    cuda_ok(cudaDeviceSynchronize(), "SpMV");
    Verify v;
    if (o.verify_cpu) v = verify(a, x, d_y, lossy_gate(spec));

    print_matrix_header(o, m, "8 x 4");
    print_contract(spec);
    const double nnz = static_cast<double>(dev.nnz);
    std::cout << "spmv_layout: " << o.layout << "\n";
    std::cout << "spmv_effective_layout: " << o.layout << "\n";
    std::cout << "position_codec: col_bitmap64\n";
    std::cout << "position_codec_exact: true\n";
    std::cout << "position_codec_payload_bytes: " << r.position_bytes << "\n";
    std::cout << "value_codec: " << o.value_codec << "\n";
    std::cout << "value_codec_effective: " << codec_name(codec) << "\n";
    std::cout << "value_codec_auto_selected: " << (r.auto_selected ? "true" : "false") << "\n";
    std::cout << "value_codec_auto_unique_count: " << r.auto_unique_count << "\n";
    std::cout << "value_codec_auto_unique_overflow: " << (r.auto_unique_overflow ? "true" : "false") << "\n";
    std::cout << "value_codec_auto_raw_payload_bytes: " << r.auto_raw_bytes << "\n";
    std::cout << "value_codec_auto_candidate_payload_bytes: " << r.auto_candidate_bytes << "\n";
    std::cout << "value_codec_exact: " << (r.exact ? "true" : "false") << "\n";
    std::cout << "value_codec_codebook_size: " << r.codebook_size << "\n";
    std::cout << "value_codec_payload_bytes: " << r.payload_bytes << "\n";
    std::cout << "value_codec_bytes_per_nnz: " << (nnz == 0 ? 0.0 : static_cast<double>(r.payload_bytes) / nnz) << "\n";
    const size_t vo = r.value_only_valid ? r.value_only_bytes : r.payload_bytes;
    std::cout << "value_codec_value_only_payload_bytes: " << vo << "\n";
    std::cout << "value_codec_value_only_bytes_per_nnz: " << (nnz == 0 ? 0.0 : static_cast<double>(vo) / nnz) << "\n";
    std::cout << "value_codec_num_outliers: " << r.num_outliers << "\n";
    std::cout << "load_balance_policy: " << (binary_lb ? "binary_implicit_one" : "manual") << "\n";
    std::cout << "load_balance_chunk_blocks: " << plan.load_balance.chunk_blocks << "\n";
    std::cout << "load_balance_split_threshold_blocks: " << plan.load_balance.split_threshold_blocks << "\n";
    std::cout << "gpu_work_items: " << plan.load_balance.work_items.size() << "\n";
    std::cout << "gpu_output_residency: device\n";
    std::cout << "gpu_num_blocks: " << dev.num_blocks << "\n";
    std::cout << "verify_gate: " << structural::spmv_verify_gate_name(spec.verify_gate) << "\n";
    std::cout << "timing_scope: event_excludes_output_init\n";
    std::cout << std::fixed << std::setprecision(4);
    std::cout << "timing_ms: load=" << tm.load << ", cuda_context=" << tm.ctx << ", gpu_convert_host=" << tm.convert_host
              << ", gpu_convert_event=" << tm.convert_event << ", value_codec_auto_select_host=" << tm.auto_host
              << ", value_codec_auto_select_event=" << tm.auto_event << ", col_bitmap_pack_host=" << tm.pack_host
              << ", col_bitmap_pack_event=" << tm.pack_event << ", load_balance_pack_host=" << tm.lb_host
              << ", load_balance_pack_event=" << tm.lb_event << ", value_codec_pack_host=" << tm.codec_host
              << ", gpu_spmv_avg_event=" << (sum_ms / o.iterations) << ", gpu_spmv_min_event=" << min_ms
              << ", cpu_spmv=" << (o.verify_cpu ? v.cpu_ms : 0.0) << "\n";
    print_verify(v);
    return v.pass ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        const Options o = structural::parse_spmv_cli_options(argc, argv);
        return o.precision == "float" ? run<float>(o) : run<double>(o);
    } catch (const std::exception& e) {
        std::cerr << "error: " << e.what() << "\n";
        return 1;
    }
}
