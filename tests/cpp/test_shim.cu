// test_shim.cu -- the structural:: C++ API of the B200 library, exercised the
// way the reference's own tests use it (structural/tests/test_gpu_convert.cu,
// structural/src/main_gpu_csr_bitbsr_spmv.cu): GPU converter vs a host
// conversion, packed words and work-item known answers, BitBSR-only
// operators, the hybrid/joint launchers, and the device pipeline handle.
// Built and run by tests/test_gpu_shim.py (needs a GPU).
#include "structural/convert.hpp"
#include "structural/csr_bitbsr_hybrid.cuh"
#include "structural/csr_bitbsr_split.hpp"
#include "structural/gpu_value_codecs.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <cassert>
#include <cmath>
#include <cstring>
#include <cstdio>
#include <map>
#include <vector>

#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #cond); \
            std::exit(1);                                                        \
        }                                                                        \
    } while (0)

using structural::CsrMatrix;

namespace {

std::vector<double> cpu_spmv(const CsrMatrix<double>& a, const std::vector<double>& x) {
    std::vector<double> y(a.rows, 0.0);
    for (int r = 0; r < a.rows; ++r)
        for (int p = a.row_ptr[r]; p < a.row_ptr[r + 1]; ++p) y[r] += a.values[p] * x[a.col_idx[p]];
    return y;
}

template <typename V>
std::vector<V> host(const thrust::device_vector<V>& d) {
    std::vector<V> h(d.size());
    thrust::copy(d.begin(), d.end(), h.begin());
    return h;
}

void close(const std::vector<double>& a, const std::vector<double>& b, double tol) {
    CHECK(a.size() == b.size());
    for (size_t i = 0; i < a.size(); ++i) CHECK(std::abs(a[i] - b[i]) <= tol);
}

CsrMatrix<double> kat_9x4404() {  // test_gpu_convert.cu:496-563
    CsrMatrix<double> csr;
    csr.rows = 9;
    csr.cols = 4404;
    csr.row_ptr = {0, 3, 5, 6, 7, 8, 8, 9, 9, 12};
    csr.col_idx = {400, 416, 2000, 401, 417, 2001, 418, 402, 2002, 2800, 3600, 4400};
    csr.values = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12};
    return csr;
}

void test_converter_and_work_items() {
    const auto csr = kat_9x4404();
    structural::GpuBitBsrWorkspace<double> ws;
    structural::DeviceBitBsrMatrix<double> dev;
    structural::convert_to_bitbsr_gpu_warp_direct_8x4_device(csr, ws, dev);
    CHECK(dev.num_blocks == 6 && dev.nnz == 12);
    CHECK(host(dev.block_row_ptr) == (std::vector<int>{0, 3, 6}));
    const auto h = dev.to_host();
    CHECK(h.block_val_ptr.back() == 12);

    thrust::device_vector<std::uint64_t> packed;
    structural::make_bitbsr_8x4_col_bitmap_packed(dev, packed);
    structural::BitBsrLoadBalanceLayout8x4 lb;
    structural::make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(dev, lb, 2, packed);
    const auto items = host(lb.work_items);
    const auto words = host(packed);
    CHECK(items.size() == 4);
    const unsigned want[4][4] = {{0, 0, 2, 0}, {0, 2, 1, 6}, {1, 3, 2, 9}, {1, 5, 1, 11}};
    for (int i = 0; i < 4; ++i) {
        CHECK(items[i].br == want[i][0] && items[i].block_begin == want[i][1]);
        CHECK(items[i].block_count == want[i][2] && items[i].value_begin == want[i][3]);
    }
    for (int b : {0, 2, 3, 5}) CHECK(structural::gpu_detail::unpack_col_bitmap_flag(words[b]));

    structural::make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(dev, lb, 2, 4, packed);
    CHECK(lb.work_items.size() == 2);  // :913-970
    for (const auto w : host(packed)) CHECK(!structural::gpu_detail::unpack_col_bitmap_flag(w));
}

void test_bitbsr_only_operators() {
    const auto csr = kat_9x4404();
    std::vector<double> x(csr.cols);
    for (int i = 0; i < csr.cols; ++i) x[i] = ((i % 13) - 6) * 0.25;
    const auto expected = cpu_spmv(csr, x);
    structural::GpuBitBsrWorkspace<double> ws;
    const auto dev = structural::convert_to_bitbsr_gpu_warp_direct_8x4_device(csr, ws);
    thrust::device_vector<double> dx(x.begin(), x.end()), dy;

    structural::BitBsrSpmvPlan8x4<double> plan;
    structural::make_bitbsr_8x4_col_bitmap_packed(dev, plan.packed_col_bitmap_meta);
    structural::make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(
        dev, plan.load_balance, 32, plan.packed_col_bitmap_meta);
    float ms = -1.0f;
    structural::run_bitbsr_spmv_once(dev, plan, dx, dy, &ms);
    CHECK(ms >= 0.0f);
    close(expected, host(dy), 1e-12);

    // exact dictionary with per-cell 8-bit tile codes (codebook = sorted values)
    const auto h = dev.to_host();
    std::map<double, unsigned> id;
    for (double v : h.values) id.emplace(v, 0);
    std::vector<double> codebook;
    for (auto& kv : id) {
        kv.second = static_cast<unsigned>(codebook.size());
        codebook.push_back(kv.first);
    }
    std::vector<std::uint32_t> tile(static_cast<size_t>(h.num_blocks()) * 8, 0);
    for (int b = 0; b < h.num_blocks(); ++b) {
        int k = h.block_val_ptr[b];
        for (int bit = 0; bit < 32; ++bit) {
            if (!(h.bitmap_words[b] & (1u << bit))) continue;
            tile[b * 8 + bit / 4] |= id[h.values[k++]] << ((bit % 4) * 8);
        }
    }
    plan.value_codec = structural::BitBsrValueCodecKind8x4::Dict256U8;
    plan.tile_code_words = tile;
    plan.value_codebook = codebook;
    structural::run_bitbsr_spmv_once(dev, plan, dx, dy);
    close(expected, host(dy), 1e-12);

    // k256 / log-k-means are 8-bit code tiles over a 256-entry codebook
    plan.value_codec = structural::BitBsrValueCodecKind8x4::K256U8;
    std::vector<double> book256(codebook);
    book256.resize(256, 0.0);
    plan.value_codebook = book256;
    structural::run_bitbsr_spmv_once(dev, plan, dx, dy);
    close(expected, host(dy), 1e-12);
    plan.value_codec = structural::BitBsrValueCodecKind8x4::GlobalLogKmeans64;
    structural::run_bitbsr_spmv_once(dev, plan, dx, dy);
    close(expected, host(dy), 1e-12);
}

// A random 8x4-blocked matrix whose values come from `value(k)`.
CsrMatrix<double> random_csr(int rows, int cols, double density, unsigned seed,
                             double (*value)(unsigned)) {
    CsrMatrix<double> a;
    a.rows = rows;
    a.cols = cols;
    a.row_ptr.push_back(0);
    unsigned s = seed;
    auto next = [&]() { s = s * 1664525u + 1013904223u; return s >> 8; };
    for (int r = 0; r < rows; ++r) {
        for (int c = 0; c < cols; ++c) {
            if ((next() % 10000) < density * 10000) {
                a.col_idx.push_back(c);
                a.values.push_back(value(next()));
            }
        }
        a.row_ptr.push_back(static_cast<int>(a.col_idx.size()));
    }
    return a;
}

double val_one(unsigned) { return 1.0; }
double val_const(unsigned) { return 2.5; }
double val_sign(unsigned u) { return (u & 1) ? 1.0 : -1.0; }
double val_sign_scale(unsigned u) { return (u & 1) ? 0.75 : -0.75; }
double val_eighths(unsigned u) { return static_cast<double>(static_cast<int>(u % 64) - 32) / 8.0; }
double val_wide(unsigned u) { return (static_cast<double>(u % 20001) - 10000.0) * 1e-3; }

std::uint16_t half_bits(double v) {  // the values used are exact in fp16
    const __half h = __double2half(v);
    return __half_as_ushort(h);
}

// bf16 bits, round to nearest even (value_compression.hpp:105-109)
std::uint16_t bf16_bits(float f) {
    std::uint32_t u = 0;
    std::memcpy(&u, &f, 4);
    return static_cast<std::uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
float bf16_float(std::uint16_t b) {
    const std::uint32_t u = static_cast<std::uint32_t>(b) << 16;
    float f = 0.0f;
    std::memcpy(&f, &u, 4);
    return f;
}

void test_family_value_codecs() {
    using K = structural::BitBsrValueCodecKind8x4;
    struct Case {
        K codec;
        double (*value)(unsigned);
        double tol;
    };
    const Case cases[] = {{K::ImplicitOne, val_one, 1e-12},   {K::ConstC, val_const, 1e-12},
                          {K::Sign2, val_sign, 1e-12},        {K::Sign2Scale, val_sign_scale, 1e-12},
                          {K::Fp16, val_eighths, 1e-5},       {K::Bfp4, val_wide, 1e-5}};
    for (const Case& cs : cases) {
        const auto csr = random_csr(203, 301, 0.08, 7u + static_cast<unsigned>(cs.codec), cs.value);
        structural::GpuBitBsrWorkspace<double> ws;
        const auto dev = structural::convert_to_bitbsr_gpu_warp_direct_8x4_device(csr, ws);
        const auto h = dev.to_host();
        std::vector<double> x(csr.cols);
        for (int i = 0; i < csr.cols; ++i) x[i] = ((i % 17) - 8) * 0.125;
        // the matrix as the codec decodes it, in CSR order
        std::vector<double> decoded(h.values.begin(), h.values.end());
        structural::BitBsrSpmvPlan8x4<double> plan;
        plan.value_codec = cs.codec;
        const int nb = h.num_blocks();
        if (cs.codec == K::ConstC) plan.value_scale = 2.5;
        if (cs.codec == K::Sign2 || cs.codec == K::Sign2Scale) {  // build_sign2_tile32_masks
            std::vector<std::uint32_t> masks(nb, 0);
            for (int b = 0; b < nb; ++b) {
                int k = h.block_val_ptr[b];
                for (int bit = 0; bit < 32; ++bit)
                    if (h.bitmap_words[b] & (1u << bit)) {
                        if (h.values[k++] > 0) masks[b] |= 1u << bit;
                    }
            }
            plan.sign_masks = masks;
            plan.value_scale = cs.codec == K::Sign2 ? 1.0 : 0.75;
        }
        if (cs.codec == K::Fp16) {
            std::vector<std::uint16_t> v16(h.values.size());
            for (size_t i = 0; i < v16.size(); ++i) v16[i] = half_bits(h.values[i]);
            plan.values16 = v16;
        }
        if (cs.codec == K::Bfp4) {  // build_bfp4_blkscale_value_codec
            std::vector<std::uint8_t> packed((h.values.size() + 1) / 2, 0);
            std::vector<std::uint16_t> scales(nb, 0);
            for (int b = 0; b < nb; ++b) {
                double mx = 0.0;
                for (int k = h.block_val_ptr[b]; k < h.block_val_ptr[b + 1]; ++k)
                    mx = std::max(mx, std::abs(h.values[k]));
                float sc = static_cast<float>(mx / 7.0);
                if (sc == 0.0f) sc = 1.0f;
                scales[b] = bf16_bits(sc);
                const float dsc = bf16_float(scales[b]);
                for (int k = h.block_val_ptr[b]; k < h.block_val_ptr[b + 1]; ++k) {
                    const long q = std::max(-7L, std::min(7L, std::lround(h.values[k] / static_cast<double>(dsc))));
                    const std::uint8_t nib = static_cast<std::uint8_t>(q & 0xF);
                    packed[k >> 1] |= (k & 1) ? static_cast<std::uint8_t>(nib << 4) : nib;
                    decoded[k] = static_cast<double>(q) * dsc;
                }
            }
            plan.packed_int4 = packed;
            plan.block_scale_bf16 = scales;
        }
        // expected y from the decoded values in block/bit order
        std::vector<double> expected(csr.rows, 0.0);
        for (int br = 0; br < h.num_block_rows; ++br)
            for (int b = h.block_row_ptr[br]; b < h.block_row_ptr[br + 1]; ++b) {
                int k = h.block_val_ptr[b];
                for (int bit = 0; bit < 32; ++bit)
                    if (h.bitmap_words[b] & (1u << bit)) {
                        const int row = br * 8 + bit / 4, col = h.block_col_idx[b] * 4 + bit % 4;
                        expected[row] += decoded[k++] * x[col];
                    }
            }
        structural::make_bitbsr_8x4_col_bitmap_packed(dev, plan.packed_col_bitmap_meta);
        structural::make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(
            dev, plan.load_balance, 32, plan.packed_col_bitmap_meta);
        thrust::device_vector<double> dx(x.begin(), x.end()), dy;
        structural::run_bitbsr_spmv_once(dev, plan, dx, dy);
        double mx = 1e-30;
        for (double e : expected) mx = std::max(mx, std::abs(e));
        close(expected, host(dy), cs.tol * mx);
    }
}

void test_hybrid_launchers_and_plan() {
    // 4 x 8 matrix of test_gpu_csr_bitbsr_spmv_cli.sh:11-18, residual threshold 2
    CsrMatrix<double> csr;
    csr.rows = 4;
    csr.cols = 8;
    csr.row_ptr = {0, 2, 3, 4, 5};
    csr.col_idx = {0, 7, 3, 1, 6};
    csr.values = {1, 2, 3, 4, 5};
    std::vector<double> x(8);
    for (int i = 0; i < 8; ++i) x[i] = ((i % 17) - 8) * 0.125;
    const auto expected = cpu_spmv(csr, x);

    // split by hand: block (0, 0) kept (3 nnz), block (0, 1) residual (2 nnz)
    structural::BitBsrMatrix<double> kept;
    kept.rows = 4;
    kept.cols = 8;
    kept.block_rows = 8;
    kept.block_cols = 4;
    kept.num_block_rows = 1;
    kept.num_block_cols = 2;
    kept.words_per_block = 1;
    kept.block_row_ptr = {0, 1};
    kept.block_col_idx = {0};
    kept.bitmap_words = {(1u << 0) | (1u << 7) | (1u << 9)};
    kept.block_val_ptr = {0, 3};
    kept.values = {1, 3, 4};
    const auto dev = structural::copy_bitbsr_to_device(kept);
    thrust::device_vector<std::uint64_t> packed;
    structural::BitBsrLoadBalanceLayout8x4 lb;
    structural::make_fused_8x4_load_balance_layout_host(kept, lb, packed, 32, 32);
    CHECK(lb.work_items.size() == 1);
    thrust::device_vector<int> rrp(std::vector<int>{0, 1, 1, 1, 2});
    thrust::device_vector<int> rci(std::vector<int>{7, 6});
    thrust::device_vector<double> rv(std::vector<double>{2, 5});
    thrust::device_vector<int> cr, cb, cc;
    thrust::device_vector<double> dx(x.begin(), x.end()), dy(4, 0.0);
    structural::run_csr_bitbsr_fused_8x4_lb(dev, packed, lb, rrp, rci, rv, 0, cr, cb, cc, dx, dy);
    close(expected, host(dy), 1e-12);

    thrust::device_vector<std::uint8_t> kidx(std::vector<std::uint8_t>{0, 1, 2});
    thrust::device_vector<std::uint8_t> ridx(std::vector<std::uint8_t>{3, 4});
    thrust::device_vector<double> book(std::vector<double>{1, 3, 4, 2, 5});
    structural::run_csr_bitbsr_fused_8x4_lb_dict<double, std::uint8_t>(dev, packed, lb, rrp, rci, kidx,
                                                                       book, ridx, 0, cr, cb, cc, dx, dy);
    close(expected, host(dy), 1e-12);

    // the full device pipeline on the same CSR
    cove_plan_opts o;
    cove_plan_opts_default(&o);
    o.residual_threshold = 2;
    o.value_codec = COVE_CODEC_AUTO;
    structural::cove::Plan<double> p(csr, &o);
    CHECK(p.info().kept_blocks == 1 && p.info().residual_blocks == 1);
    CHECK(p.info().joint_route == COVE_ROUTE_DICT_U8);
    p.spmv(dx, dy);
    close(expected, host(dy), 1e-12);
}

// ---- family codec builders vs the reference builders' payloads -------------------
#include "codec_golden.inc"

// the matrices of oracle/ref_codec_golden.cu (same formulas)
double golden_value(int kind, int r, int c) {
    const int h = (r * 131 + c * 71) % 97;
    switch (kind) {
        case 0: return (h % 3 == 0) ? -1.5 : (h % 3 == 1 ? 0.5 : 2.0);
        case 1: return (h % 2) ? -1.5 : 2.0;
        case 2: return (h % 2) ? 1.0 : -1.0;
        case 3: return (h % 2) ? 0.75 : -0.75;
        case 4: return 3.25;
        default: {
            const double m = (h - 48) / 7.0;
            return m * std::pow(10.0, (r + c) % 7 - 3);
        }
    }
}

structural::BitBsrMatrix<double> golden_bitbsr(int kind, structural::DeviceBitBsrMatrix<double>* dev_out = nullptr) {
    CsrMatrix<double> a;
    a.rows = 37;
    a.cols = 53;
    a.row_ptr.push_back(0);
    for (int r = 0; r < a.rows; ++r) {
        for (int c = 0; c < a.cols; ++c)
            if ((r * 7 + c * 13 + r * c) % 11 < 4) {
                a.col_idx.push_back(c);
                a.values.push_back(golden_value(kind, r, c));
            }
        a.row_ptr.push_back(static_cast<int>(a.col_idx.size()));
    }
    structural::GpuBitBsrWorkspace<double> ws;
    auto dev = structural::convert_to_bitbsr_gpu_warp_direct_8x4_device(a, ws);
    auto h = dev.to_host();
    if (dev_out) *dev_out = std::move(dev);
    return h;
}

template <typename A, typename B>
void same(const std::vector<A>& got, const B* want, size_t n, const char* what) {
    if (got.size() != n) {
        std::fprintf(stderr, "%s: %zu values, golden %zu\n", what, got.size(), n);
        std::exit(1);
    }
    for (size_t i = 0; i < n; ++i)
        if (!(got[i] == static_cast<A>(want[i]))) {
            std::fprintf(stderr, "%s: value %zu differs from the reference builder\n", what, i);
            std::exit(1);
        }
}

template <typename Codec>
void same_tile(const Codec& c, const double* cb, size_t ncb, const uint32_t* w, size_t nw, const char* what) {
    same(c.codebook, cb, ncb, what);
    same(c.tile_code_words, w, nw, what);
}

void test_family_builders() {
    using namespace structural;
    const auto b0 = golden_bitbsr(0);
    same_tile(build_unique4_tile64_value_codec(b0), g_unique4_codebook, g_unique4_codebook_n, g_unique4_words,
              g_unique4_words_n, "unique4");
    same_tile(build_unique16_tile128_value_codec(b0), g_unique16_codebook, g_unique16_codebook_n, g_unique16_words,
              g_unique16_words_n, "unique16");
    same_tile(build_dict256_tile256_value_codec(b0), g_dict256_codebook, g_dict256_codebook_n, g_dict256_words,
              g_dict256_words_n, "dict256");
    same_tile(build_dict65536_tile512_value_codec(b0), g_dict65536_codebook, g_dict65536_codebook_n,
              g_dict65536_words, g_dict65536_words_n, "dict65536");
    same_tile(build_dict2_tile32_value_codec(golden_bitbsr(1)), g_dict2_codebook, g_dict2_codebook_n, g_dict2_words,
              g_dict2_words_n, "dict2");
    same(build_sign2_tile32_masks(golden_bitbsr(2)), g_sign2_masks, g_sign2_masks_n, "sign2");
    const auto s3 = build_sign2_scale_tile32_value_codec(golden_bitbsr(3));
    CHECK(s3.scale == g_sign2s_scale[0]);
    same(s3.sign_masks, g_sign2s_masks, g_sign2s_masks_n, "sign2_scale");
    CHECK(build_const_c_value(golden_bitbsr(4)) == g_const_c[0]);
    const auto b5 = golden_bitbsr(5);
    const auto q8 = build_bfp8_blkscale_value_codec(b5);
    same(std::vector<int>(q8.int8_values.begin(), q8.int8_values.end()), g_bfp8_q, g_bfp8_q_n, "bfp8 q");
    same(q8.block_scale_bf16, g_bfp8_scale, g_bfp8_scale_n, "bfp8 scale");
    const auto q4 = build_bfp4_blkscale_value_codec(b5);
    same(q4.packed_int4, g_bfp4_packed, g_bfp4_packed_n, "bfp4 packed");
    same(q4.block_scale_bf16, g_bfp4_scale, g_bfp4_scale_n, "bfp4 scale");
    const auto bf = [](double v) { return float_to_bf16_bits(static_cast<float>(v)); };
    const auto hf = [](double v) { return float_to_fp16_bits(static_cast<float>(v)); };
    same(build_round16_nnz_value_codec(b5, bf).values16, g_bf16_nnz, g_bf16_nnz_n, "bf16 nnz");
    same(build_round16_nnz_value_codec(b5, hf).values16, g_fp16_nnz, g_fp16_nnz_n, "fp16 nnz");
    same(build_round16_tile512_value_codec(b5, bf).tile_code_words, g_bf16_tile512, g_bf16_tile512_n, "bf16 tile512");

    // k-means codebooks: k256 exact (3 values) and clustered (646 values into
    // 256), global log-k-means with 16 and 128 centres and with 3 magnitudes
    const auto k0 = build_k256_tile256_build_result(b0);
    same_tile(k0.tile, g_k256_exact_codebook, g_k256_exact_codebook_n, g_k256_exact_words, g_k256_exact_words_n,
              "k256 exact");
    CHECK(k0.tile.exact && k0.used_codebook_size == g_k256_exact_used[0]);
    const auto k5 = build_k256_tile256_build_result(b5);
    same_tile(k5.tile, g_k256_kmeans_codebook, g_k256_kmeans_codebook_n, g_k256_kmeans_words, g_k256_kmeans_words_n,
              "k256 k-means");
    CHECK(!k5.tile.exact && k5.used_codebook_size == g_k256_kmeans_used[0]);
    same_tile(build_logkmeans_tile256_build_result(b5, 16).tile, g_logk16_codebook, g_logk16_codebook_n,
              g_logk16_words, g_logk16_words_n, "log-k-means 16");
    same_tile(build_logkmeans_tile256_build_result(b5, 128).tile, g_logk128_codebook, g_logk128_codebook_n,
              g_logk128_words, g_logk128_words_n, "log-k-means 128");
    same_tile(build_logkmeans_tile256_build_result(b0, 8).tile, g_logk_exact_codebook, g_logk_exact_codebook_n,
              g_logk_exact_words, g_logk_exact_words_n, "log-k-means exact");
    // BFP8 with global outliers: default fraction (2 outliers) and 5 % (31)
    {
        const auto o = build_bfp8_outlier_blkscale_value_codec(b5);
        same(std::vector<int>(o.int8_values.begin(), o.int8_values.end()), g_bfp8o_q, g_bfp8o_q_n, "bfp8o q");
        same(o.block_scale_bf16, g_bfp8o_scale, g_bfp8o_scale_n, "bfp8o scale");
        same(o.outlier_rows, g_bfp8o_rows, g_bfp8o_rows_n, "bfp8o rows");
        same(o.outlier_cols, g_bfp8o_cols, g_bfp8o_cols_n, "bfp8o cols");
        same(o.outlier_vals, g_bfp8o_vals, g_bfp8o_vals_n, "bfp8o vals");
        const auto o5 = build_bfp8_outlier_blkscale_value_codec(b5, 0.05);
        same(std::vector<int>(o5.int8_values.begin(), o5.int8_values.end()), g_bfp8o5_q, g_bfp8o5_q_n, "bfp8o5 q");
        same(o5.block_scale_bf16, g_bfp8o5_scale, g_bfp8o5_scale_n, "bfp8o5 scale");
        same(o5.outlier_rows, g_bfp8o5_rows, g_bfp8o5_rows_n, "bfp8o5 rows");
        same(o5.outlier_cols, g_bfp8o5_cols, g_bfp8o5_cols_n, "bfp8o5 cols");
        same(o5.outlier_vals, g_bfp8o5_vals, g_bfp8o5_vals_n, "bfp8o5 vals");
    }
    {
        // the clustered k256 payload runs as K256U8: y = A' x, A' the decoded values
        DeviceBitBsrMatrix<double> d5;
        golden_bitbsr(5, &d5);
        std::vector<double> x(static_cast<size_t>(b5.cols));
        for (size_t c = 0; c < x.size(); ++c) x[c] = (static_cast<int>(c % 7) - 3) * 0.25;
        std::vector<double> expected(static_cast<size_t>(b5.rows), 0.0);
        for (Index br = 0; br < b5.num_block_rows; ++br)
            for (Offset b = b5.block_row_ptr[br]; b < b5.block_row_ptr[br + 1]; ++b) {
                Offset k = b5.block_val_ptr[b];
                for (int bit = 0; bit < 32; ++bit) {
                    if (!(b5.bitmap_words[b] & (1u << bit))) continue;
                    const double v = k5.tile.codebook[k5.tile.value_ids[static_cast<size_t>(k++)]];
                    expected[static_cast<size_t>(br * 8 + bit / 4)] += v * x[static_cast<size_t>(b5.block_col_idx[b] * 4 + bit % 4)];
                }
            }
        BitBsrSpmvPlan8x4<double> plan;
        make_bitbsr_8x4_col_bitmap_packed(d5, plan.packed_col_bitmap_meta);
        make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(d5, plan.load_balance, 32,
                                                                 plan.packed_col_bitmap_meta);
        plan.value_codec = BitBsrValueCodecKind8x4::K256U8;
        plan.tile_code_words = k5.tile.tile_code_words;
        plan.value_codebook = k5.tile.codebook;
        thrust::device_vector<double> dx(x.begin(), x.end()), dy;
        run_bitbsr_spmv_once(d5, plan, dx, dy);
        close(expected, host(dy), 1e-12);
    }

    // histogram and the auto_lossless choice (main_gpu_spmv.cu:127-174)
    using K = BitBsrValueCodecKind8x4;
    const int kinds[] = {4, 2, 3, 1, 0, 5};
    const K want[] = {K::ConstC, K::Sign2, K::Sign2Scale, K::Dict2, K::Unique4, K::Raw};
    for (int i = 0; i < 6; ++i) {
        DeviceBitBsrMatrix<double> dev;
        golden_bitbsr(kinds[i], &dev);
        const auto h = build_device_exact_value_histogram(dev);
        CHECK(cove::select_auto_lossless_value_codec(h) == want[i]);
    }
    // an all-one matrix
    auto ones = golden_bitbsr(4);
    CsrMatrix<double> one = kat_9x4404();
    for (auto& v : one.values) v = 1.0;
    structural::GpuBitBsrWorkspace<double> ws;
    const auto d1 = convert_to_bitbsr_gpu_warp_direct_8x4_device(one, ws);
    CHECK(cove::select_auto_lossless_value_codec(build_device_exact_value_histogram(d1)) == K::ImplicitOne);
    (void)ones;
}

}  // namespace

// Host convert_to_bitbsr and the split API (csr_bitbsr_split.hpp) over the
// device plan: the parts reproduce A x, the counters partition the blocks,
// and a predicate on block population is applied as given.
void test_host_convert_and_split_api() {
    using namespace structural;
    const auto csr = kat_9x4404();
    const auto full = convert_to_bitbsr(csr, 8, 4);
    GpuBitBsrWorkspace<double> ws;
    DeviceBitBsrMatrix<double> dev;
    convert_to_bitbsr_gpu_warp_direct_8x4_device(csr, ws, dev);
    const auto h = dev.to_host();
    CHECK(full.block_col_idx == h.block_col_idx && full.bitmap_words == h.bitmap_words && full.values == h.values);
    CHECK(full.block_row_ptr == h.block_row_ptr && full.block_val_ptr == h.block_val_ptr);
    bool threw = false;
    try {
        convert_to_bitbsr(csr, 2, 2);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw);

    std::vector<double> x(csr.cols);
    for (int i = 0; i < csr.cols; ++i) x[i] = static_cast<double>(i % 7) - 3.0;
    const auto y0 = cpu_spmv(csr, x);
    auto split_product = [&](const CsrBitBsrSplitMatrix<double>& s) {
        std::vector<double> y = cpu_spmv(s.residual, x);
        const auto& b = s.bitbsr;
        for (int br = 0; br < b.num_block_rows; ++br)
            for (int k = b.block_row_ptr[br]; k < b.block_row_ptr[br + 1]; ++k)
                for (int bit = 0; bit < 32; ++bit)
                    if (b.bitmap_words[k] >> bit & 1u)
                        y[br * 8 + bit / 4] += b.values[b.block_val_ptr[k] + popcount_word(b.bitmap_words[k] &
                                                                                          ((1u << bit) - 1u))] *
                                               x[b.block_col_idx[k] * 4 + bit % 4];
        return y;
    };
    std::vector<int> pop;
    for (int b = 0; b < full.num_blocks(); ++b) pop.push_back(full.block_val_ptr[b + 1] - full.block_val_ptr[b]);

    const CsrBitBsrSplitCostModel model;  // moves populations <= 9
    const auto g = convert_to_csr_bitbsr_split_cost_gated(csr, 8, 4, 32, model);
    CHECK(g.kept_blocks + g.residual_blocks == full.num_blocks() && g.residual_blocks == full.num_blocks());
    CHECK(g.cost_skipped_blocks == 0 && g.kept_nnz + g.residual_nnz == full.nnz());
    close(split_product(g), y0, 0.0);

    const auto t = convert_bitbsr_to_csr_bitbsr_split(full, 1);  // only single-entry blocks move
    int singles = 0;
    for (int p : pop) singles += p <= 1;
    CHECK(t.residual_blocks == singles && t.kept_blocks == full.num_blocks() - singles && t.cost_skipped_blocks == 0);
    close(split_product(t), y0, 0.0);

    const auto e = convert_bitbsr_to_csr_bitbsr_split_if(full, 32, [](Offset p) { return p % 2 == 0; });
    int even = 0, odd_nnz = 0;
    for (int p : pop) {
        even += p % 2 == 0;
        odd_nnz += p % 2 ? p : 0;
    }
    CHECK(e.residual_blocks == even && e.cost_skipped_blocks == full.num_blocks() - even);
    CHECK(e.cost_skipped_nnz == odd_nnz && e.kept_nnz == odd_nnz);
    close(split_product(e), y0, 0.0);

    threw = false;
    try {
        convert_bitbsr_to_csr_bitbsr_split(full, -1);
    } catch (const std::runtime_error& err) {
        threw = std::strcmp(err.what(), "CSR+BitBSR residual threshold must be non-negative") == 0;
    }
    CHECK(threw);
}

int main() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        std::fprintf(stderr, "SKIP: no CUDA device\n");
        return 0;
    }
    test_converter_and_work_items();
    test_bitbsr_only_operators();
    test_family_value_codecs();
    test_family_builders();
    test_hybrid_launchers_and_plan();
    test_host_convert_and_split_api();
    std::printf("shim tests passed\n");
    return 0;
}
