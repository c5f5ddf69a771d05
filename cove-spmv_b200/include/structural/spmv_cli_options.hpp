// spmv_cli_options.hpp -- command-line options of the family SpMV runner
// (structural/include/structural/spmv_cli_options.hpp): the same options,
// defaults, accepted spellings, normalised names, checks and messages, so
// that scripts written for the reference's struct_gpu_spmv drive this
// build's binary unchanged.  The spellings live in alias tables here.
#pragma once

#include "structural/load_balance_policy.hpp"
#include "structural/operators/bitbsr_spmv_8x4_dispatch.cuh"

#include <cstdlib>
#include <iostream>
#include <stdexcept>
#include <string>

namespace structural {

struct SpmvCliOptions {
    std::string matrix_path;
    std::string precision = "double";
    std::string layout = "col_bitmap64_flag_lb";
    std::string value_codec = "original";
    int lb_chunk_blocks = 32;
    int lb_split_threshold_blocks = -1;
    std::string lb_policy = "manual";
    bool lb_chunk_blocks_explicit = false;
    bool lb_split_threshold_blocks_explicit = false;
    std::string cusparse_alg = "default";
    int warmup = 5;
    int iterations = 20;
    bool verify_cpu = false;
};

inline void print_spmv_cli_usage(const char* argv0, std::ostream& os = std::cerr) {
    os << "usage: " << argv0 << " MATRIX.mtx [--precision float|double]"
       << " [--layout col_bitmap64|col_bitmap64_flag_lb|cusparse_csr]"
       << " [--value-codec original|all_one|const_c|sign2|sign2_scale|dict2|dict4|dict16|"
          "dict256_u8|dict65536_u16|auto_lossless|fp16|bf16|codebook256_u8|"
          "global_logkmeans16|global_logkmeans32|global_logkmeans64|global_logkmeans128]"
       << " [--lb-policy manual|binary_implicit_one] [--lb-chunk-blocks N]"
       << " [--lb-split-threshold-blocks N] [--cusparse-alg default|csr_alg1|csr_alg2]"
       << " [--warmup N] [--iters N] [--verify-cpu]\n";
}

namespace cli_detail {

struct Alias {
    const char* spelling;
    const char* name;
};

template <std::size_t N>
const char* lookup(const Alias (&table)[N], const std::string& s) {
    for (const auto& a : table)
        if (s == a.spelling) return a.name;
    return nullptr;
}

// layout spellings -> (layout, cuSPARSE algorithm or nullptr to keep it)
struct LayoutAlias {
    const char* spelling;
    const char* layout;
    const char* alg;
};
constexpr LayoutAlias kLayouts[] = {
    {"col_bitmap", "col_bitmap64", nullptr},
    {"packed_abs", "col_bitmap64", nullptr},
    {"abs_packed", "col_bitmap64", nullptr},
    {"col_bitmap64", "col_bitmap64", nullptr},
    {"col_bitmap64_packed", "col_bitmap64", nullptr},
    {"col_bitmap_flag_lb", "col_bitmap64_flag_lb", nullptr},
    {"packed_abs_flag_lb", "col_bitmap64_flag_lb", nullptr},
    {"abs_packed_flag_lb", "col_bitmap64_flag_lb", nullptr},
    {"col_bitmap64_flag_lb", "col_bitmap64_flag_lb", nullptr},
    {"col_bitmap64_packed_flag_lb", "col_bitmap64_flag_lb", nullptr},
    {"cusparse", "cusparse_csr", nullptr},
    {"cusparse_spmv", "cusparse_csr", nullptr},
    {"cusparse_csr", "cusparse_csr", nullptr},
    {"cusparse_csr_alg1", "cusparse_csr", "csr_alg1"},
    {"cusparse_alg1", "cusparse_csr", "csr_alg1"},
    {"cusparse_csr_alg2", "cusparse_csr", "csr_alg2"},
    {"cusparse_alg2", "cusparse_csr", "csr_alg2"},
};

constexpr Alias kCodecs[] = {
    // canonical names
    {"original", "original"}, {"all_one", "all_one"}, {"const_c", "const_c"}, {"sign2", "sign2"},
    {"sign2_scale", "sign2_scale"}, {"dict4", "dict4"}, {"dict2", "dict2"}, {"dict16", "dict16"},
    {"dict256_u8", "dict256_u8"}, {"dict65536_u16", "dict65536_u16"}, {"auto_lossless", "auto_lossless"},
    {"fp16", "fp16"}, {"bf16", "bf16"}, {"bfp8", "bfp8"}, {"bfp8_outlier", "bfp8_outlier"}, {"bfp4", "bfp4"},
    {"codebook256_u8", "codebook256_u8"}, {"global_logkmeans16", "global_logkmeans16"},
    {"global_logkmeans32", "global_logkmeans32"}, {"global_logkmeans64", "global_logkmeans64"},
    {"global_logkmeans128", "global_logkmeans128"},
    // other spellings
    {"raw", "original"}, {"orig", "original"}, {"origin", "original"},
    {"one", "all_one"}, {"pattern", "all_one"}, {"implicit1", "all_one"}, {"implicit_one", "all_one"},
    {"dict1", "const_c"}, {"const", "const_c"}, {"constant", "const_c"}, {"constant_c", "const_c"},
    {"sign", "sign2"}, {"sign_i8", "sign2"}, {"sign_tile32", "sign2"}, {"tile_sign", "sign2"},
    {"scaled_sign", "sign2_scale"}, {"scaled_sign2", "sign2_scale"}, {"sign_scale", "sign2_scale"},
    {"sign2_c", "sign2_scale"},
    {"code1", "dict2"}, {"u1", "dict2"}, {"unique2_tile32", "dict2"}, {"tile1", "dict2"}, {"unique2", "dict2"},
    {"code2", "dict4"}, {"u2", "dict4"}, {"unique4_tile64", "dict4"}, {"ternary", "dict4"}, {"ternary3", "dict4"},
    {"tile2", "dict4"}, {"unique4", "dict4"},
    {"u4", "dict16"}, {"unique_u8", "dict16"}, {"unique16_tile128", "dict16"}, {"tile4", "dict16"},
    {"unique16", "dict16"},
    {"dict256", "dict256_u8"}, {"unique256", "dict256_u8"}, {"unique256_tile256", "dict256_u8"},
    {"dict256_tile256", "dict256_u8"}, {"exact_u8", "dict256_u8"},
    {"dict65536", "dict65536_u16"}, {"dict_u16", "dict65536_u16"}, {"unique65536", "dict65536_u16"},
    {"unique65536_tile512", "dict65536_u16"}, {"dict65536_tile512", "dict65536_u16"}, {"tile16", "dict65536_u16"},
    {"exact_u16", "dict65536_u16"},
    {"k256", "codebook256_u8"}, {"k256_uint8", "codebook256_u8"}, {"uint8", "codebook256_u8"},
    {"u8", "codebook256_u8"}, {"k256_tile256", "codebook256_u8"}, {"tile8", "codebook256_u8"},
    {"k256_u8", "codebook256_u8"},
    {"half", "fp16"}, {"fp16_tile512", "fp16"}, {"bfloat16", "bf16"}, {"bf16_tile512", "bf16"},
    {"bfp8_blkscale", "bfp8"}, {"int8_blkscale", "bfp8"}, {"int8_8x4", "bfp8"},
    {"bfp8_outlier_blkscale", "bfp8_outlier"}, {"bfp8_outlier_lb", "bfp8_outlier"}, {"int8_outlier", "bfp8_outlier"},
    {"bfp8_2pass", "bfp8_outlier"},
    {"bfp4_blkscale", "bfp4"}, {"int4_blkscale", "bfp4"}, {"int4_8x4", "bfp4"},
    {"logkmeans16", "global_logkmeans16"}, {"log_kmeans16", "global_logkmeans16"},
    {"logkmeans32", "global_logkmeans32"}, {"log_kmeans32", "global_logkmeans32"},
    {"logkmeans64", "global_logkmeans64"}, {"log_kmeans64", "global_logkmeans64"},
    {"logkmeans128", "global_logkmeans128"}, {"log_kmeans128", "global_logkmeans128"},
};

constexpr Alias kPolicies[] = {{"manual", "manual"},           {"binary_implicit_one", "binary_implicit_one"},
                               {"binary", "binary_implicit_one"}, {"implicit_one", "binary_implicit_one"},
                               {"all_one", "binary_implicit_one"}, {"binary_one", "binary_implicit_one"}};

constexpr Alias kAlgs[] = {
    {"default", "default"}, {"csr_alg1", "csr_alg1"}, {"csr_alg2", "csr_alg2"}, {"alg1", "csr_alg1"}, {"alg2", "csr_alg2"}};

// Normalised value codec name -> enum, in the enum's order ("original" is Raw).
constexpr const char* kCodecKinds[] = {
    "original",           "all_one",            "const_c",            "sign2",
    "sign2_scale",        "dict2",              "dict4",              "dict16",
    "dict256_u8",         "dict65536_u16",      "fp16",               "bf16",
    "bfp8",               "bfp8_outlier",       "bfp4",               "codebook256_u8",
    "global_logkmeans16", "global_logkmeans32", "global_logkmeans64", "global_logkmeans128"};

}  // namespace cli_detail

inline std::string normalize_spmv_layout_name(const std::string& layout, std::string& cusparse_alg) {
    for (const auto& a : cli_detail::kLayouts)
        if (layout == a.spelling) {
            if (a.alg) cusparse_alg = a.alg;
            return a.layout;
        }
    throw std::runtime_error("layout must be col_bitmap64, col_bitmap64_flag_lb, or cusparse_csr");
}

inline std::string normalize_spmv_value_codec_name(const std::string& value_codec) {
    if (const char* n = cli_detail::lookup(cli_detail::kCodecs, value_codec)) return n;
    throw std::runtime_error(
        "value-codec must be original, all_one, const_c, sign2, sign2_scale, dict2, dict4, dict16, dict256_u8, "
        "dict65536_u16, auto_lossless, fp16, bf16, codebook256_u8, or global_logkmeans{16,32,64,128}");
}

inline std::string normalize_spmv_load_balance_policy_name(const std::string& policy) {
    if (const char* n = cli_detail::lookup(cli_detail::kPolicies, policy)) return n;
    throw std::runtime_error("lb-policy must be manual or binary_implicit_one");
}

inline std::string normalize_cusparse_spmv_alg_name(const std::string& alg) {
    if (const char* n = cli_detail::lookup(cli_detail::kAlgs, alg)) return n;
    throw std::runtime_error("cusparse-alg must be default, csr_alg1, or csr_alg2");
}

inline bool spmv_has_manual_load_balance_override(const SpmvCliOptions& opts) {
    return opts.lb_chunk_blocks_explicit || opts.lb_split_threshold_blocks_explicit;
}

inline BitBsrSpmvLayoutKind8x4 spmv_layout_kind_from_name(const std::string& layout) {
    if (layout == "col_bitmap64") return BitBsrSpmvLayoutKind8x4::ColBitmap64;
    if (layout == "col_bitmap64_flag_lb") return BitBsrSpmvLayoutKind8x4::ColBitmap64FlagLb;
    if (layout == "cusparse_csr") return BitBsrSpmvLayoutKind8x4::CusparseCsr;
    throw std::runtime_error("internal error: unknown normalized layout");
}

inline BitBsrValueCodecKind8x4 spmv_value_codec_kind_from_name(const std::string& value_codec) {
    int i = 0;
    for (const char* n : cli_detail::kCodecKinds) {
        if (value_codec == n) return static_cast<BitBsrValueCodecKind8x4>(i);
        ++i;
    }
    throw std::runtime_error("internal error: unknown normalized value codec");
}

inline LoadBalancePolicy spmv_load_balance_policy_from_name(const std::string& policy) {
    if (policy == "manual") return LoadBalancePolicy::Manual;
    if (policy == "binary_implicit_one") return LoadBalancePolicy::BinaryImplicitOne;
    throw std::runtime_error("internal error: unknown normalized lb policy");
}

// argv[1] is the matrix; options follow.  No arguments or --help print the
// usage and exit (2 / 0); anything else that fails throws.
inline SpmvCliOptions parse_spmv_cli_options(int argc, char** argv) {
    SpmvCliOptions o;
    if (argc < 2) {
        print_spmv_cli_usage(argv[0]);
        std::exit(2);
    }
    o.matrix_path = argv[1];
    for (int i = 2; i < argc; ++i) {
        const std::string a = argv[i];
        const bool has_value = i + 1 < argc;
        if (a == "--precision" && has_value) {
            o.precision = argv[++i];
            if (o.precision != "float" && o.precision != "double")
                throw std::runtime_error("precision must be float or double");
        } else if (a == "--layout" && has_value) {
            o.layout = normalize_spmv_layout_name(argv[++i], o.cusparse_alg);
        } else if (a == "--value-codec" && has_value) {
            o.value_codec = normalize_spmv_value_codec_name(argv[++i]);
        } else if ((a == "--lb-chunk-blocks" || a == "--chunk-blocks") && has_value) {
            o.lb_chunk_blocks = std::stoi(argv[++i]);
            o.lb_chunk_blocks_explicit = true;
        } else if ((a == "--lb-split-threshold-blocks" || a == "--split-threshold-blocks" ||
                    a == "--lb-split-threshold") &&
                   has_value) {
            o.lb_split_threshold_blocks = std::stoi(argv[++i]);
            o.lb_split_threshold_blocks_explicit = true;
        } else if (a == "--lb-policy" && has_value) {
            o.lb_policy = normalize_spmv_load_balance_policy_name(argv[++i]);
        } else if (a == "--cusparse-alg" && has_value) {
            o.cusparse_alg = normalize_cusparse_spmv_alg_name(argv[++i]);
        } else if (a == "--warmup" && has_value) {
            o.warmup = std::stoi(argv[++i]);
        } else if ((a == "--iters" || a == "--iterations") && has_value) {
            o.iterations = std::stoi(argv[++i]);
        } else if (a == "--verify-cpu") {
            o.verify_cpu = true;
        } else if (a == "--help" || a == "-h") {
            print_spmv_cli_usage(argv[0]);
            std::exit(0);
        } else {
            throw std::runtime_error("unknown or incomplete argument: " + a);
        }
    }
    if (o.warmup < 0 || o.iterations <= 0)
        throw std::runtime_error("warmup must be non-negative and iterations must be positive");
    if (o.lb_chunk_blocks <= 0) throw std::runtime_error("lb-chunk-blocks must be positive");
    if (o.lb_split_threshold_blocks < 0) o.lb_split_threshold_blocks = o.lb_chunk_blocks;
    if (o.lb_split_threshold_blocks <= 0) throw std::runtime_error("lb-split-threshold-blocks must be positive");
    return o;
}

}  // namespace structural
