// spmv_operator_plan.hpp -- the SpMV operator contract of the structural::
// API (structural/include/structural/spmv_operator_plan.hpp): operator
// names, families, verify gates, promotion status and runner for every
// layout x value codec x load-balance policy, with the same names, checks
// and messages.  The family CLI prints these as its operator_* keys.
#pragma once

#include "structural/load_balance_policy.hpp"
#include "structural/operators/bitbsr_spmv_8x4_dispatch.cuh"

#include <map>
#include <stdexcept>
#include <string>
#include <utility>

namespace structural {

enum class SpmvOperatorFamily {
    LoadBalancedTraversal,
    NonLoadBalancedTraversal,
    LosslessValueSpecialized,
    ControlledLossyValueSpecialized,
    ExternalBaseline,
};

enum class SpmvVerifyGate {
    ExactAbsOrRel,
    SpmvMaxRel,
};

enum class SpmvPromotionStatus {
    Promoted,
    BuildableNeedsReport,
    ExternalBaseline,
};

enum class SpmvOperatorRunner {
    BitBsrRawTraversal,
    BitBsrValueSpecialized,
    CusparseCsr,
};

struct SpmvOperatorSpec {
    BitBsrSpmvLayoutKind8x4 layout = BitBsrSpmvLayoutKind8x4::ColBitmap64FlagLb;
    BitBsrValueCodecKind8x4 value_codec = BitBsrValueCodecKind8x4::Raw;
    LoadBalancePolicy requested_load_balance_policy = LoadBalancePolicy::Manual;
    bool load_balance_policy_manual_override = false;
    const char* operator_name = "original_lb";
    SpmvOperatorFamily family = SpmvOperatorFamily::LoadBalancedTraversal;
    SpmvVerifyGate verify_gate = SpmvVerifyGate::ExactAbsOrRel;
    SpmvPromotionStatus promotion_status = SpmvPromotionStatus::Promoted;
    SpmvOperatorRunner runner = SpmvOperatorRunner::BitBsrRawTraversal;
};

namespace op_detail {

template <typename E, std::size_t N>
const char* name_of(E e, const char* const (&names)[N]) {
    const auto i = static_cast<std::size_t>(e);
    return i < N ? names[i] : "unknown";
}

// The report name of each value codec, in the enum's order.
constexpr const char* kCodecNames[] = {
    "original",           "all_one",            "const_c",           "sign2",
    "sign2_scale",        "dict2",              "dict4",             "dict16",
    "dict256_u8",         "dict65536_u16",      "fp16",              "bf16",
    "bfp8",               "bfp8_outlier",       "bfp4",              "codebook256_u8",
    "global_logkmeans16", "global_logkmeans32", "global_logkmeans64", "global_logkmeans128"};

}  // namespace op_detail

inline const char* spmv_operator_family_name(SpmvOperatorFamily f) {
    static const char* const names[] = {"load_balanced_traversal", "non_load_balanced_traversal",
                                        "lossless_value_specialized", "controlled_lossy_value_specialized",
                                        "external_baseline"};
    return op_detail::name_of(f, names);
}

inline const char* spmv_verify_gate_name(SpmvVerifyGate g) {
    static const char* const names[] = {"exact_abs_or_rel", "spmv_max_rel"};
    return op_detail::name_of(g, names);
}

inline const char* spmv_promotion_status_name(SpmvPromotionStatus s) {
    static const char* const names[] = {"promoted", "buildable_needs_report", "external_baseline"};
    return op_detail::name_of(s, names);
}

inline const char* spmv_operator_runner_name(SpmvOperatorRunner r) {
    static const char* const names[] = {"bitbsr_original_traversal", "bitbsr_value_specialized", "cusparse_csr"};
    return op_detail::name_of(r, names);
}

inline LoadBalancePolicy effective_requested_load_balance_policy(LoadBalancePolicy requested, bool manual_override) {
    return manual_override ? LoadBalancePolicy::Manual : requested;
}

inline bool spmv_operator_uses_col_bitmap64_layout(BitBsrSpmvLayoutKind8x4 layout) {
    return layout == BitBsrSpmvLayoutKind8x4::ColBitmap64 || layout == BitBsrSpmvLayoutKind8x4::ColBitmap64FlagLb;
}

// "<codec>_lb" / "<codec>_nolb" ("original_*" for raw values), or
// "cusparse_csr" for raw values on the cuSPARSE layout.
inline const char* spmv_operator_name(BitBsrSpmvLayoutKind8x4 layout, BitBsrValueCodecKind8x4 value_codec) {
    const auto c = static_cast<std::size_t>(value_codec);
    if (c >= sizeof(op_detail::kCodecNames) / sizeof(op_detail::kCodecNames[0])) return "unknown";
    if (layout == BitBsrSpmvLayoutKind8x4::CusparseCsr && value_codec == BitBsrValueCodecKind8x4::Raw)
        return "cusparse_csr";
    const bool lb = layout == BitBsrSpmvLayoutKind8x4::ColBitmap64FlagLb;
    static const std::map<std::pair<std::size_t, bool>, std::string> names = [] {
        std::map<std::pair<std::size_t, bool>, std::string> m;
        for (std::size_t i = 0; i < sizeof(op_detail::kCodecNames) / sizeof(op_detail::kCodecNames[0]); ++i)
            for (const bool with_lb : {false, true})
                m[{i, with_lb}] = std::string(op_detail::kCodecNames[i]) + (with_lb ? "_lb" : "_nolb");
        return m;
    }();
    return names.at({c, lb}).c_str();
}

inline SpmvOperatorSpec make_spmv_operator_spec(BitBsrSpmvLayoutKind8x4 layout, BitBsrValueCodecKind8x4 value_codec,
                                                LoadBalancePolicy requested_load_balance_policy,
                                                bool load_balance_policy_manual_override) {
    using L = BitBsrSpmvLayoutKind8x4;
    const LoadBalancePolicy policy =
        effective_requested_load_balance_policy(requested_load_balance_policy, load_balance_policy_manual_override);
    const bool binary = policy == LoadBalancePolicy::BinaryImplicitOne;
    if (binary && (layout != L::ColBitmap64FlagLb || value_codec != BitBsrValueCodecKind8x4::ImplicitOne))
        throw std::runtime_error(
            "lb-policy binary_implicit_one requires col_bitmap64_flag_lb layout and all_one value codec");
    const bool non_raw = bitbsr_spmv_8x4_is_non_raw_value_codec(value_codec);
    if (non_raw && layout == L::CusparseCsr)
        throw std::runtime_error("compressed value codecs are only supported for BitBSR layouts");
    if (non_raw && !spmv_operator_uses_col_bitmap64_layout(layout))
        throw std::runtime_error("compressed value codecs currently require col_bitmap64 layout");

    SpmvOperatorSpec s;
    s.layout = layout;
    s.value_codec = value_codec;
    s.requested_load_balance_policy = requested_load_balance_policy;
    s.load_balance_policy_manual_override = load_balance_policy_manual_override;
    s.operator_name = spmv_operator_name(layout, value_codec);
    const bool lossy = bitbsr_spmv_8x4_is_controlled_lossy_value_codec(value_codec);
    s.verify_gate = lossy ? SpmvVerifyGate::SpmvMaxRel : SpmvVerifyGate::ExactAbsOrRel;
    using F = SpmvOperatorFamily;
    using P = SpmvPromotionStatus;
    using R = SpmvOperatorRunner;
    if (layout == L::CusparseCsr) {
        s.family = F::ExternalBaseline;
        s.promotion_status = P::ExternalBaseline;
        s.runner = R::CusparseCsr;
    } else if (lossy) {
        s.family = F::ControlledLossyValueSpecialized;
        s.promotion_status = P::BuildableNeedsReport;
        s.runner = R::BitBsrValueSpecialized;
    } else if (non_raw) {
        s.family = F::LosslessValueSpecialized;
        s.promotion_status = binary ? P::Promoted : P::BuildableNeedsReport;
        s.runner = R::BitBsrValueSpecialized;
    } else if (layout == L::ColBitmap64FlagLb) {
        s.family = F::LoadBalancedTraversal;
        s.promotion_status = P::Promoted;
        s.runner = R::BitBsrRawTraversal;
    } else {
        s.family = F::NonLoadBalancedTraversal;
        s.promotion_status = P::BuildableNeedsReport;
        s.runner = R::BitBsrRawTraversal;
    }
    return s;
}

}  // namespace structural
