// Prints the SpMV operator contract and the load-balance policy decisions
// through the public structural:: API only (spmv_operator_plan.hpp,
// load_balance_policy.hpp), so the same source builds against the
// reference's headers (oracle/Makefile -> oracle/_ref/ref_operator_plan,
// whose output tests/golden/make_operator_plan_golden.py stores in
// tests/golden/operator_plan.txt) and against this library's shim
// (tests/test_operator_plan.py), and the two outputs must be equal.
#include "structural/spmv_operator_plan.hpp"

#include <cstdio>
#include <exception>

using namespace structural;

int main() {
    const BitBsrSpmvLayoutKind8x4 layouts[] = {BitBsrSpmvLayoutKind8x4::ColBitmap64,
                                               BitBsrSpmvLayoutKind8x4::ColBitmap64FlagLb,
                                               BitBsrSpmvLayoutKind8x4::CusparseCsr};
    for (int l = 0; l < 3; ++l)
        for (int c = 0; c < 20; ++c)
            for (int p = 0; p < 2; ++p)
                for (int o = 0; o < 2; ++o) {
                    std::printf("spec %d %d %d %d ", l, c, p, o);
                    try {
                        const auto s = make_spmv_operator_spec(layouts[l], static_cast<BitBsrValueCodecKind8x4>(c),
                                                               static_cast<LoadBalancePolicy>(p), o != 0);
                        std::printf("%s %s %s %s %s %s\n", s.operator_name, spmv_operator_family_name(s.family),
                                    spmv_verify_gate_name(s.verify_gate),
                                    spmv_promotion_status_name(s.promotion_status),
                                    spmv_operator_runner_name(s.runner),
                                    load_balance_policy_name(effective_requested_load_balance_policy(
                                        s.requested_load_balance_policy, s.load_balance_policy_manual_override)));
                    } catch (const std::exception& e) {
                        std::printf("ERR %s\n", e.what());
                    }
                }
    const long long blocks[] = {-1, 0, 1, 29999, 30000, 100000, 119999, 120000, 249999, 250000, 399999, 400000,
                                699999, 700000, 2999999, 3000000, 7999999, 8000000, 20000000, 2000000000};
    const int rows[] = {-8, 0, 1, 8, 9, 64, 800, 8000, 80000, 1000000, 10000000, 2000000000};
    for (const long long b : blocks)
        for (const int r : rows) {
            const auto p = select_binary_implicit_one_load_balance_policy(static_cast<Offset>(b), r);
            std::printf("lb %lld %d %d %d %s\n", b, r, p.chunk_blocks, p.split_threshold_blocks,
                        load_balance_policy_name(p.policy));
        }
    const auto m = manual_load_balance_params(48, 96);
    std::printf("manual %d %d %s\n", m.chunk_blocks, m.split_threshold_blocks, load_balance_policy_name(m.policy));
    return 0;
}
