// load_balance_policy.hpp -- load-balance chunking policies of the
// structural:: API (structural/include/structural/load_balance_policy.hpp):
// same names and results.
//
// select_binary_implicit_one_load_balance_policy picks the chunk size (and
// equal split threshold) of the flag work items for binary all-one matrices
// from the block count and the mean blocks per 8-row block row: the
// reference's calibrated decisions, kept here as a first-match rule table.
#pragma once

#include "structural/types.hpp"

#include <algorithm>
#include <cstdint>

namespace structural {

enum class LoadBalancePolicy {
    Manual,
    BinaryImplicitOne,
};

struct LoadBalanceParams {
    int chunk_blocks = 32;
    int split_threshold_blocks = 32;
    LoadBalancePolicy policy = LoadBalancePolicy::Manual;
};

inline const char* load_balance_policy_name(LoadBalancePolicy policy) {
    return policy == LoadBalancePolicy::Manual              ? "manual"
           : policy == LoadBalancePolicy::BinaryImplicitOne ? "binary_implicit_one"
                                                            : "unknown";
}

inline LoadBalanceParams manual_load_balance_params(int chunk_blocks, int split_threshold_blocks) {
    LoadBalanceParams p;
    p.chunk_blocks = chunk_blocks;
    p.split_threshold_blocks = split_threshold_blocks;
    p.policy = LoadBalancePolicy::Manual;
    return p;
}

namespace lb_detail {

// A rule applies when blocks in [min_blocks, max_blocks) and the mean
// blocks per block row >= min_per_row; chunk 0 keeps the default 32.
struct ChunkRule {
    double min_per_row;
    std::int64_t min_blocks, max_blocks;
    int chunk;
};
constexpr std::int64_t kAny = INT64_MAX;
constexpr ChunkRule kBinaryImplicitOneRules[] = {
    {0.0, 0, 30000, 8},
    {20000.0, 700000, kAny, 128},
    {6000.0, 400000, kAny, 128},
    {6000.0, 250000, kAny, 64},
    {500.0, 0, 120000, 16},
    {500.0, 3000000, kAny, 64},
    {500.0, 0, kAny, 0},
    {128.0, 8000000, kAny, 128},
    {0.0, 3000000, kAny, 64},
};

}  // namespace lb_detail

inline LoadBalanceParams select_binary_implicit_one_load_balance_policy(Offset num_blocks, Index rows) {
    LoadBalanceParams p;
    p.policy = LoadBalancePolicy::BinaryImplicitOne;
    if (num_blocks <= 0 || rows <= 0) return p;
    const Index block_rows = (rows + 7) / 8;
    const double per_row = static_cast<double>(num_blocks) / static_cast<double>(std::max<Index>(block_rows, 1));
    for (const auto& r : lb_detail::kBinaryImplicitOneRules) {
        if (num_blocks < r.min_blocks || num_blocks >= r.max_blocks || per_row < r.min_per_row) continue;
        if (r.chunk > 0) p.chunk_blocks = p.split_threshold_blocks = r.chunk;
        break;
    }
    return p;
}

}  // namespace structural
