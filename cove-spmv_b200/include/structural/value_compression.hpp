// value_compression.hpp -- value-encoding primitives of the structural::
// API (structural/include/structural/value_compression.hpp): the bf16 /
// fp16 bit encodings, the ascending distinct-value set, the 1-D k-means
// used by the k256 and log-k-means codebooks, and the k256 uint8 value
// codebook with exact ids (:20-100, 265-497).  Same names and results;
// gpu_value_codecs.cuh builds the tile payloads on these.
#pragma once

#include "structural/types.hpp"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <vector>

namespace structural {

// ---- 16-bit encodings (value_compression.hpp:105-198) -------------------------

inline std::uint32_t float_bits(float f) {
    std::uint32_t u = 0;
    std::memcpy(&u, &f, 4);
    return u;
}

inline float bits_float(std::uint32_t u) {
    float f = 0.0f;
    std::memcpy(&f, &u, 4);
    return f;
}

// bf16: round to nearest, ties to even, on the upper half of the fp32 bits.
inline std::uint16_t float_to_bf16_bits(float value) {
    const std::uint32_t u = float_bits(value);
    return static_cast<std::uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

inline float bf16_bits_to_float(std::uint16_t bits) { return bits_float(static_cast<std::uint32_t>(bits) << 16); }

// fp16 (IEEE binary16), round to nearest, ties to even; overflow -> inf,
// NaN -> quiet NaN with the sign kept, values below half the smallest
// subnormal -> signed zero.
inline std::uint16_t float_to_fp16_bits(float value) {
    const std::uint32_t u = float_bits(value);
    const std::uint16_t sign = static_cast<std::uint16_t>((u >> 16) & 0x8000u);
    const int e8 = static_cast<int>((u >> 23) & 0xFFu);
    const std::uint32_t m23 = u & 0x7FFFFFu;
    if (e8 == 0xFF) return static_cast<std::uint16_t>(sign | (m23 ? 0x7E00u : 0x7C00u));
    int e5 = e8 - 112;  // rebias 127 -> 15
    if (e5 >= 31) return static_cast<std::uint16_t>(sign | 0x7C00u);
    // round the significand (with its hidden bit) right by `drop` bits
    auto round_shift = [](std::uint32_t v, int drop) {
        const std::uint32_t keep = v >> drop;
        const std::uint32_t rest = v & ((1u << drop) - 1u);
        const std::uint32_t half = 1u << (drop - 1);
        return keep + ((rest > half || (rest == half && (keep & 1u))) ? 1u : 0u);
    };
    if (e5 <= 0) {  // subnormal result (or zero)
        if (e5 < -10) return sign;
        return static_cast<std::uint16_t>(sign | round_shift(m23 | 0x800000u, 14 - e5));
    }
    std::uint32_t m10 = round_shift(m23, 13);
    if (m10 == 0x400u) {  // the rounding carried into the exponent
        m10 = 0;
        if (++e5 >= 31) return static_cast<std::uint16_t>(sign | 0x7C00u);
    }
    return static_cast<std::uint16_t>(sign | (static_cast<std::uint32_t>(e5) << 10) | m10);
}

// ---- value sets --------------------------------------------------------------

// Ascending distinct values, stopping once unique_cap + 1 are found.
template <typename T>
std::vector<T> sorted_unique_values(const std::vector<T>& values, int unique_cap) {
    std::vector<T> s(values);
    std::sort(s.begin(), s.end());
    std::vector<T> out;
    for (const T v : s) {
        if (!out.empty() && out.back() == v) continue;
        out.push_back(v);
        if (static_cast<int>(out.size()) > unique_cap) break;
    }
    return out;
}

// ---- k-means codebooks ---------------------------------------------------------

namespace codec_detail {

// Entry of the ascending `centers` nearest to v; at equal distance the lower.
inline int nearest_center(const std::vector<double>& centers, double v) {
    const auto it = std::lower_bound(centers.begin(), centers.end(), v);
    if (it == centers.begin()) return 0;
    if (it == centers.end()) return static_cast<int>(centers.size()) - 1;
    const int hi = static_cast<int>(it - centers.begin());
    return std::abs(v - centers[hi - 1]) <= std::abs(centers[hi] - v) ? hi - 1 : hi;
}

// One-dimensional k-means on a sample: at most k distinct values are their
// own centres; otherwise the sorted sample is binned into equal-width bins
// (bin sums in ascending order), the centres start at evenly spaced order
// statistics, and each iteration moves every centre to the mean of the bins
// whose mean lies nearest to it, then re-sorts the centres.
inline std::vector<double> binned_kmeans_1d(std::vector<double> v, int k_wanted, int bins, int iterations) {
    if (v.empty() || k_wanted <= 0) return {};
    std::sort(v.begin(), v.end());
    std::vector<double> distinct;
    bool more = false;
    for (const double a : v) {
        if (!distinct.empty() && a == distinct.back()) continue;
        if (static_cast<int>(distinct.size()) == k_wanted) {
            more = true;
            break;
        }
        distinct.push_back(a);
    }
    if (!more) return distinct;
    const int k = std::min<int>(k_wanted, static_cast<int>(v.size()));
    if (k <= 1 || v.front() == v.back()) return {v[v.size() / 2]};
    bins = std::max(k * 16, std::min(bins, static_cast<int>(v.size())));
    const double lo = v.front();
    const double per_unit = static_cast<double>(bins - 1) / (v.back() - lo);
    std::vector<Offset> count(static_cast<size_t>(bins), 0);
    std::vector<double> total(static_cast<size_t>(bins), 0.0);
    for (const double a : v) {
        const int b = std::clamp(static_cast<int>((a - lo) * per_unit), 0, bins - 1);
        ++count[static_cast<size_t>(b)];
        total[static_cast<size_t>(b)] += a;
    }
    std::vector<double> c(static_cast<size_t>(k));
    const long long last = static_cast<long long>(v.size() - 1);
    for (int i = 0; i < k; ++i) c[static_cast<size_t>(i)] = v[static_cast<size_t>((i * last) / std::max(1, k - 1))];
    std::sort(c.begin(), c.end());
    std::vector<double> acc(static_cast<size_t>(k));
    std::vector<Offset> hits(static_cast<size_t>(k));
    for (int it = 0; it < iterations; ++it) {
        std::fill(acc.begin(), acc.end(), 0.0);
        std::fill(hits.begin(), hits.end(), 0);
        for (int b = 0; b < bins; ++b) {
            const Offset n = count[static_cast<size_t>(b)];
            if (n == 0) continue;
            const int j = nearest_center(c, total[static_cast<size_t>(b)] / static_cast<double>(n));
            acc[static_cast<size_t>(j)] += total[static_cast<size_t>(b)];
            hits[static_cast<size_t>(j)] += n;
        }
        for (int i = 0; i < k; ++i)
            if (hits[static_cast<size_t>(i)] != 0)
                c[static_cast<size_t>(i)] = acc[static_cast<size_t>(i)] / static_cast<double>(hits[static_cast<size_t>(i)]);
        std::sort(c.begin(), c.end());
    }
    return c;
}

}  // namespace codec_detail

// ---- k256 uint8 value codebook (value_compression.hpp:20, 58-92, 442-497) ------

constexpr int kK256ValueCodebookSize = 256;

template <typename T>
struct K256UInt8ValueCodebook {
    std::array<T, kK256ValueCodebookSize> codebook{};
    std::vector<std::uint8_t> ids;
    int codebook_size = 0;
    bool exact = false;

    Offset nnz() const { return static_cast<Offset>(ids.size()); }
    std::size_t payload_bytes() const { return ids.size() + codebook.size() * sizeof(T); }
    std::vector<T> reconstruct() const {
        std::vector<T> v;
        v.reserve(ids.size());
        for (const std::uint8_t id : ids) v.push_back(codebook[id]);
        return v;
    }
    void validate() const {
        if (codebook_size < 0 || codebook_size > kK256ValueCodebookSize)
            throw std::runtime_error("K256 uint8 codebook size is invalid");
        for (const std::uint8_t id : ids)
            if (static_cast<int>(id) >= codebook_size)
                throw std::runtime_error("K256 uint8 value id is outside the codebook");
    }
};

// Index of `value` in `codebook` (first equal entry).
template <typename T>
int exact_value_id(const std::vector<T>& codebook, T value) {
    const auto it = std::find(codebook.begin(), codebook.end(), value);
    if (it == codebook.end()) throw std::runtime_error("K256 uint8 exact value was not found in codebook");
    return static_cast<int>(it - codebook.begin());
}

// Up to 256 distinct values: the ascending set itself, ids exact.  More:
// 256 k-means centres over a value histogram, ids to the nearest centre.
template <typename T>
K256UInt8ValueCodebook<T> build_k256_uint8_value_codebook(const std::vector<T>& values, int histogram_bins = 4096,
                                                          int iterations = 16) {
    K256UInt8ValueCodebook<T> c;
    c.ids.resize(values.size());
    if (values.empty()) return c;
    std::vector<double> sample;
    sample.reserve(values.size());
    for (const T raw : values) {
        if (!std::isfinite(static_cast<double>(raw)))
            throw std::runtime_error("K256 uint8 value codebook requires finite values");
        sample.push_back(static_cast<double>(raw));
    }
    const auto u = sorted_unique_values(values, kK256ValueCodebookSize);
    if (static_cast<int>(u.size()) <= kK256ValueCodebookSize) {
        c.exact = true;
        c.codebook_size = static_cast<int>(u.size());
        std::copy(u.begin(), u.end(), c.codebook.begin());
        for (std::size_t i = 0; i < values.size(); ++i) c.ids[i] = static_cast<std::uint8_t>(exact_value_id(u, values[i]));
    } else {
        const auto centers =
            codec_detail::binned_kmeans_1d(std::move(sample), kK256ValueCodebookSize, histogram_bins, iterations);
        c.codebook_size = static_cast<int>(centers.size());
        for (std::size_t i = 0; i < centers.size(); ++i) c.codebook[i] = static_cast<T>(centers[i]);
        for (std::size_t i = 0; i < values.size(); ++i)
            c.ids[i] = static_cast<std::uint8_t>(codec_detail::nearest_center(centers, static_cast<double>(values[i])));
    }
    c.validate();
    return c;
}

}  // namespace structural
