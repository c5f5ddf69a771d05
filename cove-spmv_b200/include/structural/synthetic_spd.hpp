// structural/synthetic_spd.hpp -- the CG bench's seeded SPD test matrices
// (structural/src/bench_cg_solve.cu:199-278, file-static there) and its
// right-hand side (:593-601), host only.
//
//   make_synthetic_spd(n, halfbw, seed, delta): symmetric band of half
//     width halfbw, off-diagonals uniform(-1, 1), diagonal = sum of the
//     row's |off-diagonals| + delta (strictly diagonally dominant, SPD).
//   make_synthetic_laplacian_spd(n, halfbw, seed, sigma): weighted graph
//     Laplacian of the same band, weights uniform(0.1, 1), off-diagonals
//     -w, diagonal = weighted degree + sigma.
//
// A matrix is the same for a given seed as the reference's: the band's
// upper-triangle values are drawn from std::mt19937_64(seed) through
// std::uniform_real_distribution, row by row and left to right, and every
// diagonal sums its row's terms in ascending column order.
#pragma once

#include "structural/csr.hpp"

#include <algorithm>
#include <cmath>
#include <random>
#include <vector>

namespace structural {

namespace synth_detail {

// Draws the upper band: entry (i, i + 1 + k) for k < width(i) sits at
// upper[start[i] + k].
struct UpperBand {
    int n = 0, halfbw = 0;
    std::vector<std::size_t> start;
    std::vector<double> upper;
    int width(int i) const { return std::max(0, std::min(n - 1, i + halfbw) - i); }
    double at(int i, int j) const { return upper[start[i] + static_cast<std::size_t>(j - i - 1)]; }
};

inline UpperBand draw_upper_band(int n, int halfbw, unsigned seed, double lo, double hi) {
    UpperBand b;
    b.n = std::max(n, 0);
    b.halfbw = std::max(halfbw, 0);  // no band: the diagonal alone
    n = b.n;
    b.start.assign(static_cast<std::size_t>(n) + 1, 0);
    for (int i = 0; i < n; ++i) b.start[i + 1] = b.start[i] + static_cast<std::size_t>(b.width(i));
    b.upper.resize(b.start[n]);
    std::mt19937_64 rng(seed);
    std::uniform_real_distribution<double> u(lo, hi);
    for (double& v : b.upper) v = u(rng);
    return b;
}

// CSR of the symmetric band: off-diagonal (i, j) = sign * w(min, max),
// diagonal = sum over the row's off-diagonal columns, ascending, of
// |w| + shift.
inline CsrMatrix<double> band_csr(const UpperBand& b, double sign, double shift) {
    const int n = b.n;
    CsrMatrix<double> a;
    a.rows = n;
    a.cols = n;
    a.row_ptr.assign(static_cast<std::size_t>(n) + 1, 0);
    for (int i = 0; i < n; ++i) {
        const int lower = i - std::max(0, i - b.halfbw);
        a.row_ptr[i + 1] = a.row_ptr[i] + static_cast<Offset>(lower + 1 + b.width(i));
    }
    a.col_idx.resize(static_cast<std::size_t>(a.row_ptr[n]));
    a.values.resize(static_cast<std::size_t>(a.row_ptr[n]));
    for (int i = 0; i < n; ++i) {
        Offset p = a.row_ptr[i];
        double diag = 0.0;
        Offset diag_at = 0;
        for (int j = std::max(0, i - b.halfbw); j <= std::min(n - 1, i + b.halfbw); ++j) {
            a.col_idx[p] = j;
            if (j == i) {
                diag_at = p++;
                continue;
            }
            const double w = j < i ? b.at(j, i) : b.at(i, j);
            diag += std::abs(w);
            a.values[p++] = sign * w;
        }
        a.values[diag_at] = diag + shift;
    }
    return a;
}

}  // namespace synth_detail

inline CsrMatrix<double> make_synthetic_spd(int n, int halfbw, unsigned seed, double delta) {
    return synth_detail::band_csr(synth_detail::draw_upper_band(n, halfbw, seed, -1.0, 1.0), 1.0, delta);
}

inline CsrMatrix<double> make_synthetic_laplacian_spd(int n, int halfbw, unsigned seed, double sigma) {
    return synth_detail::band_csr(synth_detail::draw_upper_band(n, halfbw, seed, 0.1, 1.0), -1.0, sigma);
}

// x_true ~ N(0, 1) from std::mt19937_64(seed), the bench's known solution.
inline std::vector<double> synthetic_solution(int n, unsigned seed) {
    std::vector<double> x(static_cast<std::size_t>(std::max(n, 0)));
    std::mt19937_64 rng(seed);
    std::normal_distribution<double> nd(0.0, 1.0);
    for (double& v : x) v = nd(rng);
    return x;
}

}  // namespace structural
