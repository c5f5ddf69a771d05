// synth.cu -- seeded synthetic matrices and vectors (see include/cove_synth.h).
//
// Host generators (OpenMP) produce the CSR inputs of the parity tests and
// benchmarks; the device generator writes the large 7-point Laplacian row
// blocks straight into HBM.
#include "cove_internal.cuh"
#include "cove_synth.h"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <vector>

namespace {

__host__ __device__ inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__host__ __device__ inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return splitmix64(splitmix64(seed) ^ stream);
}

__host__ __device__ inline double u01_key(uint64_t key, uint64_t index) {
    return static_cast<double>(splitmix64(key ^ index) >> 11) * 0x1.0p-53;
}

inline uint16_t bf16_rne(float v) {
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    const uint32_t lsb = (bits >> 16) & 1u;
    return static_cast<uint16_t>((bits + 0x7fffu + lsb) >> 16);
}

inline float bf16_float(uint16_t b) {
    const uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

inline int lapl3d_count(int64_t row, int32_t nx, int32_t ny, int32_t nz) {
    const int64_t plane = static_cast<int64_t>(nx) * ny;
    const int64_t k = row / plane;
    const int64_t rem = row - k * plane;
    const int64_t j = rem / nx;
    const int64_t i = rem - j * nx;
    return 1 + (i > 0) + (i < nx - 1) + (j > 0) + (j < ny - 1) + (k > 0) + (k < nz - 1);
}

__global__ void lapl3d_count_kernel(int32_t nx, int32_t ny, int32_t nz, int64_t row_begin,
                                    int64_t rows, int32_t* __restrict__ cnt) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= rows) return;
    const int64_t row = row_begin + t;
    const int64_t plane = static_cast<int64_t>(nx) * ny;
    const int64_t k = row / plane;
    const int64_t rem = row - k * plane;
    const int64_t j = rem / nx;
    const int64_t i = rem - j * nx;
    cnt[t] = 1 + (i > 0) + (i < nx - 1) + (j > 0) + (j < ny - 1) + (k > 0) + (k < nz - 1);
}

__global__ void lapl3d_fill_kernel(int32_t nx, int32_t ny, int32_t nz, int64_t row_begin,
                                   int64_t rows, int64_t col_shift,
                                   const int32_t* __restrict__ rp, int32_t* __restrict__ col,
                                   double* __restrict__ val) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= rows) return;
    const int64_t row = row_begin + t;
    const int64_t plane = static_cast<int64_t>(nx) * ny;
    const int64_t k = row / plane;
    const int64_t rem = row - k * plane;
    const int64_t j = rem / nx;
    const int64_t i = rem - j * nx;
    int64_t p = rp[t];
    auto put = [&](int64_t c, double v) {
        col[p] = static_cast<int32_t>(c - col_shift);
        val[p] = v;
        ++p;
    };
    if (k > 0) put(row - plane, -1.0);
    if (j > 0) put(row - nx, -1.0);
    if (i > 0) put(row - 1, -1.0);
    put(row, 6.0);
    if (i < nx - 1) put(row + 1, -1.0);
    if (j < ny - 1) put(row + nx, -1.0);
    if (k < nz - 1) put(row + plane, -1.0);
}

__global__ void vector_kernel(int32_t kind, uint64_t key, int64_t begin, int64_t n,
                              double* __restrict__ out) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n) return;
    const double u = u01_key(key, static_cast<uint64_t>(begin + t));
    out[t] = kind == 0 ? 2.0 * u - 1.0 : u;
}

// ---- 8x4 block-sparse rows (the host generator's draws, on the device) ----------
// One warp per block row scans the block columns (a lane per column, a
// Bernoulli draw each); a present block's 32 cells are one lane each.

struct BlockSparseKeys {
    uint64_t kb, ke, kv, ko, ks, km;
};

__host__ __device__ inline BlockSparseKeys blocksparse_keys(uint64_t seed) {
    return {stream_key(seed, 0), stream_key(seed, 1), stream_key(seed, 2),
            stream_key(seed, 3), stream_key(seed, 4), stream_key(seed, 5)};
}

// The value of cell `cell` (block * 32 + bit).  The outlier magnitude is a
// separate multiply and add on the device too (the host compiler does not
// contract it), so both give the same double.
__device__ inline double blocksparse_value_dev(const BlockSparseKeys& k, double outlier_fraction, uint64_t cell) {
    if (u01_key(k.ko, cell) < outlier_fraction) {
        const double sgn = u01_key(k.ks, cell) < 0.5 ? -1.0 : 1.0;
        return sgn * __dadd_rn(1e5, __dmul_rn(9e5, u01_key(k.km, cell)));
    }
    for (int t = 0; t < 8; ++t) {
        const float f = static_cast<float>(__dadd_rn(__dmul_rn(16.0, u01_key(k.kv, cell * 8 + t)), -8.0));
        const uint32_t bits = __float_as_uint(f);
        const uint32_t r = ((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16) << 16;  // bf16, ties to even
        if (__uint_as_float(r) != 0.0f) return static_cast<double>(__uint_as_float(r));
    }
    return 1.0;
}

__global__ void blocksparse_count_kernel(int32_t n, int64_t nbc, double p_block, double p_entry,
                                         BlockSparseKeys k, int64_t br0, int64_t nbr_local,
                                         int64_t row_begin, int32_t* __restrict__ cnt) {
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= nbr_local) return;  // whole warp
    const int64_t br = br0 + w;
    int c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t bc = lane; bc < nbc; bc += 32) {
        const uint64_t blk = static_cast<uint64_t>(br * nbc + bc);
        if (u01_key(k.kb, blk) < p_block) {
#pragma unroll
            for (int lr = 0; lr < 8; ++lr)
#pragma unroll
                for (int lc = 0; lc < 4; ++lc)
                    c[lr] += (bc * 4 + lc < n && u01_key(k.ke, blk * 32 + lr * 4 + lc) < p_entry) ? 1 : 0;
        }
    }
#pragma unroll
    for (int lr = 0; lr < 8; ++lr) {
        const int t = __reduce_add_sync(0xffffffffu, c[lr]);
        const int64_t row = br * 8 + lr;
        if (lane == 0 && row < n) cnt[row - row_begin] = t;
    }
}

__global__ void blocksparse_fill_kernel(int32_t n, int64_t nbc, double p_block, double p_entry,
                                        double outlier_fraction, BlockSparseKeys k, int64_t br0,
                                        int64_t nbr_local, int64_t row_begin,
                                        const int32_t* __restrict__ rp, int32_t* __restrict__ ci,
                                        double* __restrict__ v) {
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= nbr_local) return;
    const int64_t br = br0 + w;
    const int lr = lane >> 2, lc = lane & 3;
    // lane i < 8 carries row i's next write position
    int32_t pos = (lane < 8 && br * 8 + lane < n) ? rp[br * 8 + lane - row_begin] : 0;
    for (int64_t base = 0; base < nbc; base += 32) {
        const int64_t bc = base + lane;
        const bool present = bc < nbc && u01_key(k.kb, static_cast<uint64_t>(br * nbc + bc)) < p_block;
        unsigned pb = __ballot_sync(0xffffffffu, present);
        while (pb) {
            const int src = __ffs(pb) - 1;
            pb &= pb - 1;
            const int64_t pbc = base + src;
            const uint64_t blk = static_cast<uint64_t>(br * nbc + pbc);
            const bool cell = pbc * 4 + lc < n && br * 8 + lr < n && u01_key(k.ke, blk * 32 + lane) < p_entry;
            const unsigned cb = __ballot_sync(0xffffffffu, cell);
            const int32_t row_pos = __shfl_sync(0xffffffffu, pos, lr);
            if (cell) {
                const int32_t p = row_pos + __popc(cb & (0xFu << (4 * lr)) & ((1u << lane) - 1u));
                ci[p] = static_cast<int32_t>(pbc * 4 + lc);
                v[p] = blocksparse_value_dev(k, outlier_fraction, blk * 32 + lane);
            }
            if (lane < 8) pos += __popc(cb & (0xFu << (4 * lane)));
        }
    }
}

}  // namespace

extern "C" {

uint64_t cove_rng_u64(uint64_t seed, uint64_t stream, uint64_t index) {
    return splitmix64(stream_key(seed, stream) ^ index);
}

double cove_rng_uniform01(uint64_t seed, uint64_t stream, uint64_t index) {
    return u01_key(stream_key(seed, stream), index);
}

int64_t cove_synth_lapl2d(int32_t nx, int32_t ny, int64_t* rp, int32_t* ci, double* v) {
    const int64_t n = static_cast<int64_t>(nx) * ny;
    if (!rp) {
        int64_t nnz = 0;
        for (int64_t r = 0; r < n; ++r) {
            const int64_t j = r / nx, i = r - j * nx;
            nnz += 1 + (i > 0) + (i < nx - 1) + (j > 0) + (j < ny - 1);
        }
        return nnz;
    }
    rp[0] = 0;
    for (int64_t r = 0; r < n; ++r) {
        const int64_t j = r / nx, i = r - j * nx;
        rp[r + 1] = rp[r] + 1 + (i > 0) + (i < nx - 1) + (j > 0) + (j < ny - 1);
    }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        const int64_t j = r / nx, i = r - j * nx;
        int64_t p = rp[r];
        auto put = [&](int64_t c, double val) {
            ci[p] = static_cast<int32_t>(c);
            v[p] = val;
            ++p;
        };
        if (j > 0) put(r - nx, -1.0);
        if (i > 0) put(r - 1, -1.0);
        put(r, 4.0);
        if (i < nx - 1) put(r + 1, -1.0);
        if (j < ny - 1) put(r + nx, -1.0);
    }
    return rp[n];
}

int64_t cove_synth_lapl3d(int32_t nx, int32_t ny, int32_t nz, int64_t rb, int64_t re,
                          int64_t shift, int64_t* rp, int32_t* ci, double* v) {
    const int64_t rows = re - rb;
    if (!rp) {
        int64_t nnz = 0;
#pragma omp parallel for reduction(+ : nnz) schedule(static)
        for (int64_t t = 0; t < rows; ++t) nnz += lapl3d_count(rb + t, nx, ny, nz);
        return nnz;
    }
    rp[0] = 0;
    for (int64_t t = 0; t < rows; ++t) rp[t + 1] = rp[t] + lapl3d_count(rb + t, nx, ny, nz);
    const int64_t plane = static_cast<int64_t>(nx) * ny;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < rows; ++t) {
        const int64_t row = rb + t;
        const int64_t k = row / plane, rem = row - k * plane, j = rem / nx, i = rem - j * nx;
        int64_t p = rp[t];
        auto put = [&](int64_t c, double val) {
            ci[p] = static_cast<int32_t>(c - shift);
            v[p] = val;
            ++p;
        };
        if (k > 0) put(row - plane, -1.0);
        if (j > 0) put(row - nx, -1.0);
        if (i > 0) put(row - 1, -1.0);
        put(row, 6.0);
        if (i < nx - 1) put(row + 1, -1.0);
        if (j < ny - 1) put(row + nx, -1.0);
        if (k < nz - 1) put(row + plane, -1.0);
    }
    return rp[rows];
}

static double normal_draw(uint64_t key, uint64_t idx) {
    const double u1 = 1.0 - u01_key(key, 2 * idx);
    const double u2 = u01_key(key, 2 * idx + 1);
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

int64_t cove_synth_fem27_rows(int32_t nx, int32_t ny, int32_t nz, int32_t dof, uint64_t seed,
                              int64_t row_begin, int64_t row_end, int64_t col_shift,
                              int64_t* rp, int32_t* ci, double* v) {
    const int64_t nodes = static_cast<int64_t>(nx) * ny * nz;
    const int64_t n = nodes * dof;
    const int64_t rows = row_end - row_begin;
    auto node_nbrs = [&](int64_t node) {
        const int64_t k = node / (static_cast<int64_t>(nx) * ny);
        const int64_t rem = node - k * nx * static_cast<int64_t>(ny);
        const int64_t j = rem / nx, i = rem - j * nx;
        int c = 0;
        for (int dk = -1; dk <= 1; ++dk)
            for (int dj = -1; dj <= 1; ++dj)
                for (int di = -1; di <= 1; ++di)
                    if (k + dk >= 0 && k + dk < nz && j + dj >= 0 && j + dj < ny && i + di >= 0 &&
                        i + di < nx)
                        ++c;
        return c;
    };
    if (!rp) {
        int64_t nnz = 0;
#pragma omp parallel for reduction(+ : nnz) schedule(static)
        for (int64_t t = 0; t < rows; ++t) nnz += static_cast<int64_t>(node_nbrs((row_begin + t) / dof)) * dof;
        return nnz;
    }
    rp[0] = 0;
    for (int64_t t = 0; t < rows; ++t)
        rp[t + 1] = rp[t] + static_cast<int64_t>(node_nbrs((row_begin + t) / dof)) * dof;
    const uint64_t key = stream_key(seed, 0);
#pragma omp parallel for schedule(dynamic, 256)
    for (int64_t t = 0; t < rows; ++t) {
        const int64_t row = row_begin + t;
        const int64_t node = row / dof;
        const int64_t k = node / (static_cast<int64_t>(nx) * ny);
        const int64_t rem = node - k * nx * static_cast<int64_t>(ny);
        const int64_t j = rem / nx, i = rem - j * nx;
        int64_t p = rp[t];
        int64_t diag_p = -1;
        double off_sum = 0.0;
        for (int dk = -1; dk <= 1; ++dk)
            for (int dj = -1; dj <= 1; ++dj)
                for (int di = -1; di <= 1; ++di) {
                    if (k + dk < 0 || k + dk >= nz || j + dj < 0 || j + dj >= ny || i + di < 0 ||
                        i + di >= nx)
                        continue;
                    const int64_t nb = ((k + dk) * ny + (j + dj)) * static_cast<int64_t>(nx) + (i + di);
                    for (int b = 0; b < dof; ++b) {
                        const int64_t col = nb * dof + b;
                        ci[p] = static_cast<int32_t>(col - col_shift);
                        if (col == row) {
                            diag_p = p;
                            v[p] = 0.0;
                        } else {
                            const int64_t lo = std::min(row, col), hi = std::max(row, col);
                            const double val = 0.05 * normal_draw(key, static_cast<uint64_t>(lo * n + hi));
                            v[p] = val;
                            off_sum += std::fabs(val);
                        }
                        ++p;
                    }
                }
        v[diag_p] = 1.0 + off_sum;
    }
    return rp[rows];
}

int64_t cove_synth_fem27(int32_t nx, int32_t ny, int32_t nz, int32_t dof, uint64_t seed,
                         int64_t* rp, int32_t* ci, double* v) {
    const int64_t n = static_cast<int64_t>(nx) * ny * nz * dof;
    return cove_synth_fem27_rows(nx, ny, nz, dof, seed, 0, n, 0, rp, ci, v);
}

int64_t cove_synth_rmat(int32_t scale, int32_t edge_factor, double a, double b, double c,
                        uint64_t seed, int64_t* rp, int32_t* ci, float* v) {
    const int64_t n = int64_t{1} << scale;
    const int64_t E = static_cast<int64_t>(edge_factor) << scale;
    std::vector<int32_t> er(E), ec(E);
    std::vector<float> ev(E);
    std::vector<uint64_t> keys(scale + 1);
    for (int l = 0; l <= scale; ++l) keys[l] = stream_key(seed, static_cast<uint64_t>(l));
    const double ab = a + b, abc = a + b + c;
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < E; ++e) {
        int64_t r = 0, cc = 0;
        for (int l = 0; l < scale; ++l) {
            const double u = u01_key(keys[l + 1], static_cast<uint64_t>(e));
            int rb, cb;
            if (u < a) { rb = 0; cb = 0; }
            else if (u < ab) { rb = 0; cb = 1; }
            else if (u < abc) { rb = 1; cb = 0; }
            else { rb = 1; cb = 1; }
            r = (r << 1) | rb;
            cc = (cc << 1) | cb;
        }
        er[e] = static_cast<int32_t>(r);
        ec[e] = static_cast<int32_t>(cc);
        ev[e] = static_cast<float>(1.0 - u01_key(keys[0], static_cast<uint64_t>(e)));
    }
    // stable counting sort by row, then per-row stable sort by column and
    // summation of duplicates in draw order
    std::vector<int64_t> start(n + 1, 0);
    for (int64_t e = 0; e < E; ++e) ++start[er[e] + 1];
    for (int64_t r = 0; r < n; ++r) start[r + 1] += start[r];
    std::vector<int32_t> sc(E);
    std::vector<float> sv(E);
    {
        std::vector<int64_t> pos(start.begin(), start.end() - 1);
        for (int64_t e = 0; e < E; ++e) {
            const int64_t p = pos[er[e]]++;
            sc[p] = ec[e];
            sv[p] = ev[e];
        }
    }
    std::vector<int64_t> merged(n, 0);
#pragma omp parallel
    {
        std::vector<int64_t> idx;
#pragma omp for schedule(dynamic, 256)
        for (int64_t r = 0; r < n; ++r) {
            const int64_t b0 = start[r], b1 = start[r + 1];
            idx.resize(b1 - b0);
            std::iota(idx.begin(), idx.end(), b0);
            std::stable_sort(idx.begin(), idx.end(), [&](int64_t x, int64_t y) { return sc[x] < sc[y]; });
            std::vector<int32_t> cols;
            std::vector<float> vals;
            for (int64_t q : idx) {
                if (!cols.empty() && cols.back() == sc[q]) vals.back() += sv[q];
                else { cols.push_back(sc[q]); vals.push_back(sv[q]); }
            }
            for (size_t q = 0; q < cols.size(); ++q) {
                sc[b0 + q] = cols[q];
                sv[b0 + q] = vals[q];
            }
            merged[r] = static_cast<int64_t>(cols.size());
        }
    }
    int64_t nnz = 0;
    for (int64_t r = 0; r < n; ++r) nnz += merged[r];
    if (!rp) return nnz;
    rp[0] = 0;
    for (int64_t r = 0; r < n; ++r) rp[r + 1] = rp[r] + merged[r];
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        std::memcpy(ci + rp[r], sc.data() + start[r], merged[r] * sizeof(int32_t));
        std::memcpy(v + rp[r], sv.data() + start[r], merged[r] * sizeof(float));
    }
    return nnz;
}

int64_t cove_synth_blocksparse(int32_t n, double p_block, double p_entry, double outlier_fraction,
                               uint64_t seed, int64_t* rp, int32_t* ci, double* v) {
    return cove_synth_blocksparse_rows(n, p_block, p_entry, outlier_fraction, seed, 0, n, rp, ci, v);
}

int64_t cove_synth_blocksparse_rows(int32_t n, double p_block, double p_entry, double outlier_fraction,
                                    uint64_t seed, int64_t rb, int64_t re, int64_t* rp, int32_t* ci,
                                    double* v) {
    if (n < 0 || rb < 0 || re < rb || re > n || rb % 8 != 0 || (re % 8 != 0 && re != n)) return -1;
    const int64_t nbc = (n + 3) / 4;
    const int64_t br0 = rb / 8, br1 = (re + 7) / 8;
    const uint64_t kb = stream_key(seed, 0), ke = stream_key(seed, 1), kv = stream_key(seed, 2);
    const uint64_t ko = stream_key(seed, 3), ks = stream_key(seed, 4), km = stream_key(seed, 5);
    auto present_blocks = [&](int64_t br, std::vector<int32_t>& out) {
        out.clear();
        for (int64_t bc = 0; bc < nbc; ++bc)
            if (u01_key(kb, static_cast<uint64_t>(br * nbc + bc)) < p_block) out.push_back(static_cast<int32_t>(bc));
    };
    auto cell_present = [&](int64_t blk, int bit) {
        return u01_key(ke, static_cast<uint64_t>(blk * 32 + bit)) < p_entry;
    };
    auto cell_value = [&](int64_t cell) -> double {
        if (u01_key(ko, static_cast<uint64_t>(cell)) < outlier_fraction) {
            const double sgn = u01_key(ks, static_cast<uint64_t>(cell)) < 0.5 ? -1.0 : 1.0;
            return sgn * (1e5 + 9e5 * u01_key(km, static_cast<uint64_t>(cell)));
        }
        for (int t = 0; t < 8; ++t) {
            const float f = static_cast<float>(16.0 * u01_key(kv, static_cast<uint64_t>(cell * 8 + t)) - 8.0);
            const float r = bf16_float(bf16_rne(f));
            if (r != 0.0f) return static_cast<double>(r);
        }
        return 1.0;
    };
    const int64_t rows = re - rb;
    std::vector<int64_t> rowcnt(rows, 0);
#pragma omp parallel
    {
        std::vector<int32_t> blocks;
#pragma omp for schedule(dynamic, 16)
        for (int64_t br = br0; br < br1; ++br) {
            present_blocks(br, blocks);
            for (int lr = 0; lr < 8; ++lr) {
                const int64_t row = br * 8 + lr;
                if (row >= n) break;
                int64_t cnt = 0;
                for (int32_t bc : blocks)
                    for (int lc = 0; lc < 4; ++lc)
                        if (bc * 4 + lc < n && cell_present(br * nbc + bc, lr * 4 + lc)) ++cnt;
                rowcnt[row - rb] = cnt;
            }
        }
    }
    int64_t nnz = 0;
    for (int64_t r = 0; r < rows; ++r) nnz += rowcnt[r];
    if (!rp) return nnz;
    rp[0] = 0;
    for (int64_t r = 0; r < rows; ++r) rp[r + 1] = rp[r] + rowcnt[r];
#pragma omp parallel
    {
        std::vector<int32_t> blocks;
#pragma omp for schedule(dynamic, 16)
        for (int64_t br = br0; br < br1; ++br) {
            present_blocks(br, blocks);
            for (int lr = 0; lr < 8; ++lr) {
                const int64_t row = br * 8 + lr;
                if (row >= n) break;
                int64_t p = rp[row - rb];
                for (int32_t bc : blocks)
                    for (int lc = 0; lc < 4; ++lc) {
                        const int64_t blk = br * nbc + bc;
                        const int bit = lr * 4 + lc;
                        if (bc * 4 + lc < n && cell_present(blk, bit)) {
                            ci[p] = bc * 4 + lc;
                            v[p] = cell_value(blk * 32 + bit);
                            ++p;
                        }
                    }
            }
        }
    }
    return nnz;
}

void cove_synth_vector(int32_t kind, uint64_t seed, uint64_t stream, int64_t n, int32_t dtype,
                       void* out) {
    const uint64_t key = stream_key(seed, stream);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        double val;
        if (kind == 2) {
            val = normal_draw(key, static_cast<uint64_t>(i));
        } else {
            const double u = u01_key(key, static_cast<uint64_t>(i));
            val = kind == 0 ? 2.0 * u - 1.0 : u;
        }
        if (dtype == 0) static_cast<double*>(out)[i] = val;
        else static_cast<float*>(out)[i] = static_cast<float>(val);
    }
}

int cove_synth_lapl3d_device(int32_t nx, int32_t ny, int32_t nz, int64_t rb, int64_t re,
                             int64_t shift, int32_t* rp, int32_t* ci, double* v,
                             int64_t* nnz_out, void* stream) {
    return cove::guarded([&] {
        const int64_t rows = re - rb;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cove::DevBuf cnt;
        cove::alloc_n<int32_t>(cnt, rows);
        if (rows > 0) {
            lapl3d_count_kernel<<<cove::grid_for(rows, 256), 256, 0, s>>>(nx, ny, nz, rb, rows,
                                                                          cnt.as<int32_t>());
            CUDA_LAUNCH_OK();
        }
        cove::DevBuf tmp;
        int32_t* dst = rp;
        if (!dst) {
            cove::alloc_n<int64_t>(tmp, rows + 1);
            const int64_t nnz = cove::exclusive_scan_total<int32_t, int64_t>(
                cnt.as<int32_t>(), tmp.as<int64_t>(), rows, s);
            if (nnz_out) *nnz_out = nnz;
            return;
        }
        const int64_t nnz = cove::exclusive_scan_total<int32_t, int32_t>(cnt.as<int32_t>(), dst, rows, s);
        if (nnz > INT32_MAX) COVE_THROW(COVE_ERR_OVERFLOW, "row block exceeds int32 nnz");
        if (nnz_out) *nnz_out = nnz;
        if (rows > 0) {
            lapl3d_fill_kernel<<<cove::grid_for(rows, 256), 256, 0, s>>>(nx, ny, nz, rb, rows, shift,
                                                                         dst, ci, v);
            CUDA_LAUNCH_OK();
        }
        CUDA_OK(cudaStreamSynchronize(s));
    });
}

int cove_synth_blocksparse_device(int32_t n, double p_block, double p_entry, double outlier_fraction,
                                  uint64_t seed, int64_t rb, int64_t re, int32_t* rp, int32_t* ci,
                                  double* v, int64_t* nnz_out, void* stream) {
    return cove::guarded([&] {
        if (n < 0 || rb < 0 || re < rb || re > n) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "bad row range");
        if (rb % 8 != 0 || (re % 8 != 0 && re != n)) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "row range must cover whole 8-row block rows");
        }
        const int64_t rows = re - rb;
        const int64_t nbc = (static_cast<int64_t>(n) + 3) / 4;
        const int64_t br0 = rb / 8, nbr_local = (re + 7) / 8 - br0;
        const BlockSparseKeys k = blocksparse_keys(seed);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cove::DevBuf cnt;
        cove::alloc_n<int32_t>(cnt, rows);
        const int grid = cove::grid_for(nbr_local * 32, 256);
        if (rows > 0) {
            blocksparse_count_kernel<<<grid, 256, 0, s>>>(n, nbc, p_block, p_entry, k, br0, nbr_local, rb,
                                                          cnt.as<int32_t>());
            CUDA_LAUNCH_OK();
        }
        cove::DevBuf tmp;
        if (!rp) {
            cove::alloc_n<int64_t>(tmp, rows + 1);
            const int64_t nnz = cove::exclusive_scan_total<int32_t, int64_t>(cnt.as<int32_t>(), tmp.as<int64_t>(),
                                                                            rows, s);
            if (nnz_out) *nnz_out = nnz;
            return;
        }
        // count into an int64 scan first: a block of more than INT32_MAX entries is refused
        // before any int32 offset is written
        cove::alloc_n<int64_t>(tmp, rows + 1);
        const int64_t nnz = cove::exclusive_scan_total<int32_t, int64_t>(cnt.as<int32_t>(), tmp.as<int64_t>(), rows, s);
        if (nnz > INT32_MAX) COVE_THROW(COVE_ERR_OVERFLOW, "row block exceeds int32 nnz");
        cove::exclusive_scan_total<int32_t, int32_t>(cnt.as<int32_t>(), rp, rows, s);
        if (nnz_out) *nnz_out = nnz;
        if (rows > 0 && nnz > 0) {
            if (!ci || !v) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null col_idx/values");
            blocksparse_fill_kernel<<<grid, 256, 0, s>>>(n, nbc, p_block, p_entry, outlier_fraction, k, br0,
                                                         nbr_local, rb, rp, ci, v);
            CUDA_LAUNCH_OK();
        }
        CUDA_OK(cudaStreamSynchronize(s));
    });
}

int cove_synth_vector_device(int32_t kind, uint64_t seed, uint64_t stream, int64_t begin,
                             int64_t n, double* out, void* cuda_stream) {
    return cove::guarded([&] {
        if (n <= 0) return;
        vector_kernel<<<cove::grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(cuda_stream)>>>(
            kind, stream_key(seed, stream), begin, n, out);
        CUDA_LAUNCH_OK();
    });
}

}  // extern "C"
