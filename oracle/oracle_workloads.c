/*
 * oracle_workloads.c -- CPU restatement of the seeded benchmark inputs.
 *
 * TEST INFRASTRUCTURE ONLY.  The reference measures on SuiteSparse files,
 * which are not present; the benchmark configurations are generated from a
 * counter-based SplitMix64 stream instead (Steele, Lea and Flood, OOPSLA
 * 2014): u = splitmix64(splitmix64(splitmix64(seed) ^ stream) ^ index),
 * uniform01 = (u >> 11) * 2^-53.  The library defines the same generators
 * (cove_synth.h); this file restates them in plain C so that the CPU
 * baseline and the reference arm of the benchmark can build their inputs
 * without loading the library they are compared with.  tests/ check that
 * both give identical arrays.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>

#define OC_EXPORT __attribute__((visibility("default")))

static uint64_t sm64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static uint64_t key_of(uint64_t seed, uint64_t stream) { return sm64(sm64(seed) ^ stream); }

static double u01(uint64_t key, uint64_t index) {
    return (double)(sm64(key ^ index) >> 11) * 0x1.0p-53;
}

/* Box-Muller on two uniforms of the pair (2i, 2i + 1). */
static double normal01(uint64_t key, uint64_t idx) {
    const double u1 = 1.0 - u01(key, 2 * idx);
    const double u2 = u01(key, 2 * idx + 1);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

/* kind 0: U[-1,1]; 1: U[0,1]; 2: N(0,1) over global indices [begin, begin + n). */
OC_EXPORT void oc_vector(int32_t kind, uint64_t seed, uint64_t stream, int64_t begin, int64_t n,
                         double* out) {
    const uint64_t key = key_of(seed, stream);
    for (int64_t t = 0; t < n; ++t) {
        const uint64_t i = (uint64_t)(begin + t);
        if (kind == 2) {
            out[t] = normal01(key, i);
        } else {
            const double u = u01(key, i);
            out[t] = kind == 0 ? 2.0 * u - 1.0 : u;
        }
    }
}

/* 3D 7-point Laplacian on nx x ny x nz (natural ordering, Dirichlet):
 * rows [rb, re), columns shifted by -shift, diagonal 6, neighbours -1,
 * columns ascending.  Null row_ptr: returns nnz only. */
OC_EXPORT int64_t oc_lapl3d_rows(int32_t nx, int32_t ny, int32_t nz, int64_t rb, int64_t re,
                                 int64_t shift, int64_t* row_ptr, int32_t* col, double* val) {
    const int64_t plane = (int64_t)nx * ny;
    int64_t p = 0;
    if (row_ptr) row_ptr[0] = 0;
    for (int64_t row = rb; row < re; ++row) {
        const int64_t k = row / plane, rem = row - k * plane, j = rem / nx, i = rem - j * nx;
        const int64_t c[7] = {row - plane, row - nx, row - 1, row, row + 1, row + nx, row + plane};
        const int on[7] = {k > 0, j > 0, i > 0, 1, i < nx - 1, j < ny - 1, k < nz - 1};
        for (int e = 0; e < 7; ++e) {
            if (!on[e]) continue;
            if (row_ptr) {
                col[p] = (int32_t)(c[e] - shift);
                val[p] = e == 3 ? 6.0 : -1.0;
            }
            ++p;
        }
        if (row_ptr) row_ptr[row - rb + 1] = p;
    }
    return p;
}

/* 2D 5-point Laplacian on nx x ny, Dirichlet: diagonal 4, neighbours -1. */
OC_EXPORT int64_t oc_lapl2d(int32_t nx, int32_t ny, int64_t* row_ptr, int32_t* col, double* val) {
    const int64_t n = (int64_t)nx * ny;
    int64_t p = 0;
    if (row_ptr) row_ptr[0] = 0;
    for (int64_t row = 0; row < n; ++row) {
        const int64_t j = row / nx, i = row - j * nx;
        const int64_t c[5] = {row - nx, row - 1, row, row + 1, row + nx};
        const int on[5] = {j > 0, i > 0, 1, i < nx - 1, j < ny - 1};
        for (int e = 0; e < 5; ++e) {
            if (!on[e]) continue;
            if (row_ptr) {
                col[p] = (int32_t)c[e];
                val[p] = e == 2 ? 4.0 : -1.0;
            }
            ++p;
        }
        if (row_ptr) row_ptr[row + 1] = p;
    }
    return p;
}

/* FEM-like 27-point stencil, nx x ny x nz nodes, dof unknowns per node with
 * dense dof x dof couplings; off-diagonal 0.05 N(0,1) keyed by the index
 * pair (min, max) (so the matrix is symmetric), diagonal 1 + the row's sum
 * of |off-diagonal|.  Rows [rb, re), columns shifted by -shift. */
OC_EXPORT int64_t oc_fem27_rows(int32_t nx, int32_t ny, int32_t nz, int32_t dof, uint64_t seed,
                                int64_t rb, int64_t re, int64_t shift, int64_t* row_ptr,
                                int32_t* col, double* val) {
    const int64_t n = (int64_t)nx * ny * nz * dof;
    const uint64_t key = key_of(seed, 0);
    int64_t p = 0;
    if (row_ptr) row_ptr[0] = 0;
    for (int64_t row = rb; row < re; ++row) {
        const int64_t node = row / dof;
        const int64_t k = node / ((int64_t)nx * ny);
        const int64_t rem = node - k * (int64_t)nx * ny;
        const int64_t j = rem / nx, i = rem - j * nx;
        int64_t diag = -1;
        double off = 0.0;
        for (int dk = -1; dk <= 1; ++dk)
            for (int dj = -1; dj <= 1; ++dj)
                for (int di = -1; di <= 1; ++di) {
                    if (k + dk < 0 || k + dk >= nz || j + dj < 0 || j + dj >= ny || i + di < 0 ||
                        i + di >= nx)
                        continue;
                    const int64_t nb = ((k + dk) * ny + (j + dj)) * (int64_t)nx + (i + di);
                    for (int b = 0; b < dof; ++b) {
                        const int64_t c = nb * dof + b;
                        if (row_ptr) {
                            col[p] = (int32_t)(c - shift);
                            if (c == row) {
                                diag = p;
                                val[p] = 0.0;
                            } else {
                                const int64_t lo = row < c ? row : c, hi = row < c ? c : row;
                                const double v = 0.05 * normal01(key, (uint64_t)(lo * n + hi));
                                val[p] = v;
                                off += fabs(v);
                            }
                        }
                        ++p;
                    }
                }
        if (row_ptr) {
            val[diag] = 1.0 + off;
            row_ptr[row - rb + 1] = p;
        }
    }
    return p;
}

/* MatrixMarket coordinate file of a CSR (1-based, "general"), values with
 * %.17g (esz 8) or %.9g (esz 4) so they read back exactly.  Returns 0, or -1
 * when the file cannot be written. */
OC_EXPORT int oc_write_mtx(const char* path, int64_t rows, int64_t cols, const int64_t* row_ptr,
                           const int32_t* col, const void* val, int32_t esz) {
    FILE* f = fopen(path, "w");
    if (!f) return -1;
    static char buf[1 << 20];
    setvbuf(f, buf, _IOFBF, sizeof(buf));
    fprintf(f, "%%%%MatrixMarket matrix coordinate real general\n");
    fprintf(f, "%lld %lld %lld\n", (long long)rows, (long long)cols, (long long)row_ptr[rows]);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
            if (esz == 8)
                fprintf(f, "%lld %d %.17g\n", (long long)(r + 1), col[p] + 1, ((const double*)val)[p]);
            else
                fprintf(f, "%lld %d %.9g\n", (long long)(r + 1), col[p] + 1, (double)((const float*)val)[p]);
        }
    return fclose(f) == 0 ? 0 : -1;
}
