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
#include <stdlib.h>
#include <string.h>

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

/* ---- 8x4 block-sparse rows and the R-MAT graph ----------------------------- */

static uint16_t oc_bf16_rne(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

static float oc_bf16_float(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Value of cell `cell` (block * 32 + bit): an outlier +-U(1e5, 1e6) with
 * probability `outlier_fraction`, else the first nonzero of eight draws
 * U[-8, 8] rounded to bf16 (ties to even), else 1. */
static double bs_value(const uint64_t* k, double outlier_fraction, uint64_t cell) {
    if (u01(k[3], cell) < outlier_fraction) {
        const double sgn = u01(k[4], cell) < 0.5 ? -1.0 : 1.0;
        return sgn * (1e5 + 9e5 * u01(k[5], cell));
    }
    for (int t = 0; t < 8; ++t) {
        const float f = (float)(16.0 * u01(k[2], cell * 8 + (uint64_t)t) - 8.0);
        const float r = oc_bf16_float(oc_bf16_rne(f));
        if (r != 0.0f) return (double)r;
    }
    return 1.0;
}

/* Rows [rb, re) of the random 8x4 block-sparse n x n matrix: block (br, bc)
 * present iff U(stream 0, br * nbc + bc) < p_block, cell bit of a present
 * block iff U(stream 1, block * 32 + bit) < p_entry (bit = local_row * 4 +
 * local_col), columns beyond n dropped.  rb a multiple of 8, re a multiple
 * of 8 or n; row_ptr relative to rb, global columns.  Returns nnz (-1 for a
 * bad range); null row_ptr counts only. */
OC_EXPORT int64_t oc_blocksparse_rows(int32_t n, double p_block, double p_entry, double outlier_fraction,
                                      uint64_t seed, int64_t rb, int64_t re, int64_t* row_ptr,
                                      int32_t* col, double* val) {
    if (n < 0 || rb < 0 || re < rb || re > n || rb % 8 != 0 || (re % 8 != 0 && re != n)) return -1;
    const int64_t nbc = ((int64_t)n + 3) / 4;
    uint64_t k[6];
    for (int s = 0; s < 6; ++s) k[s] = key_of(seed, (uint64_t)s);
    int64_t nnz = 0;
    if (row_ptr) row_ptr[0] = 0;
    int32_t* blocks = (int32_t*)malloc((size_t)(nbc > 0 ? nbc : 1) * sizeof(int32_t));
    if (!blocks) return -1;
    for (int64_t br = rb / 8; br < (re + 7) / 8; ++br) {
        int64_t nb = 0;
        for (int64_t bc = 0; bc < nbc; ++bc)
            if (u01(k[0], (uint64_t)(br * nbc + bc)) < p_block) blocks[nb++] = (int32_t)bc;
        for (int lr = 0; lr < 8; ++lr) {
            const int64_t row = br * 8 + lr;
            if (row >= re) break;
            for (int64_t i = 0; i < nb; ++i) {
                const int64_t blk = br * nbc + blocks[i];
                for (int lc = 0; lc < 4; ++lc) {
                    const int64_t c = (int64_t)blocks[i] * 4 + lc;
                    const uint64_t cell = (uint64_t)(blk * 32 + lr * 4 + lc);
                    if (c >= n || !(u01(k[1], cell) < p_entry)) continue;
                    if (row_ptr) {
                        col[nnz] = (int32_t)c;
                        val[nnz] = bs_value(k, outlier_fraction, cell);
                    }
                    ++nnz;
                }
            }
            if (row_ptr) row_ptr[row - rb + 1] = nnz;
        }
    }
    free(blocks);
    return nnz;
}

static int cmp_u64(const void* a, const void* b) {
    const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return (x > y) - (x < y);
}

/* R-MAT graph: 2^scale rows, edge_factor * 2^scale edge draws; draw e picks
 * one quadrant per level l from U(stream l + 1, e) against (a, a + b,
 * a + b + c) and takes the value float(1 - U(stream 0, e)); duplicates are
 * merged by float summation in draw order.  Null row_ptr counts only. */
OC_EXPORT int64_t oc_rmat(int32_t scale, int32_t edge_factor, double a, double b, double c, uint64_t seed,
                          int64_t* row_ptr, int32_t* col, float* val) {
    const int64_t n = (int64_t)1 << scale;
    const int64_t E = (int64_t)edge_factor << scale;
    int32_t* er = (int32_t*)malloc((size_t)E * sizeof(int32_t));
    int32_t* ec = (int32_t*)malloc((size_t)E * sizeof(int32_t));
    float* ev = (float*)malloc((size_t)E * sizeof(float));
    int64_t* start = (int64_t*)calloc((size_t)n + 1, sizeof(int64_t));
    uint64_t* keys = (uint64_t*)malloc((size_t)(scale + 1) * sizeof(uint64_t));
    int32_t* sc = (int32_t*)malloc((size_t)E * sizeof(int32_t));
    float* sv = (float*)malloc((size_t)E * sizeof(float));
    int64_t* merged = (int64_t*)calloc((size_t)n, sizeof(int64_t));
    int64_t nnz = -1;
    if (!er || !ec || !ev || !start || !keys || !sc || !sv || !merged) goto done;
    for (int l = 0; l <= scale; ++l) keys[l] = key_of(seed, (uint64_t)l);
    const double ab = a + b, abc = a + b + c;
    for (int64_t e = 0; e < E; ++e) {
        int64_t r = 0, cc = 0;
        for (int l = 0; l < scale; ++l) {
            const double u = u01(keys[l + 1], (uint64_t)e);
            const int rbit = u < ab ? 0 : 1;
            const int cbit = (u < a || (u >= ab && u < abc)) ? 0 : 1;
            r = (r << 1) | rbit;
            cc = (cc << 1) | cbit;
        }
        er[e] = (int32_t)r;
        ec[e] = (int32_t)cc;
        ev[e] = (float)(1.0 - u01(keys[0], (uint64_t)e));
    }
    /* stable counting sort by row */
    for (int64_t e = 0; e < E; ++e) ++start[er[e] + 1];
    for (int64_t r = 0; r < n; ++r) start[r + 1] += start[r];
    {
        int64_t* pos = (int64_t*)malloc((size_t)n * sizeof(int64_t));
        if (!pos) goto done;
        memcpy(pos, start, (size_t)n * sizeof(int64_t));
        for (int64_t e = 0; e < E; ++e) {
            const int64_t p = pos[er[e]]++;
            sc[p] = ec[e];
            sv[p] = ev[e];
        }
        free(pos);
    }
    /* per row: order by (column, draw position), then sum duplicates in that order */
    {
        uint64_t* key = NULL;
        int64_t cap = 0;
        int32_t* tc = NULL;
        float* tv = NULL;
        for (int64_t r = 0; r < n; ++r) {
            const int64_t b0 = start[r], len = start[r + 1] - b0;
            if (len > cap) {
                cap = len;
                free(key);
                free(tc);
                free(tv);
                key = (uint64_t*)malloc((size_t)cap * sizeof(uint64_t));
                tc = (int32_t*)malloc((size_t)cap * sizeof(int32_t));
                tv = (float*)malloc((size_t)cap * sizeof(float));
                if (!key || !tc || !tv) { free(key); free(tc); free(tv); goto done; }
            }
            for (int64_t q = 0; q < len; ++q) key[q] = ((uint64_t)(uint32_t)sc[b0 + q] << 32) | (uint64_t)q;
            qsort(key, (size_t)len, sizeof(uint64_t), cmp_u64);
            int64_t m = 0;
            for (int64_t q = 0; q < len; ++q) {
                const int64_t src = b0 + (int64_t)(key[q] & 0xffffffffu);
                if (m > 0 && tc[m - 1] == sc[src]) {
                    tv[m - 1] += sv[src];
                } else {
                    tc[m] = sc[src];
                    tv[m] = sv[src];
                    ++m;
                }
            }
            memcpy(sc + b0, tc, (size_t)m * sizeof(int32_t));
            memcpy(sv + b0, tv, (size_t)m * sizeof(float));
            merged[r] = m;
        }
        free(key);
        free(tc);
        free(tv);
    }
    nnz = 0;
    for (int64_t r = 0; r < n; ++r) nnz += merged[r];
    if (row_ptr) {
        row_ptr[0] = 0;
        for (int64_t r = 0; r < n; ++r) {
            row_ptr[r + 1] = row_ptr[r] + merged[r];
            memcpy(col + row_ptr[r], sc + start[r], (size_t)merged[r] * sizeof(int32_t));
            memcpy(val + row_ptr[r], sv + start[r], (size_t)merged[r] * sizeof(float));
        }
    }
done:
    free(er);
    free(ec);
    free(ev);
    free(start);
    free(keys);
    free(sc);
    free(sv);
    free(merged);
    return nnz;
}
