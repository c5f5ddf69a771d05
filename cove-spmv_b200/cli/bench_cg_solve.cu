// bench_cg_solve -- CG solver comparison of the value codecs
// (structural/src/bench_cg_solve.cu): the same arguments, synthetic
// matrices, variants, CSV files and printed table, over this library's
// operators.
//
//   usage: bench_cg_solve matrix.mtx out.csv [append=0] [maxiter=5000] [seed=12345]
//     matrix may be 'synth:N:halfbw:delta' (diagonally dominant SPD) or
//     'lapl:N:halfbw:sigma' (shifted graph Laplacian SPD)
//
// Every variant runs a textbook CG with fp64 working vectors (cuBLAS) and its
// own matvec: cuSPARSE CSR in double and in float (p rounded to float, Ap
// widened back), and the BitBSR 8x4 operator with raw fp64, per-nonzero bf16,
// BFP8 and BFP8-with-outliers values (structural/operators/bitbsr_spmv_8x4.cuh
// over cove_hybrid_spmv).  b = A x_true with the exact operator and x_true ~
// N(0, 1).  Per variant (:112-163): the true relative residual
// ||b - A_exact x|| / ||b|| after every step, its floor (best value), the
// first step reaching 1e-2 / 1e-3 / 1e-6 / 1e-8, the final solution error,
// and the per-step time of the bare recurrence over max(50, min(steps, 400))
// steps (:166-197).  A run stops at 1e-12, at 1e-8, after 200 steps without a
// 1e-4 relative gain in the floor, or when p.Ap <= 0 (then "NOT SPD").
// Then mixed-precision iterative refinement (:287-351) and flexible
// Polak-Ribiere CG (:355-448): bf16 or BFP8 inner CG of k steps, exact outer
// residual, timed to a true residual of 1e-8.
#include "structural/gpu_convert.cuh"
#include "structural/gpu_value_codecs.cuh"
#include "structural/matrix_market.hpp"
#include "structural/operators/bitbsr_spmv_8x4.cuh"
#include "structural/synthetic_spd.hpp"

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <cusparse.h>
#include <thrust/device_vector.h>
#include <thrust/fill.h>
#include <thrust/transform.h>

#include <algorithm>
#include <array>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

using DVec = thrust::device_vector<double>;
using Matvec = std::function<void(const DVec& p, DVec& Ap)>;
constexpr std::array<double, 4> kTols = {1e-2, 1e-3, 1e-6, 1e-8};

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void blas_ok(cublasStatus_t s, const char* what) {
    if (s != CUBLAS_STATUS_SUCCESS) throw std::runtime_error(std::string("cuBLAS ") + what + " failed");
}
void sparse_ok(cusparseStatus_t s, const char* what) {
    if (s != CUSPARSE_STATUS_SUCCESS) throw std::runtime_error(std::string("cuSPARSE ") + what + " failed");
}
double* ptr(DVec& v) { return thrust::raw_pointer_cast(v.data()); }
const double* ptr(const DVec& v) { return thrust::raw_pointer_cast(v.data()); }

// Length-n fp64 vector operations with host-side scalars (the recurrences
// below need each dot product on the host to branch on it).
class Blas {
  public:
    explicit Blas(int n) : n_(n) { blas_ok(cublasCreate(&h_), "create"); }
    ~Blas() { cublasDestroy(h_); }
    Blas(const Blas&) = delete;
    Blas& operator=(const Blas&) = delete;
    double dot(const DVec& a, const DVec& b) {
        double r = 0.0;
        blas_ok(cublasDdot(h_, n_, ptr(a), 1, ptr(b), 1, &r), "dot");
        return r;
    }
    double nrm2(const DVec& a) {
        double r = 0.0;
        blas_ok(cublasDnrm2(h_, n_, ptr(a), 1, &r), "nrm2");
        return r;
    }
    void axpy(double a, const DVec& x, DVec& y) { blas_ok(cublasDaxpy(h_, n_, &a, ptr(x), 1, ptr(y), 1), "axpy"); }
    void scal(double a, DVec& x) { blas_ok(cublasDscal(h_, n_, &a, ptr(x), 1), "scal"); }
    void copy(const DVec& x, DVec& y) { blas_ok(cublasDcopy(h_, n_, ptr(x), 1, ptr(y), 1), "copy"); }
    // out = b - A_exact x, returns ||out||
    double residual(const Matvec& exact, const DVec& b, const DVec& x, DVec& ax, DVec& out) {
        exact(x, ax);
        copy(b, out);
        axpy(-1.0, ax, out);
        return nrm2(out);
    }

  private:
    int n_;
    cublasHandle_t h_ = nullptr;
};

class EventPair {
  public:
    EventPair() {
        cuda_ok(cudaEventCreate(&a_), "event");
        cuda_ok(cudaEventCreate(&b_), "event");
    }
    ~EventPair() {
        cudaEventDestroy(a_);
        cudaEventDestroy(b_);
    }
    void start() {
        cuda_ok(cudaDeviceSynchronize(), "synchronize");
        cuda_ok(cudaEventRecord(a_), "event");
    }
    double stop_ms() {
        cuda_ok(cudaEventRecord(b_), "event");
        cuda_ok(cudaEventSynchronize(b_), "event");
        float ms = 0.0f;
        cuda_ok(cudaEventElapsedTime(&ms, a_, b_), "event");
        return ms;
    }

  private:
    cudaEvent_t a_ = nullptr, b_ = nullptr;
};

struct Problem {
    int n = 0;
    Matvec exact;
    DVec b, x_true;
    double bnorm = 0.0, xtnorm = 0.0;
};

struct Curve {
    std::string variant;
    double bytes_per_nnz = 0.0;
    bool spd_ok = true;
    int total_iters = 0;
    double floor = 1.0, sol_err = 1.0, ms_per_iter = 0.0;
    std::array<int, 4> iters_to_tol{{-1, -1, -1, -1}};
    double time_to(std::size_t t) const {
        return iters_to_tol[t] > 0 ? iters_to_tol[t] * ms_per_iter : -1.0;
    }
};

// Untimed CG with `mv`, tracking the true residual after every step.
Curve cg_curve(Blas& blas, const Problem& pb, const Matvec& mv, int maxiter, const std::string& name, double bpn) {
    Curve c;
    c.variant = name;
    c.bytes_per_nnz = bpn;
    const int n = pb.n;
    DVec x(n, 0.0), r(pb.b), p(pb.b), ap(n, 0.0), ax(n, 0.0), t(n, 0.0);
    double rs = blas.dot(r, r), best = 1.0, last_gain = 2.0;
    int stale = 0;
    for (int k = 1; k <= maxiter; ++k) {
        mv(p, ap);
        const double pap = blas.dot(p, ap);
        if (!(pap > 0.0)) {
            c.spd_ok = false;
            c.total_iters = k - 1;
            c.floor = best;
            return c;
        }
        const double alpha = rs / pap;
        blas.axpy(alpha, p, x);
        blas.axpy(-alpha, ap, r);
        const double rel = blas.residual(pb.exact, pb.b, x, ax, t) / (pb.bnorm + 1e-300);
        best = std::min(best, rel);
        for (std::size_t i = 0; i < kTols.size(); ++i)
            if (c.iters_to_tol[i] < 0 && rel <= kTols[i]) c.iters_to_tol[i] = k;
        c.total_iters = k;
        if (best < last_gain * (1.0 - 1e-4)) {
            last_gain = best;
            stale = 0;
        } else {
            ++stale;
        }
        if (rel <= 1e-12 || c.iters_to_tol.back() > 0 || stale > 200) break;
        const double rs_next = blas.dot(r, r);
        blas.scal(rs_next / rs, p);
        blas.axpy(1.0, r, p);
        rs = rs_next;
    }
    c.floor = best;
    blas.copy(x, t);
    blas.axpy(-1.0, pb.x_true, t);
    c.sol_err = blas.nrm2(t) / (pb.xtnorm + 1e-300);
    return c;
}

// The bare recurrence for `iters` steps, device time per step.
double cg_step_ms(Blas& blas, const Problem& pb, const Matvec& mv, int iters) {
    if (iters <= 0) return 0.0;
    const int n = pb.n;
    DVec x(n, 0.0), r(pb.b), p(pb.b), ap(n, 0.0);
    double rs = blas.dot(r, r);
    EventPair ev;
    ev.start();
    for (int k = 0; k < iters; ++k) {
        mv(p, ap);
        const double pap = blas.dot(p, ap);
        const double alpha = pap != 0.0 ? rs / pap : 0.0;
        blas.axpy(alpha, p, x);
        blas.axpy(-alpha, ap, r);
        const double rs_next = blas.dot(r, r);
        blas.scal(rs != 0.0 ? rs_next / rs : 0.0, p);
        blas.axpy(1.0, r, p);
        rs = rs_next;
    }
    return ev.stop_ms() / iters;
}

struct Solve {
    std::string name;
    double time_ms = 0.0, final_relres = 1.0;
    int outer = 0, inner_total = 0;
    bool reached = false;
};

// Up to k steps of CG on A d = rhs from d = 0 with `mv`, stopping early when
// p.Ap is not positive; returns the steps taken.
struct InnerCg {
    DVec ri, p, ap;
    explicit InnerCg(int n) : ri(n, 0.0), p(n, 0.0), ap(n, 0.0) {}
    int run(Blas& blas, const Matvec& mv, const DVec& rhs, DVec& d, int k) {
        thrust::fill(d.begin(), d.end(), 0.0);
        blas.copy(rhs, ri);
        blas.copy(rhs, p);
        double rs = blas.dot(ri, ri);
        int steps = 0;
        for (; steps < k; ++steps) {
            mv(p, ap);
            const double pap = blas.dot(p, ap);
            if (!(pap > 0.0)) break;
            const double a = rs / pap;
            blas.axpy(a, p, d);
            blas.axpy(-a, ap, ri);
            const double rs_next = blas.dot(ri, ri);
            blas.scal(rs_next / rs, p);
            blas.axpy(1.0, ri, p);
            rs = rs_next;
        }
        return steps;
    }
};

// Iterative refinement: x += (k inner steps on A d = r), r = b - A_exact x.
Solve refine(Blas& blas, const Problem& pb, const Matvec& inner, double tol, int k, int max_outer, std::string name) {
    Solve s;
    s.name = std::move(name);
    const int n = pb.n;
    DVec x(n, 0.0), r(pb.b), d(n, 0.0), ax(n, 0.0);
    InnerCg cg(n);
    EventPair ev;
    ev.start();
    for (s.outer = 0; s.outer < max_outer; ++s.outer) {
        if (blas.nrm2(r) / pb.bnorm < tol) break;
        s.inner_total += cg.run(blas, inner, r, d, k);
        blas.axpy(1.0, d, x);
        blas.residual(pb.exact, pb.b, x, ax, r);
    }
    s.time_ms = ev.stop_ms();
    s.final_relres = blas.nrm2(r) / pb.bnorm;
    s.reached = s.final_relres <= tol;
    return s;
}

// Flexible CG: exact outer matvec, preconditioner z = (k inner steps) r,
// beta = max(0, (r'.z' - r'.z) / (r.z)).
Solve flexible_cg(Blas& blas, const Problem& pb, const Matvec& inner, double tol, int k, int max_outer,
                  std::string name) {
    Solve s;
    s.name = std::move(name);
    const int n = pb.n;
    DVec x(n, 0.0), r(pb.b), z(n, 0.0), p(n, 0.0), ap(n, 0.0), r_next(n, 0.0), z_next(n, 0.0);
    InnerCg cg(n);
    EventPair ev;
    ev.start();
    s.inner_total += cg.run(blas, inner, r, z, k);
    blas.copy(z, p);
    double rz = blas.dot(r, z);
    for (s.outer = 0; s.outer < max_outer; ++s.outer) {
        pb.exact(p, ap);
        const double pap = blas.dot(p, ap);
        if (!(pap > 0.0)) break;
        const double a = rz / pap;
        blas.axpy(a, p, x);
        blas.copy(r, r_next);
        blas.axpy(-a, ap, r_next);
        if (blas.nrm2(r_next) / pb.bnorm < tol) {
            ++s.outer;
            break;
        }
        s.inner_total += cg.run(blas, inner, r_next, z_next, k);
        const double rz_next = blas.dot(r_next, z_next);
        const double beta = std::max(0.0, (rz_next - blas.dot(r_next, z)) / rz);
        blas.scal(beta, p);
        blas.axpy(1.0, z_next, p);
        rz = rz_next;
        blas.copy(r_next, r);
        blas.copy(z_next, z);
    }
    s.time_ms = ev.stop_ms();
    s.final_relres = blas.residual(pb.exact, pb.b, x, ap, r_next) / pb.bnorm;
    s.reached = s.final_relres <= tol;
    return s;
}

struct Narrow {
    __host__ __device__ float operator()(double v) const { return static_cast<float>(v); }
};
struct Widen {
    __host__ __device__ double operator()(float v) const { return static_cast<double>(v); }
};

// cuSPARSE CSR SpMV of the loaded matrix, in double or in float.
class CusparseCsr {
  public:
    CusparseCsr(const structural::CsrMatrix<double>& a)
        : n_(a.rows), rp_(a.row_ptr), ci_(a.col_idx), vd_(a.values),
          vf_(std::vector<float>(a.values.begin(), a.values.end())), pf_(a.rows, 0.0f), yf_(a.rows, 0.0f) {
        sparse_ok(cusparseCreate(&h_), "create");
        make(md_, ptr(vd_), CUDA_R_64F);
        make(mf_, thrust::raw_pointer_cast(vf_.data()), CUDA_R_32F);
        static double dummy = 0.0;
        sparse_ok(cusparseCreateDnVec(&xd_, n_, &dummy, CUDA_R_64F), "vector");
        sparse_ok(cusparseCreateDnVec(&yd_, n_, &dummy, CUDA_R_64F), "vector");
        sparse_ok(cusparseCreateDnVec(&xf_, n_, thrust::raw_pointer_cast(pf_.data()), CUDA_R_32F), "vector");
        sparse_ok(cusparseCreateDnVec(&yf_desc_, n_, thrust::raw_pointer_cast(yf_.data()), CUDA_R_32F), "vector");
        const double one = 1.0, zero = 0.0;
        const float onef = 1.0f, zerof = 0.0f;
        size_t bd = 0, bf = 0;
        sparse_ok(cusparseSpMV_bufferSize(h_, CUSPARSE_OPERATION_NON_TRANSPOSE, &one, md_, xd_, &zero, yd_,
                                          CUDA_R_64F, CUSPARSE_SPMV_ALG_DEFAULT, &bd), "buffer size");
        sparse_ok(cusparseSpMV_bufferSize(h_, CUSPARSE_OPERATION_NON_TRANSPOSE, &onef, mf_, xf_, &zerof, yf_desc_,
                                          CUDA_R_32F, CUSPARSE_SPMV_ALG_DEFAULT, &bf), "buffer size");
        bufd_.resize(std::max<size_t>(bd, 1));
        buff_.resize(std::max<size_t>(bf, 1));
    }
    ~CusparseCsr() {
        cusparseDestroyDnVec(yf_desc_);
        cusparseDestroyDnVec(xf_);
        cusparseDestroyDnVec(yd_);
        cusparseDestroyDnVec(xd_);
        cusparseDestroySpMat(mf_);
        cusparseDestroySpMat(md_);
        cusparseDestroy(h_);
    }
    CusparseCsr(const CusparseCsr&) = delete;
    CusparseCsr& operator=(const CusparseCsr&) = delete;

    void apply_double(const DVec& p, DVec& ap) {
        ap.resize(n_);
        const double one = 1.0, zero = 0.0;
        sparse_ok(cusparseDnVecSetValues(xd_, const_cast<double*>(ptr(p))), "set x");
        sparse_ok(cusparseDnVecSetValues(yd_, ptr(ap)), "set y");
        sparse_ok(cusparseSpMV(h_, CUSPARSE_OPERATION_NON_TRANSPOSE, &one, md_, xd_, &zero, yd_, CUDA_R_64F,
                               CUSPARSE_SPMV_ALG_DEFAULT, thrust::raw_pointer_cast(bufd_.data())), "SpMV");
    }
    void apply_float(const DVec& p, DVec& ap) {
        ap.resize(n_);
        const float one = 1.0f, zero = 0.0f;
        thrust::transform(p.begin(), p.end(), pf_.begin(), Narrow());
        sparse_ok(cusparseSpMV(h_, CUSPARSE_OPERATION_NON_TRANSPOSE, &one, mf_, xf_, &zero, yf_desc_, CUDA_R_32F,
                               CUSPARSE_SPMV_ALG_DEFAULT, thrust::raw_pointer_cast(buff_.data())), "SpMV");
        thrust::transform(yf_.begin(), yf_.end(), ap.begin(), Widen());
    }

  private:
    void make(cusparseSpMatDescr_t& m, void* values, cudaDataType t) {
        sparse_ok(cusparseCreateCsr(&m, n_, n_, static_cast<int64_t>(ci_.size()), thrust::raw_pointer_cast(rp_.data()),
                                    thrust::raw_pointer_cast(ci_.data()), values, CUSPARSE_INDEX_32I,
                                    CUSPARSE_INDEX_32I, CUSPARSE_INDEX_BASE_ZERO, t),
                  "create CSR");
    }
    int n_;
    thrust::device_vector<structural::Offset> rp_;
    thrust::device_vector<structural::Index> ci_;
    DVec vd_;
    thrust::device_vector<float> vf_, pf_, yf_;
    thrust::device_vector<std::uint8_t> bufd_, buff_;
    cusparseHandle_t h_ = nullptr;
    cusparseSpMatDescr_t md_ = nullptr, mf_ = nullptr;
    cusparseDnVecDescr_t xd_ = nullptr, yd_ = nullptr, xf_ = nullptr, yf_desc_ = nullptr;
};

// 'synth:N:halfbw:delta', 'lapl:N:halfbw:sigma' or a MatrixMarket path; the
// name the reports use.
structural::CsrMatrix<double> load(const std::string& spec, unsigned seed, std::string& name) {
    char buf[96];
    if (spec.rfind("synth:", 0) == 0) {
        long n = 400000, bw = 32;
        double delta = 1.0;
        std::sscanf(spec.c_str() + 6, "%ld:%ld:%lf", &n, &bw, &delta);
        std::snprintf(buf, sizeof buf, "synth_n%ld_bw%ld_d%.3g", n, bw, delta);
        name = buf;
        return structural::make_synthetic_spd(static_cast<int>(n), static_cast<int>(bw), seed, delta);
    }
    if (spec.rfind("lapl:", 0) == 0) {
        long n = 400000, bw = 32;
        double sigma = 0.01;
        std::sscanf(spec.c_str() + 5, "%ld:%ld:%lf", &n, &bw, &sigma);
        std::snprintf(buf, sizeof buf, "lapl_n%ld_bw%ld_s%.4g", n, bw, sigma);
        name = buf;
        return structural::make_synthetic_laplacian_spd(static_cast<int>(n), static_cast<int>(bw), seed, sigma);
    }
    name = spec.substr(spec.find_last_of('/') == std::string::npos ? 0 : spec.find_last_of('/') + 1);
    if (name.size() > 4 && name.compare(name.size() - 4, 4, ".mtx") == 0) name.resize(name.size() - 4);
    return structural::read_matrix_market<double>(spec);
}

int run(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr,
                     "usage: %s matrix.mtx out.csv [append=0] [maxiter=5000] [seed=12345]\n"
                     "  matrix may be 'synth:N:halfbw:delta' (diag-dominant SPD) or\n"
                     "  'lapl:N:halfbw:sigma' (shifted-Laplacian SPD, spread spectrum)\n",
                     argv[0]);
        return 2;
    }
    const std::string spec = argv[1], csv_path = argv[2];
    const bool append = argc > 3 && std::atoi(argv[3]) != 0;
    const int maxiter = argc > 4 ? std::atoi(argv[4]) : 5000;
    const unsigned seed = argc > 5 ? static_cast<unsigned>(std::strtoul(argv[5], nullptr, 10)) : 12345u;

    std::string mname;
    const auto csr = load(spec, seed, mname);
    if (csr.rows != csr.cols) {
        std::fprintf(stderr, "%s not square -> CG N/A\n", mname.c_str());
        return 0;
    }
    const int n = csr.rows;
    structural::GpuBitBsrWorkspace<double> ws;
    structural::DeviceBitBsrMatrix<double> dev;
    structural::convert_to_bitbsr_gpu_warp_direct_8x4_device(csr, ws, dev);
    const auto host = dev.to_host();
    thrust::device_vector<std::uint64_t> words;
    structural::make_bitbsr_8x4_col_bitmap_packed(dev, words);
    structural::BitBsrLoadBalanceLayout8x4 lb;
    structural::make_bitbsr_8x4_col_bitmap_flag_load_balance_work_items(dev, lb, 32, 32, words);
    const double nnz = static_cast<double>(dev.nnz);

    const auto bfp8 = structural::build_checked_bfp8_blkscale_value_codec(host);
    const auto outl = structural::build_checked_bfp8_outlier_blkscale_value_codec(host, 0.005);
    const auto bf16 = structural::build_checked_bf16_nnz_value_codec(host);
    const thrust::device_vector<signed char> q8(bfp8.int8_values.begin(), bfp8.int8_values.end());
    const thrust::device_vector<std::uint16_t> s8(bfp8.block_scale_bf16.begin(), bfp8.block_scale_bf16.end());
    const thrust::device_vector<signed char> q8o(outl.int8_values.begin(), outl.int8_values.end());
    const thrust::device_vector<std::uint16_t> s8o(outl.block_scale_bf16.begin(), outl.block_scale_bf16.end());
    const thrust::device_vector<std::int32_t> orow(outl.outlier_rows.begin(), outl.outlier_rows.end());
    const thrust::device_vector<std::int32_t> ocol(outl.outlier_cols.begin(), outl.outlier_cols.end());
    const DVec oval(outl.outlier_vals.begin(), outl.outlier_vals.end());
    const thrust::device_vector<std::uint16_t> v16(bf16.values16.begin(), bf16.values16.end());

    CusparseCsr cusp(csr);
    Blas blas(n);
    const Matvec mv_cusp_d = [&](const DVec& p, DVec& ap) { cusp.apply_double(p, ap); };
    const Matvec mv_cusp_f = [&](const DVec& p, DVec& ap) { cusp.apply_float(p, ap); };
    const Matvec mv_exact = [&](const DVec& p, DVec& ap) {
        structural::spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_device(dev, words, lb, p, ap);
    };
    const Matvec mv_bf16 = [&](const DVec& p, DVec& ap) {
        structural::spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_round16_nnz_device<true>(
            dev, words, lb, v16, "bf16_nnz", p, ap);
    };
    const Matvec mv_bfp8 = [&](const DVec& p, DVec& ap) {
        structural::spmv_bitbsr_gpu_8x4_col_bitmap_packed_flag_load_balance_bfp8_blkscale_device(dev, words, lb, q8,
                                                                                               s8, p, ap);
    };
    const Matvec mv_outl = [&](const DVec& p, DVec& ap) {
        structural::spmv_bitbsr_gpu_8x4_bfp8_outlier_flag_load_balance_device(dev, words, lb, q8o, s8o, orow, ocol,
                                                                              oval, p, ap);
    };

    Problem pb;
    pb.n = n;
    pb.exact = mv_exact;
    const auto xt = structural::synthetic_solution(n, seed);
    pb.x_true.assign(xt.begin(), xt.end());
    mv_exact(pb.x_true, pb.b);
    pb.bnorm = blas.nrm2(pb.b);
    pb.xtnorm = blas.nrm2(pb.x_true);

    struct Variant {
        const char* name;
        const Matvec* mv;
        double bpn;
    };
    const Variant variants[] = {{"cusparse_double", &mv_cusp_d, 8.0},
                                {"cusparse_float", &mv_cusp_f, 4.0},
                                {"cove_lossless", &mv_exact, 8.0},
                                {"cove_bf16", &mv_bf16, bf16.payload_bytes() / nnz},
                                {"cove_bfp8", &mv_bfp8, bfp8.payload_bytes() / nnz},
                                {"cove_bfp8_outlier", &mv_outl, outl.payload_bytes() / nnz}};
    std::vector<Curve> curves;
    for (const auto& v : variants) {
        Curve c = cg_curve(blas, pb, *v.mv, maxiter, v.name, v.bpn);
        c.ms_per_iter = cg_step_ms(blas, pb, *v.mv, std::max(50, std::min(c.total_iters, 400)));
        curves.push_back(c);
    }

    FILE* f = std::fopen(csv_path.c_str(), append ? "a" : "w");
    if (!f) {
        std::fprintf(stderr, "cannot open %s\n", csv_path.c_str());
        return 1;
    }
    if (!append)
        std::fprintf(f, "matrix,n,nnz,variant,bytes_per_nnz,spd_ok,ms_per_iter,floor,sol_err,"
                        "iter_1e-2,iter_1e-3,iter_1e-6,iter_1e-8,total_iters,time_1e-3_ms,time_1e-6_ms\n");
    for (const auto& c : curves)
        std::fprintf(f, "%s,%d,%lld,%s,%.4f,%d,%.6f,%.3e,%.3e,%d,%d,%d,%d,%d,%.4f,%.4f\n", mname.c_str(), n,
                     static_cast<long long>(dev.nnz), c.variant.c_str(), c.bytes_per_nnz, c.spd_ok ? 1 : 0,
                     c.ms_per_iter, c.floor, c.sol_err, c.iters_to_tol[0], c.iters_to_tol[1], c.iters_to_tol[2],
                     c.iters_to_tol[3], c.total_iters, c.time_to(1), c.time_to(2));
    std::fclose(f);

    std::printf("== %-14s n=%d nnz=%lld | b=A*x_true seed=%u maxiter=%d ==\n", mname.c_str(), n,
                static_cast<long long>(dev.nnz), seed, maxiter);
    std::printf("  %-18s %6s %8s %10s | iters@[1e-2 1e-3 1e-6 1e-8] | t@1e-3 t@1e-6(ms)\n", "variant", "B/nnz",
                "ms/iter", "floor");
    for (const auto& c : curves) {
        if (!c.spd_ok) {
            std::printf("  %-18s  NOT SPD (p^T A p<=0 at iter %d)\n", c.variant.c_str(), c.total_iters);
            continue;
        }
        std::printf("  %-18s %6.2f %8.4f %10.2e | %6d %6d %6d %6d | %7.2f %7.2f\n", c.variant.c_str(),
                    c.bytes_per_nnz, c.ms_per_iter, c.floor, c.iters_to_tol[0], c.iters_to_tol[1], c.iters_to_tol[2],
                    c.iters_to_tol[3], c.time_to(1), c.time_to(2));
    }

    // mixed precision: low-precision inner solves, exact outer residual
    const double base6 = curves[0].time_to(2), base8 = curves[0].time_to(3);  // cusparse_double
    const double tol = 1e-8;
    std::vector<Solve> solves;
    for (int k : {20, 40, 80}) solves.push_back(refine(blas, pb, mv_bf16, tol, k, 600, "ir_bf16_k" + std::to_string(k)));
    for (int k : {5, 10, 20, 40})
        solves.push_back(flexible_cg(blas, pb, mv_bf16, tol, k, 2000, "fcg_bf16_k" + std::to_string(k)));
    for (int k : {5, 10})
        solves.push_back(flexible_cg(blas, pb, mv_bfp8, tol, k, 2000, "fcg_bfp8_k" + std::to_string(k)));
    const auto speedup = [&](const Solve& s) { return base8 > 0 && s.time_ms > 0 ? base8 / s.time_ms : -1.0; };
    std::printf("  --- IR vs FCG (target true relres %.0e) | baseline double: t@1e-6=%.2f t@1e-8=%.2fms ---\n", tol,
                base6, base8);
    for (const auto& s : solves)
        std::printf("  %-14s outer=%4d inner=%5d final=%9.2e %s | time=%8.2fms  speedup@1e-8 vs double=%.2fx\n",
                    s.name.c_str(), s.outer, s.inner_total, s.final_relres, s.reached ? "OK" : "NO", s.time_ms,
                    speedup(s));

    std::string ir_csv = csv_path;
    if (ir_csv.size() > 4 && ir_csv.compare(ir_csv.size() - 4, 4, ".csv") == 0) ir_csv.resize(ir_csv.size() - 4);
    ir_csv += "_ir.csv";
    if (FILE* fi = std::fopen(ir_csv.c_str(), append ? "a" : "w")) {
        if (!append)
            std::fprintf(fi, "matrix,n,nnz,solver,outer,inner_total,final_relres,reached,"
                             "time_ms,base_double_t1e8_ms,speedup_1e8\n");
        for (const auto& s : solves)
            std::fprintf(fi, "%s,%d,%lld,%s,%d,%d,%.3e,%d,%.4f,%.4f,%.4f\n", mname.c_str(), n,
                         static_cast<long long>(dev.nnz), s.name.c_str(), s.outer, s.inner_total, s.final_relres,
                         s.reached ? 1 : 0, s.time_ms, base8, speedup(s));
        std::fclose(fi);
    }
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        return run(argc, argv);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
}
