// cg.cu -- textbook CG over the fused SpMV, on one GPU or a row-block
// partition across GPUs (one process per GPU, NCCL over NVLink).
//
// Recurrence of the reference's timed CG (structural/src/bench_cg_solve.cu:
// 165-197): x0 = 0, r = p = b, rs = r.r; per iteration Ap = A p,
// alpha = rs / (p.Ap) (0 if p.Ap == 0), x += alpha p, r -= alpha Ap,
// rs' = r.r, beta = rs'/rs (0 if rs == 0), p = r + beta p.
//
// B200 layout: alpha and beta never leave the device (the reference reads
// every dot product back to the host, two syncs per iteration).  Dots are
// two-stage deterministic reductions (fixed grid, per-CTA partials, one
// final CTA).  On a partition each dot's partial sum is allreduced with
// ncclAllReduce on the compute stream, and the SpMV's x window gets its halo
// with ncclSend/ncclRecv from the neighbouring ranks first.
#include "cove_plan.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

namespace cove {
namespace {

constexpr int kThreads = 256;
constexpr int kDotCtas = 148 * 4;

// ---- textbook CG vector passes ---------------------------------------------------
// Each pass streams n-vectors once with 16-byte loads (kU independent pairs
// in flight per thread) over the fixed kDotCtas x kThreads grid; the dot
// partials of a pass are one per CTA in a fixed order, so every sum is
// deterministic.  Vectors that are not 16-byte aligned take the scalar path.

constexpr int kU = 4;
constexpr int kVecCtasPerSm = kDotCtas / 148;  // the whole grid resident at once

__device__ __forceinline__ bool al16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// the CTA's sum of s into partial[blockIdx.x]
__device__ __forceinline__ void cta_partial(double s, double* __restrict__ partial) {
    __shared__ double sh[kThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < kThreads / 32; ++w) t += sh[w];
        partial[blockIdx.x] = t;
    }
}

// Visit every index of [0, n) once over the grid: with 16-byte aligned
// vectors f2(j, nt) takes the U pairs j, j + nt, ... (pair j = elements 2j,
// 2j + 1), the leftovers go elementwise to f1(i), as does everything when
// the vectors are not aligned.
template <int U, typename F2, typename F1>
__device__ __forceinline__ void stream_pairs(int64_t n, bool vec, F2 f2, F1 f1) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nt = static_cast<int64_t>(gridDim.x) * blockDim.x;
    if (vec) {
        const int64_t n2 = n >> 1;
        int64_t j = tid;
        for (; j + (U - 1) * nt < n2; j += U * nt) f2(j, nt);
        for (; j < n2; j += nt) f1(2 * j), f1(2 * j + 1);
        if ((n & 1) && tid == 0) f1(n - 1);
    } else {
        for (int64_t i = tid; i < n; i += nt) f1(i);
    }
}

// partial sums of a . b; partial[blockIdx.x]
__global__ void __launch_bounds__(kThreads, kVecCtasPerSm)
dot_partial_kernel(int64_t n, const double* __restrict__ a, const double* __restrict__ b,
                   double* __restrict__ partial) {
    double s = 0.0;
    const double2* a2 = reinterpret_cast<const double2*>(a);
    const double2* b2 = reinterpret_cast<const double2*>(b);
    stream_pairs<kU>(
        n, al16(a) && al16(b),
        [&](int64_t j, int64_t nt) {
            double2 va[kU], vb[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                va[u] = a2[j + u * nt];
                vb[u] = b2[j + u * nt];
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                s += va[u].x * vb[u].x;
                s += va[u].y * vb[u].y;
            }
        },
        [&](int64_t i) { s += a[i] * b[i]; });
    cta_partial(s, partial);
}

__global__ void dot_final_kernel(const double* __restrict__ partial, int m,
                                 double* __restrict__ out) {
    __shared__ double sh[kThreads];
    double s = 0.0;
    for (int i = threadIdx.x; i < m; i += blockDim.x) s += partial[i];
    sh[threadIdx.x] = s;
    __syncthreads();
    for (int o = kThreads / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) *out = sh[0];
}

__device__ __forceinline__ double cg_alpha(const double* __restrict__ scal, int rs_slot) {
    const double pap = scal[2];
    return pap != 0.0 ? scal[rs_slot] / pap : 0.0;
}

// r -= alpha Ap and the partials of the new r.r   (alpha = rs / pAp on device)
__global__ void __launch_bounds__(kThreads, kVecCtasPerSm)
cg_r_kernel(int64_t n, const double* __restrict__ scal, int rs_slot, const double* __restrict__ ap,
            double* __restrict__ r, double* __restrict__ partial) {
    const double alpha = cg_alpha(scal, rs_slot);
    double s = 0.0;
    const double2* ap2 = reinterpret_cast<const double2*>(ap);
    double2* r2 = reinterpret_cast<double2*>(r);
    stream_pairs<kU>(
        n, al16(ap) && al16(r),
        [&](int64_t j, int64_t nt) {
            double2 va[kU], vr[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                va[u] = ap2[j + u * nt];
                vr[u] = r2[j + u * nt];
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                vr[u].x -= alpha * va[u].x;
                vr[u].y -= alpha * va[u].y;
                r2[j + u * nt] = vr[u];
                s += vr[u].x * vr[u].x;
                s += vr[u].y * vr[u].y;
            }
        },
        [&](int64_t i) {
            const double ri = r[i] - alpha * ap[i];
            r[i] = ri;
            s += ri * ri;
        });
    cta_partial(s, partial);
}

// x += alpha p (the p of this iteration), then p = r + beta p with
// beta = rs_new / rs: the iteration's x update and the next direction in one
// pass over x, p and r
__global__ void __launch_bounds__(kThreads, kVecCtasPerSm)
cg_xp_kernel(int64_t n, const double* __restrict__ scal, int rs_slot, int new_slot,
             const double* __restrict__ r, double* __restrict__ p, double* __restrict__ x) {
    const double alpha = cg_alpha(scal, rs_slot);
    const double rs = scal[rs_slot];
    const double beta = rs != 0.0 ? scal[new_slot] / rs : 0.0;
    const double2* r2 = reinterpret_cast<const double2*>(r);
    double2* p2 = reinterpret_cast<double2*>(p);
    double2* x2 = reinterpret_cast<double2*>(x);
    constexpr int U = kU / 2;  // three streams: fewer pairs in flight keep it in 64 registers
    stream_pairs<U>(
        n, al16(r) && al16(p) && al16(x),
        [&](int64_t j, int64_t nt) {
            double2 vr[U], vp[U], vx[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                vp[u] = p2[j + u * nt];
                vx[u] = x2[j + u * nt];
                vr[u] = r2[j + u * nt];
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                vx[u].x += alpha * vp[u].x;
                vx[u].y += alpha * vp[u].y;
                x2[j + u * nt] = vx[u];
                vp[u].x = vr[u].x + beta * vp[u].x;
                vp[u].y = vr[u].y + beta * vp[u].y;
                p2[j + u * nt] = vp[u];
            }
        },
        [&](int64_t i) {
            const double pi = p[i];
            x[i] += alpha * pi;
            p[i] = r[i] + beta * pi;
        });
}


// ---- mixed-precision solver kernels (IR / flexible CG) --------------------------
// Scalar slots: [0], [1] inner r.r (alternating), [2] p.Ap, [3] outer r.r,
// [4] ||b||^2, [6] inner stop flag, [7] inner iterations run, [8] r.z,
// [9] rn.zn, [10] rn.z, [11] outer p.Ap.

// Inner bounded CG step (bench_cg_solve.cu:311-330): stop for good once
// p.Ap is not positive; else d += alpha p, ri -= alpha Ap and the ri.ri
// partials.  Every CTA takes the same decision from the same scalars.
__global__ void ir_update_kernel(int64_t n, double* __restrict__ scal, int rs_slot,
                                 const double* __restrict__ p, const double* __restrict__ ap,
                                 double* __restrict__ d, double* __restrict__ ri,
                                 double* __restrict__ partial) {
    const double pap = scal[2];
    const bool stop = scal[6] != 0.0 || !(pap > 0.0);
    const double alpha = stop ? 0.0 : scal[rs_slot] / pap;
    double s = 0.0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        if (!stop) {
            d[i] += alpha * p[i];
            ri[i] -= alpha * ap[i];
        }
        s += ri[i] * ri[i];
    }
    __shared__ double sh[kThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < kThreads / 32; ++w) t += sh[w];
        partial[blockIdx.x] = t;
        if (blockIdx.x == 0) {
            scal[6] = stop ? 1.0 : 0.0;
            if (!stop) scal[7] += 1.0;
        }
    }
}

// p = ri + (rs'/rs) p unless the inner solve has stopped
__global__ void ir_p_kernel(int64_t n, const double* __restrict__ scal, int rs_slot, int new_slot,
                            const double* __restrict__ ri, double* __restrict__ p) {
    if (scal[6] != 0.0) return;
    const double rs = scal[rs_slot];
    const double beta = rs != 0.0 ? scal[new_slot] / rs : 0.0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        p[i] = ri[i] + beta * p[i];
}

// y = a + s * b   (s = +1 / -1)
__global__ void axpy_kernel(int64_t n, const double* __restrict__ a, double s,
                            const double* __restrict__ b, double* __restrict__ y) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = a[i] + s * b[i];
}

// flexible CG outer step: alpha = rz / pAp (0 if pAp <= 0), x += alpha p,
// rn = r - alpha Ap, rn.rn partials
__global__ void fcg_update_kernel(int64_t n, const double* __restrict__ scal,
                                  const double* __restrict__ p, const double* __restrict__ ap,
                                  const double* __restrict__ r, double* __restrict__ x,
                                  double* __restrict__ rn, double* __restrict__ partial) {
    const double pap = scal[11];
    const double alpha = pap > 0.0 ? scal[8] / pap : 0.0;
    double s = 0.0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        x[i] += alpha * p[i];
        const double v = r[i] - alpha * ap[i];
        rn[i] = v;
        s += v * v;
    }
    __shared__ double sh[kThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < kThreads / 32; ++w) t += sh[w];
        partial[blockIdx.x] = t;
    }
}

// flexible Polak-Ribiere: beta = max(0, (rn.zn - rn.z) / rz); p = zn + beta p;
// then rz = rn.zn (bench_cg_solve.cu:430-436)
__global__ void fcg_p_kernel(int64_t n, double* __restrict__ scal, const double* __restrict__ zn,
                             double* __restrict__ p) {
    double beta = (scal[9] - scal[10]) / scal[8];
    if (!(beta > 0.0)) beta = 0.0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        p[i] = zn[i] + beta * p[i];
}

__global__ void fcg_rz_kernel(double* __restrict__ scal) { scal[8] = scal[9]; }

// NCCL is resolved at run time: a process that already holds libnccl.so.2
// (PyTorch loads its own) keeps using that copy, and the library itself
// never forces a second NCCL version into the process.
struct NcclApi {
    bool loaded = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
    static NcclApi api;
    if (api.loaded) return api;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) COVE_THROW(COVE_ERR_NCCL, std::string("cannot load libnccl.so.2: ") + dlerror());
    auto sym = [&](const char* name) {
        void* f = dlsym(h, name);
        if (!f) COVE_THROW(COVE_ERR_NCCL, std::string("libnccl.so.2 lacks ") + name);
        return f;
    };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRankConfig = reinterpret_cast<decltype(api.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
    api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
    api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(sym("ncclCommAbort"));
    api.CommFinalize = reinterpret_cast<decltype(api.CommFinalize)>(sym("ncclCommFinalize"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
    api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
    api.Send = reinterpret_cast<decltype(api.Send)>(sym("ncclSend"));
    api.Recv = reinterpret_cast<decltype(api.Recv)>(sym("ncclRecv"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym("ncclAllReduce"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
    api.loaded = true;
    return api;
}

inline void nccl_ok(ncclResult_t r, const char* what) {
    if (r != ncclSuccess && r != ncclInProgress) {
        COVE_THROW(COVE_ERR_NCCL, std::string(what) + ": " + nccl().GetErrorString(r));
    }
}

void wait_comm_ready(ncclComm_t comm, int timeout_ms);

}  // namespace
}  // namespace cove

using namespace cove;

struct cove_dist {
    int rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    std::vector<cove_plan*> plans;
    int64_t global_rows = 0, row_begin = 0, row_end = 0, wb = 0, wl = 0;
    cove::CgWorkspace cg_ws;  // CG work vectors, kept between solves
    int timeout_ms = 60000;
    struct Xfer {
        int peer;
        int64_t send_off, send_n, recv_off, recv_n;  // offsets into this rank's window
    };
    std::vector<Xfer> xfers;
    // Halo overlap: per plan, block-row ranges that read only the rank's own
    // columns (run while the halo is in flight on s_comm) and ranges that
    // read halo columns (run after it lands).
    struct Range {
        int32_t b0, b1;
        bool halo;
    };
    std::vector<std::vector<Range>> ranges;
    bool overlap = false;
    cudaStream_t s_comm = nullptr;
    cudaEvent_t x_ready = nullptr, halo_done = nullptr;
};

namespace cove {
namespace {

// A non-blocking communicator finishes enqueuing an operation within
// microseconds: poll tightly first (every launch after it waits for this),
// then back off so a stalled peer does not burn a core until the deadline.
void wait_comm_ready(ncclComm_t comm, int timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        ncclResult_t st = ncclSuccess;
        nccl_ok(nccl().CommGetAsyncError(comm, &st), "ncclCommGetAsyncError");
        if (st == ncclSuccess) return;
        if (st != ncclInProgress) {
            nccl().CommAbort(comm);
            COVE_THROW(COVE_ERR_NCCL, std::string("NCCL communicator error: ") + nccl().GetErrorString(st));
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) {
            nccl().CommAbort(comm);
            COVE_THROW(COVE_ERR_TIMEOUT, "NCCL communicator did not become ready in time");
        }
        if (ms < 5) {
            std::this_thread::yield();
        } else {
            std::this_thread::sleep_for(std::chrono::microseconds(100));
        }
    }
}

// Wait for the stream with a host deadline; on timeout or an asynchronous
// NCCL error the communicator is aborted so no rank waits forever.
void wait_stream(cove_dist* d, cudaStream_t s) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t q = cudaStreamQuery(s);
        if (q == cudaSuccess) return;
        if (q != cudaErrorNotReady) CUDA_OK(q);
        if (d && d->comm) {
            ncclResult_t st = ncclSuccess;
            nccl().CommGetAsyncError(d->comm, &st);
            if (st != ncclSuccess && st != ncclInProgress) {
                nccl().CommAbort(d->comm);
                d->comm = nullptr;
                COVE_THROW(COVE_ERR_NCCL, std::string("NCCL async error: ") + nccl().GetErrorString(st));
            }
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (d && ms > d->timeout_ms) {
            if (d->comm) nccl().CommAbort(d->comm);
            d->comm = nullptr;
            COVE_THROW(COVE_ERR_TIMEOUT, "stream did not finish before the deadline");
        }
        if (ms < 5) {
            std::this_thread::yield();
        } else {
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
}

void halo(cove_dist* d, double* xw, cudaStream_t s) {
    if (!d || d->world == 1 || d->xfers.empty()) return;
    nccl_ok(nccl().GroupStart(), "ncclGroupStart");
    for (const auto& x : d->xfers) {
        if (x.send_n > 0)
            nccl_ok(nccl().Send(xw + x.send_off, static_cast<size_t>(x.send_n), ncclFloat64, x.peer,
                             d->comm, s), "ncclSend");
        if (x.recv_n > 0)
            nccl_ok(nccl().Recv(xw + x.recv_off, static_cast<size_t>(x.recv_n), ncclFloat64, x.peer,
                             d->comm, s), "ncclRecv");
    }
    const ncclResult_t r = nccl().GroupEnd();
    nccl_ok(r, "ncclGroupEnd");
    if (r == ncclInProgress) wait_comm_ready(d->comm, d->timeout_ms);
}

void allreduce_scalar(cove_dist* d, double* v, cudaStream_t s) {
    if (!d || d->world == 1) return;
    const ncclResult_t r = nccl().AllReduce(v, v, 1, ncclFloat64, ncclSum, d->comm, s);
    nccl_ok(r, "ncclAllReduce");
    if (r == ncclInProgress) wait_comm_ready(d->comm, d->timeout_ms);
}

// The route a plan runs for `route` (< 0: its dispatched route).
int route_of(const cove_plan* P, int route) { return route < 0 ? P->dispatched_route : route; }

// y_local = A_local x_window over the rank's plans (consecutive row blocks);
// returns the kernel launches
int spmv_plans(const std::vector<cove_plan*>& plans, const double* xw, double* y,
               cudaStream_t s, int route = -1) {
    int64_t off = 0;
    int launches = 0;
    for (const cove_plan* P : plans) {
        launches += launch_hybrid_spmv(P->shape(), P->route_values(route_of(P, route)), xw, y + off, s);
        off += P->rows;
    }
    return launches;
}

// y_local = A_local x_window on a partition: the block rows that read only
// own columns are launched first, so the GPU computes them while the host
// enqueues the halo on the (highest-priority) comm stream.  The halo block
// rows follow the exchange on that same stream, beside the interior pass's
// remaining waves (a short launch of its own would expose one block row's
// serial load chain); the two passes write disjoint rows.  The compute
// stream joins before any overflow pass.
int spmv_dist(cove_dist* d, double* xw, double* y, cudaStream_t s, int route = -1) {
    if (!d->overlap) {
        halo(d, xw, s);
        return spmv_plans(d->plans, xw, y, s, route);
    }
    int launches = 0;
    auto launch_ranges = [&](bool halo_rows, cudaStream_t st) {
        int64_t off = 0;
        for (size_t i = 0; i < d->plans.size(); ++i) {
            const cove_plan* P = d->plans[i];
            const KernelShape k = P->shape();
            const RouteValues rv = P->route_values(route_of(P, route));
            for (const auto& r : d->ranges[i]) {
                if (r.halo != halo_rows) continue;
                KernelShape kr = k;
                kr.part = 1;
                kr.br_begin = r.b0;
                kr.nbr = r.b1;
                launches += launch_hybrid_spmv(kr, rv, xw, y + off, st);
            }
            off += P->rows;
        }
    };
    CUDA_OK(cudaEventRecord(d->x_ready, s));
    launch_ranges(false, s);
    CUDA_OK(cudaStreamWaitEvent(d->s_comm, d->x_ready, 0));
    halo(d, xw, d->s_comm);
    launch_ranges(true, d->s_comm);
    CUDA_OK(cudaEventRecord(d->halo_done, d->s_comm));
    CUDA_OK(cudaStreamWaitEvent(s, d->halo_done, 0));
    int64_t off = 0;
    for (const cove_plan* P : d->plans) {
        const KernelShape k = P->shape();
        const RouteValues rv = P->route_values(route_of(P, route));
        if (hybrid_spmv_launch_count(k, rv) > 1) {
            KernelShape ko = k;
            ko.part = 2;
            launches += launch_hybrid_spmv(ko, rv, xw, y + off, s);
        }
        off += P->rows;
    }
    return launches;
}

// Split each plan's block rows into runs that read only the rank's own
// columns [own_lo, own_hi) of the window and runs that read halo columns.
void plan_overlap(cove_dist* d) {
    d->ranges.clear();
    d->overlap = false;
    if (d->world == 1 || d->xfers.empty()) return;
    const int64_t own_lo = d->row_begin - d->wb, own_hi = d->row_end - d->wb;
    size_t runs = 0;
    bool any_interior = false;
    for (const cove_plan* P : d->plans) {
        std::vector<int32_t> lo, hi;
        block_row_col_bounds(P, &lo, &hi);
        std::vector<cove_dist::Range> rs;
        for (int32_t b = 0; b < P->nbr; ++b) {
            const bool h = hi[b] >= 0 && (lo[b] < own_lo || hi[b] >= own_hi);
            if (!rs.empty() && rs.back().halo == h) {
                rs.back().b1 = b + 1;
            } else {
                rs.push_back({b, b + 1, h});
            }
            any_interior |= !h;
        }
        runs += rs.size();
        d->ranges.push_back(std::move(rs));
    }
    // many short runs would cost more launches than the overlap saves
    if (!any_interior || runs > 16) {
        d->ranges.clear();
        return;
    }
    // NCCL's kernel on this stream should not queue behind the interior
    // pass's remaining CTAs
    int least = 0, greatest = 0;
    CUDA_OK(cudaDeviceGetStreamPriorityRange(&least, &greatest));
    CUDA_OK(cudaStreamCreateWithPriority(&d->s_comm, cudaStreamNonBlocking, greatest));
    CUDA_OK(cudaEventCreateWithFlags(&d->x_ready, cudaEventDisableTiming));
    CUDA_OK(cudaEventCreateWithFlags(&d->halo_done, cudaEventDisableTiming));
    d->overlap = true;
}

void dot(int64_t n, const double* a, const double* b, double* partial, double* out,
         cudaStream_t s) {
    dot_partial_kernel<<<kDotCtas, kThreads, 0, s>>>(n, a, b, partial);
    dot_final_kernel<<<1, kThreads, 0, s>>>(partial, kDotCtas, out);
}

// One textbook CG iteration after Ap = A p: p.Ap -> alpha; r -= alpha Ap and
// the new r.r -> beta; x += alpha p and p = r + beta p.  Scalar slots: S[cur]
// the iteration's r.r, S[cur ^ 1] the new one, S[2] p.Ap.  Ten n-vector
// passes besides the SpMV.  Returns the kernel launches.
int cg_vector_step(cove_dist* d, int64_t n, double* p, const double* ap, double* r, double* x,
                   double* partial, double* S, int cur, cudaStream_t s) {
    const int nxt = cur ^ 1;
    dot(n, p, ap, partial, S + 2, s);
    allreduce_scalar(d, S + 2, s);
    cg_r_kernel<<<kDotCtas, kThreads, 0, s>>>(n, S, cur, ap, r, partial);
    dot_final_kernel<<<1, kThreads, 0, s>>>(partial, kDotCtas, S + nxt);
    allreduce_scalar(d, S + nxt, s);
    cg_xp_kernel<<<kDotCtas, kThreads, 0, s>>>(n, S, cur, nxt, r, p, x);
    return 5;
}

// The workspace for n rows and a window of wl entries: the kept vectors when
// the sizes match (a previous solve on the same handle), else new ones.
CgWorkspace& cg_workspace(CgWorkspace& ws, int64_t n, int64_t wl) {
    if (ws.n != n || ws.wl != wl) {
        alloc_n<double>(ws.r, n);
        alloc_n<double>(ws.pw, wl);
        alloc_n<double>(ws.ap, n);
        alloc_n<double>(ws.partial, kDotCtas);
        alloc_n<double>(ws.scal, 8);
        ws.n = n;
        ws.wl = wl;
    }
    return ws;
}

void cg_run(cove_dist* d, const std::vector<cove_plan*>& plans, int64_t n_local,
            int64_t p_off, int64_t wl, const double* b, double* x, int iters,
            cove_cg_result* res, cudaStream_t s) {
    for (const cove_plan* P : plans) {
        if (P->dtype != COVE_F64) COVE_THROW(COVE_ERR_UNSUPPORTED, "CG runs in fp64");
    }
    if (res) *res = cove_cg_result{};
    if (n_local == 0 && !d) {  // nothing to solve (a partition's ranks all take the collective steps)
        if (res) res->iterations = iters;
        return;
    }
    CgWorkspace& ws = cg_workspace(d ? d->cg_ws : plans[0]->cg_ws, n_local, wl);
    DevBuf &r = ws.r, &pw = ws.pw, &ap = ws.ap, &partial = ws.partial, &scal = ws.scal;
    double* p = pw.as<double>() + p_off;
    CUDA_OK(cudaMemsetAsync(pw.p, 0, static_cast<size_t>(wl) * 8, s));
    CUDA_OK(cudaMemsetAsync(x, 0, static_cast<size_t>(n_local) * 8, s));
    CUDA_OK(cudaMemcpyAsync(r.p, b, static_cast<size_t>(n_local) * 8, cudaMemcpyDeviceToDevice, s));
    CUDA_OK(cudaMemcpyAsync(p, b, static_cast<size_t>(n_local) * 8, cudaMemcpyDeviceToDevice, s));
    double* S = scal.as<double>();
    dot(n_local, r.as<double>(), r.as<double>(), partial.as<double>(), S + 0, s);
    allreduce_scalar(d, S + 0, s);
    CUDA_LAUNCH_OK();
    wait_stream(d, s);
    double rs0 = 0.0;
    CUDA_OK(cudaMemcpy(&rs0, S, 8, cudaMemcpyDeviceToHost));
    int64_t launches = 2;

    cudaEvent_t e0, e1;
    CUDA_OK(cudaEventCreate(&e0));
    CUDA_OK(cudaEventCreate(&e1));
    std::vector<cudaEvent_t> ev(2 * static_cast<size_t>(iters));
    for (auto& e : ev) CUDA_OK(cudaEventCreate(&e));
    double spmv_ms = 0.0;
    CUDA_OK(cudaEventRecord(e0, s));
    for (int k = 0; k < iters; ++k) {
        // the distributed SpMV: halo exchange overlapped with own-column rows
        CUDA_OK(cudaEventRecord(ev[2 * k], s));
        launches += d ? spmv_dist(d, pw.as<double>(), ap.as<double>(), s)
                      : spmv_plans(plans, pw.as<double>(), ap.as<double>(), s);
        CUDA_OK(cudaEventRecord(ev[2 * k + 1], s));
        launches += cg_vector_step(d, n_local, p, ap.as<double>(), r.as<double>(), x, partial.as<double>(),
                                   S, k & 1, s);
        CUDA_LAUNCH_OK();
    }
    CUDA_OK(cudaEventRecord(e1, s));
    wait_stream(d, s);
    float total = 0.0f;
    CUDA_OK(cudaEventElapsedTime(&total, e0, e1));
    for (int k = 0; k < iters; ++k) {
        float ms = 0.0f;
        CUDA_OK(cudaEventElapsedTime(&ms, ev[2 * k], ev[2 * k + 1]));
        spmv_ms += ms;
    }
    for (auto& e : ev) cudaEventDestroy(e);
    double rsf = 0.0;
    CUDA_OK(cudaMemcpy(&rsf, S + (iters & 1), 8, cudaMemcpyDeviceToHost));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (res) {
        res->iterations = iters;
        res->rs_initial = rs0;
        res->rs_final = rsf;
        res->ms_total = total;
        res->ms_spmv = spmv_ms;
        res->launches = launches;
    }
}

// ---- mixed-precision iterative refinement and flexible CG ------------------------
// (bench_cg_solve.cu:280-448).  The outer level uses an exact (lossless)
// route, the inner bounded CG a cheaper one; both run on one plan or on a
// row-block partition (halo + allreduce as in cg_run).  Inner alpha, beta and
// the breakdown stop stay on the device; the host reads one residual norm per
// outer step.

struct MpSolver {
    cove_dist* d = nullptr;
    std::vector<cove_plan*> plans;
    int64_t n = 0, p_off = 0, wl = 0;
    int exact_route = COVE_ROUTE_HYBRID, inner_route = COVE_ROUTE_HYBRID;
    cudaStream_t s = nullptr;
    DevBuf xw, pw, r, dvec, ri, ap, z, zn, rn, partial, scal;
    int ug = 1;

    double* S() { return scal.as<double>(); }
    double* p() { return pw.as<double>() + p_off; }
    double* x() { return xw.as<double>() + p_off; }

    void setup() {
        alloc_n<double>(xw, wl);
        alloc_n<double>(pw, wl);
        for (DevBuf* b : {&r, &dvec, &ri, &ap, &z, &zn, &rn}) alloc_n<double>(*b, n);
        alloc_n<double>(partial, kDotCtas);
        alloc_n<double>(scal, 16);
        CUDA_OK(cudaMemsetAsync(xw.p, 0, static_cast<size_t>(wl) * 8, s));
        CUDA_OK(cudaMemsetAsync(pw.p, 0, static_cast<size_t>(wl) * 8, s));
        CUDA_OK(cudaMemsetAsync(scal.p, 0, 16 * 8, s));
        ug = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid_for(n, kThreads), kDotCtas)));
    }
    void matvec(int route, double* window, double* y) {
        if (d) {
            spmv_dist(d, window, y, s, route);
        } else {
            spmv_plans(plans, window, y, s, route);
        }
    }
    void dot_to(const double* a, const double* b, int slot) {
        dot(n, a, b, partial.as<double>(), S() + slot, s);
        allreduce_scalar(d, S() + slot, s);
    }
    double read(int slot) {
        double v = 0.0;
        CUDA_LAUNCH_OK();
        wait_stream(d, s);
        CUDA_OK(cudaMemcpy(&v, S() + slot, 8, cudaMemcpyDeviceToHost));
        return v;
    }
    // out ~= A^-1 rhs: k_inner steps of CG on the inner route, from out = 0
    void inner(const double* rhs, double* out, int k_inner) {
        CUDA_OK(cudaMemsetAsync(out, 0, static_cast<size_t>(n) * 8, s));
        CUDA_OK(cudaMemcpyAsync(ri.p, rhs, static_cast<size_t>(n) * 8, cudaMemcpyDeviceToDevice, s));
        CUDA_OK(cudaMemcpyAsync(p(), rhs, static_cast<size_t>(n) * 8, cudaMemcpyDeviceToDevice, s));
        CUDA_OK(cudaMemsetAsync(S() + 6, 0, 8, s));  // not stopped
        dot_to(ri.as<double>(), ri.as<double>(), 0);
        for (int j = 0; j < k_inner; ++j) {
            const int cur = j & 1, nxt = cur ^ 1;
            matvec(inner_route, pw.as<double>(), ap.as<double>());
            dot_to(p(), ap.as<double>(), 2);
            ir_update_kernel<<<kDotCtas, kThreads, 0, s>>>(n, S(), cur, p(), ap.as<double>(), out,
                                                         ri.as<double>(), partial.as<double>());
            dot_final_kernel<<<1, kThreads, 0, s>>>(partial.as<double>(), kDotCtas, S() + nxt);
            allreduce_scalar(d, S() + nxt, s);
            ir_p_kernel<<<ug, kThreads, 0, s>>>(n, S(), cur, nxt, ri.as<double>(), p());
        }
        CUDA_LAUNCH_OK();
    }
    // ||b - A_exact x||^2 into `res` (the outer residual) and slot 3
    void exact_residual(const double* b, double* res) {
        matvec(exact_route, xw.as<double>(), ap.as<double>());
        axpy_kernel<<<ug, kThreads, 0, s>>>(n, b, -1.0, ap.as<double>(), res);
        dot_to(res, res, 3);
    }
};

void mp_solve(MpSolver& m, bool flexible, const double* b, double* x_out, double tol, int k_inner,
              int max_outer, cove_ir_result* res) {
    m.setup();
    cudaEvent_t e0, e1;
    CUDA_OK(cudaEventCreate(&e0));
    CUDA_OK(cudaEventCreate(&e1));
    m.dot_to(b, b, 4);
    const double bnorm = std::sqrt(m.read(4));
    const double denom = bnorm > 0.0 ? bnorm : 1.0;
    CUDA_OK(cudaEventRecord(e0, m.s));
    int outer = 0;
    double* r = m.r.as<double>();
    if (!flexible) {
        // iterative refinement: r = b; repeat {d = inner(r); x += d; r = b - A x}
        CUDA_OK(cudaMemcpyAsync(r, b, static_cast<size_t>(m.n) * 8, cudaMemcpyDeviceToDevice, m.s));
        m.dot_to(r, r, 3);
        for (outer = 0; outer < max_outer; ++outer) {
            if (std::sqrt(m.read(3)) / denom < tol) break;
            m.inner(r, m.dvec.as<double>(), k_inner);
            axpy_kernel<<<m.ug, kThreads, 0, m.s>>>(m.n, m.x(), 1.0, m.dvec.as<double>(), m.x());
            m.exact_residual(b, r);
        }
    } else {
        // flexible CG: z = M r, p = z; per step exact Ap, x += a p, rn = r - a Ap,
        // zn = M rn, beta = max(0, (rn.zn - rn.z) / r.z), p = zn + beta p
        double* z = m.z.as<double>();
        double* zn = m.zn.as<double>();
        double* rn = m.rn.as<double>();
        CUDA_OK(cudaMemcpyAsync(r, b, static_cast<size_t>(m.n) * 8, cudaMemcpyDeviceToDevice, m.s));
        m.inner(r, z, k_inner);
        CUDA_OK(cudaMemcpyAsync(m.p(), z, static_cast<size_t>(m.n) * 8, cudaMemcpyDeviceToDevice, m.s));
        m.dot_to(r, z, 8);
        for (outer = 0; outer < max_outer; ++outer) {
            m.matvec(m.exact_route, m.pw.as<double>(), m.ap.as<double>());
            m.dot_to(m.p(), m.ap.as<double>(), 11);
            fcg_update_kernel<<<kDotCtas, kThreads, 0, m.s>>>(m.n, m.S(), m.p(), m.ap.as<double>(), r,
                                                             m.x(), rn, m.partial.as<double>());
            dot_final_kernel<<<1, kThreads, 0, m.s>>>(m.partial.as<double>(), kDotCtas, m.S() + 3);
            allreduce_scalar(m.d, m.S() + 3, m.s);
            const double pap = m.read(11);
            if (!(pap > 0.0)) break;
            if (std::sqrt(m.read(3)) / denom < tol) {
                ++outer;
                break;
            }
            // the p window is the inner solve's work vector: keep p in dvec meanwhile
            CUDA_OK(cudaMemcpyAsync(m.dvec.p, m.p(), static_cast<size_t>(m.n) * 8,
                                    cudaMemcpyDeviceToDevice, m.s));
            m.inner(rn, zn, k_inner);
            CUDA_OK(cudaMemcpyAsync(m.p(), m.dvec.p, static_cast<size_t>(m.n) * 8,
                                    cudaMemcpyDeviceToDevice, m.s));
            m.dot_to(rn, zn, 9);
            m.dot_to(rn, z, 10);
            fcg_p_kernel<<<m.ug, kThreads, 0, m.s>>>(m.n, m.S(), zn, m.p());
            fcg_rz_kernel<<<1, 1, 0, m.s>>>(m.S());
            std::swap(r, rn);
            std::swap(z, zn);
        }
        // the true residual with the exact operator
        m.exact_residual(b, m.rn.as<double>());
    }
    CUDA_OK(cudaEventRecord(e1, m.s));
    const double rs = m.read(3);
    float ms = 0.0f;
    CUDA_OK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    CUDA_OK(cudaMemcpyAsync(x_out, m.x(), static_cast<size_t>(m.n) * 8, cudaMemcpyDeviceToDevice, m.s));
    const double inner_total = m.read(7);
    if (res) {
        res->outer = outer;
        res->inner_total = static_cast<int32_t>(inner_total);
        res->final_relres = std::sqrt(rs) / denom;
        res->reached = res->final_relres <= tol ? 1 : 0;
        res->ms_total = ms;
    }
}

// exact = the lossless hybrid when the plan keeps it, else a lossless dispatched route
int exact_route_of(const std::vector<cove_plan*>& plans) {
    const cove_plan* P = plans.front();
    if (P->has_route(COVE_ROUTE_HYBRID)) return COVE_ROUTE_HYBRID;
    if (P->dispatched_route == COVE_ROUTE_DICT_U8 || P->dispatched_route == COVE_ROUTE_DICT_U16)
        return P->dispatched_route;
    COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "the plan holds no lossless route for the outer solve");
}

void check_mp(const std::vector<cove_plan*>& plans, int inner_route, double tol, int k_inner, int max_outer) {
    if (plans.empty()) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "no plan");
    for (const cove_plan* P : plans) {
        if (P->dtype != COVE_F64) COVE_THROW(COVE_ERR_UNSUPPORTED, "the mixed-precision solvers run in fp64");
        if (!P->has_route(inner_route)) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "the plan does not hold the inner route");
        if (hybrid_spmv_launch_count(P->shape(), P->route_values(inner_route)) < 1 && P->nbr > 0)
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "inner route not runnable");
    }
    if (!(tol > 0.0) || k_inner < 1 || max_outer < 0)
        COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "tol must be positive, k_inner >= 1, max_outer >= 0");
}

}  // namespace
}  // namespace cove

extern "C" {

cove_status cove_ir_solve(const cove_plan* P, int32_t inner_route, const void* b, void* x, double tol,
                          int32_t k_inner, int32_t max_outer, cove_ir_result* result, void* stream) {
    return guarded([&] {
        if (!P || !b || !x) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        if (P->rows != P->cols) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "the solvers need a square matrix");
        MpSolver m;
        m.plans = {const_cast<cove_plan*>(P)};
        check_mp(m.plans, inner_route, tol, k_inner, max_outer);
        m.n = P->rows;
        m.wl = P->cols;
        m.exact_route = exact_route_of(m.plans);
        m.inner_route = inner_route;
        m.s = static_cast<cudaStream_t>(stream);
        mp_solve(m, false, static_cast<const double*>(b), static_cast<double*>(x), tol, k_inner, max_outer, result);
    });
}

cove_status cove_fcg_solve(const cove_plan* P, int32_t inner_route, const void* b, void* x, double tol,
                           int32_t k_inner, int32_t max_outer, cove_ir_result* result, void* stream) {
    return guarded([&] {
        if (!P || !b || !x) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        if (P->rows != P->cols) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "the solvers need a square matrix");
        MpSolver m;
        m.plans = {const_cast<cove_plan*>(P)};
        check_mp(m.plans, inner_route, tol, k_inner, max_outer);
        m.n = P->rows;
        m.wl = P->cols;
        m.exact_route = exact_route_of(m.plans);
        m.inner_route = inner_route;
        m.s = static_cast<cudaStream_t>(stream);
        mp_solve(m, true, static_cast<const double*>(b), static_cast<double*>(x), tol, k_inner, max_outer, result);
    });
}

cove_status cove_cg_solve(const cove_plan* P, const void* b, void* x, int32_t iters,
                          cove_cg_result* result, void* stream) {
    return guarded([&] {
        if (!P || !b || !x) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        if (P->rows != P->cols) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "CG needs a square matrix");
        if (iters < 0) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "iterations must be non-negative");
        std::vector<cove_plan*> plans{const_cast<cove_plan*>(P)};
        cg_run(nullptr, plans, P->rows, 0, P->cols, static_cast<const double*>(b),
               static_cast<double*>(x), iters, result, static_cast<cudaStream_t>(stream));
    });
}

int32_t cove_dist_halo_plan(int32_t rank, int32_t world, const int64_t* blocks4, int64_t* xfers5,
                            int32_t cap) {
    if (!blocks4 || !xfers5 || rank < 0 || rank >= world) return -1;
    const int64_t row_begin = blocks4[4 * rank], row_end = blocks4[4 * rank + 1];
    const int64_t wb = blocks4[4 * rank + 2], wl = blocks4[4 * rank + 3];
    int n = 0;
    int64_t covered = row_end - row_begin;
    for (int q = 0; q < world; ++q) {
        if (q == rank) continue;
        const int64_t qb = blocks4[4 * q], qe = blocks4[4 * q + 1];
        const int64_t qwb = blocks4[4 * q + 2], qwl = blocks4[4 * q + 3];
        // my rows inside q's window go to q; q's rows inside my window come from q
        const int64_t sb = std::max(row_begin, qwb), se = std::min(row_end, qwb + qwl);
        const int64_t rb = std::max(qb, wb), re = std::min(qe, wb + wl);
        const int64_t sn = std::max<int64_t>(0, se - sb), rn = std::max<int64_t>(0, re - rb);
        if (sn == 0 && rn == 0) continue;
        if (n >= cap) return -1;
        xfers5[5 * n + 0] = q;
        xfers5[5 * n + 1] = sn > 0 ? sb - wb : 0;
        xfers5[5 * n + 2] = sn;
        xfers5[5 * n + 3] = rn > 0 ? rb - wb : 0;
        xfers5[5 * n + 4] = rn;
        covered += rn;
        ++n;
    }
    return covered == wl ? n : -1;
}

size_t cove_dist_id_bytes(void) { return sizeof(ncclUniqueId); }

cove_status cove_dist_make_id(void* id_out) {
    return guarded([&] {
        if (!id_out) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null id");
        ncclUniqueId id;
        nccl_ok(nccl().GetUniqueId(&id), "ncclGetUniqueId");
        std::memcpy(id_out, &id, sizeof(id));
    });
}

cove_status cove_dist_create(int32_t rank, int32_t world, const void* nccl_id,
                             cove_plan* const* plans, int32_t num_plans, int64_t global_rows,
                             int64_t row_begin, int64_t row_end, int64_t window_begin,
                             int64_t window_len, int32_t timeout_ms, cove_dist** out) {
    return guarded([&] {
        if (!out || !nccl_id || (num_plans > 0 && !plans)) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        if (world < 1 || rank < 0 || rank >= world) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "bad rank/world");
        if (row_begin < window_begin || row_end > window_begin + window_len || row_end < row_begin) {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "row block must lie inside the window");
        }
        int64_t rows = 0;
        for (int i = 0; i < num_plans; ++i) {
            if (plans[i]->cols != window_len) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plan columns must equal the window length");
            rows += plans[i]->rows;
        }
        if (rows != row_end - row_begin) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "plans must cover the row block");
        auto* d = new cove_dist();
        d->rank = rank;
        d->world = world;
        d->plans.assign(plans, plans + num_plans);
        d->global_rows = global_rows;
        d->row_begin = row_begin;
        d->row_end = row_end;
        d->wb = window_begin;
        d->wl = window_len;
        d->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
        try {
            ncclUniqueId id;
            std::memcpy(&id, nccl_id, sizeof(id));
            ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
            cfg.blocking = 0;
            nccl_ok(nccl().CommInitRankConfig(&d->comm, world, id, rank, &cfg), "ncclCommInitRankConfig");
            wait_comm_ready(d->comm, d->timeout_ms);
            // share every rank's (row_begin, row_end, window_begin, window_len)
            DevBuf all;
            alloc_n<int64_t>(all, 4 * world);
            int64_t mine[4] = {row_begin, row_end, window_begin, window_len};
            cudaStream_t s = nullptr;
            CUDA_OK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
            CUDA_OK(cudaMemcpyAsync(all.as<int64_t>() + 4 * rank, mine, sizeof(mine),
                                    cudaMemcpyHostToDevice, s));
            const ncclResult_t ag =
                nccl().AllGather(all.as<int64_t>() + 4 * rank, all.p, 4, ncclInt64, d->comm, s);
            nccl_ok(ag, "ncclAllGather");
            if (ag == ncclInProgress) wait_comm_ready(d->comm, d->timeout_ms);
            wait_stream(d, s);
            std::vector<int64_t> h(4 * world);
            CUDA_OK(cudaMemcpy(h.data(), all.p, h.size() * 8, cudaMemcpyDeviceToHost));
            cudaStreamDestroy(s);
            std::vector<int64_t> xf(5 * static_cast<size_t>(world));
            const int nx = cove_dist_halo_plan(rank, world, h.data(), xf.data(), world);
            if (nx < 0) {
                COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "halo is not covered by other ranks' row blocks");
            }
            for (int i = 0; i < nx; ++i) {
                d->xfers.push_back(cove_dist::Xfer{static_cast<int>(xf[5 * i]), xf[5 * i + 1], xf[5 * i + 2],
                                                   xf[5 * i + 3], xf[5 * i + 4]});
            }
            plan_overlap(d);
        } catch (...) {
            if (d->comm) nccl().CommAbort(d->comm);
            if (d->x_ready) cudaEventDestroy(d->x_ready);
            if (d->halo_done) cudaEventDestroy(d->halo_done);
            if (d->s_comm) cudaStreamDestroy(d->s_comm);
            delete d;
            throw;
        }
        *out = d;
    });
}

cove_status cove_dist_destroy(cove_dist* d) {
    return guarded([&] {
        if (!d) return;
        if (d->comm) {
            nccl().CommFinalize(d->comm);
            wait_comm_ready(d->comm, d->timeout_ms);
            nccl().CommDestroy(d->comm);
        }
        if (d->x_ready) cudaEventDestroy(d->x_ready);
        if (d->halo_done) cudaEventDestroy(d->halo_done);
        if (d->s_comm) cudaStreamDestroy(d->s_comm);
        delete d;
    });
}

cove_status cove_dist_halo(cove_dist* d, void* x_window, void* stream) {
    return guarded([&] {
        if (!d || !x_window) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        halo(d, static_cast<double*>(x_window), static_cast<cudaStream_t>(stream));
    });
}

cove_status cove_dist_spmv(cove_dist* d, void* x_window, void* y_local, void* stream) {
    return guarded([&] {
        if (!d || !x_window || !y_local) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        spmv_dist(d, static_cast<double*>(x_window), static_cast<double*>(y_local),
                  static_cast<cudaStream_t>(stream));
    });
}

int32_t cove_dist_spmv_launches(const cove_dist* d) {
    if (!d) return -1;
    int32_t n = 0;
    for (size_t i = 0; i < d->plans.size(); ++i) {
        const cove_plan* P = d->plans[i];
        const KernelShape k = P->shape();
        const RouteValues rv = P->route_values(P->dispatched_route);
        const int full = hybrid_spmv_launch_count(k, rv);
        if (!d->overlap) {
            n += full;
            continue;
        }
        for (const auto& r : d->ranges[i]) n += r.b1 > r.b0 ? 1 : 0;  // main pass per range
        n += full - (k.nbr > 0 ? 1 : 0);                              // the overflow pass
    }
    return n;
}

cove_status cove_dist_mp_solve(cove_dist* d, int32_t flexible, int32_t inner_route, const void* b_local,
                               void* x_local, double tol, int32_t k_inner, int32_t max_outer,
                               cove_ir_result* result, void* stream) {
    return guarded([&] {
        if (!d || !b_local || !x_local) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        MpSolver m;
        m.d = d;
        m.plans = d->plans;
        check_mp(m.plans, inner_route, tol, k_inner, max_outer);
        m.n = d->row_end - d->row_begin;
        m.p_off = d->row_begin - d->wb;
        m.wl = d->wl;
        m.exact_route = exact_route_of(m.plans);
        m.inner_route = inner_route;
        m.s = static_cast<cudaStream_t>(stream);
        mp_solve(m, flexible != 0, static_cast<const double*>(b_local), static_cast<double*>(x_local), tol,
                 k_inner, max_outer, result);
    });
}

cove_status cove_dist_cg_solve(cove_dist* d, const void* b_local, void* x_local, int32_t iters,
                               cove_cg_result* result, void* stream) {
    return guarded([&] {
        if (!d || !b_local || !x_local) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        cg_run(d, d->plans, d->row_end - d->row_begin, d->row_begin - d->wb, d->wl,
               static_cast<const double*>(b_local), static_cast<double*>(x_local), iters, result,
               static_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// CG that allocates no device memory.
//
// Some callers cannot call cudaMalloc once they are running: applications
// whose device memory is owned by their own arena or pool allocator (all of
// HBM reserved at start-up, so a library's cudaMalloc fails or escapes their
// accounting), and loops with a latency budget, where cudaMalloc and
// cudaFree may synchronize the device and take unbounded time.  For them,
// cove_cg_solve_noalloc runs the same recurrence as cove_cg_solve with its
// work vectors in the fixed array below instead of freshly allocated
// buffers.  The array is a module global: every GPU on which this file's
// device code is loaded holds it until the process exits, and every call on
// that GPU shares it.
// ---------------------------------------------------------------------------

namespace cove {
namespace {
// one vector segment per work vector (p, r, Ap); a multiple of 32 doubles,
// so every segment starts 256-byte aligned like the array itself
constexpr int64_t kNoAllocSeg = COVE_CG_NOALLOC_MAX_ROWS;
static_assert(kNoAllocSeg % 32 == 0, "segments must stay 256-byte aligned");
constexpr int64_t kNoAllocDoubles = 3 * kNoAllocSeg + kDotCtas + 8;
}  // namespace
}  // namespace cove

// p | r | Ap | dot partials (kDotCtas) | scalar slots (8): about 3 MiB
static __device__ __align__(256) double cove_cg_noalloc_scratch[cove::kNoAllocDoubles];

namespace cove {
namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
struct NoAllocSlot {
    double* base = nullptr;
    unsigned long long ctx_id = 0;  // the context the address belongs to
};
NoAllocSlot g_noalloc[kNoAllocMaxDevices];

// Unique id of the current CUDA context (driver entry point, resolved at run
// time so the library does not link the driver library); 0 if unavailable.
unsigned long long current_context_id() {
    using GetCurrent = int (*)(void**);
    using GetId = int (*)(void*, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(f);
    });
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&ctx) == 0 && ctx && get_id(ctx, &id) == 0) return id;
    return 0;
}

// Device address of the scratch array on the current device (the host-side
// name is only a stand-in for the symbol).  It is looked up once per device
// and looked up again if the device's context was replaced since
// (cudaDeviceReset), since the array then lives at a new address.
double* noalloc_scratch() {
    int dev = -1;
    CUDA_OK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        COVE_THROW(COVE_ERR_UNSUPPORTED, "device ordinal beyond the no-allocation scratch table");
    const unsigned long long ctx = current_context_id();  // 0 before the context exists
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocSlot& slot = g_noalloc[dev];
    if (!slot.base || slot.ctx_id != ctx || ctx == 0) {
        double* ptr = nullptr;
        CUDA_OK(cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), cove_cg_noalloc_scratch));
        slot.base = ptr;
        slot.ctx_id = ctx;
    }
    return slot.base;
}

void cg_run_noalloc(const cove_plan* P, const double* b, double* x, int iters,
                    cove_cg_result* res, cudaStream_t s) {
    const int64_t n = P->rows;
    double* base = noalloc_scratch();
    double* p = base;
    double* r = base + kNoAllocSeg;
    double* ap = base + 2 * kNoAllocSeg;
    double* partial = base + 3 * kNoAllocSeg;
    double* S = partial + kDotCtas;  // [0,1] rs slots, [2] p.Ap, [4] rs0
    // The array keeps the previous call's contents.  x accumulates, so it is
    // cleared; the scalar slots are cleared too.  p and r are copied from b,
    // and Ap and the partials are written in full before they are read.
    CUDA_OK(cudaMemsetAsync(S, 0, 8 * sizeof(double), s));
    CUDA_OK(cudaMemsetAsync(x, 0, static_cast<size_t>(n) * 8, s));
    CUDA_OK(cudaMemcpyAsync(r, b, static_cast<size_t>(n) * 8, cudaMemcpyDeviceToDevice, s));
    CUDA_OK(cudaMemcpyAsync(p, b, static_cast<size_t>(n) * 8, cudaMemcpyDeviceToDevice, s));
    dot(n, r, r, partial, S + 0, s);
    CUDA_OK(cudaMemcpyAsync(S + 4, S + 0, sizeof(double), cudaMemcpyDeviceToDevice, s));
    const KernelShape shape = P->shape();
    const RouteValues vals = P->route_values(P->dispatched_route);
    int64_t launches = 2;
    for (int k = 0; k < iters; ++k) {
        launches += launch_hybrid_spmv(shape, vals, p, ap, s);
        launches += cg_vector_step(nullptr, n, p, ap, r, x, partial, S, k & 1, s);
    }
    CUDA_LAUNCH_OK();
    double h[8];
    CUDA_OK(cudaMemcpyAsync(h, S, sizeof(h), cudaMemcpyDeviceToHost, s));
    CUDA_OK(cudaStreamSynchronize(s));
    if (res) {
        res->iterations = iters;
        res->rs_initial = h[4];
        res->rs_final = h[iters & 1];
        res->ms_total = 0.0;
        res->ms_spmv = 0.0;
        res->launches = launches;
    }
}

}  // namespace
}  // namespace cove

extern "C" cove_status cove_cg_solve_noalloc(const cove_plan* P, const void* b, void* x,
                                             int32_t iters, cove_cg_result* result, void* stream) {
    return guarded([&] {
        if (!P || !b || !x) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        if (P->dtype != COVE_F64) COVE_THROW(COVE_ERR_UNSUPPORTED, "CG runs in fp64");
        if (P->rows != P->cols) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "CG needs a square matrix");
        if (iters < 0) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "iterations must be non-negative");
        if (P->rows > COVE_CG_NOALLOC_MAX_ROWS)
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT,
                       "cove_cg_solve_noalloc: " + std::to_string(P->rows) +
                           " rows exceed its fixed scratch of " +
                           std::to_string(COVE_CG_NOALLOC_MAX_ROWS) +
                           " rows; use cove_cg_solve for larger systems");
        cg_run_noalloc(P, static_cast<const double*>(b), static_cast<double*>(x), iters, result,
                       static_cast<cudaStream_t>(stream));
    });
}
