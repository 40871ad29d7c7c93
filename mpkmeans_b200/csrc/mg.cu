/* mg.cu -- single-process multi-GPU Lloyd over row shards (mpkMeansMixedMG).
 *
 * One engine per device holds its shard's split points.  Per iteration every
 * device assigns its rows and adds its exact int64 fixed-point sums and
 * counts; one NCCL allreduce (int64 sum, in place) combines them; every device
 * then finalises the same centroids redundantly.  Integer sums make the result
 * independent of the number of devices and of the reduction order.
 *
 * NCCL is resolved at run time (dlopen of libnccl.so.2, or the copy already
 * loaded by the host process), so the library links without it and callers
 * that never use this entry point never load it.
 *
 * Failure detection: the host never blocks on a device.  It polls every
 * stream and every communicator's asynchronous error; on an error, or when a
 * wait exceeds MPK_MG_TIMEOUT_S seconds (default 600), it aborts the
 * communicators (ncclCommAbort) and returns MPK_ERR_CUDA.
 */
#include "engine.cuh"
#include "mpkmeans.h"
#include "mpkmeans_debug.h"

#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

namespace mpk {
/* mpkmeans_api.cu: excl_cond3 (or excl_cond6) of the reference's mpkStats from
 * S->tested, the rows the bound left to the refinement and the FP32 candidates
 * evaluated. */
void fill_exclusions(mpkStats* S, const mpkParams& P, long long rows_refined, long long cands);
}  /* namespace mpk */

namespace {

struct Nccl {
    ncclResult_t (*commInitAll)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*groupStart)() = nullptr;
    ncclResult_t (*groupEnd)() = nullptr;
    const char* (*errStr)(ncclResult_t) = nullptr;
    ncclResult_t (*asyncError)(ncclComm_t, ncclResult_t*) = nullptr;   /* optional */
    ncclResult_t (*abort)(ncclComm_t) = nullptr;                        /* optional */
    bool ok = false;
};

const Nccl& nccl() {
    static Nccl n;
    static bool tried = false;
    if (tried) return n;
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        fprintf(stderr, "mpkMeansMixedMG: cannot load NCCL: %s\n", dlerror());
        return n;
    }
    n.commInitAll = (decltype(n.commInitAll))dlsym(h, "ncclCommInitAll");
    n.commDestroy = (decltype(n.commDestroy))dlsym(h, "ncclCommDestroy");
    n.allReduce = (decltype(n.allReduce))dlsym(h, "ncclAllReduce");
    n.groupStart = (decltype(n.groupStart))dlsym(h, "ncclGroupStart");
    n.groupEnd = (decltype(n.groupEnd))dlsym(h, "ncclGroupEnd");
    n.errStr = (decltype(n.errStr))dlsym(h, "ncclGetErrorString");
    n.asyncError = (decltype(n.asyncError))dlsym(h, "ncclCommGetAsyncError");
    n.abort = (decltype(n.abort))dlsym(h, "ncclCommAbort");
    n.ok = n.commInitAll && n.commDestroy && n.allReduce && n.groupStart && n.groupEnd && n.errStr;
    return n;
}

__global__ void k_max_abs_host_visible(const float* A, long long count, float* out) {
    float m = 0.f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (long long)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(A[i]));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(reinterpret_cast<unsigned int*>(out), __float_as_uint(m));
}

float device_maxabs(const float* A, long long count, cudaStream_t s) {
    float* d = nullptr;
    float h = 0.f;
    if (count <= 0 || cudaMalloc(&d, sizeof(float)) != cudaSuccess) return 0.f;
    cudaMemsetAsync(d, 0, sizeof(float), s);
    long long blocks = (count + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    k_max_abs_host_visible<<<(int)blocks, 256, 0, s>>>(A, count, d);
    cudaMemcpyAsync(&h, d, sizeof(float), cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    cudaFree(d);
    return h;
}

/* Test hook (mpkDebugMGFailNextWait): the next wait that finds every stream
 * idle reports an asynchronous error anyway, so the abort path runs with no
 * collective in flight. */
std::atomic<bool> g_mg_fail{false};

double wait_limit_s() {
    const char* v = std::getenv("MPK_MG_TIMEOUT_S");
    const double t = v ? std::atof(v) : 0.0;
    return t > 0.0 ? t : 600.0;
}

/* Wait for every device's stream without blocking on any: poll the streams
 * and the communicators' asynchronous errors.  On an error or a timeout,
 * abort every communicator (the handles are gone afterwards) and return
 * MPK_ERR_CUDA. */
mpkStatus mg_wait(int ngpu, const int* devices, const std::vector<cudaStream_t>& st,
                  std::vector<ncclComm_t>& comm, const Nccl& N) {
    const auto t0 = std::chrono::steady_clock::now();
    const double limit = wait_limit_s();
    const char* why = nullptr;
    for (;;) {
        bool idle = true;
        for (int g = 0; g < ngpu && !why; ++g) {
            cudaSetDevice(devices[g]);
            const cudaError_t q = cudaStreamQuery(st[g]);
            if (q == cudaErrorNotReady) idle = false;
            else if (q != cudaSuccess) why = cudaGetErrorString(q);
            if (!why && comm[g] && N.asyncError) {
                ncclResult_t ae = ncclSuccess;
                if (N.asyncError(comm[g], &ae) != ncclSuccess) why = "ncclCommGetAsyncError failed";
                else if (ae != ncclSuccess && ae != ncclInProgress) why = N.errStr(ae);
            }
        }
        if (!why && idle) {
            if (!g_mg_fail.exchange(false)) return MPK_OK;
            why = "injected asynchronous error (test hook)";
        }
        if (!why && std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit)
            why = "timed out waiting for the devices";
        if (why) break;
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    fprintf(stderr, "mpkMeansMixedMG: %s; aborting the communicators\n", why);
    for (int g = 0; g < ngpu; ++g)
        if (comm[g]) {
            cudaSetDevice(devices[g]);
            if (N.abort) N.abort(comm[g]);
            else N.commDestroy(comm[g]);
            comm[g] = nullptr;
        }
    return MPK_ERR_CUDA;
}

}  /* namespace */

extern "C" mpkStatus mpkDebugMGFailNextWait(void) {
    g_mg_fail.store(true);
    return MPK_OK;
}

extern "C" mpkStatus mpkMeansMixedMG(int ngpu, const int* devices, const float* const* dPshard, const int* nshard,
                                     int d, int k, float* const* dC, int* const* dAssign, const mpkParams* params,
                                     mpkStats* stats) {
    if (ngpu < 1 || !devices || !dPshard || !nshard || !dC || !dAssign || d <= 0 || k <= 0) return MPK_ERR_INVALID;
    long long n_total = 0;
    for (int g = 0; g < ngpu; ++g) {
        if (nshard[g] < 0 || (nshard[g] > 0 && (!dPshard[g] || !dAssign[g])) || !dC[g]) return MPK_ERR_INVALID;
        n_total += nshard[g];
    }
    if (n_total < k) return MPK_ERR_INVALID;
    const Nccl& N = nccl();
    if (!N.ok) return MPK_ERR_INVALID;
    mpkParams P;
    if (params) P = *params; else mpkParamsInit(&P);
    mpkStats local;
    mpkStats* S = stats ? stats : &local;
    std::memset(S, 0, sizeof(*S));
    const int refine = (P.use_cond3 || P.use_cond6) ? 1 : 0;
    int prev_dev = 0;
    cudaGetDevice(&prev_dev);

    std::vector<cudaStream_t> st(ngpu, nullptr);
    std::vector<mpkEngine> eng(ngpu, nullptr);
    std::vector<long long*> sums(ngpu, nullptr);
    std::vector<float*> moved(ngpu, nullptr);
    std::vector<ncclComm_t> comm(ngpu, nullptr);
    std::vector<float> h_moved((size_t)k);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    mpkStatus rc = MPK_OK;
    const long long len = (long long)k * d + k;
    int it = 0;

    /* one global operand scale: max |P| over every shard and the start C */
    float pmax = 0.f;
    for (int g = 0; g < ngpu; ++g) {
        cudaSetDevice(devices[g]);
        if (cudaStreamCreateWithFlags(&st[g], cudaStreamNonBlocking) != cudaSuccess) { rc = MPK_ERR_CUDA; goto done; }
        pmax = fmaxf(pmax, device_maxabs(dPshard[g], (long long)nshard[g] * d, st[g]));
        if (g == 0) pmax = fmaxf(pmax, device_maxabs(dC[g], (long long)k * d, st[g]));
    }
    for (int g = 0; g < ngpu; ++g) {
        cudaSetDevice(devices[g]);
        rc = mpkEngineCreate(&eng[g], dPshard[g], nshard[g], d, k, nullptr, pmax > 0.f ? pmax : 1.f, n_total, st[g]);
        if (rc != MPK_OK) goto done;
        if (mpk::dev_alloc((void**)&sums[g], (size_t)len * sizeof(long long), st[g]) != cudaSuccess ||
            mpk::dev_alloc((void**)&moved[g], (size_t)k * sizeof(float), st[g]) != cudaSuccess) {
            rc = MPK_ERR_ALLOC;
            goto done;
        }
    }
    {
        const ncclResult_t r = N.commInitAll(comm.data(), ngpu, devices);
        if (r != ncclSuccess) {
            fprintf(stderr, "mpkMeansMixedMG: ncclCommInitAll: %s\n", N.errStr(r));
            rc = MPK_ERR_CUDA;
            goto done;
        }
    }
    /* NCCL connects its peers at a communicator's first collective: one
     * allreduce here, waited for, keeps that out of the timed iterations */
    for (int g = 0; g < ngpu; ++g) {
        cudaSetDevice(devices[g]);
        cudaMemsetAsync(sums[g], 0, (size_t)len * sizeof(long long), st[g]);
    }
    N.groupStart();
    for (int g = 0; g < ngpu; ++g)
        N.allReduce(sums[g], sums[g], (size_t)len, ncclInt64, ncclSum, comm[g], st[g]);
    {
        const ncclResult_t r = N.groupEnd();
        if (r != ncclSuccess) {
            fprintf(stderr, "mpkMeansMixedMG: ncclAllReduce: %s\n", N.errStr(r));
            rc = MPK_ERR_CUDA;
            goto done;
        }
    }
    if ((rc = mg_wait(ngpu, devices, st, comm, N)) != MPK_OK) goto done;
    cudaSetDevice(devices[0]);
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st[0]);
    for (it = 0; it < P.max_iter; ++it) {
        for (int g = 0; g < ngpu; ++g) {
            cudaSetDevice(devices[g]);
            /* assign, refine, accumulate: three CUDA graphs replayed per device */
            if ((rc = mpkEngineStep(eng[g], dC[g], dAssign[g], sums[g], refine)) != MPK_OK) goto done;
        }
        N.groupStart();
        for (int g = 0; g < ngpu; ++g)
            N.allReduce(sums[g], sums[g], (size_t)len, ncclInt64, ncclSum, comm[g], st[g]);
        {
            const ncclResult_t r = N.groupEnd();
            if (r != ncclSuccess) {
                fprintf(stderr, "mpkMeansMixedMG: ncclAllReduce: %s\n", N.errStr(r));
                rc = MPK_ERR_CUDA;
                goto done;
            }
        }
        for (int g = 0; g < ngpu; ++g) {
            cudaSetDevice(devices[g]);
            if ((rc = mpkEngineFinalize(eng[g], sums[g], dC[g], moved[g])) != MPK_OK) goto done;
        }
        S->hp_baseline += n_total * k;
        S->tested += n_total * (k - 1);
        if (P.tol > 0.f || P.verbose) {
            cudaSetDevice(devices[0]);
            cudaMemcpyAsync(h_moved.data(), moved[0], (size_t)k * sizeof(float), cudaMemcpyDeviceToHost, st[0]);
            if ((rc = mg_wait(ngpu, devices, st, comm, N)) != MPK_OK) goto done;
            double fro2 = 0.0;
            for (int j = 0; j < k; ++j) fro2 += (double)h_moved[j];
            if (P.verbose) fprintf(stderr, "[mg] iter %3d  ||dC||_F^2 %.6e\n", it, fro2);
            if (P.tol > 0.f && fro2 < (double)P.tol * (double)P.tol) { ++it; break; }
        }
    }
    S->iters = it;
    cudaSetDevice(devices[0]);
    cudaEventRecord(e1, st[0]);
    if ((rc = mg_wait(ngpu, devices, st, comm, N)) != MPK_OK) goto done;
    {
        float ms = 0.f;
        cudaSetDevice(devices[0]);
        cudaEventElapsedTime(&ms, e0, e1);
        S->t_total_ms = ms;
        long long rows_all = 0;
        for (int g = 0; g < ngpu; ++g) {
            cudaSetDevice(devices[g]);
            long long rows = 0, cands = 0, full = 0;
            int status = 0;
            double ine = 0.0;
            mpkEngineCounters(eng[g], &rows, &cands, &full, &status);
            if (status) { rc = MPK_ERR_CUDA; goto done; }
            S->hp_update += cands;
            rows_all += rows;
            if (nshard[g] > 0 && mpkEngineInertia(eng[g], dC[g], dAssign[g], &ine) != MPK_OK) { rc = MPK_ERR_CUDA; goto done; }
            S->inertia += ine;
        }
        if (refine) mpk::fill_exclusions(S, P, rows_all, S->hp_update);
    }
done:
    /* Invariant before the synchronisations below: no stream holds a collective that
     * could wait for ever.  On success every collective has completed (mg_wait).  On
     * an error a collective may be in flight (a group launch that failed part way, or
     * a step that failed after others' allreduces were enqueued), so any communicator
     * still alive is aborted first, which ends its kernels; mg_wait's own failures
     * have aborted theirs already (comm[g] is then null). */
    if (rc != MPK_OK)
        for (int g = 0; g < ngpu; ++g)
            if (comm[g]) {
                cudaSetDevice(devices[g]);
                if (N.abort) N.abort(comm[g]);
                else N.commDestroy(comm[g]);
                comm[g] = nullptr;
            }
    for (int g = 0; g < ngpu; ++g) {
        cudaSetDevice(devices[g]);
        if (st[g]) cudaStreamSynchronize(st[g]);
        if (comm[g]) N.commDestroy(comm[g]);
        if (eng[g]) mpkEngineDestroy(eng[g]);
        mpk::dev_free(sums[g], st[g]);
        mpk::dev_free(moved[g], st[g]);
        if (st[g]) {
            cudaStreamSynchronize(st[g]);
            cudaStreamDestroy(st[g]);
        }
    }
    cudaSetDevice(devices[0]);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaSetDevice(prev_dev);
    return rc;
}
