/* peer.cu -- combining the ranks' sums over NVLink peer memory, fused with the
 * finalisation (mpkPeer*).
 *
 * One Lloyd iteration over row shards ends with every GPU holding int64
 * fixed-point sums and counts of its own rows; the new centroids need the sum
 * over GPUs.  Instead of an allreduce of the whole k*d + k buffer followed by
 * the finalisation on every GPU, one kernel per GPU does both:
 *
 *   1. barrier: the rank announces that its sums are complete (an epoch value
 *      stored into a flag in every peer's memory) and waits until every peer
 *      has announced the same;
 *   2. the rank finalises its own slice of the clusters, [r k / N, (r+1) k / N),
 *      reading every peer's sums and counts of those clusters directly over
 *      NVLink (integer adds, exact in any order), with the arithmetic of
 *      k_finalize_fixed, into its centroids and into its exchange block;
 *   3. barrier: every rank has finalised its slice;
 *   4. the rank reads the other ranks' finalised slices (centroids and moved^2)
 *      from their exchange blocks into its own centroids.
 *
 * Each GPU moves about (k d + k) 8 bytes / N in and k d 4 bytes (N-1) / N out
 * instead of an allreduce's 2 (N-1) / N (k d + k) 8 bytes each way, and the
 * finalisation's launch goes away.  Every wait is bounded by the global timer
 * (kWaitLimitNs); a wait that runs out sets MPK_DEV_TIMEOUT in the engine's
 * status word and the kernel finishes without the data it waited for.  Loads
 * and stores of peer memory are plain (no multicast, no bulk copies).
 *
 * The exchange block of a rank (cudaMalloc, so it can be exported as a CUDA IPC
 * handle to the other ranks' processes):
 *   [0, 1024)      flags[2][kPeerMax] u64: written by the peers (barriers 1, 2)
 *   [1024, 1040)   epoch u64 (the barrier value of the next combine), done u32
 *   [2048, ...)    S: k*d + k int64 sums then counts (the engine's dSums)
 *   then           X: k*d FP32 finalised centroids of this rank's slice
 *   then           M: k FP32 moved^2 of this rank's slice
 * The epoch lives on the device and moves on by one per combine, so the
 * kernel's arguments do not change between iterations.
 */
#include "engine.cuh"
#include "mpkmeans.h"

#include <cstdio>
#include <cstring>

namespace mpk {
namespace {

constexpr size_t kOffFlags = 0, kOffCtrl = 1024, kOffS = 2048;

__host__ __device__ inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }
__host__ __device__ inline size_t off_x(int k, int d) { return kOffS + align256(((size_t)k * d + k) * sizeof(long long)); }
__host__ __device__ inline size_t off_m(int k, int d) { return off_x(k, d) + align256((size_t)k * d * sizeof(float)); }
__host__ __device__ inline size_t block_bytes(int k, int d) { return off_m(k, d) + align256((size_t)k * sizeof(float)); }

/* Flags are stored and polled with relaxed system-scope accesses; the one
 * __threadfence_system() before a rank's stores (release) and the one after its
 * wait (acquire) order the data around them. */
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

/* Release: this thread's (and, cumulatively, its block's) earlier writes, then
 * flag `slot` of every rank's block set to ep. */
__device__ __forceinline__ void announce(const PeerBases& bases, int world, int slot, unsigned long long ep) {
    __threadfence_system();
    for (int p = 0; p < world; ++p)
        st_relaxed_sys(reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(bases.p[p]) + kOffFlags) + slot,
                       ep);
}

/* Thread 0: every rank's flag at or past ep, within the time limit; then acquire. */
__device__ bool wait_flags(const unsigned long long* flags, int world, unsigned long long ep, int* status) {
    const unsigned long long t0 = globaltimer();
    for (int p = 0; p < world; ++p) {
        while (ld_relaxed_sys(flags + p) < ep) {
            if (globaltimer() - t0 > kWaitLimitNs) {
                atomicOr(status, MPK_DEV_TIMEOUT);
                return false;
            }
        }
    }
    __threadfence_system();
    return true;
}

/* The sum over ranks of one int64 of the sums region, the loads of all ranks
 * issued before any is used (eight at a time).  Plain L2-level loads: a peer's
 * memory is not cached in this GPU's L2, and the flag wait ordered them. */
__device__ __forceinline__ long long sum_over_ranks(const PeerBases& bases, int world, size_t index) {
    long long total = 0;
    for (int p0 = 0; p0 < world; p0 += 8) {
        long long v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            v[u] = p0 + u < world
                       ? __ldcg(reinterpret_cast<const long long*>(reinterpret_cast<const uint8_t*>(bases.p[p0 + u]) +
                                                                   kOffS) + index)
                       : 0;
#pragma unroll
        for (int u = 0; u < 8; ++u) total += v[u];
    }
    return total;
}

__global__ void __launch_bounds__(256)
k_peer_combine(PeerBases bases, int rank, int world, int k, int d, const DevParams* __restrict__ prm, int* status,
               float* __restrict__ C, float* __restrict__ moved2) {
    __shared__ float sh[256];
    __shared__ unsigned long long ep_s;
    __shared__ int ok_s;
    const int t = threadIdx.x;
    uint8_t* own = reinterpret_cast<uint8_t*>(bases.p[rank]);
    unsigned long long* flags = reinterpret_cast<unsigned long long*>(own + kOffFlags);
    unsigned long long* epoch = reinterpret_cast<unsigned long long*>(own + kOffCtrl);
    unsigned int* done = reinterpret_cast<unsigned int*>(own + kOffCtrl + 8);
    const size_t ox = off_x(k, d), om = off_m(k, d);
    const long long kd = (long long)k * d;

    /* ---- 1: announce, then wait for every rank's sums ---- */
    if (t == 0) {
        ep_s = *reinterpret_cast<volatile unsigned long long*>(epoch);
        if (blockIdx.x == 0) announce(bases, world, rank, ep_s);
        ok_s = wait_flags(flags, world, ep_s, status) ? 1 : 0;
    }
    __syncthreads();
    const unsigned long long ep = ep_s;
    bool ok = ok_s != 0;

    /* ---- 2: this rank's slice of the clusters, summed over the ranks and finalised ---- */
    const int j0 = (int)((long long)rank * k / world), j1 = (int)((long long)(rank + 1) * k / world);
    float* X = reinterpret_cast<float*>(own + ox);
    float* Mv = reinterpret_cast<float*>(own + om);
    if (ok) {
        const double inv = ldexp(1.0, -prm->frac);
        for (int j = j0 + (int)blockIdx.x; j < j1; j += (int)gridDim.x) {
            const long long cnt = sum_over_ranks(bases, world, (size_t)kd + j);
            float acc = 0.f;
            for (int f = t; f < d; f += 256) {
                const size_t o = (size_t)j * d + f;
                const long long sum = sum_over_ranks(bases, world, o);
                const float old = C[o];
                const float nv = cnt > 0 ? (float)(((double)sum * inv) / (double)cnt) : old;
                C[o] = nv;
                X[o] = nv;
                const float dv = nv - old;
                acc = fmaf(dv, dv, acc);
            }
            sh[t] = acc;
            __syncthreads();
            for (int off = 128; off > 0; off >>= 1) {
                if (t < off) sh[t] = sh[t] + sh[t + off];
                __syncthreads();
            }
            if (t == 0) {
                Mv[j] = sh[0];
                if (moved2) moved2[j] = sh[0];
            }
            __syncthreads();
        }
    }

    /* ---- 3: the last block of this rank announces the slice, and moves the epoch on ---- */
    __threadfence_system();
    __syncthreads();
    if (t == 0) {
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0;
            *reinterpret_cast<volatile unsigned long long*>(epoch) = ep + 1;
            announce(bases, world, kPeerMax + rank, ep);
        }
        ok_s = (ok && wait_flags(flags + kPeerMax, world, ep, status)) ? 1 : 0;
    }
    __syncthreads();
    if (!ok_s) return;

    /* ---- 4: the other ranks' finalised slices ---- */
    const long long nthr = (long long)gridDim.x * blockDim.x;
    const long long tid = (long long)blockIdx.x * blockDim.x + t;
    for (int p = 0; p < world; ++p) {
        if (p == rank) continue;
        const int q0 = (int)((long long)p * k / world), q1 = (int)((long long)(p + 1) * k / world);
        const uint8_t* pb = reinterpret_cast<const uint8_t*>(bases.p[p]);
        const float* Xp = reinterpret_cast<const float*>(pb + ox);
        const float* Mp = reinterpret_cast<const float*>(pb + om);
        const long long e0 = (long long)q0 * d, e1 = (long long)q1 * d;
        if ((d & 3) == 0) {                       /* rows of 16-byte multiples: float4 copies */
            const float4* src = reinterpret_cast<const float4*>(Xp + e0);
            float4* dst = reinterpret_cast<float4*>(C + e0);
            const long long nv = (e1 - e0) >> 2;
            for (long long e = tid; e < nv; e += nthr) dst[e] = __ldcg(src + e);
        } else {
            for (long long e = e0 + tid; e < e1; e += nthr) C[e] = __ldcg(Xp + e);
        }
        if (moved2)
            for (long long j = q0 + tid; j < q1; j += nthr) moved2[j] = __ldcg(Mp + j);
    }
}

}  /* namespace */

size_t peer_block_bytes(int k, int d) { return block_bytes(k, d); }
size_t peer_sums_offset() { return kOffS; }

cudaError_t launch_peer_combine(const PeerBases& bases, int rank, int world, int k, int d, const DevParams* prm,
                                int* status, float* C, float* moved2, int num_sms, cudaStream_t s) {
    const int slice = (int)(((long long)(rank + 1) * k) / world - ((long long)rank * k) / world);
    int nb = slice < 1 ? 1 : slice;
    if (nb > num_sms * 4) nb = num_sms * 4;
    k_peer_combine<<<nb, 256, 0, s>>>(bases, rank, world, k, d, prm, status, C, moved2);
    return cudaGetLastError();
}

}  /* namespace mpk */

/* ------------------------------------------------------------- the ABI ---- */

struct mpkPeerGroup_s {
    int rank = 0, world = 0, k = 0, d = 0, dev = 0;
    void* base = nullptr;                 /* this rank's exchange block */
    mpk::PeerBases bases{};               /* every rank's block, this one included */
    bool imported[mpk::kPeerMax] = {};    /* opened from an IPC handle (closed on destroy) */
    bool connected = false;
};

/* Runs `fn` with the group's device current, then restores the caller's. */
template <typename F>
static mpkStatus on_device(int dev, F&& fn) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) return MPK_ERR_CUDA;
    const mpkStatus st = fn();
    if (prev != dev) cudaSetDevice(prev);
    return st;
}

extern "C" {

mpkStatus mpkPeerCreate(mpkPeerGroup* out, int rank, int world, int k, int d) {
    if (!out || world < 1 || world > mpk::kPeerMax || rank < 0 || rank >= world || k < 1 || d < 1)
        return MPK_ERR_INVALID;
    *out = nullptr;
    mpkPeerGroup g = new mpkPeerGroup_s();
    g->rank = rank;
    g->world = world;
    g->k = k;
    g->d = d;
    cudaGetDevice(&g->dev);
    const size_t bytes = mpk::peer_block_bytes(k, d);
    if (cudaMalloc(&g->base, bytes) != cudaSuccess) {
        cudaGetLastError();
        delete g;
        return MPK_ERR_ALLOC;
    }
    /* flags 0, epoch 1 (the first combine's barrier value), done 0 */
    const unsigned long long one = 1;
    if (cudaMemset(g->base, 0, mpk::peer_sums_offset()) != cudaSuccess ||
        cudaMemcpy(static_cast<uint8_t*>(g->base) + 1024, &one, sizeof(one), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(g->base);
        delete g;
        return MPK_ERR_CUDA;
    }
    g->bases.p[rank] = g->base;
    *out = g;
    return MPK_OK;
}

mpkStatus mpkPeerExportHandle(mpkPeerGroup g, void* handle64) {
    if (!g || !handle64) return MPK_ERR_INVALID;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, g->base) != cudaSuccess) return MPK_ERR_CUDA;
    static_assert(sizeof(h) == 64, "IPC handle size");
    std::memcpy(handle64, &h, sizeof(h));
    return MPK_OK;
}

mpkStatus mpkPeerLocalBase(mpkPeerGroup g, void** base) {
    if (!g || !base) return MPK_ERR_INVALID;
    *base = g->base;
    return MPK_OK;
}

mpkStatus mpkPeerConnect(mpkPeerGroup g, const void* const* handles64, void* const* bases, const int* devices) {
    if (!g || g->connected || (!handles64 && !bases)) return MPK_ERR_INVALID;
    /* peer access and IPC mappings belong to the context of the group's device */
    return on_device(g->dev, [&]() -> mpkStatus {
    for (int p = 0; p < g->world; ++p) {
        if (p == g->rank) continue;
        if (bases && bases[p]) {
            /* a block of this process on another device: its memory through peer access */
            if (devices && devices[p] >= 0 && devices[p] != g->dev) {
                const cudaError_t e = cudaDeviceEnablePeerAccess(devices[p], 0);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
                    fprintf(stderr, "mpkPeerConnect: no peer access from device %d to %d: %s\n", g->dev, devices[p],
                            cudaGetErrorString(e));
                    return MPK_ERR_CUDA;
                }
                cudaGetLastError();
            }
            g->bases.p[p] = bases[p];
        } else if (handles64 && handles64[p]) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, handles64[p], sizeof(h));
            void* ptr = nullptr;
            const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                fprintf(stderr, "mpkPeerConnect: cannot open rank %d's block: %s\n", p, cudaGetErrorString(e));
                return MPK_ERR_CUDA;
            }
            g->bases.p[p] = ptr;
            g->imported[p] = true;
        } else {
            return MPK_ERR_INVALID;
        }
    }
    g->connected = true;
    return MPK_OK;
    });
}

long long* mpkPeerSums(mpkPeerGroup g) {
    return g ? reinterpret_cast<long long*>(static_cast<uint8_t*>(g->base) + mpk::peer_sums_offset()) : nullptr;
}

mpkStatus mpkPeerDestroy(mpkPeerGroup g) {
    if (!g) return MPK_ERR_INVALID;
    const mpkStatus st = on_device(g->dev, [&]() -> mpkStatus {
        /* no combine of this rank may still read the peers' blocks or its own */
        cudaDeviceSynchronize();
        for (int p = 0; p < g->world; ++p)
            if (g->imported[p]) cudaIpcCloseMemHandle(g->bases.p[p]);
        cudaFree(g->base);
        return MPK_OK;
    });
    delete g;
    return st;
}

}  /* extern "C" */

/* the engine side (mpkmeans_api.cu) launches the combine on its own stream */
namespace mpk {
bool peer_ready(mpkPeerGroup g, int k, int d) { return g && g->connected && g->k == k && g->d == d; }
const PeerBases& peer_bases(mpkPeerGroup g) { return g->bases; }
int peer_rank(mpkPeerGroup g) { return g->rank; }
int peer_world(mpkPeerGroup g) { return g->world; }
}  /* namespace mpk */
