/* update.cu -- exact segmented-sum centroid update.
 *
 * Replaces the reference's mpkLaunchZero / mpkLaunchAccumulate
 * (kmeans/src/kernels.cu:683-703: one FP64 global atomic per coordinate) with
 * a counting sort of the rows by label followed by a segmented sum:
 *
 *   k_label_hist     labels -> per-cluster counts (shared-memory histogram)
 *   k_bin_scan       counts -> bin starts; counts written to the sums buffer
 *   k_label_scatter  row indices grouped by label (perm)
 *   k_segsum         each warp walks a contiguous run of perm, reading whole
 *                    point rows (coalesced, 16 B per lane), quantising every
 *                    coordinate once to q = rint(x * 2^frac) and adding into
 *                    int64 registers; at a label boundary (and at the end of
 *                    its run) the warp adds its registers into the global
 *                    int64 sums.
 *
 * Integer sums are exact, so the result does not depend on the order of the
 * rows within a cluster, on the split of the work, or on the number of GPUs
 * whose buffers are later summed; the points are read from HBM once.
 */
#include "engine.cuh"

namespace mpk {
namespace {

constexpr int kSmemHistMax = 48 * 1024;   /* labels per shared-memory histogram */

template <bool SMEM>
__global__ void k_label_hist(const int* __restrict__ labels, long long n, int k, int* __restrict__ hist,
                             DevParams* __restrict__ prm) {
    extern __shared__ int h[];
    if (SMEM) {
        for (int j = threadIdx.x; j < k; j += blockDim.x) h[j] = 0;
        __syncthreads();
    }
    bool bad = false;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int a = labels[i];
        if ((unsigned)a >= (unsigned)k) { bad = true; continue; }
        if (SMEM) atomicAdd(&h[a], 1);
        else atomicAdd(&hist[a], 1);
    }
    if (bad) atomicOr(&prm->status, MPK_DEV_LABEL_RANGE);
    if (SMEM) {
        __syncthreads();
        for (int j = threadIdx.x; j < k; j += blockDim.x)
            if (h[j]) atomicAdd(&hist[j], h[j]);
    }
}

/* One 1024-thread block: exclusive scan of the k counts. */
__global__ void k_bin_scan(const int* __restrict__ hist, int k, int* __restrict__ bin_start,
                           int* __restrict__ cursor, long long* __restrict__ counts) {
    __shared__ long long part[1024];
    const int t = threadIdx.x;
    const int per = (k + 1023) / 1024;
    const int j0 = t * per, j1 = min(k, j0 + per);
    long long s = 0;
    for (int j = j0; j < j1; ++j) s += hist[j];
    part[t] = s;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
        const long long v = t >= off ? part[t - off] : 0;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    long long run = part[t] - s;   /* exclusive prefix of this thread's chunk */
    for (int j = j0; j < j1; ++j) {
        bin_start[j] = (int)run;
        cursor[j] = (int)run;
        counts[j] = hist[j];
        run += hist[j];
    }
    if (t == 1023) bin_start[k] = (int)part[1023];
}

/* Rows [r0, r1) of one block: a local histogram reserves one range per label
 * in the global order, then every row takes the next slot of its range. */
template <bool SMEM>
__global__ void k_label_scatter(const int* __restrict__ labels, long long n, int k, int* __restrict__ cursor,
                                int* __restrict__ perm, long long rows_per_block) {
    extern __shared__ int h[];
    const long long r0 = (long long)blockIdx.x * rows_per_block;
    const long long r1 = min(n, r0 + rows_per_block);
    if constexpr (!SMEM) {
        for (long long i = r0 + threadIdx.x; i < r1; i += blockDim.x) {
            const int a = labels[i];
            if ((unsigned)a < (unsigned)k) perm[atomicAdd(&cursor[a], 1)] = (int)i;
        }
    } else {
        for (int j = threadIdx.x; j < k; j += blockDim.x) h[j] = 0;
        __syncthreads();
        for (long long i = r0 + threadIdx.x; i < r1; i += blockDim.x) {
            const int a = labels[i];
            if ((unsigned)a < (unsigned)k) atomicAdd(&h[a], 1);
        }
        __syncthreads();
        for (int j = threadIdx.x; j < k; j += blockDim.x)
            if (h[j]) h[j] = atomicAdd(&cursor[j], h[j]);
        __syncthreads();
        for (long long i = r0 + threadIdx.x; i < r1; i += blockDim.x) {
            const int a = labels[i];
            if ((unsigned)a < (unsigned)k) perm[atomicAdd(&h[a], 1)] = (int)i;
        }
    }
}

__device__ __forceinline__ long long quantise(float x, float sc) {
    /* x * 2^frac is exact in FP32 (a power-of-two scale that cannot overflow
     * by the choice of frac); the conversion rounds to nearest, ties even. */
    return __float2ll_rn(x * sc);
}

/* Segmented sum over the label-sorted rows.  VEC = 4: lane l owns features
 * 4l..4l+3 of every 128-feature group (float4 loads); VEC = 1: lane l owns
 * features l, l+32, ...  NG groups per lane cover d.  U rows are loaded at
 * once; a narrow row (d <= 64: half the lanes or fewer hold a feature) takes
 * U = 8, since each load then moves little. */
template <int VEC, int NG, int U = (NG <= 2 ? 4 : (NG <= 4 ? 2 : 1))>
__global__ void __launch_bounds__(256)
k_segsum(const float* __restrict__ P, int d, int f0, const int* __restrict__ perm, const int* __restrict__ bin_start,
         int k, const DevParams* __restrict__ prm, long long* __restrict__ sums) {
    constexpr int SPAN = 32 * VEC;                 /* features per group */
    const int lane = threadIdx.x & 31;
    const long long total = bin_start[k];
    const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
    const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const long long e0 = total * w / nw, e1 = total * (w + 1) / nw;
    if (e0 >= e1) return;
    const float sc = ldexpf(1.0f, prm->frac);

    /* the cluster holding entry e0: the last bin whose start is <= e0 */
    int lo = 0, hi = k - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (bin_start[mid] <= e0) lo = mid; else hi = mid - 1;
    }
    int bin = lo;
    long long next = bin_start[bin + 1];
    while (next <= e0) { ++bin; next = bin_start[bin + 1]; }

    long long acc[NG][VEC];
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[g][v] = 0;

    auto flush = [&](int b) {
#pragma unroll
        for (int g = 0; g < NG; ++g)
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
                const int f = f0 + g * SPAN + (VEC == 4 ? 4 * lane + v : lane);
                if (f < d && acc[g][v])
                    atomicAdd(reinterpret_cast<unsigned long long*>(&sums[(size_t)b * d + f]),
                              (unsigned long long)acc[g][v]);
                acc[g][v] = 0;
            }
    };

    for (long long e = e0; e < e1; e += U) {
        float x[U][NG][VEC];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const bool live = e + u < e1;
            const int row = live ? perm[e + u] : 0;
            const float* p = P + (size_t)row * d;
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                if (VEC == 4) {
                    const int f = f0 + g * SPAN + 4 * lane;
                    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (live && f < d) t = __ldg(reinterpret_cast<const float4*>(p + f));
                    x[u][g][0] = t.x; x[u][g][1] = t.y; x[u][g][2] = t.z; x[u][g][3] = t.w;
                } else {
                    const int f = f0 + g * SPAN + lane;
                    x[u][g][0] = (live && f < d) ? __ldg(p + f) : 0.f;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (e + u >= e1) break;
            while (e + u >= next) {       /* warp-uniform: every lane holds the same e */
                flush(bin);
                ++bin;
                next = bin_start[bin + 1];
            }
#pragma unroll
            for (int g = 0; g < NG; ++g)
#pragma unroll
                for (int v = 0; v < VEC; ++v) acc[g][v] += quantise(x[u][g][v], sc);
        }
    }
    flush(bin);
}

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

template <int VEC>
void launch_segsum_window(const float* P, int d, int f0, int ng, const int* perm, const int* bin_start, int k,
                          const DevParams* prm, long long* sums, int blocks, cudaStream_t s) {
    switch (ng) {
        case 1:
            if (d <= 64) k_segsum<VEC, 1, 8><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums);
            else k_segsum<VEC, 1><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums);
            break;
        case 2: k_segsum<VEC, 2><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums); break;
        case 3: k_segsum<VEC, 3><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums); break;
        case 4: k_segsum<VEC, 4><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums); break;
        case 5: k_segsum<VEC, 5><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums); break;
        case 6: k_segsum<VEC, 6><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums); break;
        case 7: k_segsum<VEC, 7><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums); break;
        default: k_segsum<VEC, 8><<<blocks, 256, 0, s>>>(P, d, f0, perm, bin_start, k, prm, sums); break;
    }
}

/* One launch per window of up to 8 groups of features. */
template <int VEC>
int launch_segsum(const float* P, int d, const int* perm, const int* bin_start, int k, const DevParams* prm,
                  long long* sums, int blocks, cudaStream_t s) {
    constexpr int WIN = 8 * 32 * VEC;
    int launches = 0;
    for (int f0 = 0; f0 < d; f0 += WIN, ++launches) {
        const int ng = ceil_div(min(WIN, d - f0), 32 * VEC);
        launch_segsum_window<VEC>(P, d, f0, ng, perm, bin_start, k, prm, sums, blocks, s);
    }
    return launches;
}

}  /* namespace */

int launch_update_sorted(const float* P, long long n, int d, const int* labels, int k, DevParams* prm,
                         long long* sums, long long* counts, UpdateScratch sc, int num_sms, cudaStream_t s) {
    cudaMemsetAsync(sc.hist, 0, sizeof(int) * (size_t)k, s);
    const bool smem = k <= kSmemHistMax;
    const size_t hb = smem ? sizeof(int) * (size_t)k : 0;
    if (hb > 48 * 1024) {
        cudaFuncSetAttribute(k_label_hist<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hb);
        cudaFuncSetAttribute(k_label_scatter<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hb);
    }
    const int blocks = num_sms * 4;
    if (n > 0) {
        if (smem) k_label_hist<true><<<blocks, 512, hb, s>>>(labels, n, k, sc.hist, prm);
        else k_label_hist<false><<<blocks, 512, 0, s>>>(labels, n, k, sc.hist, prm);
    }
    k_bin_scan<<<1, 1024, 0, s>>>(sc.hist, k, sc.bin_start, sc.cursor, counts);
    if (n <= 0) return 1;
    const long long rpb = (n + blocks - 1) / blocks;
    if (smem) k_label_scatter<true><<<blocks, 512, hb, s>>>(labels, n, k, sc.cursor, sc.perm, rpb);
    else k_label_scatter<false><<<blocks, 512, 0, s>>>(labels, n, k, sc.cursor, sc.perm, rpb);
    const bool vec = (d % 4 == 0) && ((reinterpret_cast<uintptr_t>(P) & 15) == 0);
    /* eight warps a block; at least 32 rows a warp, so that a small problem does not pay
     * a bin search and a flush of atomics for every handful of rows */
    const int sblocks = (int)std::max<long long>(1, std::min<long long>((long long)num_sms * 8, (n + 255) / 256));
    const int seg = vec ? launch_segsum<4>(P, d, sc.perm, sc.bin_start, k, prm, sums, sblocks, s)
                        : launch_segsum<1>(P, d, sc.perm, sc.bin_start, k, prm, sums, sblocks, s);
    return 3 + seg;                       /* hist, scan, scatter, segmented sums */
}

}  /* namespace mpk */
