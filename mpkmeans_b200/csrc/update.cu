/* update.cu -- exact segmented-sum centroid update.
 *
 * Replaces the reference's mpkLaunchZero / mpkLaunchAccumulate
 * (kmeans/src/kernels.cu:683-703: one FP64 global atomic per coordinate) with
 * a counting sort of the rows by label followed by a segmented sum:
 *
 *   k_label_hist     labels -> per-cluster counts (shared-memory histogram)
 *   k_bin_scan       counts -> bin starts; counts written to the sums buffer
 *   k_label_scatter_local   row indices grouped by label (perm): each block
 *                    sorts 8192-row chunks in shared memory and writes every
 *                    label's run contiguously (k <= 4096; k_label_scatter,
 *                    row by row, above)
 *   k_segsum         each warp walks a contiguous run of perm over one
 *                    128-feature slice of the rows (coalesced, 16 B per lane),
 *                    quantising every coordinate once to q = rint(x * 2^frac)
 *                    and adding into int64 registers; at a label boundary (and
 *                    at the end of its run) the warp adds its registers into
 *                    the global int64 sums.
 *
 * Integer sums are exact, so the result does not depend on the order of the
 * rows within a cluster, on the split of the work, or on the number of GPUs
 * whose buffers are later summed; the points are read from HBM once.  The
 * same exactness lets the refinement run beside the segmented sum:
 * k_refine_snapshot keeps the listed rows' labels before it, and
 * k_refine_correct moves every row it relabelled between the clusters'
 * sums and counts afterwards.
 */
#include "engine.cuh"

namespace mpk {
namespace {

constexpr int kSmemHistMax = 48 * 1024;   /* labels per shared-memory histogram */
constexpr unsigned FULL = 0xffffffffu;

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

/* The scatter with coalesced writes (k <= kLocalSortMaxK): each block sorts
 * its rows by label in chunks of kChunkRows in shared memory (a counting sort:
 * local histogram, local starts, one global reservation per label and chunk
 * from the cursors, placement), then writes each label's run of row indices
 * to its reserved slots in order, so consecutive threads write consecutive
 * perm entries.  (Scattering row by row writes one isolated 4-byte word per
 * row.)  Shared memory: 2k ints + kChunkRows (int + short). */
constexpr int kLocalSortMaxK = 4096;
constexpr int kChunkRows = 8192;
constexpr int kScatterThreads = 512;

__global__ void __launch_bounds__(kScatterThreads)
k_label_scatter_local(const int* __restrict__ labels, long long n, int k, int* __restrict__ cursor,
                      int* __restrict__ perm, long long rows_per_block) {
    extern __shared__ int sm[];
    int* cnt = sm;                                   /* k: counts, then run starts, then run ends */
    int* gb = sm + k;                                /* k: global slot of each run's first row */
    int* idx = gb + k;                               /* kChunkRows row indices, sorted by label */
    unsigned short* lab = reinterpret_cast<unsigned short*>(idx + kChunkRows);
    __shared__ int part[kScatterThreads / 32];
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    const long long r0 = min(n, (long long)blockIdx.x * rows_per_block);
    const long long r1 = min(n, r0 + rows_per_block);
    const int per = (k + kScatterThreads - 1) / kScatterThreads;
    const int j0 = min(k, t * per), j1 = min(k, j0 + per);
    for (long long c0 = r0; c0 < r1; c0 += kChunkRows) {
        const int m = (int)min((long long)kChunkRows, r1 - c0);
        for (int j = t; j < k; j += kScatterThreads) cnt[j] = 0;
        __syncthreads();
        for (int i = t; i < m; i += kScatterThreads) {
            const int a = labels[c0 + i];
            if ((unsigned)a < (unsigned)k) atomicAdd(&cnt[a], 1);
        }
        __syncthreads();
        /* exclusive scan of the counts (thread t owns labels [j0, j1)), and the reservations */
        int sum = 0;
        for (int j = j0; j < j1; ++j) sum += cnt[j];
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(FULL, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) part[w] = incl;
        __syncthreads();
        int run = incl - sum;
        for (int q = 0; q < w; ++q) run += part[q];
        for (int j = j0; j < j1; ++j) {
            const int c = cnt[j];
            cnt[j] = run;
            gb[j] = c ? atomicAdd(&cursor[j], c) : 0;
            run += c;
        }
        __syncthreads();
        for (int i = t; i < m; i += kScatterThreads) {
            const int a = labels[c0 + i];
            if ((unsigned)a < (unsigned)k) {
                const int q = atomicAdd(&cnt[a], 1);
                idx[q] = (int)(c0 + i);
                lab[q] = (unsigned short)a;
            }
        }
        __syncthreads();
        /* cnt[j] is now the end of run j, the start of run j + 1 */
        const int total = cnt[k - 1];
        for (int q = t; q < total; q += kScatterThreads) {
            const int a = lab[q];
            const int st = a ? cnt[a - 1] : 0;
            perm[gb[a] + (q - st)] = idx[q];
        }
        __syncthreads();
    }
}

__device__ __forceinline__ long long quantise(float x, float sc) {
    /* x * 2^frac is exact in FP32 (a power-of-two scale that cannot overflow
     * by the choice of frac); the conversion rounds to nearest, ties even. */
    return __float2ll_rn(x * sc);
}

/* Segmented sum over the label-sorted rows, one feature slice per warp: slice
 * blockIdx.y covers features [y * SPAN, (y + 1) * SPAN), SPAN = 32 * VEC.
 * VEC = 4: lane l owns features 4l..4l+3 of the slice (float4 loads); VEC = 1:
 * lane l owns feature l.  Wide rows are thus read by several warps at once,
 * each a 512-byte (or 128-byte) piece, rather than by one warp with fewer
 * rows in flight.
 *
 * A warp walks its contiguous run of perm 32 entries at a time: lane l loads
 * entry e + l (one coalesced load, issued a chunk ahead), and the row indices
 * reach the loads by shuffle, so no row load waits on a perm load; U = 8 rows
 * are loaded at once. */
template <int VEC, int U = 8>
__global__ void __launch_bounds__(256, 4)
k_segsum(const float* __restrict__ P, int d, const int* __restrict__ perm, const int* __restrict__ bin_start,
         int k, const DevParams* __restrict__ prm, long long* __restrict__ sums) {
    static_assert(32 % U == 0, "row batches tile a chunk of 32 entries");
    constexpr int SPAN = 32 * VEC;                 /* features per slice */
    const int lane = threadIdx.x & 31;
    const int f = blockIdx.y * SPAN + (VEC == 4 ? 4 * lane : lane);   /* this lane's first feature */
    const bool has = f < d;
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

    long long acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = 0;

    auto flush = [&](int b) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
            if (has && acc[v])
                atomicAdd(reinterpret_cast<unsigned long long*>(&sums[(size_t)b * d + f + v]),
                          (unsigned long long)acc[v]);
            acc[v] = 0;
        }
    };

    int idx = e0 + lane < e1 ? perm[e0 + lane] : 0;
    for (long long e = e0; e < e1; e += 32) {
        const int cnt = (int)min(32LL, e1 - e);
        const int cur = idx;
        idx = e + 32 + lane < e1 ? perm[e + 32 + lane] : 0;      /* the next chunk's entries */
#pragma unroll 1
        for (int u0 = 0; u0 < cnt; u0 += U) {
            float x[U][VEC];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const bool live = has && u0 + u < cnt;
                const float* p = P + (size_t)__shfl_sync(FULL, cur, (u0 + u) & 31) * d + f;
                if constexpr (VEC == 4) {
                    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (live) t = __ldg(reinterpret_cast<const float4*>(p));
                    x[u][0] = t.x; x[u][1] = t.y; x[u][2] = t.z; x[u][3] = t.w;
                } else {
                    x[u][0] = live ? __ldg(p) : 0.f;
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (u0 + u >= cnt) break;
                while (e + u0 + u >= next) {   /* warp-uniform: every lane holds the same entry */
                    flush(bin);
                    ++bin;
                    next = bin_start[bin + 1];
                }
#pragma unroll
                for (int v = 0; v < VEC; ++v) acc[v] += quantise(x[u][v], sc);
            }
        }
    }
    flush(bin);
}

/* The listed rows' labels as the assignment left them (before the refinement
 * may change them): old[e] = labels[list[e].row], e < nflag. */
__global__ void k_refine_snapshot(const RefineEntry* __restrict__ list, const DevParams* __restrict__ prm,
                                  const int* __restrict__ labels, int* __restrict__ old, long long cap) {
    const long long nf = min((long long)prm->nflag, cap);
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < nf; e += (long long)gridDim.x * blockDim.x)
        old[e] = labels[list[e].row];
}

/* After the refinement: every listed row whose label it changed from a to b
 * moves its fixed-point coordinates from cluster a's sums to b's and one count
 * with them.  One thread checks each entry; the warp then moves its changed
 * rows one at a time, its lanes over the row's features.  Integer adds
 * commute, so this may run beside the segmented sum of the same update, and
 * the result equals an update from the refined labels exactly. */
__global__ void k_refine_correct(const float* __restrict__ P, int d, const RefineEntry* __restrict__ list,
                                 const DevParams* __restrict__ prm, const int* __restrict__ labels,
                                 const int* __restrict__ old, long long cap, int k, long long* __restrict__ sums) {
    const long long nf = min((long long)prm->nflag, cap);
    const int lane = threadIdx.x & 31;
    const long long nthr = (long long)gridDim.x * blockDim.x;
    const float sc = ldexpf(1.0f, prm->frac);
    long long* counts = sums + (size_t)k * d;
    /* warp-uniform trip count: every lane of a warp runs the same bases */
    for (long long base = (long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31); base < nf; base += nthr) {
        const long long e = base + lane;
        int row = 0, a = 0, b = 0;
        bool moved = false;
        if (e < nf) {
            row = list[e].row;
            a = old[e];
            b = labels[row];
            moved = a != b && (unsigned)a < (unsigned)k && (unsigned)b < (unsigned)k;
        }
        unsigned m = __ballot_sync(FULL, moved);
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const int r = __shfl_sync(FULL, row, src), ra = __shfl_sync(FULL, a, src), rb = __shfl_sync(FULL, b, src);
            const float* p = P + (size_t)r * d;
            for (int f = lane; f < d; f += 32) {
                const long long q = quantise(p[f], sc);
                if (q) {
                    atomicAdd(reinterpret_cast<unsigned long long*>(&sums[(size_t)rb * d + f]), (unsigned long long)q);
                    atomicAdd(reinterpret_cast<unsigned long long*>(&sums[(size_t)ra * d + f]), (unsigned long long)(-q));
                }
            }
            if (lane == 0) {
                atomicAdd(reinterpret_cast<unsigned long long*>(&counts[rb]), 1ull);
                atomicAdd(reinterpret_cast<unsigned long long*>(&counts[ra]), ~0ull);   /* -1 */
            }
        }
    }
}

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

}  /* namespace */

int launch_update_sort(long long n, const int* labels, int k, DevParams* prm, long long* counts, UpdateScratch sc,
                       int num_sms, cudaStream_t s) {
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
    if (k <= kLocalSortMaxK) {
        const size_t sb = 2 * sizeof(int) * (size_t)k + (size_t)kChunkRows * (sizeof(int) + sizeof(short));
        if (sb > 48 * 1024) cudaFuncSetAttribute(k_label_scatter_local, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sb);
        /* as many blocks as fit a SM (four at k = 1024), each chunk's phases latency-bound */
        const int sblocks = num_sms * std::max(1, std::min(4, (int)((227 * 1024) / (sb + 1024))));
        const long long srpb = (n + sblocks - 1) / sblocks;
        k_label_scatter_local<<<sblocks, kScatterThreads, sb, s>>>(labels, n, k, sc.cursor, sc.perm, srpb);
        return 3;
    }
    const long long rpb = (n + blocks - 1) / blocks;
    if (smem) k_label_scatter<true><<<blocks, 512, hb, s>>>(labels, n, k, sc.cursor, sc.perm, rpb);
    else k_label_scatter<false><<<blocks, 512, 0, s>>>(labels, n, k, sc.cursor, sc.perm, rpb);
    return 3;                             /* hist, scan, scatter */
}

int launch_update_sum(const float* P, long long n, int d, int k, DevParams* prm, long long* sums, UpdateScratch sc,
                      int num_sms, cudaStream_t s, bool leave_room) {
    if (n <= 0) return 0;
    const bool vec = (d % 4 == 0) && ((reinterpret_cast<uintptr_t>(P) & 15) == 0);
    /* eight warps a block, over all feature slices about eight blocks per SM (two waves of
     * four, which fill the register file); leave_room: one wave of three blocks per SM, so
     * that a kernel running beside it (the refinement) keeps a block's worth of each SM.
     * At least 32 rows a warp, so that a small problem does not pay a bin search and a
     * flush of atomics for every handful of rows. */
    const int ny = ceil_div(d, vec ? 128 : 32);
    const long long want = std::max<long long>(1, (long long)num_sms * (leave_room ? 3 : 8) / ny);   /* whole waves */
    const dim3 grid((unsigned)std::max<long long>(1, std::min<long long>(want, (n + 255) / 256)), (unsigned)ny);
    if (vec) k_segsum<4><<<grid, 256, 0, s>>>(P, d, sc.perm, sc.bin_start, k, prm, sums);
    else k_segsum<1><<<grid, 256, 0, s>>>(P, d, sc.perm, sc.bin_start, k, prm, sums);
    return 1;
}

int launch_update_sorted(const float* P, long long n, int d, const int* labels, int k, DevParams* prm,
                         long long* sums, long long* counts, UpdateScratch sc, int num_sms, cudaStream_t s) {
    const int a = launch_update_sort(n, labels, k, prm, counts, sc, num_sms, s);
    return a + launch_update_sum(P, n, d, k, prm, sums, sc, num_sms, s, false);
}

int launch_refine_snapshot(const RefineEntry* list, const DevParams* prm, const int* labels, int* old, long long cap,
                           int num_sms, cudaStream_t s) {
    k_refine_snapshot<<<num_sms * 2, 256, 0, s>>>(list, prm, labels, old, cap);
    return 1;
}

int launch_refine_correct(const float* P, int d, const RefineEntry* list, const DevParams* prm, const int* labels,
                          const int* old, long long cap, int k, long long* sums, int num_sms, cudaStream_t s) {
    k_refine_correct<<<num_sms * 2, 256, 0, s>>>(P, d, list, prm, labels, old, cap, k, sums);
    return 1;
}

}  /* namespace mpk */
