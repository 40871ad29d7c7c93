/* assign_tc.cu -- fused split-precision distance GEMM + row argmin (sm_100a).
 *
 * Replaces, for the Lloyd assignment step, the reference's
 *   cublasGemmEx FP16 -> G (n x k in HBM)      kmeans/src/mpkmeans.cu:477-488
 *   k_argmin_count (argmin + exclusion test)    kmeans/src/kernels.cu:264-547
 * with one persistent kernel in which the n x k distance matrix never leaves
 * the SM:
 *
 *   warp 0      TMA producer: the 128-row tile of the point planes (hi, lo) is
 *               loaded once per tile and stays resident; centroid planes
 *               stream through a ring of 64-wide K chunks.
 *   warp 1      MMA issuer: per 128 x BN output tile, for every K chunk,
 *               hi*hi + lo*hi + hi*lo as tcgen05.mma kind::f16 (FP16
 *               operands, FP32 accumulation) into a double-buffered TMEM
 *               accumulator.
 *   warps 2-5   epilogue: tcgen05.ld of the accumulator, D = ||c||^2 - 2 x.c
 *               (the ||x||^2 term is a per-row constant and is dropped, as in
 *               the reference), and a running top-4 (value, index) per row.
 *
 * After the last centroid tile of a row tile, every row writes its argmin.  A
 * row whose runner-up lies within the certified error bound T of the best is
 * appended to the refinement list with every top-4 candidate inside T (and an
 * overflow mark when the 4th is also inside T, in which case the refinement
 * scans all k).  The bound covers (a) the FP16x2 split and the dropped lo*lo
 * term, (b) the tensor-core FP32 accumulation, (c) the rounding of the FP32
 * distance that any FP32 evaluation of ||c||^2 - 2 x.c would make; so a row
 * that is not refined has the same argmin under any FP32 summation order, and
 * a refined row gets the exact FP32 answer from the refinement kernel.
 */
#include "engine.cuh"

#include <cstdio>

namespace mpk {
namespace {

constexpr int BM = 128;
constexpr int KC = 64;                  /* FP16 elements per 128-byte swizzle row */
constexpr int ROW_BYTES = 128;
constexpr int kThreads = 192;           /* 6 warps */
constexpr int kSmemBudget = 224 * 1024;

template <int BN, int NKC>
struct Cfg {
    static constexpr int A_CHUNK = BM * ROW_BYTES;            /* one plane, one K chunk */
    static constexpr int A_TILE = 2 * NKC * A_CHUNK;          /* hi + lo                */
    static constexpr int B_STAGE = BN * ROW_BYTES;
    static constexpr int A_BUFS = (2 * A_TILE + 2 * B_STAGE <= kSmemBudget) ? 2 : 1;
    static constexpr int B_RAW = (kSmemBudget - A_BUFS * A_TILE) / B_STAGE;
    static constexpr int B_STAGES = B_RAW > 8 ? 8 : B_RAW;
    static constexpr int SMEM_BYTES = A_BUFS * A_TILE + B_STAGES * B_STAGE + 1024;
    static constexpr int TMEM_COLS = 2 * BN;
    static_assert(B_STAGES >= 2, "shared memory too small for two B stages");
    static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512, "TMEM columns");
};

__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, status) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

/* Bounded wait that ignores the abort flag (used to drain in-flight work). */
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > kWaitLimitNs) return;
    }
}

template <int BN, int NKC>
__global__ void __launch_bounds__(kThreads, 1)
k_assign_tc(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmC,
            long long n, int k, const float* __restrict__ xnorm, const float* __restrict__ cn,
            DevParams* __restrict__ prm, int* __restrict__ labels, RefineEntry* __restrict__ list,
            int refine, BoundConsts bc, float4* __restrict__ dbg) {
    using Cf = Cfg<BN, NKC>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smA = smem;
    uint8_t* smB = smem + Cf::A_BUFS * Cf::A_TILE;

    __shared__ __align__(8) uint64_t a_full[2], a_empty[2], b_full[8], b_empty[8], t_full[2], t_empty[2], fin_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    __shared__ float s_wmax[kThreads / 32];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long num_mt = (n + BM - 1) / BM;
    const int NT = (k + BN - 1) / BN;
    int* status = &prm->status;

    if (threadIdx.x == 0) {
        for (int i = 0; i < Cf::A_BUFS; ++i) { mbar_init(&a_full[i], 1); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < Cf::B_STAGES; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&t_full[i], 1); mbar_init(&t_empty[i], 128); }
        mbar_init(&fin_bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmX); tma_prefetch_desc(&tmC); }
    if (warp == 1) tmem_alloc(&tmem_slot, Cf::TMEM_COLS);

    /* max_j ||c_j||, for the error bound; cn holds ||c_j||^2 */
    {
        float m = 0.f;
        for (int j = threadIdx.x; j < k; j += kThreads) m = fmaxf(m, cn[j]);
        m = warp_max(m);
        if (lane == 0) s_wmax[warp] = m;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_slot;

    if (warp == 0) {
        /* ------------------------------------------------ TMA producer --- */
        if (lane == 0) {
            uint32_t a_last[2] = {0xffffffffu, 0xffffffffu};
            uint32_t b_last[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) b_last[i] = 0xffffffffu;
            uint32_t bs = 0;
            int lt = 0;
            bool ok = true;
            for (long long mt = blockIdx.x; mt < num_mt && ok; mt += gridDim.x, ++lt) {
                const int ab = lt % Cf::A_BUFS;
                const uint32_t au = (uint32_t)(lt / Cf::A_BUFS);
                if (!mbar_wait(&a_empty[ab], (au & 1u) ^ 1u, &abort_flag, status)) { ok = false; break; }
                mbar_expect_tx(&a_full[ab], Cf::A_TILE);
                a_last[ab] = au;
                for (int p = 0; p < 2; ++p)
                    for (int kc = 0; kc < NKC; ++kc)
                        tma_load_3d(&tmX, &a_full[ab], smA + ab * Cf::A_TILE + (p * NKC + kc) * Cf::A_CHUNK,
                                    kc * KC, (int)(mt * BM), p);
                for (int nt = 0; nt < NT && ok; ++nt)
                    for (int kc = 0; kc < NKC && ok; ++kc)
                        for (int p = 0; p < 2; ++p) {
                            const int st = (int)(bs % Cf::B_STAGES);
                            const uint32_t bu = bs / Cf::B_STAGES;
                            if (!mbar_wait(&b_empty[st], (bu & 1u) ^ 1u, &abort_flag, status)) { ok = false; break; }
                            mbar_expect_tx(&b_full[st], Cf::B_STAGE);
                            b_last[st] = bu;
                            tma_load_3d(&tmC, &b_full[st], smB + st * Cf::B_STAGE, kc * KC, nt * BN, p);
                            ++bs;
                        }
            }
            if (!ok) {
                /* let every load already issued land before the CTA exits */
                for (int i = 0; i < Cf::A_BUFS; ++i)
                    if (a_last[i] != 0xffffffffu) drain_wait(&a_full[i], a_last[i] & 1u);
                for (int i = 0; i < Cf::B_STAGES; ++i)
                    if (b_last[i] != 0xffffffffu) drain_wait(&b_full[i], b_last[i] & 1u);
            }
        }
    } else if (warp == 1) {
        /* ------------------------------------------------- MMA issuer ---- */
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(BM, BN, 0, 0, 0);
            uint32_t bs = 0, ts = 0;
            int lt = 0;
            bool ok = true;
            for (long long mt = blockIdx.x; mt < num_mt && ok; mt += gridDim.x, ++lt) {
                const int ab = lt % Cf::A_BUFS;
                const uint32_t au = (uint32_t)(lt / Cf::A_BUFS);
                if (!mbar_wait(&a_full[ab], au & 1u, &abort_flag, status)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smA + ab * Cf::A_TILE);
                for (int nt = 0; nt < NT && ok; ++nt, ++ts) {
                    const int tb = (int)(ts & 1u);
                    const uint32_t tu = ts >> 1;
                    if (!mbar_wait(&t_empty[tb], (tu & 1u) ^ 1u, &abort_flag, status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + (uint32_t)(tb * BN);
                    uint32_t accum = 0;
                    for (int kc = 0; kc < NKC && ok; ++kc) {
                        const uint32_t ah = a_addr + (uint32_t)(kc * Cf::A_CHUNK);
                        const uint32_t al = a_addr + (uint32_t)((NKC + kc) * Cf::A_CHUNK);
                        /* centroid hi plane: x_hi * c_hi and x_lo * c_hi */
                        int st = (int)(bs % Cf::B_STAGES);
                        uint32_t bu = bs / Cf::B_STAGES;
                        if (!mbar_wait(&b_full[st], bu & 1u, &abort_flag, status)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t bh = smem_u32(smB + st * Cf::B_STAGE);
#pragma unroll
                        for (int ks = 0; ks < KC / 16; ++ks) {
                            umma_f16(d_tmem, sw128_desc(ah + ks * 32, 16, 1024), sw128_desc(bh + ks * 32, 16, 1024),
                                     idesc, accum);
                            accum = 1;
                        }
#pragma unroll
                        for (int ks = 0; ks < KC / 16; ++ks)
                            umma_f16(d_tmem, sw128_desc(al + ks * 32, 16, 1024), sw128_desc(bh + ks * 32, 16, 1024),
                                     idesc, 1);
                        umma_commit(&b_empty[st]);
                        ++bs;
                        /* centroid lo plane: x_hi * c_lo */
                        st = (int)(bs % Cf::B_STAGES);
                        bu = bs / Cf::B_STAGES;
                        if (!mbar_wait(&b_full[st], bu & 1u, &abort_flag, status)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t bl = smem_u32(smB + st * Cf::B_STAGE);
#pragma unroll
                        for (int ks = 0; ks < KC / 16; ++ks)
                            umma_f16(d_tmem, sw128_desc(ah + ks * 32, 16, 1024), sw128_desc(bl + ks * 32, 16, 1024),
                                     idesc, 1);
                        umma_commit(&b_empty[st]);
                        ++bs;
                    }
                    if (ok) umma_commit(&t_full[tb]);
                }
                if (ok) umma_commit(&a_empty[ab]);
            }
            /* every MMA issued by this thread has completed once fin_bar flips */
            umma_commit(&fin_bar);
            drain_wait(&fin_bar, 0);
        }
    } else {
        /* --------------------------------------------------- epilogue ---- */
        const int q = warp & 3;                       /* TMEM lane quarter */
        const int r_loc = q * 32 + lane;
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
        const float ns = prm->neg2_inv_s2;
        const float eta = prm->eta;
        float cmax = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) cmax = fmaxf(cmax, s_wmax[w]);
        cmax = sqrtf(cmax);
        uint32_t ts = 0;
        bool ok = true;
        for (long long mt = blockIdx.x; mt < num_mt && ok; mt += gridDim.x) {
            float v0 = INFINITY, v1 = INFINITY, v2 = INFINITY, v3 = INFINITY;
            int j0 = -1, j1 = -1, j2 = -1, j3 = -1;
            for (int nt = 0; nt < NT; ++nt, ++ts) {
                const int tb = (int)(ts & 1u);
                const uint32_t tu = ts >> 1;
                if (!wait_warp(&t_full[tb], tu & 1u, &abort_flag, status)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(t_lane + (uint32_t)(tb * BN + c * 32), r);
                    tmem_ld_wait();
                    const int jb = nt * BN + c * 32;
                    const float4* cn4 = reinterpret_cast<const float4*>(cn + jb);
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const float4 cc = __ldg(cn4 + u);
                        const float cv[4] = {cc.x, cc.y, cc.z, cc.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float D = fmaf(__uint_as_float(r[4 * u + e]), ns, cv[e]);
                            if (D < v3) {
                                const int jj = jb + 4 * u + e;
                                if (D < v2) {
                                    v3 = v2; j3 = j2;
                                    if (D < v1) {
                                        v2 = v1; j2 = j1;
                                        if (D < v0) { v1 = v0; j1 = j0; v0 = D; j0 = jj; }
                                        else { v1 = D; j1 = jj; }
                                    } else { v2 = D; j2 = jj; }
                                } else { v3 = D; j3 = jj; }
                            }
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&t_empty[tb]);
            }
            if (!ok) break;

            const long long row = mt * BM + r_loc;
            bool flag = false;
            int ovf = 0, c1 = -1, c2 = -1, c3 = -1;
            if (row < n) {
                labels[row] = j0;
                if (dbg) dbg[row] = make_float4(v0, v1, __int_as_float(j0), __int_as_float(j1));
                if (refine && j1 >= 0) {
                    const float xn = xnorm[row];
                    const float T0 = bc.c1 * xn * cmax + bc.c2 * eta * (xn + cmax);
                    const float av0 = fabsf(v0);
                    const float t1 = (T0 + 0x1.0p-22f * (fabsf(v1) + av0)) * (1.0f + 0x1.0p-20f);
                    flag = (v1 - v0) <= t1;
                    if (flag) {
                        c1 = j1;
                        if (j2 >= 0 && (v2 - v0) <= (T0 + 0x1.0p-22f * (fabsf(v2) + av0)) * (1.0f + 0x1.0p-20f)) c2 = j2;
                        if (j3 >= 0 && (v3 - v0) <= (T0 + 0x1.0p-22f * (fabsf(v3) + av0)) * (1.0f + 0x1.0p-20f)) { c3 = j3; ovf = 1; }
                    }
                }
            }
            const unsigned m = __ballot_sync(0xffffffffu, flag);
            if (m) {
                unsigned base = 0;
                if (lane == 0) base = atomicAdd(&prm->nflag, (unsigned)__popc(m));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (flag) {
                    RefineEntry e;
                    e.row = (int)row;
                    e.ovf = ovf;
                    e.c[0] = j0; e.c[1] = c1; e.c[2] = c2; e.c[3] = c3;
                    list[base + __popc(m & ((1u << lane) - 1u))] = e;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cf::TMEM_COLS);
    }
}

template <int BN, int NKC>
cudaError_t launch_t(const AssignArgs& a, cudaStream_t s) {
    using Cf = Cfg<BN, NKC>;
    auto kern = k_assign_tc<BN, NKC>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const long long num_mt = (a.n + BM - 1) / BM;
    const int grid = (int)(num_mt < a.num_sms ? num_mt : a.num_sms);
    kern<<<grid, kThreads, Cf::SMEM_BYTES, s>>>(*a.tmX, *a.tmC, a.n, a.k, a.xnorm, a.cn, a.prm, a.labels,
                                                 a.list, a.refine, a.bc, a.dbg);
    return cudaGetLastError();
}

template <int BN>
cudaError_t launch_bn(const AssignArgs& a, cudaStream_t s) {
    switch (a.dp / KC) {
        case 1: return launch_t<BN, 1>(a, s);
        case 2: return launch_t<BN, 2>(a, s);
        case 3: return launch_t<BN, 3>(a, s);
        case 4: return launch_t<BN, 4>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  /* namespace */

int assign_bn_for(int k) { return k <= 64 ? 64 : (k <= 128 ? 128 : 256); }
int assign_supported(int d) { return d >= 1 && d <= 4 * KC; }

cudaError_t launch_assign(const AssignArgs& a, cudaStream_t s) {
    if (a.n <= 0) return cudaSuccess;
    switch (assign_bn_for(a.k)) {
        case 64: return launch_bn<64>(a, s);
        case 128: return launch_bn<128>(a, s);
        default: return launch_bn<256>(a, s);
    }
}

}  /* namespace mpk */
