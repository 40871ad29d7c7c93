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
 *   warps 2-9   epilogue, two warps per TMEM lane quarter, each taking half
 *               the columns of a tile: tcgen05.ld of the accumulator,
 *               D = ||c||^2 - 2 x.c (fma.rn.f32x2 on column pairs; the ||x||^2
 *               term is a per-row constant and is dropped, as in the
 *               reference), and, without branches, for each of 8 column
 *               classes (column mod 8) the best value with its column and the
 *               runner-up value.
 *
 * The pair variant (k > 128) runs the same roles on a cluster of two
 * CTAs: CTA 0's MMA warp issues tcgen05.mma.cta_group::2 over 256 rows (128
 * from each CTA's point tile) and 256 centroids (each CTA stages 128), every
 * CTA's epilogue reads its own 128 rows of the accumulator from its own TMEM.
 *
 * After the last centroid tile of a row tile the two halves exchange their
 * summaries through shared memory and every row writes its argmin (smaller
 * index on ties).  A row whose runner-up lies within the certified error
 * bound T of the best is appended to the refinement list with every class
 * best inside T; when some class's runner-up is also inside T that class may
 * hold further candidates and the entry marks it for a scan of its columns.  The bound
 * covers (a) the FP16x2 split and the dropped lo*lo term, (b) the tensor-core
 * FP32 accumulation, (c) the rounding any FP32 evaluation of ||c||^2 - 2 x.c
 * makes; so an unrefined row has the same argmin under any FP32 summation
 * order, and a refined row gets the exact FP32 answer from the refinement.
 */
#include "engine.cuh"

namespace mpk {
namespace {

constexpr int BM = 128;
constexpr int KC = 64;                  /* FP16 elements per 128-byte swizzle row */
constexpr int ROW_BYTES = 128;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSmemMax = 232448;        /* 227 KB, no static shared memory */
constexpr int kMiscBytes = 2048;        /* barriers + the epilogue exchange */
constexpr int kClasses = 8;
constexpr int kMaxDim = 1 << 16;        /* TMA coordinates and the error-bound model */

/* NKC > 0: the point tile (hi, lo planes, NKC chunks of 64) stays resident
 * while every centroid tile streams past it.  NKC == 0 (d > 256): the point
 * chunks stream too, through their own ring of (hi, lo) stages, next to the
 * centroid ring.  PAIR: two CTAs on two SMs share every MMA (M = 256 rows,
 * 128 per CTA); each CTA stages only its half (BN / 2 centroids) of every
 * centroid tile, which halves the shared-memory and L2 traffic per MMA. */
template <int BN, int NKC, bool PAIR = false>
struct Cfg {
    static constexpr bool STREAM = NKC == 0;
    static constexpr int A_CHUNK = BM * ROW_BYTES;            /* one plane, one K chunk */
    static constexpr int A_TILE = STREAM ? 2 * A_CHUNK : 2 * NKC * A_CHUNK;   /* hi + lo: a tile or a stage */
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;         /* centroid rows a stage holds here */
    static constexpr int B_STAGE = B_ROWS * ROW_BYTES;
    static constexpr int BUDGET = kSmemMax - kMiscBytes;
    static constexpr int A_BUFS = STREAM ? 3 : ((2 * A_TILE + 3 * B_STAGE <= BUDGET) ? 2 : 1);
    static constexpr int B_RAW = (BUDGET - A_BUFS * A_TILE) / B_STAGE;
    static constexpr int B_STAGES = B_RAW > 8 ? 8 : B_RAW;
    static constexpr int TILE_BYTES = A_BUFS * A_TILE + B_STAGES * B_STAGE;
    static constexpr int SMEM_BYTES = TILE_BYTES + kMiscBytes;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int HALF = BN / 2;                       /* columns per epilogue warp */
    static constexpr int CHUNKS = HALF / 32;
    static_assert(B_STAGES >= 2, "shared memory too small for two B stages");
    static_assert(SMEM_BYTES <= kSmemMax, "shared memory");
    static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512, "TMEM columns");
    static_assert(HALF % 32 == 0, "epilogue half must be whole 32-column chunks");
    static_assert(!PAIR || BN == 256, "CTA pairs: 256-wide tiles");
};

/* Shared-memory block after the tiles. */
struct Misc {
    uint64_t a_full[4], a_empty[4], b_full[8], b_empty[8], t_full[2], t_empty[2], fin;
    uint32_t tmem_slot;
    int abort_flag;
    float wmax[kThreads / 32];
    /* Row r is exchanged by thread r of the two halves only.  Half 1 writes
     * (best value, runner-up, best column) before the first named barrier;
     * half 0 reads them and overwrites the same words with (row best, bound,
     * refinement slot) for half 1 before the second. */
    float xa[BM], xb[BM];
    int xc[BM];
};
static_assert(sizeof(Misc) <= kMiscBytes, "misc block");

__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          uint32_t lim) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, status, lim) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

/* Bounded wait that ignores the abort flag (used to drain in-flight work). */
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > kWaitLimitNs) return;
    }
}

__device__ __forceinline__ void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(count) : "memory");
}

/* Two FP32 fused multiply-adds in one instruction: (a0,a1)*(b,b)+(c0,c1). */
__device__ __forceinline__ void fma2(float a0, float a1, uint64_t bb, float c0, float c1, float& d0, float& d1) {
    uint64_t a, c, d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(c0), "f"(c1));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(bb), "l"(c));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ float thr_of(float T0, float v, float v0) {
    return (T0 + 0x1.0p-22f * (fabsf(v) + fabsf(v0))) * (1.0f + 0x1.0p-20f);
}

/* EMIT: the wide-refinement pass.  The rows are the first prm->nwide rows of
 * tmX (copies of wide rows' planes); instead of an argmin, every column whose
 * emulated value lies within the row's bound (v0, T0 from its refinement
 * entry) is written to the row's candidate list. */
template <int BN, int NKC, bool EMIT, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
k_assign_tc(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmC,
            long long n, int k, int nkc_rt, const float* __restrict__ xnorm, const float* __restrict__ cn,
            DevParams* __restrict__ prm, int* __restrict__ labels, RefineEntry* __restrict__ list,
            int refine, BoundConsts bc, float4* __restrict__ dbg, const int* __restrict__ went,
            int* __restrict__ cand, int* __restrict__ ccount, long long wbase, int stall_stage) {
    using Cf = Cfg<BN, NKC, PAIR>;
    static_assert(!(EMIT && PAIR), "the wide pass runs on single CTAs");
    /* limit of one wait (a test may shorten it to make a left-out stage time out quickly) */
    const uint32_t lim = (uint32_t)((!EMIT && prm->wait_ns ? prm->wait_ns : kWaitLimitNs) / 1000);   /* microseconds */
    if (EMIT) {
        /* this round's rows: queued rows [wbase, wbase + n) that exist */
        const long long nw = (long long)*reinterpret_cast<volatile unsigned int*>(&prm->nwide) - wbase;
        n = nw < n ? (nw > 0 ? nw : 0) : n;
    }
    static_assert(Cf::A_BUFS <= 4, "A ring");
    const int nkc = Cf::STREAM ? nkc_rt : NKC;   /* K chunks of 64 */
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* smA = smem;
    uint8_t* smB = smem + Cf::A_BUFS * Cf::A_TILE;
    Misc& ms = *reinterpret_cast<Misc*>(smem + Cf::TILE_BYTES);
    volatile int* abort_flag = &ms.abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    /* PAIR: the unit of work is a pair of 128-row tiles, 2 mt and 2 mt + 1,
     * the even one in the cluster's CTA 0; tiles go to clusters round robin */
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    const long long num_mt = PAIR ? (n + 2 * BM - 1) / (2 * BM) : (n + BM - 1) / BM;
    const long long mt0 = PAIR ? (long long)(blockIdx.x >> 1) : (long long)blockIdx.x;
    const long long mt_step = PAIR ? (long long)(gridDim.x >> 1) : (long long)gridDim.x;
    const int NT = (k + BN - 1) / BN;
    int* status = &prm->status;

    /* the 128-byte swizzle needs 1024-byte aligned tiles */
    if (smem_u32(smem) & 1023u) {
        if (threadIdx.x == 0) atomicOr(status, MPK_DEV_TIMEOUT);
        return;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < Cf::A_BUFS; ++i) { mbar_init(&ms.a_full[i], 1); mbar_init(&ms.a_empty[i], 1); }
        for (int i = 0; i < Cf::B_STAGES; ++i) { mbar_init(&ms.b_full[i], 1); mbar_init(&ms.b_empty[i], 1); }
        /* PAIR: CTA 0's t_empty counts one arrival per epilogue warp of both CTAs */
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ms.t_full[i], 1);
            mbar_init(&ms.t_empty[i], PAIR ? 2 * kEpiWarps : 32 * kEpiWarps);
        }
        mbar_init(&ms.fin, 1);
        ms.abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmX); tma_prefetch_desc(&tmC); }
    if (warp == 1) {
        if (PAIR) tmem_alloc_pair(&ms.tmem_slot, Cf::TMEM_COLS);
        else tmem_alloc(&ms.tmem_slot, Cf::TMEM_COLS);
    }

    /* max_j ||c_j||, for the error bound; cn holds ||c_j||^2 */
    {
        float m = 0.f;
        for (int j = threadIdx.x; j < k; j += kThreads) m = fmaxf(m, cn[j]);
        m = warp_max(m);
        if (lane == 0) ms.wmax[warp] = m;
    }
    tc_fence_before();
    if (PAIR) cluster_sync();       /* the peer's barriers are initialised before any remote signal */
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = ms.tmem_slot;

    if (warp == 0) {
        /* ------------------------------------------------ TMA producer --- */
        if (lane == 0) {
            uint32_t a_last[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
            uint32_t b_last[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) b_last[i] = 0xffffffffu;
            uint32_t bs = 0, as = 0;
            int lt = 0;
            bool ok = true;
            auto load_b = [&](int nt, int kc) {
                for (int p = 0; p < 2; ++p) {
                    const int st = (int)(bs % Cf::B_STAGES);
                    const uint32_t bu = bs / Cf::B_STAGES;
                    if (!mbar_wait(&ms.b_empty[st], (bu & 1u) ^ 1u, abort_flag, status, lim)) { ok = false; return; }
                    if (!EMIT && (int)bs == stall_stage) {    /* test hook: this stage is never loaded */
                        ++bs;
                        continue;
                    }
                    b_last[st] = bu;
                    if (PAIR) {
                        /* this CTA's half of the tile; CTA 0's barrier counts both halves */
                        if (rank == 0) mbar_expect_tx(&ms.b_full[st], 2 * Cf::B_STAGE);
                        tma_load_3d_pair(&tmC, peer_addr(&ms.b_full[st], 0), smB + st * Cf::B_STAGE, kc * KC,
                                         nt * BN + (int)rank * Cf::B_ROWS, p);
                    } else {
                        mbar_expect_tx(&ms.b_full[st], Cf::B_STAGE);
                        tma_load_3d(&tmC, &ms.b_full[st], smB + st * Cf::B_STAGE, kc * KC, nt * BN, p);
                    }
                    ++bs;
                }
            };
            for (long long mt = mt0; mt < num_mt && ok; mt += mt_step, ++lt) {
                if (Cf::STREAM) {
                    /* PAIR: as for the resident tile below, CTA 1 loads its chunks only when
                     * the pair's second tile holds rows */
                    const bool rows1 = (2 * mt + 1) * BM < n;
                    for (int nt = 0; nt < NT && ok; ++nt)
                        for (int kc = 0; kc < nkc && ok; ++kc, ++as) {
                            const int ab = (int)(as % Cf::A_BUFS);
                            const uint32_t au = as / Cf::A_BUFS;
                            if (!mbar_wait(&ms.a_empty[ab], (au & 1u) ^ 1u, abort_flag, status, lim)) { ok = false; break; }
                            a_last[ab] = au;
                            if (PAIR) {
                                if (rank == 0) mbar_expect_tx(&ms.a_full[ab], (rows1 ? 2 : 1) * Cf::A_TILE);
                                if (rank == 0 || rows1)
                                    for (int p = 0; p < 2; ++p)
                                        tma_load_3d_pair(&tmX, peer_addr(&ms.a_full[ab], 0),
                                                         smA + ab * Cf::A_TILE + p * Cf::A_CHUNK, kc * KC,
                                                         (int)((2 * mt + rank) * BM), p);
                            } else {
                                mbar_expect_tx(&ms.a_full[ab], Cf::A_TILE);
                                for (int p = 0; p < 2; ++p)
                                    tma_load_3d(&tmX, &ms.a_full[ab], smA + ab * Cf::A_TILE + p * Cf::A_CHUNK,
                                                kc * KC, (int)(mt * BM), p);
                            }
                            load_b(nt, kc);
                        }
                    continue;
                }
                const int ab = lt % Cf::A_BUFS;
                const uint32_t au = (uint32_t)(lt / Cf::A_BUFS);
                if (!mbar_wait(&ms.a_empty[ab], (au & 1u) ^ 1u, abort_flag, status, lim)) { ok = false; break; }
                a_last[ab] = au;
                if (PAIR) {
                    /* CTA 1 loads its rows only when the pair's second tile holds any (its
                     * MMA rows are then never read); CTA 0's barrier counts both tiles */
                    const bool rows1 = (2 * mt + 1) * BM < n;
                    if (rank == 0) mbar_expect_tx(&ms.a_full[ab], (rows1 ? 2 : 1) * Cf::A_TILE);
                    if (rank == 0 || rows1)
                        for (int p = 0; p < 2; ++p)
                            for (int kc = 0; kc < nkc; ++kc)
                                tma_load_3d_pair(&tmX, peer_addr(&ms.a_full[ab], 0),
                                                 smA + ab * Cf::A_TILE + (p * nkc + kc) * Cf::A_CHUNK, kc * KC,
                                                 (int)((2 * mt + rank) * BM), p);
                } else {
                    mbar_expect_tx(&ms.a_full[ab], Cf::A_TILE);
                    for (int p = 0; p < 2; ++p)
                        for (int kc = 0; kc < nkc; ++kc)
                            tma_load_3d(&tmX, &ms.a_full[ab], smA + ab * Cf::A_TILE + (p * nkc + kc) * Cf::A_CHUNK,
                                        kc * KC, (int)(mt * BM), p);
                }
                for (int nt = 0; nt < NT && ok; ++nt)
                    for (int kc = 0; kc < nkc && ok; ++kc) load_b(nt, kc);
            }
            if (!ok && !PAIR) {
                /* let every load already issued land before the CTA exits */
                for (int i = 0; i < Cf::A_BUFS; ++i)
                    if (a_last[i] != 0xffffffffu) drain_wait(&ms.a_full[i], a_last[i] & 1u);
                for (int i = 0; i < Cf::B_STAGES; ++i)
                    if (b_last[i] != 0xffffffffu) drain_wait(&ms.b_full[i], b_last[i] & 1u);
            } else if (!ok) {
                /* a pair's loads complete on CTA 0's barriers, which CTA 1 cannot
                 * wait on, and a phase CTA 0 never armed does not complete: give
                 * every load in flight a fixed time (each takes microseconds) */
                const unsigned long long t_end = globaltimer() + 20000000ull;
                while (globaltimer() < t_end) {
                }
            }
        }
    } else if (warp == 1) {
        /* ------------------------------------------------- MMA issuer ---- */
        /* PAIR: CTA 0 issues for both; its commits arrive on the barriers of both CTAs */
        auto mma = [&](uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
            if (PAIR) umma_f16_pair(d_tmem, a, b, idesc_f16(2 * BM, BN, 0, 0, 0), accumulate);
            else umma_f16(d_tmem, a, b, idesc_f16(BM, BN, 0, 0, 0), accumulate);
        };
        auto commit = [&](uint64_t* bar) {
            if (PAIR) {
                umma_commit_pair(peer_addr(bar, 0));
                umma_commit_pair(peer_addr(bar, 1));
            } else {
                umma_commit(bar);
            }
        };
        if (lane == 0 && rank == 0) {
            uint32_t bs = 0, ts = 0, as = 0;
            int lt = 0;
            bool ok = true;
            /* hi*hi + lo*hi + hi*lo of one 64-deep chunk; the point planes at ah / al */
            auto chunk = [&](uint32_t d_tmem, uint32_t ah, uint32_t al, uint32_t& accum) {
                /* centroid hi plane: x_hi * c_hi and x_lo * c_hi */
                int st = (int)(bs % Cf::B_STAGES);
                uint32_t bu = bs / Cf::B_STAGES;
                if (!mbar_wait(&ms.b_full[st], bu & 1u, abort_flag, status, lim)) { ok = false; return; }
                tc_fence_after();
                const uint32_t bh = smem_u32(smB + st * Cf::B_STAGE);
#pragma unroll
                for (int ks = 0; ks < KC / 16; ++ks) {
                    mma(d_tmem, sw128_desc(ah + ks * 32, 16, 1024), sw128_desc(bh + ks * 32, 16, 1024), accum);
                    accum = 1;
                }
#pragma unroll
                for (int ks = 0; ks < KC / 16; ++ks)
                    mma(d_tmem, sw128_desc(al + ks * 32, 16, 1024), sw128_desc(bh + ks * 32, 16, 1024), 1);
                commit(&ms.b_empty[st]);
                ++bs;
                /* centroid lo plane: x_hi * c_lo */
                st = (int)(bs % Cf::B_STAGES);
                bu = bs / Cf::B_STAGES;
                if (!mbar_wait(&ms.b_full[st], bu & 1u, abort_flag, status, lim)) { ok = false; return; }
                tc_fence_after();
                const uint32_t bl = smem_u32(smB + st * Cf::B_STAGE);
#pragma unroll
                for (int ks = 0; ks < KC / 16; ++ks)
                    mma(d_tmem, sw128_desc(ah + ks * 32, 16, 1024), sw128_desc(bl + ks * 32, 16, 1024), 1);
                commit(&ms.b_empty[st]);
                ++bs;
            };
            for (long long mt = mt0; mt < num_mt && ok; mt += mt_step, ++lt) {
                const int ab = lt % Cf::A_BUFS;
                const uint32_t au = (uint32_t)(lt / Cf::A_BUFS);
                if (!Cf::STREAM) {
                    if (!mbar_wait(&ms.a_full[ab], au & 1u, abort_flag, status, lim)) { ok = false; break; }
                    tc_fence_after();
                }
                const uint32_t a_addr = smem_u32(smA + ab * Cf::A_TILE);
                for (int nt = 0; nt < NT && ok; ++nt, ++ts) {
                    const int tb = (int)(ts & 1u);
                    const uint32_t tu = ts >> 1;
                    if (!mbar_wait(&ms.t_empty[tb], (tu & 1u) ^ 1u, abort_flag, status, lim)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + (uint32_t)(tb * BN);
                    uint32_t accum = 0;
                    for (int kc = 0; kc < nkc && ok; ++kc) {
                        if (Cf::STREAM) {
                            const int sa = (int)(as % Cf::A_BUFS);
                            if (!mbar_wait(&ms.a_full[sa], (as / Cf::A_BUFS) & 1u, abort_flag, status, lim)) { ok = false; break; }
                            tc_fence_after();
                            const uint32_t ah = smem_u32(smA + sa * Cf::A_TILE);
                            chunk(d_tmem, ah, ah + Cf::A_CHUNK, accum);
                            if (ok) commit(&ms.a_empty[sa]);
                            ++as;
                        } else {
                            chunk(d_tmem, a_addr + (uint32_t)(kc * Cf::A_CHUNK),
                                  a_addr + (uint32_t)((nkc + kc) * Cf::A_CHUNK), accum);
                        }
                    }
                    if (ok) commit(&ms.t_full[tb]);
                }
                if (ok && !Cf::STREAM) commit(&ms.a_empty[ab]);
            }
            /* every MMA issued by this thread has completed once fin flips */
            if (PAIR) umma_commit_pair(peer_addr(&ms.fin, 0));
            else umma_commit(&ms.fin);
            drain_wait(&ms.fin, 0);
        }
    } else {
        /* --------------------------------------------------- epilogue ---- */
        const int ew = warp - 2;                       /* 0..7 */
        const int half = ew >> 2;                      /* column half of every tile */
        const int q = warp & 3;                        /* TMEM lane quarter */
        const int r_loc = q * 32 + lane;
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
        const float ns = prm->neg2_inv_s2;
        uint64_t ns2;
        asm("mov.b64 %0, {%1, %1};" : "=l"(ns2) : "f"(ns));
        const float eta = prm->eta;
        float cmax = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) cmax = fmaxf(cmax, ms.wmax[w]);
        cmax = sqrtf(cmax);
        uint32_t ts = 0;
        bool ok = true;
        /* The loop runs every tile even after a failed wait (ok == false, the
         * kernel is aborting): both halves must reach the same named barriers. */
        if (EMIT) {
            for (long long mt = mt0; mt < num_mt; mt += mt_step) {
                const long long row = mt * BM + r_loc;
                const bool live = row < n;
                /* Every column the filter could admit, (D - v0) <= thr_of(T0, D, v0), has
                 * D <= Dmax: with g = D - v0 >= 0 and |D| <= |v0| + g the admission test
                 * implies g <= (T0 + 2^-21 |v0|)(1 + 2^-20) / (1 - 2^-22 (1 + 2^-20)); the
                 * 2^-16 inflation and two ulps cover the FP32 evaluation of both sides.
                 * One compare per element instead of the threshold arithmetic. */
                float Dmax = -INFINITY;
                if (live) {
                    const RefineEntry* E = list + went[wbase + row];
                    const float v0 = E->v0, T0 = E->T0;
                    const float G = (T0 + 0x1.0p-21f * fabsf(v0)) * (1.0f + 0x1.0p-20f) /
                                    (1.0f - 0x1.0p-22f * (1.0f + 0x1.0p-20f));
                    Dmax = v0 + G * (1.0f + 0x1.0p-16f);
                    Dmax = nextafterf(nextafterf(Dmax, INFINITY), INFINITY);
                }
                int* cl = cand + (size_t)(live ? row : 0) * kWideCand + half * (kWideCand / 2);
                int cnt = 0;
                for (int nt = 0; nt < NT; ++nt, ++ts) {
                    const int tb = (int)(ts & 1u);
                    const uint32_t tu = ts >> 1;
                    if (ok) ok = wait_warp(&ms.t_full[tb], tu & 1u, abort_flag, status, lim);
                    if (!ok) continue;
                    tc_fence_after();
                    const int col0 = half * Cf::HALF;
#pragma unroll
                    for (int cc = 0; cc < Cf::CHUNKS; ++cc) {
                        uint32_t r[32];
                        tmem_ld32(t_lane + (uint32_t)(tb * BN + col0 + cc * 32), r);
                        tmem_ld_wait();
                        const int jt = col0 + cc * 32;
                        const float4* cn4 = reinterpret_cast<const float4*>(cn + nt * BN + jt);
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const float4 cv = __ldg(cn4 + u);
                            float D[4];
                            fma2(__uint_as_float(r[4 * u]), __uint_as_float(r[4 * u + 1]), ns2, cv.x, cv.y, D[0], D[1]);
                            fma2(__uint_as_float(r[4 * u + 2]), __uint_as_float(r[4 * u + 3]), ns2, cv.z, cv.w, D[2],
                                 D[3]);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                if (D[e] <= Dmax) {
                                    const int j = nt * BN + jt + 4 * u + e;
                                    if (j < k) {
                                        if (cnt < kWideCand / 2) cl[cnt] = j;
                                        ++cnt;
                                    }
                                }
                            }
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(&ms.t_empty[tb]);
                }
                if (ok && live) ccount[row * 2 + half] = cnt;
            }
        } else
        for (long long mt = mt0; mt < num_mt; mt += mt_step) {
            float a0[kClasses], a1[kClasses];
            int i0[kClasses];
#pragma unroll
            for (int c = 0; c < kClasses; ++c) { a0[c] = INFINITY; a1[c] = INFINITY; i0[c] = -1; }
            for (int nt = 0; nt < NT; ++nt, ++ts) {
                const int tb = (int)(ts & 1u);
                const uint32_t tu = ts >> 1;
                if (ok) ok = wait_warp(&ms.t_full[tb], tu & 1u, abort_flag, status, lim);
                if (!ok) continue;
                tc_fence_after();
                const int col0 = half * Cf::HALF;              /* first column of this warp */
                int pos[kClasses];                               /* column in this tile, -1 */
#pragma unroll
                for (int c = 0; c < kClasses; ++c) pos[c] = -1;
#pragma unroll
                for (int cc = 0; cc < Cf::CHUNKS; cc += 2) {
                    uint32_t r[2][32];
                    tmem_ld32(t_lane + (uint32_t)(tb * BN + col0 + cc * 32), r[0]);
                    if (cc + 1 < Cf::CHUNKS) tmem_ld32(t_lane + (uint32_t)(tb * BN + col0 + (cc + 1) * 32), r[1]);
                    tmem_ld_wait();
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (cc + h >= Cf::CHUNKS) break;
                        const int jt = col0 + (cc + h) * 32;     /* tile-relative column of r[h][0] */
                        const float4* cn4 = reinterpret_cast<const float4*>(cn + nt * BN + jt);
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const float4 cv = __ldg(cn4 + u);
                            float D[4];
                            fma2(__uint_as_float(r[h][4 * u]), __uint_as_float(r[h][4 * u + 1]), ns2, cv.x, cv.y,
                                 D[0], D[1]);
                            fma2(__uint_as_float(r[h][4 * u + 2]), __uint_as_float(r[h][4 * u + 3]), ns2, cv.z, cv.w,
                                 D[2], D[3]);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int c = (4 * u + e) & (kClasses - 1);
                                const bool p = D[e] < a0[c];
                                a1[c] = fminf(a1[c], fmaxf(a0[c], D[e]));
                                pos[c] = p ? (jt + 4 * u + e) : pos[c];
                                a0[c] = fminf(a0[c], D[e]);
                            }
                        }
                    }
                }
                tc_fence_before();
                if (PAIR) {
                    /* one arrival per warp, on CTA 0's barrier */
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(peer_addr(&ms.t_empty[tb], 0));
                } else {
                    mbar_arrive(&ms.t_empty[tb]);
                }
#pragma unroll
                for (int c = 0; c < kClasses; ++c)
                    if (pos[c] >= 0) i0[c] = nt * BN + pos[c];
            }

            /* this half's best (smaller column on ties) and runner-up value */
            float hv0 = a0[0], hv1 = a1[0];
            int hj0 = i0[0];
#pragma unroll
            for (int c = 1; c < kClasses; ++c) {
                const bool better = a0[c] < hv0 || (a0[c] == hv0 && (unsigned)i0[c] < (unsigned)hj0);
                hv1 = fminf(hv1, fminf(a1[c], better ? hv0 : a0[c]));
                hv0 = better ? a0[c] : hv0;
                hj0 = better ? i0[c] : hj0;
            }
            const int bar_id = 1 + q;
            if (half == 1) {
                ms.xa[r_loc] = hv0;
                ms.xb[r_loc] = hv1;
                ms.xc[r_loc] = hj0;
            }
            named_bar(bar_id, 64);
            const long long row = (PAIR ? 2 * mt + rank : mt) * BM + r_loc;
            if (half == 0) {
                const float ov0 = ms.xa[r_loc], ov1 = ms.xb[r_loc];
                const int oj0 = ms.xc[r_loc];
                const bool other = ov0 < hv0 || (ov0 == hv0 && (unsigned)oj0 < (unsigned)hj0);
                const float v1 = fminf(fminf(hv1, ov1), other ? hv0 : ov0);
                const float v0 = other ? ov0 : hv0;
                const int j0 = other ? oj0 : hj0;
                float T0 = 0.f;
                bool flag = false;
                if (ok && row < n) {
                    labels[row] = j0;
                    if (dbg) dbg[row] = make_float4(v0, v1, __int_as_float(j0), __int_as_float(0));
                    if (refine) {
                        const float xn = xnorm[row];
                        T0 = bc.c1 * xn * cmax + bc.c2 * eta * (xn + cmax);
                        flag = (v1 - v0) <= thr_of(T0, v1, v0);
                    }
                }
                int slot = -1;
                const unsigned m = __ballot_sync(0xffffffffu, flag);
                if (m) {
                    unsigned base = 0;
                    if (lane == 0) base = atomicAdd(&prm->nflag, (unsigned)__popc(m));
                    base = __shfl_sync(0xffffffffu, base, 0);
                    if (flag) slot = (int)(base + __popc(m & ((1u << lane) - 1u)));
                }
                ms.xa[r_loc] = v0;
                ms.xb[r_loc] = T0;
                ms.xc[r_loc] = slot;
                if (slot >= 0) {
                    RefineEntry* E = list + slot;
                    int ovf = 0;
#pragma unroll
                    for (int c = 0; c < kClasses; ++c) {
                        const bool in0 = i0[c] >= 0 && (a0[c] - v0) <= thr_of(T0, a0[c], v0);
                        E->c[c] = in0 ? i0[c] : -1;
                        ovf |= (a1[c] < INFINITY && (a1[c] - v0) <= thr_of(T0, a1[c], v0)) ? (1 << c) : 0;
                    }
                    E->row = (int)row;
                    E->ovf[0] = (unsigned short)ovf;
                    E->v0 = v0;
                    E->T0 = T0;
                }
            }
            named_bar(bar_id, 64);
            if (half == 1) {
                const int slot = ms.xc[r_loc];
                if (slot >= 0) {
                    const float v0 = ms.xa[r_loc], T0 = ms.xb[r_loc];
                    RefineEntry* E = list + slot;
                    int ovf = 0;
#pragma unroll
                    for (int c = 0; c < kClasses; ++c) {
                        const bool in0 = i0[c] >= 0 && (a0[c] - v0) <= thr_of(T0, a0[c], v0);
                        E->c[kClasses + c] = in0 ? i0[c] : -1;
                        ovf |= (a1[c] < INFINITY && (a1[c] - v0) <= thr_of(T0, a1[c], v0)) ? (1 << c) : 0;
                    }
                    E->ovf[1] = (unsigned short)ovf;
                }
            }
        }
    }

    tc_fence_before();
    /* PAIR: neither CTA leaves while the other may still signal its barriers or
     * the pair's MMAs may read its shared memory */
    if (PAIR) cluster_sync();
    else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, Cf::TMEM_COLS);
        else tmem_dealloc(tmem_base, Cf::TMEM_COLS);
    }
}

template <int BN, int NKC, bool EMIT, bool PAIR>
cudaError_t launch_t(const AssignArgs& a, cudaStream_t s) {
    using Cf = Cfg<BN, NKC, PAIR>;
    auto kern = k_assign_tc<BN, NKC, EMIT, PAIR>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const int* went = EMIT ? a.wide->went : nullptr;
    int* cand = EMIT ? a.wide->cand : nullptr;
    int* ccount = EMIT ? a.wide->ccount : nullptr;
    const long long wbase = EMIT ? a.wbase : 0;
    const int stall = EMIT ? -1 : a.stall;
    if (!PAIR) {
        const long long num_mt = (a.n + BM - 1) / BM;
        const int grid = (int)(num_mt < a.num_sms ? num_mt : a.num_sms);
        kern<<<grid, kThreads, Cf::SMEM_BYTES, s>>>(*a.tmX, *a.tmC, a.n, a.k, a.dp / KC, a.xnorm, a.cn, a.prm,
                                                     a.labels, a.list, a.refine, a.bc, a.dbg, went, cand, ccount,
                                                     wbase, stall);
        return cudaGetLastError();
    }
    /* clusters of two CTAs, as many as can be resident at once, each running
     * pairs of row tiles round robin */
    const long long pairs = (a.n + 2 * BM - 1) / (2 * BM);
    const int nclus = (int)(pairs < a.pair_clusters ? pairs : a.pair_clusters);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * nclus, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cf::SMEM_BYTES;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, *a.tmX, *a.tmCh, a.n, a.k, a.dp / KC, a.xnorm, a.cn, a.prm, a.labels,
                           a.list, a.refine, a.bc, a.dbg, went, cand, ccount, wbase, stall);
    return e != cudaSuccess ? e : cudaGetLastError();
}

/* Clusters of two that can be resident at once for the pair kernel of this
 * depth (0: it cannot run). */
template <int NKC>
int pair_clusters_t(int num_sms) {
    using Cf = Cfg<256, NKC, true>;
    auto kern = k_assign_tc<256, NKC, false, true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cf::SMEM_BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return nc;
}

template <int BN, bool EMIT>
cudaError_t launch_bn(const AssignArgs& a, cudaStream_t s) {
    /* the pair kernel: 256-wide tiles, no test hook */
    const bool pair = BN == 256 && !EMIT && a.pair != 0 && a.pair_clusters > 0 && a.stall < 0;
    switch (a.dp / KC) {
        case 1: return pair ? launch_t<256, 1, false, true>(a, s) : launch_t<BN, 1, EMIT, false>(a, s);
        case 2: return pair ? launch_t<256, 2, false, true>(a, s) : launch_t<BN, 2, EMIT, false>(a, s);
        case 3: return pair ? launch_t<256, 3, false, true>(a, s) : launch_t<BN, 3, EMIT, false>(a, s);
        case 4: return pair ? launch_t<256, 4, false, true>(a, s) : launch_t<BN, 4, EMIT, false>(a, s);
        default:                                                  /* d > 256: streaming point chunks */
            return pair ? launch_t<256, 0, false, true>(a, s) : launch_t<BN, 0, EMIT, false>(a, s);
    }
}

}  /* namespace */

int assign_bn_for(int k) { return k <= 64 ? 64 : (k <= 128 ? 128 : 256); }

int assign_pair_clusters(int k, int dp, int num_sms) {
    if (assign_bn_for(k) != 256) return 0;
    switch (dp / KC) {
        case 1: return pair_clusters_t<1>(num_sms);
        case 2: return pair_clusters_t<2>(num_sms);
        case 3: return pair_clusters_t<3>(num_sms);
        case 4: return pair_clusters_t<4>(num_sms);
        default: return pair_clusters_t<0>(num_sms);
    }
}
int assign_supported(int d) { return d >= 1 && d <= kMaxDim; }

cudaError_t launch_assign(const AssignArgs& a, cudaStream_t s) {
    if (a.n <= 0) return cudaSuccess;
    if (a.emit) {
        /* the wide path exists only for k > kWideMinK, where the tiles are 256 wide */
        if (assign_bn_for(a.k) != 256 || !a.wide) return cudaErrorInvalidValue;
        return launch_bn<256, true>(a, s);
    }
    switch (assign_bn_for(a.k)) {
        case 64: return launch_bn<64, false>(a, s);
        case 128: return launch_bn<128, false>(a, s);
        default: return launch_bn<256, false>(a, s);
    }
}

}  /* namespace mpk */
