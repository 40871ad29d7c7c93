/* gemm_tc.cu -- emulated FP32 GEMM on tcgen05: C := alpha * sum_t op(A_it) op(B_jt) + beta * C.
 *
 * Replaces the reference's per-term cublasGemmEx_64 loop
 * (gemm-emulation/src/gemm.cu:62-103, gemm_fp16.cu:32-78): one persistent
 * kernel accumulates every cross product of the requested term range into
 * an FP32 TMEM accumulator, term by term (term-major, K ascending within a
 * term), with FP16 or BF16 split planes staged by TMA.  Column-major planes
 * become K-major operands (op = T for A, op = N for B) or MN-major operands
 * (op = N for A, op = T for B) in 128-byte swizzle; the instruction
 * descriptor carries the majors.
 *
 * Output tiles are 128 x 256.  Each 512-deep K slice of each term is
 * accumulated by the tensor cores into a fresh TMEM partial (two buffers of
 * 256 columns, so the MMAs of the next slice overlap the read-out of this
 * one); the epilogue adds every partial into a running FP32 sum held in
 * registers with round-to-nearest.  The tensor cores' own FP32 accumulation
 * (truncating, its error growing with the number of MMA steps that add into
 * one accumulator) therefore only ever spans 32 steps of a partial, and the
 * long sum behaves like an FP32 SGEMM's.  (Measured at M = N = K = 8192 and
 * 2048: 256- to 512-deep partials give the smallest error; shorter ones add
 * more round-to-nearest sums, longer ones more truncation.)  When alpha is a power of two
 * and beta is 0 or 1 the sum starts from beta * C / alpha (exact) and alpha *
 * sum is stored (exact): a range continued by another range then reproduces,
 * bit for bit, the single range -- the property the reference's per-term
 * accumulation through C gives (gemm-emulation/bench/test_refine.cu).
 * Otherwise the epilogue stores fmaf(alpha, sum, beta * C).
 *
 *   warp 0 TMA producer, warp 1 MMA issuer, warps 2-9 epilogue (two warps per
 *   TMEM lane quarter, 128 columns and a 128-float running sum each).
 */
#include "engine.cuh"
#include "gemm_tc.cuh"


namespace mpk {
namespace {

constexpr int BM = 128, BK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int A_STAGE = BM * BK * 2;             /* 16 KB */
constexpr int kSmemMax = 232448;
constexpr int kMisc = 1024;
constexpr int BOX = 64 * 64 * 2;                 /* one 64 x 64 MN-major box: 8 KB */
#ifndef GEMM_CHUNKS_PER_PARTIAL
#define GEMM_CHUNKS_PER_PARTIAL 8
#endif
/* 64-deep K chunks the tensor cores accumulate into one TMEM partial before
 * the epilogue folds it into the round-to-nearest sum (a partial never spans
 * two terms). */
constexpr int CPP = GEMM_CHUNKS_PER_PARTIAL;
constexpr int kGroupM = 16;                      /* tile rows per raster group */

/* Tile order: groups of kGroupM tile rows, column by column inside a group,
 * so the CTAs resident at one time share a few A row panels and B column
 * panels (L2 reuse) instead of sweeping all of A for every column. */
__device__ __forceinline__ void tile_coords(long long tile, int tiles_m, int tiles_n, int& tm, int& tn) {
    const long long per_group = (long long)kGroupM * tiles_n;
    const int g = (int)(tile / per_group);
    const int r = (int)(tile - (long long)g * per_group);
    const int rows = min(kGroupM, tiles_m - g * kGroupM);
    tm = g * kGroupM + r % rows;
    tn = r / rows;
}

/* Epilogue modes: how C enters and leaves the running sum. */
enum : int {
    EPI_PLAIN = 0,    /* beta = 0: C := alpha * sum */
    EPI_RESUME = 1,   /* alpha a power of two, beta = 1: sum starts at C / alpha, C := alpha * sum */
    EPI_GENERAL = 2,  /* C := fmaf(alpha, sum, beta * C) */
};

template <int BN>
struct Cfg {
    static constexpr int HALF = BN / 2;                        /* columns per epilogue warp */
    static constexpr int B_STAGE = BN * BK * 2;
    static constexpr int STAGE = A_STAGE + B_STAGE;
    static constexpr int STAGES = (kSmemMax - kMisc) / STAGE;
    static constexpr int SMEM_BYTES = STAGES * STAGE + kMisc;
    static constexpr int TMEM_COLS = 2 * BN;                   /* two partial buffers */
};

template <int STAGES>
struct GMisc {
    uint64_t full[STAGES], empty[STAGES], p_full[2], p_empty[2], fin;
    uint32_t tmem_slot;
    int abort_flag;
};

__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, status) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() - t0 > kWaitLimitNs) return;
}

template <int BN, bool A_MN, bool B_MN, int FMT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int m, int n, int kdim,
          GemmTerms terms, float alpha, float beta, float* __restrict__ C, long long ldc,
          int* status) {
    using K = Cfg<BN>;
    constexpr int HALF = K::HALF, STAGE = K::STAGE, STAGES = K::STAGES;
    static_assert(sizeof(GMisc<STAGES>) <= kMisc, "misc");
    extern __shared__ __align__(1024) uint8_t smem[];
    GMisc<STAGES>& ms = *reinterpret_cast<GMisc<STAGES>*>(smem + STAGES * STAGE);
    volatile int* abort_flag = &ms.abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (m + BM - 1) / BM, tiles_n = (n + BN - 1) / BN;
    const long long num_tiles = (long long)tiles_m * tiles_n;
    const int KCH = (kdim + BK - 1) / BK;

    if (smem_u32(smem) & 1023u) {
        if (threadIdx.x == 0) atomicOr(status, MPK_DEV_TIMEOUT);
        return;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) { mbar_init(&ms.full[i], 1); mbar_init(&ms.empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&ms.p_full[i], 1); mbar_init(&ms.p_empty[i], 32 * kEpiWarps); }
        mbar_init(&ms.fin, 1);
        ms.abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
    if (warp == 1) tmem_alloc(&ms.tmem_slot, K::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = ms.tmem_slot;

    if (warp < 2) {
      if (warp == 0) {
        /* ------------------------------------------------- producer ---- */
        if (lane == 0) {
            uint32_t last[STAGES];
#pragma unroll
            for (int i = 0; i < STAGES; ++i) last[i] = 0xffffffffu;
            uint32_t it = 0;
            bool ok = true;
            for (long long tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                int tm, tn;
                tile_coords(tile, tiles_m, tiles_n, tm, tn);
                for (int t = 0; t < terms.n && ok; ++t)
                    for (int kc = 0; kc < KCH; ++kc, ++it) {
                        const int st = (int)(it % STAGES);
                        const uint32_t u = it / STAGES;
                        if (!mbar_wait(&ms.empty[st], (u & 1u) ^ 1u, abort_flag, status)) { ok = false; break; }
                        mbar_expect_tx(&ms.full[st], STAGE);
                        last[st] = u;
                        uint8_t* sa = smem + st * STAGE;
                        uint8_t* sb = sa + A_STAGE;
                        if (A_MN) {
                            tma_load_3d(&tmA, &ms.full[st], sa, tm * BM, kc * BK, terms.ia[t]);
                            tma_load_3d(&tmA, &ms.full[st], sa + BOX, tm * BM + 64, kc * BK, terms.ia[t]);
                        } else {
                            tma_load_3d(&tmA, &ms.full[st], sa, kc * BK, tm * BM, terms.ia[t]);
                        }
                        if (B_MN) {
#pragma unroll
                            for (int q = 0; q < BN / 64; ++q)
                                tma_load_3d(&tmB, &ms.full[st], sb + q * BOX, tn * BN + 64 * q, kc * BK, terms.ib[t]);
                        } else {
                            tma_load_3d(&tmB, &ms.full[st], sb, kc * BK, tn * BN, terms.ib[t]);
                        }
                    }
            }
            if (!ok)
                for (int i = 0; i < STAGES; ++i)
                    if (last[i] != 0xffffffffu) drain_wait(&ms.full[i], last[i] & 1u);
        }
      } else if (warp == 1) {
        /* ------------------------------------------------- MMA issuer --- */
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(BM, BN, FMT, A_MN ? 1 : 0, B_MN ? 1 : 0);
            uint32_t it = 0, pi = 0;                    /* stage counter, partial counter */
            bool ok = true;
            for (long long tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x)
                for (int t = 0; t < terms.n && ok; ++t)
                    for (int kc = 0; kc < KCH; ++kc, ++it) {
                        const int st = (int)(it % STAGES);
                        const int pb = (int)(pi & 1u);          /* partial buffer of this chunk */
                        const int kin = kc % CPP;               /* chunk index inside the partial */
                        const bool last_of_partial = kin == CPP - 1 || kc == KCH - 1;
                        if (!mbar_wait(&ms.full[st], (it / STAGES) & 1u, abort_flag, status)) { ok = false; break; }
                        if (kin == 0 &&
                            !mbar_wait(&ms.p_empty[pb], ((pi >> 1) & 1u) ^ 1u, abort_flag, status)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t sa = smem_u32(smem + st * STAGE);
                        const uint32_t sb = sa + A_STAGE;
                        const uint32_t d_tmem = tmem_base + (uint32_t)(pb * BN);
#pragma unroll
                        for (int ks = 0; ks < BK / 16; ++ks) {
                            const uint64_t ad = A_MN ? sw128_desc(sa + ks * 2048, BOX, 1024)
                                                     : sw128_desc(sa + ks * 32, 16, 1024);
                            const uint64_t bd = B_MN ? sw128_desc(sb + ks * 2048, BOX, 1024)
                                                     : sw128_desc(sb + ks * 32, 16, 1024);
                            umma_f16(d_tmem, ad, bd, idesc, (kin > 0 || ks > 0) ? 1u : 0u);
                        }
                        umma_commit(&ms.empty[st]);
                        if (last_of_partial) {
                            umma_commit(&ms.p_full[pb]);
                            ++pi;
                        }
                    }
            umma_commit(&ms.fin);
            drain_wait(&ms.fin, 0);
        }
      }
    } else {
        /* --------------------------------------------------- epilogue --- */
        const int ew = warp - 2;
        const int half = ew >> 2;                 /* which 128 columns of the tile */
        const int q = warp & 3;                   /* TMEM lane quarter */
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * HALF);
        const float inv_alpha = 1.0f / alpha;     /* exact in EPI_RESUME (alpha a power of two) */
        bool ok = true;
        uint32_t pi = 0;
        for (long long tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            int tm, tn;
            tile_coords(tile, tiles_m, tiles_n, tm, tn);
            const int row = tm * BM + q * 32 + lane;
            const int col0 = tn * BN + half * HALF;
            const int ncol = min(HALF, n - col0);
            float S[HALF];
            if (EPI == EPI_RESUME) {
                /* an opaque copy of C keeps these column addresses from being
                 * shared with (and kept alive until) the final store */
                const float* Cr;
                asm volatile("mov.b64 %0, %1;" : "=l"(Cr) : "l"(C));
                const float* src = Cr + (size_t)col0 * ldc + row;
                const bool load_c = row < m;
#pragma unroll
                for (int e = 0; e < HALF; ++e) {
                    S[e] = (load_c && e < ncol) ? *src * inv_alpha : 0.f;
                    src += ldc;
                }
            } else {
#pragma unroll
                for (int e = 0; e < HALF; ++e) S[e] = 0.f;
            }
            for (int t = 0; t < terms.n; ++t)
                for (int kc = 0; kc < KCH; kc += CPP, ++pi) {
                    const int pb = (int)(pi & 1u);
                    if (ok) ok = wait_warp(&ms.p_full[pb], (pi >> 1) & 1u, abort_flag, status);
                    if (!ok) continue;
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < HALF / 32; ++c) {
                        uint32_t r[32];
                        tmem_ld32(t_lane + (uint32_t)(pb * BN + c * 32), r);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e) S[c * 32 + e] = S[c * 32 + e] + __uint_as_float(r[e]);
                    }
                    tc_fence_before();
                    mbar_arrive(&ms.p_empty[pb]);
                }
            if (ok && row < m) {
                float* Cw;
                asm volatile("mov.b64 %0, %1;" : "=l"(Cw) : "l"(C));
                float* dst = Cw + (size_t)col0 * ldc + row;
#pragma unroll
                for (int e = 0; e < HALF; ++e) {
                    if (e < ncol) *dst = EPI == EPI_GENERAL ? fmaf(alpha, S[e], beta * *dst) : alpha * S[e];
                    dst += ldc;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, K::TMEM_COLS);
    }
}

template <int BN, bool A_MN, bool B_MN, int FMT, int EPI>
cudaError_t launch_t(const GemmArgs& g, cudaStream_t s) {
    using K = Cfg<BN>;
    auto kern = k_gemm_tc<BN, A_MN, B_MN, FMT, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, K::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const long long tiles = (long long)((g.m + BM - 1) / BM) * ((g.n + BN - 1) / BN);
    const int grid = (int)(tiles < g.num_sms ? tiles : g.num_sms);
    kern<<<grid, kThreads, K::SMEM_BYTES, s>>>(*g.tmA, *g.tmB, g.m, g.n, g.k, g.terms, g.alpha, g.beta, g.C, g.ldc,
                                                g.status);
    return cudaGetLastError();
}

template <int BN, int FMT, int EPI>
cudaError_t launch_epi(const GemmArgs& g, cudaStream_t s) {
    if (g.a_mn) return g.b_mn ? launch_t<BN, true, true, FMT, EPI>(g, s) : launch_t<BN, true, false, FMT, EPI>(g, s);
    return g.b_mn ? launch_t<BN, false, true, FMT, EPI>(g, s) : launch_t<BN, false, false, FMT, EPI>(g, s);
}

/* 128 x 256 tiles, except in the resuming mode: there the sums start from C,
 * and 128 running sums per thread plus the loads of C do not fit the register
 * file, so its tiles are 128 x 128.  An element's arithmetic (the partial of
 * each 64-deep chunk, then the round-to-nearest sum) does not depend on the
 * tile width, so ranges run in different modes still chain bit for bit. */
int epi_mode(float beta, int init_mode) {
    if (beta == 0.f) return EPI_PLAIN;
    return (init_mode && beta == 1.f) ? EPI_RESUME : EPI_GENERAL;
}

template <int FMT>
cudaError_t launch_fmt(const GemmArgs& g, cudaStream_t s) {
    switch (epi_mode(g.beta, g.init_mode)) {
        case EPI_PLAIN: return launch_epi<256, FMT, EPI_PLAIN>(g, s);
        case EPI_RESUME: return launch_epi<128, FMT, EPI_RESUME>(g, s);
        default: return launch_epi<256, FMT, EPI_GENERAL>(g, s);
    }
}

}  /* namespace */

int gemm_tile_m() { return BM; }
int gemm_tile_n(float beta, int init_mode) { return epi_mode(beta, init_mode) == EPI_RESUME ? 128 : 256; }
int gemm_tile_k() { return BK; }

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t s) {
    if (g.m <= 0 || g.n <= 0) return cudaSuccess;
    return g.bf16 ? launch_fmt<1>(g, s) : launch_fmt<0>(g, s);
}

}  /* namespace mpk */
