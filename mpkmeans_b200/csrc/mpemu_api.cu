/* mpemu_api.cu -- the split-precision GEMM C ABI (include/mpemu.h).
 *
 * Splits, AutoScale and the split check are bandwidth-bound SIMT kernels; the
 * GEMM drivers validate exactly as the reference does (gemm.cu:62-103,
 * gemm_fp16.cu:32-78, split.cu:124-147, split_fp16.cu:205-289), build TMA
 * descriptors over the packed split planes and launch the tcgen05 kernel of
 * gemm_tc.cu once per call.  Layouts TMA cannot address (a leading dimension
 * or plane stride that is not a multiple of 8 elements, a misaligned base)
 * take a plain SIMT kernel with the same term order.
 */
#include "engine.cuh"
#include "gemm_tc.cuh"
#include "mpemu.h"
#include "mpkmeans_debug.h"

#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <mutex>
#include <unordered_map>
#include <vector>

using namespace mpk;

namespace {

constexpr int kBlock = 256;

/* ------------------------------------------------------------- splits ---- */

template <typename W>
__device__ __forceinline__ W to_word(float a);
template <>
__device__ __forceinline__ __nv_bfloat16 to_word<__nv_bfloat16>(float a) { return __float2bfloat16_rn(a); }
template <>
__device__ __forceinline__ __half to_word<__half>(float a) { return __float2half_rn(a); }
__device__ __forceinline__ float from_word(__nv_bfloat16 w) { return __bfloat162float(w); }
__device__ __forceinline__ float from_word(__half w) { return __half2float(w); }

/* Every element of a column-major rows x cols matrix: a = scale * A(r, c);
 * word s = round(a), a -= word (exact), for s = 0..nsplits-1.  Columns go to
 * blockIdx.y, four consecutive rows to a thread: VEC (A 16-byte aligned with
 * lda % 4 == 0, S 8-byte aligned with lds and stride % 4 == 0) loads the four
 * with one float4 and stores each plane's four words with one 8-byte store;
 * the arithmetic per element is the same either way. */
template <typename W, bool VEC>
__global__ void k_split(const float* __restrict__ A, long long lda, long long rows, long long cols, int nsplits,
                        float scale, W* __restrict__ S, long long lds, long long stride) {
    const long long rstep = (long long)gridDim.x * blockDim.x * 4;
    for (long long c = blockIdx.y; c < cols; c += gridDim.y) {
        const float* a_col = A + c * lda;
        W* s_col = S + c * lds;
        for (long long r0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4; r0 < rows; r0 += rstep) {
            const bool full = r0 + 3 < rows;
            float v[4];
            if (VEC && full) {
                const float4 t = *reinterpret_cast<const float4*>(a_col + r0);
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = r0 + u < rows ? a_col[r0 + u] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = v[u] * scale;
            for (int sp = 0; sp < nsplits; ++sp) {
                W w[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    w[u] = to_word<W>(v[u]);
                    v[u] = v[u] - from_word(w[u]);
                }
                W* dst = s_col + (long long)sp * stride + r0;
                if (VEC && full) {
                    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(w);
                } else {
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (r0 + u < rows) dst[u] = w[u];
                }
            }
        }
    }
}

__global__ void k_maxabs_finite(const float* __restrict__ A, long long lda, long long rows, long long cols,
                                float* out) {
    float m = 0.f;
    const long long total = rows * cols;
    const long long step = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += step) {
        const long long c = e / rows, r = e - c * rows;
        const float v = fabsf(A[c * lda + r]);
        if (v > m && isfinite(v)) m = v;
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(reinterpret_cast<unsigned int*>(out), __float_as_uint(m));
}

/* Classifies each FP16 word: [0] not finite, [1] zero while the residual was
 * not, or subnormal, [2] clean. */
__global__ void k_check_split(const float* __restrict__ A, long long lda, long long rows, long long cols,
                              int nsplits, float scale, const __half* __restrict__ S, long long lds, long long stride,
                              unsigned long long* counts) {
    unsigned long long over = 0, sub = 0, ok = 0;
    const long long total = rows * cols;
    const long long step = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += step) {
        const long long c = e / rows, r = e - c * rows;
        float res = A[c * lda + r] * scale;
        for (int s = 0; s < nsplits; ++s) {
            const float w = __half2float(S[(long long)s * stride + c * lds + r]);
            const float aw = fabsf(w);
            if (!isfinite(w)) ++over;
            else if ((aw == 0.f && res != 0.f) || (aw > 0.f && aw < 6.103515625e-05f)) ++sub;
            else ++ok;
            res -= w;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        over += __shfl_xor_sync(0xffffffffu, over, o);
        sub += __shfl_xor_sync(0xffffffffu, sub, o);
        ok += __shfl_xor_sync(0xffffffffu, ok, o);
    }
    if ((threadIdx.x & 31) == 0) {
        if (over) atomicAdd(&counts[0], over);
        if (sub) atomicAdd(&counts[1], sub);
        if (ok) atomicAdd(&counts[2], ok);
    }
}

/* C := beta * C (an empty term range, or k = 0; BLAS semantics). */
__global__ void k_scale_c(float* C, long long ldc, int m, int n, float beta) {
    const long long total = (long long)m * n;
    const long long step = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += step) {
        const long long c = e / m, r = e - c * m;
        float* p = C + c * ldc + r;
        *p = beta == 0.f ? 0.f : beta * *p;
    }
}

/* Fallback for layouts TMA cannot take: one thread per output, the same
 * term-major, K-ascending FP32 accumulation. */
template <typename W>
__global__ void k_gemm_simt(bool ta, bool tb, int m, int n, int k, const W* __restrict__ A, long long lda,
                            long long sa, const W* __restrict__ B, long long ldb, long long sb, GemmTerms terms,
                            float alpha, float beta, int init_mode, float* C, long long ldc) {
    const long long total = (long long)m * n;
    const long long step = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += step) {
        const int j = (int)(e / m), i = (int)(e - (long long)j * m);
        float* dst = C + (long long)j * ldc + i;
        float acc = (init_mode && beta != 0.f) ? beta * *dst / alpha : 0.f;
        for (int t = 0; t < terms.n; ++t) {
            const W* a = A + terms.ia[t] * sa;
            const W* b = B + terms.ib[t] * sb;
            for (int kk = 0; kk < k; ++kk) {
                const float av = from_word(ta ? a[(long long)i * lda + kk] : a[(long long)kk * lda + i]);
                const float bv = from_word(tb ? b[(long long)kk * ldb + j] : b[(long long)j * ldb + kk]);
                acc = fmaf(av, bv, acc);
            }
        }
        if (init_mode) *dst = acc * alpha;
        else *dst = beta != 0.f ? fmaf(alpha, acc, beta * *dst) : alpha * acc;
    }
}

int grid_for(long long items) {
    long long b = (items + kBlock - 1) / kBlock;
    if (b < 1) b = 1;
    return (int)(b > 148 * 16 ? 148 * 16 : b);
}

cudaStream_t stream_of(cublasHandle_t h) {
    cudaStream_t s = nullptr;
    if (h) cublasGetStream(h, &s);
    return s;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

/* 3D map over nplanes column-major planes: (contiguous dim, other dim, plane). */
bool plane_map(CUtensorMap* map, const void* base, bool bf16, long long inner, long long outer, long long ld,
               long long pstride, int nplanes, int box_inner, int box_outer) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)nplanes};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)pstride * 2};
    cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
              const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

/* One device int per GPU for the kernel's status word (bounded waits). */
int* gemm_status(int* sms) {
    static std::mutex m;
    static int* st[64] = {};
    static int nsm[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(m);
    if (!st[dev]) {
        if (cudaMalloc(&st[dev], sizeof(int)) != cudaSuccess) return nullptr;
        cudaMemset(st[dev], 0, sizeof(int));
        cudaDeviceGetAttribute(&nsm[dev], cudaDevAttrMultiProcessorCount, dev);
    }
    *sms = nsm[dev];
    return st[dev];
}

bool power_of_two(float a) {
    if (!(a > 0.f) || !std::isfinite(a)) return false;
    int e = 0;
    return std::frexp(a, &e) == 0.5f;
}

/* The planes of one operand: plane p starts p * pstride elements after base;
 * each is a column-major matrix with leading dimension ld. */
struct Planes {
    const void* base;
    int64_t ld, pstride;
    int nplanes;
};

/* dC := alpha * sum_t op(A_{ia[t]}) op(B_{ib[t]}) + beta * dC, terms in order,
 * one launch.  Shapes and leading dimensions are already validated. */
mpemuStatus_t run_terms(cudaStream_t s, bool ta, bool tb, int64_t m, int64_t n, int64_t k, float alpha,
                        const Planes& A, const Planes& B, const GemmTerms& terms, float beta, float* dC,
                        int64_t ldc, bool bf16) {
    const int init_mode = (power_of_two(alpha) && (beta == 0.f || beta == 1.f)) ? 1 : 0;
    const bool tma_ok = ((reinterpret_cast<uintptr_t>(A.base) | reinterpret_cast<uintptr_t>(B.base)) % 16 == 0) &&
                        A.ld % 8 == 0 && B.ld % 8 == 0 && A.pstride % 8 == 0 && B.pstride % 8 == 0 &&
                        (A.nplanes == 1 || A.pstride > 0) && (B.nplanes == 1 || B.pstride > 0);
    int sms = 0;
    int* status = gemm_status(&sms);
    if (!status) return MPEMU_STATUS_CUDA_ERROR;
    CUtensorMap tmA, tmB;
    const bool a_mn = !ta, b_mn = tb;
    /* stored shapes: A is m x k (op N) or k x m (op T); B is k x n (op N) or n x k (op T) */
    bool use_tma = tma_ok;
    if (use_tma) {
        const int64_t pa = A.pstride > 0 ? A.pstride : A.ld * (a_mn ? k : m);
        const int64_t pb = B.pstride > 0 ? B.pstride : B.ld * (b_mn ? k : n);
        use_tma = (a_mn ? plane_map(&tmA, A.base, bf16, m, k, A.ld, pa, A.nplanes, 64, 64)
                        : plane_map(&tmA, A.base, bf16, k, m, A.ld, pa, A.nplanes, 64, 128)) &&
                  (b_mn ? plane_map(&tmB, B.base, bf16, n, k, B.ld, pb, B.nplanes, 64, 64)
                        : plane_map(&tmB, B.base, bf16, k, n, B.ld, pb, B.nplanes, 64,
                                    mpk::gemm_tile_n(beta, init_mode)));
    }
    if (!use_tma) {
        if (bf16)
            k_gemm_simt<__nv_bfloat16><<<grid_for(m * n), kBlock, 0, s>>>(
                ta, tb, (int)m, (int)n, (int)k, (const __nv_bfloat16*)A.base, A.ld, A.pstride,
                (const __nv_bfloat16*)B.base, B.ld, B.pstride, terms, alpha, beta, init_mode, dC, ldc);
        else
            k_gemm_simt<__half><<<grid_for(m * n), kBlock, 0, s>>>(ta, tb, (int)m, (int)n, (int)k,
                                                                   (const __half*)A.base, A.ld, A.pstride,
                                                                   (const __half*)B.base, B.ld, B.pstride, terms,
                                                                   alpha, beta, init_mode, dC, ldc);
        return cudaGetLastError() == cudaSuccess ? MPEMU_STATUS_SUCCESS : MPEMU_STATUS_CUDA_ERROR;
    }
    GemmArgs g;
    g.tmA = &tmA;
    g.tmB = &tmB;
    g.m = (int)m;
    g.n = (int)n;
    g.k = (int)k;
    g.a_mn = a_mn;
    g.b_mn = b_mn;
    g.bf16 = bf16;
    g.terms = terms;
    g.alpha = alpha;
    g.beta = beta;
    g.init_mode = init_mode;
    g.C = dC;
    g.ldc = ldc;
    g.status = status;
    g.num_sms = sms;
    return launch_gemm_tc(g, s) == cudaSuccess ? MPEMU_STATUS_SUCCESS : MPEMU_STATUS_CUDA_ERROR;
}

/* C := beta * C for an empty sum (BLAS semantics; beta == 1 leaves C alone). */
mpemuStatus_t scale_only(cudaStream_t s, int64_t m, int64_t n, float beta, float* dC, int64_t ldc) {
    if (beta == 1.0f) return MPEMU_STATUS_SUCCESS;
    k_scale_c<<<grid_for(m * n), kBlock, 0, s>>>(dC, ldc, (int)m, (int)n, beta);
    return cudaGetLastError() == cudaSuccess ? MPEMU_STATUS_SUCCESS : MPEMU_STATUS_CUDA_ERROR;
}

/* Shared driver: dC := alpha * sum over schedule positions [b, e) + beta * dC.
 * Checks follow the reference's order and results: bad split count or range
 * -> INVALID_VALUE; an empty range with beta == 1 succeeds untouched; a
 * missing handle -> INVALID_VALUE (gemm.cu:7-18); a leading dimension cuBLAS
 * would reject -> CUBLAS_ERROR. */
mpemuStatus_t gemm_range(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB, int64_t m, int64_t n,
                         int64_t k, float alpha, const void* dSA, int64_t lda, int64_t strideA, const void* dSB,
                         int64_t ldb, int64_t strideB, int nsplits, int b, int e, float beta, float* dC,
                         int64_t ldc, bool bf16) {
    if (nsplits < 1 || nsplits > MPEMU_MAX_SPLITS) return MPEMU_STATUS_INVALID_VALUE;
    const int total = nsplits * nsplits;
    if (e == MPEMU_ALL_MACS) e = total;
    if (b < 0 || e > total || b > e) return MPEMU_STATUS_INVALID_VALUE;
    if (b == e && beta == 1.0f) return MPEMU_STATUS_SUCCESS;
    if (!handle || !dC) return MPEMU_STATUS_INVALID_VALUE;
    if (m < 0 || n < 0 || k < 0) return MPEMU_STATUS_INVALID_VALUE;
    if (b < e && k > 0 && (!dSA || !dSB)) return MPEMU_STATUS_INVALID_VALUE;
    if (m == 0 || n == 0) return MPEMU_STATUS_SUCCESS;
    if (ldc < m) return MPEMU_STATUS_CUBLAS_ERROR;
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return MPEMU_STATUS_INVALID_VALUE;
    const cudaStream_t s = stream_of(handle);
    if (b == e || k == 0) return scale_only(s, m, n, beta, dC, ldc);
    mpemuTerm_t sched[MPEMU_MAX_SPLITS * MPEMU_MAX_SPLITS];
    mpemuTermSchedule(nsplits, e, sched);
    GemmTerms terms;
    terms.n = e - b;
    for (int t = b; t < e; ++t) {
        terms.ia[t - b] = sched[t].i;
        terms.ib[t - b] = sched[t].j;
    }
    const bool ta = (opA != CUBLAS_OP_N), tb = (opB != CUBLAS_OP_N);
    const int64_t a_rows = ta ? k : m, b_rows = tb ? n : k;
    if (lda < a_rows || ldb < b_rows) return MPEMU_STATUS_CUBLAS_ERROR;
    return run_terms(s, ta, tb, m, n, k, alpha, Planes{dSA, lda, strideA, nsplits},
                     Planes{dSB, ldb, strideB, nsplits}, terms, beta, dC, ldc, bf16);
}

template <typename W>
mpemuStatus_t split_impl(const float* dA, int64_t lda, int64_t rows, int64_t cols, int nsplits, float scale,
                         W* dS, int64_t lds, int64_t stride, cudaStream_t s) {
    if (!dA || !dS) return MPEMU_STATUS_INVALID_VALUE;
    if (rows < 0 || cols < 0) return MPEMU_STATUS_INVALID_VALUE;
    if (nsplits < 1 || nsplits > MPEMU_MAX_SPLITS) return MPEMU_STATUS_INVALID_VALUE;
    if (lda < rows || lds < rows) return MPEMU_STATUS_INVALID_VALUE;
    if (stride < lds * cols) return MPEMU_STATUS_INVALID_VALUE;
    if (rows == 0 || cols == 0) return MPEMU_STATUS_SUCCESS;
    /* blocks over the rows of a column (four rows a thread), columns on y; about 16 blocks
     * a SM in all */
    const long long xb = std::max<long long>(1, std::min<long long>((rows + 4 * kBlock - 1) / (4 * kBlock), 148 * 16));
    const long long yb = std::max<long long>(1, std::min<long long>(cols, std::max<long long>(1, 148 * 16 / xb)));
    const dim3 grid((unsigned)xb, (unsigned)std::min<long long>(yb, 65535));
    const bool vec = (reinterpret_cast<uintptr_t>(dA) % 16 == 0) && lda % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(dS) % 8 == 0) && lds % 4 == 0 && stride % 4 == 0;
    if (vec) k_split<W, true><<<grid, kBlock, 0, s>>>(dA, lda, rows, cols, nsplits, scale, dS, lds, stride);
    else k_split<W, false><<<grid, kBlock, 0, s>>>(dA, lda, rows, cols, nsplits, scale, dS, lds, stride);
    return cudaGetLastError() == cudaSuccess ? MPEMU_STATUS_SUCCESS : MPEMU_STATUS_CUDA_ERROR;
}

/* Stacked, reversed split of B (k x n): word j of B(r, c) goes to row
 * (nsplits - 1 - j) * k + r of column c. */
template <typename W>
__global__ void k_split_stacked(const float* __restrict__ B, long long ldb, long long k, long long n, int nsplits,
                                float scale, W* __restrict__ S, long long lds) {
    const long long total = k * n;
    const long long step = (long long)gridDim.x * blockDim.x;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += step) {
        const long long c = e / k, r = e - c * k;
        float a = B[c * ldb + r] * scale;
        W* col = S + c * lds + r;
        for (int j = 0; j < nsplits; ++j) {
            const W w = to_word<W>(a);
            col[(long long)(nsplits - 1 - j) * k] = w;
            a = a - from_word(w);
        }
    }
}

template <typename W>
mpemuStatus_t split_stacked(const float* dB, int64_t ldb, int64_t k, int64_t n, int nsplits, float scale, W* dS,
                            int64_t lds, cudaStream_t s) {
    if (!dB || !dS) return MPEMU_STATUS_INVALID_VALUE;
    if (k < 0 || n < 0) return MPEMU_STATUS_INVALID_VALUE;
    if (nsplits < 1 || nsplits > MPEMU_MAX_SPLITS) return MPEMU_STATUS_INVALID_VALUE;
    if (ldb < k) return MPEMU_STATUS_INVALID_VALUE;
    if (lds < (int64_t)nsplits * k) return MPEMU_STATUS_INVALID_VALUE;
    if (!(scale > 0.0f)) return MPEMU_STATUS_INVALID_VALUE;
    if (k == 0 || n == 0) return MPEMU_STATUS_SUCCESS;
    k_split_stacked<W><<<grid_for(k * n), kBlock, 0, s>>>(dB, ldb, k, n, nsplits, scale, dS, lds);
    return cudaGetLastError() == cudaSuccess ? MPEMU_STATUS_SUCCESS : MPEMU_STATUS_CUDA_ERROR;
}

/* Concatenated-k drivers: the products of bins [0, nbins), B in the stacked
 * reversed layout, both ops N.  The reference validates in this order
 * (concat.cu concatGemm); cuBLAS's own argument checks become CUBLAS_ERROR. */
mpemuStatus_t concat_run(cublasHandle_t handle, int64_t m, int64_t n, int64_t k, float alpha, const void* dSA,
                         int64_t lda, const void* dSB, int64_t ldsb, int nsplits, int nbins, float beta, float* dC,
                         int64_t ldc, bool bf16) {
    if (!handle || !dC || !dSA || !dSB) return MPEMU_STATUS_INVALID_VALUE;
    if (nsplits < 1 || nbins < 1 || nbins > nsplits) return MPEMU_STATUS_INVALID_VALUE;
    if (nsplits > MPEMU_MAX_SPLITS) return MPEMU_STATUS_INVALID_VALUE;
    if (m < 0 || n < 0 || k < 0) return MPEMU_STATUS_CUBLAS_ERROR;
    if (lda < (m > 1 ? m : 1) || ldsb < (nbins * k > 1 ? nbins * k : 1) || ldc < (m > 1 ? m : 1))
        return MPEMU_STATUS_CUBLAS_ERROR;
    if (m == 0 || n == 0) return MPEMU_STATUS_SUCCESS;
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return MPEMU_STATUS_INVALID_VALUE;
    const cudaStream_t s = stream_of(handle);
    if (k == 0) return scale_only(s, m, n, beta, dC, ldc);
    mpemuTerm_t sched[MPEMU_MAX_SPLITS * MPEMU_MAX_SPLITS];
    const int nt = nbins * (nbins + 1) / 2;      /* bins 0..nbins-1: the schedule's first terms */
    mpemuTermSchedule(nsplits, nt, sched);
    GemmTerms terms;
    terms.n = nt;
    for (int t = 0; t < nt; ++t) {
        terms.ia[t] = sched[t].i;
        terms.ib[t] = nsplits - 1 - sched[t].j;  /* B plane j sits at row block nsplits - 1 - j */
    }
    return run_terms(s, false, false, m, n, k, alpha, Planes{dSA, lda, lda * k, nsplits},
                     Planes{dSB, ldsb, k, nsplits}, terms, beta, dC, ldc, bf16);
}

/* What mpemuBatchPlan recorded for a workspace, keyed by its pointer arrays'
 * device address: the batched call needs the plane bases and the term range
 * on the host to build its one launch. */
struct PlanRecord {
    const void* dSA;
    int64_t strideA;
    const void* dSB;
    int64_t strideB;
    int nsplits, macBegin, count, elemBytes;
};
std::mutex g_plan_mu;
std::unordered_map<const void*, PlanRecord>& plans() {
    static std::unordered_map<const void*, PlanRecord> p;
    return p;
}

mpemuStatus_t batched_run(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB, int64_t m, int64_t n,
                          int64_t k, float alpha, int planBegin, int planCount, float beta, float* dC, int64_t ldc,
                          const mpemuBatchWorkspace_t* bw, cudaStream_t stream, bool bf16) {
    if (!bw || !dC) return MPEMU_STATUS_INVALID_VALUE;
    if (planBegin < 0 || planCount < 1 || planBegin + planCount > bw->planned) return MPEMU_STATUS_INVALID_VALUE;
    PlanRecord pr;
    {
        std::lock_guard<std::mutex> lock(g_plan_mu);
        auto it = plans().find((const void*)bw->aptr);
        if (it == plans().end()) return MPEMU_STATUS_INVALID_VALUE;   /* not planned by mpemuBatchPlan */
        pr = it->second;
    }
    if (pr.elemBytes != 2 || planBegin + planCount > pr.count) return MPEMU_STATUS_INVALID_VALUE;
    if (!handle) return MPEMU_STATUS_CUBLAS_ERROR;
    const bool ta = (opA != CUBLAS_OP_N), tb = (opB != CUBLAS_OP_N);
    const int64_t lda = mpemuSplitLd(m), ldb = mpemuSplitLd(k);
    if (m < 0 || n < 0 || k < 0) return MPEMU_STATUS_CUBLAS_ERROR;
    if (lda < (ta ? k : m) || ldb < (tb ? n : k) || ldc < m) return MPEMU_STATUS_CUBLAS_ERROR;
    if (m == 0 || n == 0) return MPEMU_STATUS_SUCCESS;
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return MPEMU_STATUS_INVALID_VALUE;
    if (k == 0) return scale_only(stream, m, n, beta, dC, ldc);
    mpemuTerm_t sched[MPEMU_MAX_TERM_SPLITS * MPEMU_MAX_TERM_SPLITS];
    const int end = pr.macBegin + planBegin + planCount;
    if (mpemuTermSchedule(pr.nsplits, end, sched) < end || planCount > 16) return MPEMU_STATUS_INVALID_VALUE;
    GemmTerms terms;
    terms.n = planCount;
    int maxa = 0, maxb = 0;
    for (int t = 0; t < planCount; ++t) {
        terms.ia[t] = sched[pr.macBegin + planBegin + t].i;
        terms.ib[t] = sched[pr.macBegin + planBegin + t].j;
        maxa = terms.ia[t] > maxa ? terms.ia[t] : maxa;
        maxb = terms.ib[t] > maxb ? terms.ib[t] : maxb;
    }
    return run_terms(stream, ta, tb, m, n, k, alpha, Planes{pr.dSA, lda, pr.strideA, maxa + 1},
                     Planes{pr.dSB, ldb, pr.strideB, maxb + 1}, terms, beta, dC, ldc, bf16);
}

constexpr size_t kArenaAlign = 256;
inline size_t align_up(size_t v) { return (v + kArenaAlign - 1) / kArenaAlign * kArenaAlign; }

}  /* namespace */

struct mpemuContext_s {
    void* arena;
    size_t capacity;
    int allocs;
};

/* Split-plane views of A (m x k) then B (k x n) from the start of the arena. */
template <typename WS, typename W>
static mpemuStatus_t carve_planes(mpemuContext_t ctx, int64_t m, int64_t n, int64_t k, int nsplits, WS* ws) {
    if (!ctx || !ws || nsplits < 1) return MPEMU_STATUS_INVALID_VALUE;
    ws->ldA = mpemuSplitLd(m);
    ws->strideA = ws->ldA * k;
    ws->ldB = mpemuSplitLd(k);
    ws->strideB = ws->ldB * n;
    const size_t a = (size_t)ws->strideA * nsplits * sizeof(W), b = (size_t)ws->strideB * nsplits * sizeof(W);
    const size_t need = align_up(a) + b;
    if (!ctx->arena || need > ctx->capacity) return MPEMU_STATUS_INVALID_VALUE;
    ws->sA = reinterpret_cast<W*>(ctx->arena);
    ws->sB = reinterpret_cast<W*>(static_cast<char*>(ctx->arena) + align_up(a));
    ws->nsplits = nsplits;
    return MPEMU_STATUS_SUCCESS;
}

extern "C" {

const char* mpemuStatusString(mpemuStatus_t s) {
    switch (s) {
        case MPEMU_STATUS_SUCCESS: return "MPEMU_STATUS_SUCCESS";
        case MPEMU_STATUS_INVALID_VALUE: return "MPEMU_STATUS_INVALID_VALUE";
        case MPEMU_STATUS_CUDA_ERROR: return "MPEMU_STATUS_CUDA_ERROR";
        case MPEMU_STATUS_CUBLAS_ERROR: return "MPEMU_STATUS_CUBLAS_ERROR";
        default: return "MPEMU_STATUS_UNKNOWN";
    }
}

int64_t mpemuSplitLd(int64_t rows) { return (rows + 7) / 8 * 8; }
int64_t mpemuSplitStride(int64_t lds, int64_t cols) { return lds * cols; }
size_t mpemuSplitBytes(int64_t rows, int64_t cols, int nsplits) {
    if (nsplits < 1 || nsplits > MPEMU_MAX_SPLITS) return 0;
    return (size_t)mpemuSplitStride(mpemuSplitLd(rows), cols) * (size_t)nsplits * 2;
}

int mpemuTermCount(int nsplits) {
    return (nsplits < 1 || nsplits > MPEMU_MAX_TERM_SPLITS) ? 0 : nsplits * nsplits;
}

int mpemuTermSchedule(int nsplits, int maxTerms, mpemuTerm_t* terms) {
    if (nsplits < 1 || nsplits > MPEMU_MAX_TERM_SPLITS || maxTerms <= 0 || !terms) return 0;
    int w = 0;
    for (int bin = 0; bin <= 2 * (nsplits - 1) && w < maxTerms; ++bin)
        for (int i = 0; i <= bin && w < maxTerms; ++i) {
            const int j = bin - i;
            if (i < nsplits && j < nsplits) terms[w++] = mpemuTerm_t{i, j};
        }
    return w;
}

int mpemuMultiwordMacs(int p) { return (p < 1 || p > MPEMU_MAX_SPLITS) ? 0 : p * (p + 1) / 2; }

mpemuStatus_t mpemuSplitBF16(const float* dA, int64_t lda, int64_t rows, int64_t cols, int nsplits,
                             __nv_bfloat16* dS, int64_t lds, int64_t splitStride, cudaStream_t stream) {
    return split_impl<__nv_bfloat16>(dA, lda, rows, cols, nsplits, 1.0f, dS, lds, splitStride, stream);
}

mpemuStatus_t mpemuSplitFP16(const float* dA, int64_t lda, int64_t rows, int64_t cols, int nsplits, float scale,
                             __half* dS, int64_t lds, int64_t splitStride, cudaStream_t stream) {
    if (!(scale > 0.0f)) return MPEMU_STATUS_INVALID_VALUE;
    return split_impl<__half>(dA, lda, rows, cols, nsplits, scale, dS, lds, splitStride, stream);
}

mpemuStatus_t mpemuAutoScaleFP16(const float* dA, int64_t lda, int64_t rows, int64_t cols, float* hScale,
                                 cudaStream_t stream) {
    if (!dA || !hScale) return MPEMU_STATUS_INVALID_VALUE;
    *hScale = 1.0f;
    if (rows <= 0 || cols <= 0) return MPEMU_STATUS_SUCCESS;
    static std::mutex m;
    static float* scratch[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return MPEMU_STATUS_CUDA_ERROR;
    std::lock_guard<std::mutex> lock(m);   /* one scratch word per device: serialise */
    if (!scratch[dev] && cudaMalloc(&scratch[dev], sizeof(float)) != cudaSuccess) return MPEMU_STATUS_CUDA_ERROR;
    if (cudaMemsetAsync(scratch[dev], 0, sizeof(float), stream) != cudaSuccess) return MPEMU_STATUS_CUDA_ERROR;
    k_maxabs_finite<<<grid_for(rows * cols), kBlock, 0, stream>>>(dA, lda, rows, cols, scratch[dev]);
    float hmax = 0.f;
    cudaMemcpyAsync(&hmax, scratch[dev], sizeof(float), cudaMemcpyDeviceToHost, stream);
    if (cudaStreamSynchronize(stream) != cudaSuccess) return MPEMU_STATUS_CUDA_ERROR;
    if (!(hmax > 0.f)) return MPEMU_STATUS_SUCCESS;
    int e = 0;
    std::frexp(4096.0f / hmax, &e);
    const float sc = std::ldexp(1.0f, e - 1);
    *hScale = (sc > 0.f && std::isfinite(sc)) ? sc : 1.0f;
    return MPEMU_STATUS_SUCCESS;
}

mpemuStatus_t mpemuCheckSplitFP16(const float* dA, int64_t lda, int64_t rows, int64_t cols, int nsplits,
                                  float scale, const __half* dS, int64_t lds, int64_t splitStride,
                                  unsigned long long* dCounts, cudaStream_t stream) {
    if (!dA || !dS || !dCounts) return MPEMU_STATUS_INVALID_VALUE;
    if (nsplits < 1 || nsplits > MPEMU_MAX_SPLITS) return MPEMU_STATUS_INVALID_VALUE;
    if (rows <= 0 || cols <= 0) return MPEMU_STATUS_SUCCESS;
    k_check_split<<<grid_for(rows * cols), kBlock, 0, stream>>>(dA, lda, rows, cols, nsplits, scale, dS, lds,
                                                                 splitStride, dCounts);
    return cudaGetLastError() == cudaSuccess ? MPEMU_STATUS_SUCCESS : MPEMU_STATUS_CUDA_ERROR;
}

mpemuStatus_t mpemuGemmBF16(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB, int64_t m,
                            int64_t n, int64_t k, float alpha, const __nv_bfloat16* dAi, int64_t lda,
                            const __nv_bfloat16* dBj, int64_t ldb, float beta, float* dC, int64_t ldc) {
    return gemm_range(handle, opA, opB, m, n, k, alpha, dAi, lda, 0, dBj, ldb, 0, 1, 0, 1, beta, dC, ldc, true);
}

mpemuStatus_t mpemuGemmFP16(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB, int64_t m,
                            int64_t n, int64_t k, float alpha, const __half* dAi, int64_t lda, const __half* dBj,
                            int64_t ldb, float beta, float* dC, int64_t ldc) {
    return gemm_range(handle, opA, opB, m, n, k, alpha, dAi, lda, 0, dBj, ldb, 0, 1, 0, 1, beta, dC, ldc, false);
}

mpemuStatus_t mpemuGemmEmulatedRange(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                     int64_t m, int64_t n, int64_t k, float alpha, const __nv_bfloat16* dSA,
                                     int64_t lda, int64_t strideA, const __nv_bfloat16* dSB, int64_t ldb,
                                     int64_t strideB, int nsplits, int macBegin, int macEnd, float beta, float* dC,
                                     int64_t ldc) {
    return gemm_range(handle, opA, opB, m, n, k, alpha, dSA, lda, strideA, dSB, ldb, strideB, nsplits, macBegin,
                      macEnd, beta, dC, ldc, true);
}

mpemuStatus_t mpemuGemmEmulated(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB, int64_t m,
                                int64_t n, int64_t k, float alpha, const __nv_bfloat16* dSA, int64_t lda,
                                int64_t strideA, const __nv_bfloat16* dSB, int64_t ldb, int64_t strideB,
                                int nsplits, int nmacs, float beta, float* dC, int64_t ldc) {
    return mpemuGemmEmulatedRange(handle, opA, opB, m, n, k, alpha, dSA, lda, strideA, dSB, ldb, strideB, nsplits, 0,
                                  nmacs, beta, dC, ldc);
}

mpemuStatus_t mpemuGemmMultiwordRange(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                      int64_t m, int64_t n, int64_t k, float alpha, const __half* dSA, int64_t lda,
                                      int64_t strideA, float scaleA, const __half* dSB, int64_t ldb,
                                      int64_t strideB, float scaleB, int nsplits, int macBegin, int macEnd,
                                      float beta, float* dC, int64_t ldc) {
    if (!(scaleA > 0.0f) || !(scaleB > 0.0f)) return MPEMU_STATUS_INVALID_VALUE;
    /* the words carry scaleA * scaleB; powers of two in normal use, so exact */
    const float a = alpha / (scaleA * scaleB);
    return gemm_range(handle, opA, opB, m, n, k, a, dSA, lda, strideA, dSB, ldb, strideB, nsplits, macBegin, macEnd,
                      beta, dC, ldc, false);
}

mpemuStatus_t mpemuGemmMultiword(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB, int64_t m,
                                 int64_t n, int64_t k, float alpha, const __half* dSA, int64_t lda, int64_t strideA,
                                 float scaleA, const __half* dSB, int64_t ldb, int64_t strideB, float scaleB,
                                 int nsplits, int nmacs, float beta, float* dC, int64_t ldc) {
    return mpemuGemmMultiwordRange(handle, opA, opB, m, n, k, alpha, dSA, lda, strideA, scaleA, dSB, ldb, strideB,
                                   scaleB, nsplits, 0, nmacs, beta, dC, ldc);
}


/* ------------------------------------------------------------- status ---- */

int mpkDebugGemmStatus(int clear) {
    int sms = 0;
    int* st = gemm_status(&sms);
    if (!st || cudaDeviceSynchronize() != cudaSuccess) return -1;
    int h = 0;
    if (cudaMemcpy(&h, st, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (clear && cudaMemset(st, 0, sizeof(int)) != cudaSuccess) return -1;
    return h;
}

/* ------------------------------------------------------------ context ---- */

mpemuStatus_t mpemuContextCreate(mpemuContext_t* ctx) {
    if (!ctx) return MPEMU_STATUS_INVALID_VALUE;
    *ctx = new (std::nothrow) mpemuContext_s{nullptr, 0, 0};
    return *ctx ? MPEMU_STATUS_SUCCESS : MPEMU_STATUS_CUDA_ERROR;
}

mpemuStatus_t mpemuContextDestroy(mpemuContext_t ctx) {
    if (!ctx) return MPEMU_STATUS_SUCCESS;
    if (ctx->arena) cudaFree(ctx->arena);
    delete ctx;
    return MPEMU_STATUS_SUCCESS;
}

mpemuStatus_t mpemuContextReserve(mpemuContext_t ctx, size_t bytes) {
    if (!ctx) return MPEMU_STATUS_INVALID_VALUE;
    if (bytes <= ctx->capacity) return MPEMU_STATUS_SUCCESS;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return MPEMU_STATUS_CUDA_ERROR;
    if (ctx->arena) cudaFree(ctx->arena);
    ctx->arena = p;
    ctx->capacity = bytes;
    ++ctx->allocs;
    return MPEMU_STATUS_SUCCESS;
}

size_t mpemuContextCapacity(mpemuContext_t ctx) { return ctx ? ctx->capacity : 0; }
void* mpemuContextBase(mpemuContext_t ctx) { return ctx ? ctx->arena : nullptr; }
int mpemuContextAllocCount(mpemuContext_t ctx) { return ctx ? ctx->allocs : 0; }

size_t mpemuBf16WorkspaceBytes(int64_t m, int64_t n, int64_t k, int nsplits) {
    if (nsplits < 1 || m < 0 || n < 0 || k < 0) return 0;
    const size_t a = (size_t)mpemuSplitLd(m) * (size_t)k * (size_t)nsplits * 2;
    const size_t b = (size_t)mpemuSplitLd(k) * (size_t)n * (size_t)nsplits * 2;
    return align_up(a) + align_up(b);
}

size_t mpemuFp16WorkspaceBytes(int64_t m, int64_t n, int64_t k, int nsplits) {
    return mpemuBf16WorkspaceBytes(m, n, k, nsplits);    /* both words are 2 bytes, same layout */
}

mpemuStatus_t mpemuBf16WorkspaceInit(mpemuContext_t ctx, int64_t m, int64_t n, int64_t k, int nsplits,
                                     mpemuBf16Workspace_t* ws) {
    return carve_planes<mpemuBf16Workspace_t, __nv_bfloat16>(ctx, m, n, k, nsplits, ws);
}

mpemuStatus_t mpemuFp16WorkspaceInit(mpemuContext_t ctx, int64_t m, int64_t n, int64_t k, int nsplits,
                                     mpemuFp16Workspace_t* ws) {
    return carve_planes<mpemuFp16Workspace_t, __half>(ctx, m, n, k, nsplits, ws);
}

/* ------------------------------------------------------------ batched ---- */

size_t mpemuBatchWorkspaceBytes(int64_t m, int64_t n, int capacity, int elemBytes) {
    if (capacity < 1 || m < 0 || n < 0 || elemBytes < 1) return 0;
    const int64_t ldt = (m + 15) / 16 * 16;
    const size_t slices = (size_t)ldt * (size_t)n * (size_t)capacity * (size_t)elemBytes;
    const size_t ptrs = (size_t)capacity * sizeof(void*);
    return align_up(slices) + 3 * align_up(ptrs) + align_up((size_t)capacity * sizeof(int));
}

mpemuStatus_t mpemuBatchWorkspaceInit(mpemuContext_t ctx, int64_t m, int64_t n, int capacity, int elemBytes,
                                      size_t arenaOffset, mpemuBatchWorkspace_t* bw) {
    if (!ctx || !bw || capacity < 1 || elemBytes < 1) return MPEMU_STATUS_INVALID_VALUE;
    const size_t need = mpemuBatchWorkspaceBytes(m, n, capacity, elemBytes);
    const size_t start = align_up(arenaOffset);
    if (!ctx->arena || start + need > ctx->capacity) return MPEMU_STATUS_INVALID_VALUE;
    char* base = static_cast<char*>(ctx->arena) + start;
    bw->ldt = (m + 15) / 16 * 16;
    bw->strideT = bw->ldt * n;
    bw->capacity = capacity;
    bw->planned = 0;
    bw->elemBytes = elemBytes;
    size_t off = 0;
    bw->tmp = base;
    off = align_up((size_t)bw->strideT * capacity * elemBytes);
    bw->aptr = reinterpret_cast<const void**>(base + off);
    off = align_up(off + (size_t)capacity * sizeof(void*));
    bw->bptr = reinterpret_cast<const void**>(base + off);
    off = align_up(off + (size_t)capacity * sizeof(void*));
    bw->cptr = reinterpret_cast<void**>(base + off);
    off = align_up(off + (size_t)capacity * sizeof(void*));
    bw->bins = reinterpret_cast<int*>(base + off);
    return MPEMU_STATUS_SUCCESS;
}

mpemuStatus_t mpemuBatchPlan(mpemuBatchWorkspace_t* bw, const void* dSA, int64_t strideA, const void* dSB,
                             int64_t strideB, int splitElemBytes, int nsplits, int macBegin, int macEnd,
                             cudaStream_t stream) {
    if (!bw || !dSA || !dSB || splitElemBytes < 1) return MPEMU_STATUS_INVALID_VALUE;
    if (macEnd == MPEMU_ALL_MACS) macEnd = mpemuTermCount(nsplits);
    const int count = macEnd - macBegin;
    if (macBegin < 0 || count < 1 || count > bw->capacity) return MPEMU_STATUS_INVALID_VALUE;
    std::vector<mpemuTerm_t> sched((size_t)macEnd);
    if (mpemuTermSchedule(nsplits, macEnd, sched.data()) < macEnd) return MPEMU_STATUS_INVALID_VALUE;
    /* the same device arrays the reference fills (plane pointers, slice
     * pointers, bins), for callers that read them */
    std::vector<const void*> ha((size_t)count), hb((size_t)count);
    std::vector<void*> hc((size_t)count);
    std::vector<int> hbin((size_t)count);
    for (int t = 0; t < count; ++t) {
        const mpemuTerm_t& tm = sched[(size_t)(macBegin + t)];
        ha[t] = static_cast<const char*>(dSA) + (size_t)tm.i * strideA * splitElemBytes;
        hb[t] = static_cast<const char*>(dSB) + (size_t)tm.j * strideB * splitElemBytes;
        hc[t] = static_cast<char*>(bw->tmp) + (size_t)t * bw->strideT * bw->elemBytes;
        hbin[t] = tm.i + tm.j;
    }
    const size_t pb = (size_t)count * sizeof(void*);
    if (cudaMemcpyAsync((void*)bw->aptr, ha.data(), pb, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync((void*)bw->bptr, hb.data(), pb, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync((void*)bw->cptr, hc.data(), pb, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync(bw->bins, hbin.data(), (size_t)count * sizeof(int), cudaMemcpyHostToDevice, stream) !=
            cudaSuccess)
        return MPEMU_STATUS_CUDA_ERROR;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return MPEMU_STATUS_CUDA_ERROR;
    {
        std::lock_guard<std::mutex> lock(g_plan_mu);
        plans()[(const void*)bw->aptr] = PlanRecord{dSA, strideA, dSB, strideB, nsplits, macBegin, count,
                                                    splitElemBytes};
    }
    bw->planned = count;
    return MPEMU_STATUS_SUCCESS;
}

mpemuStatus_t mpemuGemmEmulatedBatched(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                       int64_t m, int64_t n, int64_t k, float alpha, int planBegin, int planCount,
                                       float beta, float* dC, int64_t ldc, const mpemuBatchWorkspace_t* bw,
                                       cudaStream_t stream) {
    return batched_run(handle, opA, opB, m, n, k, alpha, planBegin, planCount, beta, dC, ldc, bw, stream, true);
}

mpemuStatus_t mpemuGemmMultiwordBatched(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                        int64_t m, int64_t n, int64_t k, float alpha, float scaleA, float scaleB,
                                        int planBegin, int planCount, float beta, float* dC, int64_t ldc,
                                        const mpemuBatchWorkspace_t* bw, cudaStream_t stream) {
    if (!(scaleA > 0.0f) || !(scaleB > 0.0f)) return MPEMU_STATUS_INVALID_VALUE;
    return batched_run(handle, opA, opB, m, n, k, alpha / (scaleA * scaleB), planBegin, planCount, beta, dC, ldc,
                       bw, stream, false);
}

/* ----------------------------------------------------- concatenated-k ---- */

int64_t mpemuStackedLd(int64_t k, int nsplits) {
    if (nsplits < 1) return 0;
    return ((int64_t)nsplits * k + 7) / 8 * 8;
}

size_t mpemuStackedBytes(int64_t k, int64_t n, int nsplits, int elemBytes) {
    if (nsplits < 1 || elemBytes < 1) return 0;
    return (size_t)mpemuStackedLd(k, nsplits) * (size_t)n * (size_t)elemBytes;
}

mpemuStatus_t mpemuSplitBF16Stacked(const float* dB, int64_t ldb, int64_t k, int64_t n, int nsplits,
                                    __nv_bfloat16* dS, int64_t lds, cudaStream_t stream) {
    return split_stacked<__nv_bfloat16>(dB, ldb, k, n, nsplits, 1.0f, dS, lds, stream);
}

mpemuStatus_t mpemuSplitFP16Stacked(const float* dB, int64_t ldb, int64_t k, int64_t n, int nsplits, float scale,
                                    __half* dS, int64_t lds, cudaStream_t stream) {
    return split_stacked<__half>(dB, ldb, k, n, nsplits, scale, dS, lds, stream);
}

mpemuStatus_t mpemuGemmEmulatedConcat(cublasHandle_t handle, int64_t m, int64_t n, int64_t k, float alpha,
                                      const __nv_bfloat16* dSA, int64_t lda, const __nv_bfloat16* dSB, int64_t ldsb,
                                      int nsplits, int nbins, float beta, float* dC, int64_t ldc) {
    return concat_run(handle, m, n, k, alpha, dSA, lda, dSB, ldsb, nsplits, nbins, beta, dC, ldc, true);
}

mpemuStatus_t mpemuGemmMultiwordConcat(cublasHandle_t handle, int64_t m, int64_t n, int64_t k, float alpha,
                                       float scaleA, float scaleB, const __half* dSA, int64_t lda,
                                       const __half* dSB, int64_t ldsb, int nsplits, int nbins, float beta,
                                       float* dC, int64_t ldc) {
    if (!(scaleA > 0.0f) || !(scaleB > 0.0f)) return MPEMU_STATUS_INVALID_VALUE;
    return concat_run(handle, m, n, k, alpha / (scaleA * scaleB), dSA, lda, dSB, ldsb, nsplits, nbins, beta, dC,
                      ldc, false);
}

}  /* extern "C" */
