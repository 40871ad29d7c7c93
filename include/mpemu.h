/* mpemu.h -- FP32 GEMM emulated on B200 tensor cores (split-precision SGEMM).
 *
 * Drop-in for the split-precision GEMM C ABI of CornellHPC/mpkmeans
 * (gemm-emulation/include/mpemu/mpemu.h:52-410): BF16 n-word and FP16
 * p-word (power-of-two scaled) splits, the ascending-bin term schedule, single
 * cross products and the range / whole drivers.  Same enums, signatures and
 * column-major, cuBLAS-style conventions (leading dimensions, op flags).
 *
 * What runs underneath is different: every cross product of a range is
 * accumulated by one tcgen05 kernel in TMEM (FP32), term by term, with the
 * operands staged by TMA -- one launch per call instead of one cuBLAS GEMM per
 * term.  With alpha = 1 and beta in {0, 1} a range [b, e) continued by
 * [e, f) gives bit for bit the result of [b, f), as in the reference.
 * The cuBLAS handle is used only for its stream.
 *
 * The workspace context, the batched and the concatenated-k variants
 * (mpemu.h:589-857) are here too, with the same signatures and struct
 * layouts, and also run the one-launch kernel: a batched call does not write
 * its temporary slices, a concatenated call issues no per-bin GEMMs.
 * Out of scope: the Ozaki-I INT8 (FP64) scheme, mpemu.h:412-586, and its
 * workspace and batched forms.
 */
#ifndef MPEMU_B200_H
#define MPEMU_B200_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cublas_v2.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* Same values as the reference (mpemu.h:52-57). */
typedef enum {
    MPEMU_STATUS_SUCCESS = 0,
    MPEMU_STATUS_INVALID_VALUE = 1,
    MPEMU_STATUS_CUDA_ERROR = 2,
    MPEMU_STATUS_CUBLAS_ERROR = 3
} mpemuStatus_t;

#define MPEMU_MAX_SPLITS 4
#define MPEMU_MAX_TERM_SPLITS 16
#define MPEMU_ALL_MACS (-1)

/* mpemu.h:69 */
const char* mpemuStatusString(mpemuStatus_t s);

/* Packed split buffer sizing (mpemu.h:79-85): plane leading dimension is rows
 * rounded up to 8 elements (16 bytes), planes are lds*cols apart. */
int64_t mpemuSplitLd(int64_t rows);
int64_t mpemuSplitStride(int64_t lds, int64_t cols);
size_t mpemuSplitBytes(int64_t rows, int64_t cols, int nsplits);

static inline __nv_bfloat16* mpemuSplitPlane(__nv_bfloat16* dS, int64_t splitStride, int s) {
    return dS + (int64_t)s * splitStride;
}
static inline const __nv_bfloat16* mpemuSplitPlaneConst(const __nv_bfloat16* dS, int64_t splitStride, int s) {
    return dS + (int64_t)s * splitStride;
}

/* b[0] = bf16(a), b[s] = bf16(a - sum_{t<s} b[t]) (round to nearest even, exact
 * FP32 residuals), column major.  mpemu.h:112-117. */
mpemuStatus_t mpemuSplitBF16(const float* dA, int64_t lda, int64_t rows, int64_t cols, int nsplits,
                             __nv_bfloat16* dS, int64_t lds, int64_t splitStride, cudaStream_t stream);

/* dC := alpha * op(dAi) * op(dBj) + beta * dC for one BF16 plane pair, FP32
 * accumulation.  mpemu.h:149-156. */
mpemuStatus_t mpemuGemmBF16(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                            int64_t m, int64_t n, int64_t k, float alpha,
                            const __nv_bfloat16* dAi, int64_t lda, const __nv_bfloat16* dBj, int64_t ldb,
                            float beta, float* dC, int64_t ldc);

typedef struct { int i; int j; } mpemuTerm_t;

/* nsplits^2 (mpemu.h:166) and the ascending-bin, then ascending-i, order of
 * the cross products (mpemu.h:173, gemm.cu:43-60). */
int mpemuTermCount(int nsplits);
int mpemuTermSchedule(int nsplits, int maxTerms, mpemuTerm_t* terms);

/* dC := alpha * sum_{t in [macBegin, macEnd)} op(A_it) op(B_jt) + beta * dC.
 * mpemu.h:218-226. */
mpemuStatus_t mpemuGemmEmulatedRange(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                     int64_t m, int64_t n, int64_t k, float alpha,
                                     const __nv_bfloat16* dSA, int64_t lda, int64_t strideA,
                                     const __nv_bfloat16* dSB, int64_t ldb, int64_t strideB,
                                     int nsplits, int macBegin, int macEnd, float beta, float* dC, int64_t ldc);

/* The first nmacs terms.  mpemu.h:235-243. */
mpemuStatus_t mpemuGemmEmulated(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                int64_t m, int64_t n, int64_t k, float alpha,
                                const __nv_bfloat16* dSA, int64_t lda, int64_t strideA,
                                const __nv_bfloat16* dSB, int64_t ldb, int64_t strideB,
                                int nsplits, int nmacs, float beta, float* dC, int64_t ldc);

/* p(p+1)/2, the i+j <= p+1 cut of the multiword scheme.  mpemu.h:289. */
int mpemuMultiwordMacs(int p);

/* FP16 words of scale*A (scale a power of two).  mpemu.h:307-312. */
mpemuStatus_t mpemuSplitFP16(const float* dA, int64_t lda, int64_t rows, int64_t cols, int nsplits, float scale,
                             __half* dS, int64_t lds, int64_t splitStride, cudaStream_t stream);

static inline __half* mpemuSplitPlaneFP16(__half* dS, int64_t splitStride, int s) {
    return dS + (int64_t)s * splitStride;
}
static inline const __half* mpemuSplitPlaneFP16Const(const __half* dS, int64_t splitStride, int s) {
    return dS + (int64_t)s * splitStride;
}

/* Largest power of two with scale * max|A| <= 4096 (finite entries); 1 for an
 * all-zero matrix; synchronises `stream`.  mpemu.h:332-334. */
mpemuStatus_t mpemuAutoScaleFP16(const float* dA, int64_t lda, int64_t rows, int64_t cols, float* hScale,
                                 cudaStream_t stream);

/* Word classification [overflow, subnormal-or-flushed, clean], accumulated
 * into dCounts (3 x uint64, device).  mpemu.h:340-346. */
mpemuStatus_t mpemuCheckSplitFP16(const float* dA, int64_t lda, int64_t rows, int64_t cols, int nsplits,
                                  float scale, const __half* dS, int64_t lds, int64_t splitStride,
                                  unsigned long long* dCounts, cudaStream_t stream);

/* One FP16 cross product.  mpemu.h:358-365. */
mpemuStatus_t mpemuGemmFP16(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                            int64_t m, int64_t n, int64_t k, float alpha,
                            const __half* dAi, int64_t lda, const __half* dBj, int64_t ldb,
                            float beta, float* dC, int64_t ldc);

/* Range / whole drivers over FP16 words; 1/(scaleA*scaleB) is folded into
 * alpha.  mpemu.h:388-410. */
mpemuStatus_t mpemuGemmMultiwordRange(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                      int64_t m, int64_t n, int64_t k, float alpha,
                                      const __half* dSA, int64_t lda, int64_t strideA, float scaleA,
                                      const __half* dSB, int64_t ldb, int64_t strideB, float scaleB,
                                      int nsplits, int macBegin, int macEnd, float beta, float* dC, int64_t ldc);
mpemuStatus_t mpemuGemmMultiword(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                 int64_t m, int64_t n, int64_t k, float alpha,
                                 const __half* dSA, int64_t lda, int64_t strideA, float scaleA,
                                 const __half* dSB, int64_t ldb, int64_t strideB, float scaleB,
                                 int nsplits, int nmacs, float beta, float* dC, int64_t ldc);

/* ---------------------------------------------- workspace context ---- */

/* One growable device arena (mpemu.h:625-638): Reserve grows it with one
 * allocation (a no-op when it fits), views are carved from it without any. */
typedef struct mpemuContext_s* mpemuContext_t;
mpemuStatus_t mpemuContextCreate(mpemuContext_t* ctx);
mpemuStatus_t mpemuContextDestroy(mpemuContext_t ctx);
mpemuStatus_t mpemuContextReserve(mpemuContext_t ctx, size_t bytes);
size_t mpemuContextCapacity(mpemuContext_t ctx);
void* mpemuContextBase(mpemuContext_t ctx);
int mpemuContextAllocCount(mpemuContext_t ctx);

/* Arena bytes of the split planes of A (m x k) and B (k x n), mpemu.h:641-642. */
size_t mpemuBf16WorkspaceBytes(int64_t m, int64_t n, int64_t k, int nsplits);
size_t mpemuFp16WorkspaceBytes(int64_t m, int64_t n, int64_t k, int nsplits);

/* Views of those planes, mpemu.h:645-655 (same layouts). */
typedef struct {
    __nv_bfloat16* sA; int64_t ldA, strideA;
    __nv_bfloat16* sB; int64_t ldB, strideB;
    int nsplits;
} mpemuBf16Workspace_t;

typedef struct {
    __half* sA; int64_t ldA, strideA;
    __half* sB; int64_t ldB, strideB;
    int nsplits;
} mpemuFp16Workspace_t;

/* Carve the views (mpemu.h:670-677); INVALID_VALUE when the arena is short. */
mpemuStatus_t mpemuBf16WorkspaceInit(mpemuContext_t ctx, int64_t m, int64_t n, int64_t k, int nsplits,
                                     mpemuBf16Workspace_t* ws);
mpemuStatus_t mpemuFp16WorkspaceInit(mpemuContext_t ctx, int64_t m, int64_t n, int64_t k, int nsplits,
                                     mpemuFp16Workspace_t* ws);

/* ------------------------------------------------------ batched ---- */

/* mpemu.h:714-724, same layout.  The plan arrays are filled as the reference
 * fills them; the product sum itself runs in the one-launch kernel, so the
 * temporary slices are never written. */
typedef struct {
    void*        tmp;
    int64_t      ldt, strideT;
    const void** aptr;
    const void** bptr;
    void**       cptr;
    int*         bins;
    int          capacity;
    int          planned;
    int          elemBytes;
} mpemuBatchWorkspace_t;

/* mpemu.h:727-737 */
size_t mpemuBatchWorkspaceBytes(int64_t m, int64_t n, int capacity, int elemBytes);
mpemuStatus_t mpemuBatchWorkspaceInit(mpemuContext_t ctx, int64_t m, int64_t n, int capacity, int elemBytes,
                                      size_t arenaOffset, mpemuBatchWorkspace_t* bw);

/* Plan schedule positions [macBegin, macEnd) over split planes at dSA / dSB
 * (mpemu.h:746-751); synchronises `stream`. */
mpemuStatus_t mpemuBatchPlan(mpemuBatchWorkspace_t* bw, const void* dSA, int64_t strideA, const void* dSB,
                             int64_t strideB, int splitElemBytes, int nsplits, int macBegin, int macEnd,
                             cudaStream_t stream);

/* dC := alpha * sum(planned products [planBegin, planBegin + planCount)) +
 * beta * dC; A planes have leading dimension mpemuSplitLd(m), B planes
 * mpemuSplitLd(k), as in the reference (mpemu.h:756-771). */
mpemuStatus_t mpemuGemmEmulatedBatched(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                       int64_t m, int64_t n, int64_t k, float alpha, int planBegin, int planCount,
                                       float beta, float* dC, int64_t ldc, const mpemuBatchWorkspace_t* bw,
                                       cudaStream_t stream);
mpemuStatus_t mpemuGemmMultiwordBatched(cublasHandle_t handle, cublasOperation_t opA, cublasOperation_t opB,
                                        int64_t m, int64_t n, int64_t k, float alpha, float scaleA, float scaleB,
                                        int planBegin, int planCount, float beta, float* dC, int64_t ldc,
                                        const mpemuBatchWorkspace_t* bw, cudaStream_t stream);

/* ------------------------------------------------- concatenated-k ---- */

/* Stacked, reversed right operand: word j of B(r, c) at row (nsplits-1-j)*k
 * + r of a (nsplits*k) x n column-major buffer (mpemu.h:819-831). */
int64_t mpemuStackedLd(int64_t k, int nsplits);
size_t mpemuStackedBytes(int64_t k, int64_t n, int nsplits, int elemBytes);
mpemuStatus_t mpemuSplitBF16Stacked(const float* dB, int64_t ldb, int64_t k, int64_t n, int nsplits,
                                    __nv_bfloat16* dS, int64_t lds, cudaStream_t stream);
mpemuStatus_t mpemuSplitFP16Stacked(const float* dB, int64_t ldb, int64_t k, int64_t n, int nsplits, float scale,
                                    __half* dS, int64_t lds, cudaStream_t stream);

/* dC := alpha * sum of the products in bins [0, nbins) + beta * dC, op N on
 * both sides; A's planes sit at column blocks i*k of dSA (mpemu.h:837-851). */
mpemuStatus_t mpemuGemmEmulatedConcat(cublasHandle_t handle, int64_t m, int64_t n, int64_t k, float alpha,
                                      const __nv_bfloat16* dSA, int64_t lda, const __nv_bfloat16* dSB, int64_t ldsb,
                                      int nsplits, int nbins, float beta, float* dC, int64_t ldc);
mpemuStatus_t mpemuGemmMultiwordConcat(cublasHandle_t handle, int64_t m, int64_t n, int64_t k, float alpha,
                                       float scaleA, float scaleB, const __half* dSA, int64_t lda,
                                       const __half* dSB, int64_t ldsb, int nsplits, int nbins, float beta,
                                       float* dC, int64_t ldc);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#endif /* MPEMU_B200_H */
