/* mpkmeans.h -- C interface of the B200-native mixed-precision k-means engine.
 *
 * Drop-in for the k-means C ABI of CornellHPC/mpkmeans
 * (kmeans/include/mpkmeans/mpkmeans.h).  Types, enum values, struct layouts
 * and function signatures are kept identical so that a caller of the
 * reference links against libmpkmeans_b200.so unchanged; each declaration
 * below names the reference declaration it replaces.
 *
 * Engine summary (what the drivers do on the device):
 *   - points and centroids are split once per fit / per iteration into FP16
 *     hi/lo words after a power-of-two scale;
 *   - one tcgen05 kernel forms hi*hi + lo*hi + hi*lo in TMEM and keeps a per
 *     row top-4 of D = ||c||^2 - 2 x.c, so the n x k matrix never reaches HBM;
 *   - rows whose runner-up is inside the certified error bound are re-decided
 *     by an FP32 recomputation of their candidate centroids only;
 *   - the centroid update is an exact fixed-point segmented sum of the points
 *     per label (order independent, identical on any number of GPUs).
 * The labels equal those of an FP32 evaluation of fmaf(-2, x.c, ||c||^2) with
 * the reference's FP32 refinement order and smaller-index tie break.
 *
 * All pointers named dX are device pointers owned by the caller.  Work runs
 * on the stream of the cuBLAS handle (cublasGetStream), or on the legacy
 * default stream when the handle is NULL.  No cuBLAS routine runs.
 */
#ifndef MPKMEANS_B200_H
#define MPKMEANS_B200_H

#include <cublas_v2.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  Same values as the reference (mpkmeans.h:32-39). */
typedef enum {
    MPK_OK = 0,
    MPK_ERR_CUDA = 1,
    MPK_ERR_CUBLAS = 2,
    MPK_ERR_CUSPARSE = 3,
    MPK_ERR_INVALID = 4,
    MPK_ERR_ALLOC = 5
} mpkStatus;

/* Accumulator request for mpkMeansMixed (reference mpkmeans.h:49-52).  The
 * engine always accumulates in FP32 on the tensor cores; MPK_ACCUM_FP16 only
 * changes what mpkEpsilon reports. */
typedef enum {
    MPK_ACCUM_FP32 = 0,
    MPK_ACCUM_FP16 = 1
} mpkAccum;

/* Run parameters; layout of the reference's mpkParams (mpkmeans.h:54-110).
 *   max_iter   iterations (exactly this many unless tol stops earlier)
 *   tol        > 0: stop once ||C - C_prev||_F < tol (checked after the
 *              update, as the reference does); 0 disables
 *   use_cond3, use_cond6
 *              both 0 selects the no-refinement mode: the emulated argmin is
 *              taken as final (no FP32 recheck); any other combination runs
 *              the certified filter and FP32 refinement
 *   cascade, accum, mw_macs, mw_gather_frac, cuvs_batch, rt_theta
 *              accepted for ABI compatibility; they select reference schemes
 *              this engine replaces and do not change its result
 *   verify     unused (the oracle lives in the test suite)
 *   verbose    per-iteration line on stderr */
typedef struct {
    int   max_iter;
    float tol;
    int   use_cond3;
    int   use_cond6;
    int   cascade;
    int   accum;
    int   mw_macs;
    float mw_gather_frac;
    int   cuvs_batch;
    float rt_theta;
    int   verify;
    int   verbose;
} mpkParams;

#define MPK_MAX_HIST 256

/* Run statistics; layout of the reference's mpkStats (mpkmeans.h:114-181).
 * This engine fills: iters, inertia, hp_baseline (n*k per iteration),
 * hp_reference (0: no per-row reference entry is needed), hp_update (FP32
 * candidate distances recomputed), tested (n*(k-1) per iteration), n_hist and
 * hist_survivors (rows refined per iteration), and the timings:
 * t_total_ms, t_prep_ms (the one-off split of the points), t_gemm_lo_ms (the
 * assignment steps: centroid split, fused split GEMM + argmin kernel and the
 * refinement, which run back to back and are timed as one), t_dist_ms
 * (t_prep_ms + t_gemm_lo_ms), t_update_ms (centroid update).  With
 * params.verify, every iteration's labels are checked (untimed) against the
 * FP32 argmin over all k in the refinement's order: verify_label_diff counts
 * the rows that differ, verify_excluded_best the same when the refinement ran
 * (a violation of the certified bound: 0 when it holds; 0 without the
 * refinement, which excludes nothing), verify_excess sums D(label) -
 * D(argmin) over them, and stats_built is 1.  Other fields are 0. */
typedef struct {
    int    iters;
    double inertia;
    long long hp_baseline;
    long long hp_reference;
    long long hp_update;
    long long mw_products;
    long long mw_refine_rows;
    long long tested;
    long long excl_cond3;
    long long excl_cond6;
    long long excl_both;
    int       n_hist;
    long long hist_survivors[MPK_MAX_HIST];
    long long verify_excluded_best;
    long long verify_label_diff;
    double    verify_excess;
    int stats_built;
    double t_total_ms;
    double t_dist_ms;
    double t_prep_ms;
    double t_gemm_lo_ms;
    double t_argmin_ms;
    double t_hp_update_ms;
    double t_assign_ms;
    double t_update_ms;
} mpkStats;

/* Defaults: max_iter 100, tol 0, use_cond3 = use_cond6 = 1, accum FP32,
 * mw_macs 3, the rest 0.  Replaces mpkParamsInit (mpkmeans.h:183,
 * kmeans/src/mpkmeans.cu:87-100). */
void mpkParamsInit(mpkParams* p);

/* Relative error bound 2*u16 + gamma_d of an FP16-operand product with the
 * named accumulator; negative when d*u >= 1.  Same formula as the reference
 * (mpkmeans.h:192, kmeans/src/mpkmeans.cu:111-119). */
double mpkEpsilon(int d, int accum);

/* P += max|P| in place; *out_shift receives max|P|.  Replaces
 * mpkShiftNonNegative (mpkmeans.h:197).  This engine does not need the shift
 * (its bound is norm based); the function is kept for callers that apply it. */
mpkStatus mpkShiftNonNegative(float* dP, int n, int d, float* out_shift);

/* Per-feature z-score in place, FP64 two pass.  Replaces mpkStandardize
 * (mpkmeans.h:213). */
mpkStatus mpkStandardize(float* dP, int n, int d);

/* Add delta to every entry of a k x d block.  Replaces mpkShiftCentroids
 * (mpkmeans.h:216). */
mpkStatus mpkShiftCentroids(float* dC, int k, int d, float delta);

/* Mixed-precision Lloyd.  dP n x d row major, dC k x d in/out (initial ->
 * final centroids), dAssign n labels out.  Labels are the assignment against
 * the centroids of the last iteration; dC holds the centroids after the last
 * update.  Replaces mpkMeansMixed (mpkmeans.h:224-227). */
mpkStatus mpkMeansMixed(cublasHandle_t blas, const float* dP, int n, int d, int k,
                        float* dC, int* dAssign, const mpkParams* params, mpkStats* stats);

/* FP32 Lloyd.  Same engine: its labels already equal the FP32 argmin, so the
 * result is that of an FP32 run with the reference's refinement dot order.
 * Replaces mpkMeansFP32 (mpkmeans.h:261-264). */
mpkStatus mpkMeansFP32(cublasHandle_t blas, const float* dP, int n, int d, int k,
                       float* dC, int* dAssign, const mpkParams* params, mpkStats* stats);

/* Reference schemes that this engine supersedes.  mpkMeansMultiword runs the
 * engine (whose split is the double-fp16 scheme with an exact FP32 recheck)
 * and reports mw_products = 3 per iteration.  mpkMeansBaselineRT and
 * mpkMeansCuvs return MPK_ERR_INVALID, as the reference does when the scheme
 * is not built in.  (mpkmeans.h:232-234, 249-251, 293-295, 309.) */
mpkStatus mpkMeansMultiword(cublasHandle_t blas, const float* dP, int n, int d, int k,
                            float* dC, int* dAssign, const mpkParams* params, mpkStats* stats);
mpkStatus mpkMeansBaselineRT(cublasHandle_t blas, const float* dP, int n, int d, int k,
                             float* dC, int* dAssign, const mpkParams* params, mpkStats* stats);
int mpkHaveCuvs(void);
mpkStatus mpkMeansCuvs(cublasHandle_t blas, const float* dP, int n, int d, int k,
                       float* dC, int* dAssign, const mpkParams* params, mpkStats* stats);
double mpkMultiwordEpsilon(int d, int macs);

/* Data helpers (mpkmeans.h:318-341).  mpkMakeBlobs and mpkInitRandomPoints
 * draw exactly the reference's random sequences (std::mt19937), so the same
 * seed yields the same points and the same initial centroids. */
mpkStatus mpkLoadBin(const char* path, int d, long long max_rows, int* out_n, float** out_P);
mpkStatus mpkLoadLibsvm(const char* path, int* out_n, int* out_d, float** out_P, int** out_labels,
                        int* out_nclasses);
void mpkMakeBlobs(int n, int d, int k, float std, float center_box, unsigned seed, float* hP, int* hLabels);
mpkStatus mpkInitRandomPoints(const float* dP, int n, int d, int k, unsigned seed, float* dC);

/* k-means++ seeding on the device: k rows of dP (n x d, row major) written to
 * dC (k x d), D^2-weighted, from `seed`.  No reference counterpart (the
 * reference seeds with mpkInitRandomPoints only; configuration 1 asks for
 * k-means++).  Distances are FP64 and the sampling uses exact integer
 * weights, so the picks do not depend on the launch shape: the same seed gives
 * the same rows on any device.  Synchronous on the default stream.
 * MPK_ERR_INVALID unless 0 < k <= n and d > 0. */
mpkStatus mpkInitKMeansPP(const float* dP, int n, int d, int k, unsigned long long seed, float* dC);

/* Engine scratch comes from one stream-ordered memory pool per device that
 * keeps freed blocks cached, so repeated fits allocate nothing new.  This
 * returns the cached blocks of `device` (-1: the current one) to the driver;
 * it synchronises that device.  No reference counterpart (the reference
 * mallocs and frees its scratch in every call). */
mpkStatus mpkTrimMemoryPool(int device);

/* ------------------------------------------------ new: explicit steps --- */

/* One assignment pass of the engine: dAssign[i] = argmin_j of the FP32
 * distance of row i to centroid j (smaller index on ties).  Replaces the
 * reference's internal launcher chain mpkLaunchToHalf + cublasGemmEx +
 * mpkLaunchArgminCount + mpkLaunchUpdateFlat + mpkLaunchUnpack
 * (kmeans/src/mpk_internal.cuh:393-447), which is not exported there. */
mpkStatus mpkAssign(cublasHandle_t blas, const float* dP, int n, int d, int k,
                    const float* dC, int* dAssign, const mpkParams* params, mpkStats* stats);

/* One centroid update: dC[j] = mean of the rows labelled j (empty clusters
 * keep dC[j]); dMoved2 (k floats, may be NULL) receives ||c_new - c_old||^2.
 * Replaces mpkLaunchZero + mpkLaunchAccumulate + mpkLaunchFinalizeCentroids
 * (kmeans/src/mpk_internal.cuh:499-510). */
mpkStatus mpkUpdate(cublasHandle_t blas, const float* dP, int n, int d, int k,
                    const int* dAssign, float* dC, float* dMoved2);

/* Single-process multi-GPU Lloyd over row shards: shard g of nshard[g] rows
 * lives on device devices[g] at dPshard[g]; dC[g] (k x d on device g) holds
 * the initial centroids on entry (identical on every device) and the final
 * centroids on return; dAssign[g] receives shard g's labels.  One NCCL
 * allreduce of the exact int64 sums and counts per iteration.  New entry
 * point (the reference is single-GPU, mpkmeans.cu:308). */
mpkStatus mpkMeansMixedMG(int ngpu, const int* devices, const float* const* dPshard, const int* nshard,
                          int d, int k, float* const* dC, int* const* dAssign,
                          const mpkParams* params, mpkStats* stats);

/* The centroid update of mpkUpdate for callers that cannot allocate device
 * memory (a device owned by a pool or custom allocator, an allocator that may
 * not be re-entered from a library, a fixed device footprint).  It calls no
 * cudaMalloc, cudaFree or allocating library routine: its scratch is one
 * fixed 32 MiB array in the library's device image, held by every GPU that
 * loads the library until exit.  Sizes are limited by that array:
 *   256 + 8*(k*d + k) + 3*4*(k + 1) + 4*n bytes (each part rounded up to
 *   256) must not exceed 32 MiB -- e.g. n up to about 8.1 million rows at
 *   d = 128, k = 1024; larger sizes return MPK_ERR_INVALID (use mpkUpdate).
 * The first call on each device looks up the array's device address (make it
 * before any stream capture); with CUDA's lazy module loading it is also the
 * call that places the 32 MiB on that device, so a caller whose footprint must
 * stay fixed makes one call at start-up.  The array is shared by every call and keeps
 * the last call's contents (cleared where needed at each call): calls that
 * overlap on the GPU race.  Synchronises `stream` to report invalid labels.
 * Same result as mpkUpdate, bit for bit.  No counterpart in the reference. */
mpkStatus mpkUpdateNoAlloc(cudaStream_t stream, const float* dP, int n, int d, int k,
                           const int* dAssign, float* dC, float* dMoved2);

/* ----------------------------------------------- new: engine handle --- */

/* A fit in explicit steps, for callers that drive the iteration themselves
 * (one process per GPU, their own collective between the steps).  The engine
 * keeps the split points and all scratch on its device; it allocates in
 * mpkEngineCreate only.
 *
 *   pmax_global   max |P| over every shard (and the initial centroids); <= 0
 *                 measures this shard's P and dC0 instead.  Shards that must
 *                 agree bit for bit pass the same value.
 *   n_global      total rows over every shard (fixes the update's fixed-point
 *                 precision); <= 0 means n.
 * Sums buffer layout: k*d int64 coordinate sums, then k int64 counts, in
 * fixed point with mpkEngineFracBits fractional bits.  Summing the buffers of
 * all shards (an int64 allreduce) and finalising gives the exact global
 * update. */
typedef struct mpkEngine_s* mpkEngine;

mpkStatus mpkEngineCreate(mpkEngine* out, const float* dP, long long n, int d, int k, const float* dC0,
                          float pmax_global, long long n_global, cudaStream_t stream);
mpkStatus mpkEngineDestroy(mpkEngine e);
/* labels of this shard against dC (k x d, device) */
mpkStatus mpkEngineAssign(mpkEngine e, const float* dC, int* dAssign, int refine);
/* zero dSums, then add this shard's fixed-point sums and counts */
mpkStatus mpkEngineAccumulate(mpkEngine e, const int* dAssign, long long* dSums);
/* dC = finalised centroids from (globally reduced) dSums; dMoved2 may be NULL */
mpkStatus mpkEngineFinalize(mpkEngine e, const long long* dSums, float* dC, float* dMoved2);
/* iters whole Lloyd iterations of this engine alone -- assign, accumulate,
 * finalize in turn, no collective between -- with exactly their result.  The
 * first call for a given (dC, dAssign, dSums, refine) captures one iteration
 * as three CUDA graphs (assignment; refinement; update) and later calls
 * replay them, so
 * small problems are not held to the host's launch rate.  On the legacy
 * default stream (not capturable) it launches the kernels directly. */
mpkStatus mpkEngineIterate(mpkEngine e, float* dC, int* dAssign, long long* dSums, int iters, int refine);
/* One multi-GPU step without the finalisation: Assign (refine as given)
 * then Accumulate into dSums, replayed from CUDA graphs like Iterate (the
 * caller then allreduces dSums and calls Finalize).  dC is only read. */
mpkStatus mpkEngineStep(mpkEngine e, const float* dC, int* dAssign, long long* dSums, int refine);
/* FP64 inertia of this shard, returned to the host (synchronises) */
mpkStatus mpkEngineInertia(mpkEngine e, const float* dC, const int* dAssign, double* out);
int mpkEngineFracBits(mpkEngine e);          /* synchronises once */
/* counters since creation: refined rows, refined candidates, full-k rows,
 * and the device status word (0 = healthy) */
mpkStatus mpkEngineCounters(mpkEngine e, long long* rows_refined, long long* cand_refined,
                            long long* rows_full_scan, int* status);
long long mpkEngineSumsLength(mpkEngine e);  /* k*d + k */

/* ---- Combining the ranks' sums over NVLink peer memory (no reference
 * counterpart: the reference has no multi-GPU path) ----
 * One group per rank (GPU), each with an exchange block in its device memory.
 * Per iteration every rank runs mpkEngineStep into mpkPeerSums(g) and then
 * mpkPeerCombine, which replaces the allreduce of the sums and
 * mpkEngineFinalize: each rank finalises its 1/world slice of the clusters
 * from every rank's sums, read over NVLink, and then copies the other ranks'
 * finalised slices; the result equals allreduce + Finalize bit for bit.
 * Set-up: mpkPeerCreate on each rank's device; either export every block as
 * an IPC handle (mpkPeerExportHandle, 64 bytes) and pass all handles to
 * mpkPeerConnect (ranks in different processes), or pass the blocks' addresses
 * (mpkPeerLocalBase) and devices (ranks of one process).  Every rank must call
 * mpkPeerCombine once per iteration: its waits on the other ranks are bounded
 * (4 s) and set the engine's device status on expiry. */
typedef struct mpkPeerGroup_s* mpkPeerGroup;
mpkStatus mpkPeerCreate(mpkPeerGroup* out, int rank, int world, int k, int d);
mpkStatus mpkPeerExportHandle(mpkPeerGroup g, void* handle64);
mpkStatus mpkPeerLocalBase(mpkPeerGroup g, void** base);
/* handles64[p] (or bases[p] with devices[p]) for every rank p but this one */
mpkStatus mpkPeerConnect(mpkPeerGroup g, const void* const* handles64, void* const* bases, const int* devices);
long long* mpkPeerSums(mpkPeerGroup g);      /* this rank's k*d + k sums buffer */
mpkStatus mpkPeerCombine(mpkPeerGroup g, mpkEngine e, float* dC, float* dMoved2);
mpkStatus mpkPeerDestroy(mpkPeerGroup g);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#endif /* MPKMEANS_B200_H */
