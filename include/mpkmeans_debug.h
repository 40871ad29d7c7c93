/* mpkmeans_debug.h -- test hooks of libmpkmeans_b200.  No counterpart in the
 * reference: they expose engine internals to the parity tests. */
#ifndef MPKMEANS_B200_DEBUG_H
#define MPKMEANS_B200_DEBUG_H

#include "mpkmeans.h"

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* While dOut4 is non-NULL, every assignment of engine e writes, per row, the
 * tensor-core best and runner-up distances and their centroids as
 * (v0, v1, j0 bits, j1 bits) to dOut4 (n float4 on the device). */
mpkStatus mpkDebugSetAssignTrace(mpkEngine e, float* dOut4);

/* Operand scale s, subnormal floor eta = 2^-25/s, fixed-point fraction bits,
 * and the two error-bound constants of the assignment filter. */
mpkStatus mpkDebugEngineInfo(mpkEngine e, float* scale, float* eta, int* frac, float* c1, float* c2);

/* Wide refinement: rows handed to the candidate-listing tensor-core pass over
 * the engine's life, rows of those that fell back to a scan of all k, and
 * the per-assignment capacity (0: the engine has no wide path, k <= 256). */
mpkStatus mpkDebugWideCounters(mpkEngine e, long long* wide_rows, long long* full_scans, long long* capacity);

/* Kernels the engine has launched over its life (its own kernels only: no
 * memsets or library calls); the bench reports the count inside its timed
 * region from this. */
long long mpkDebugEngineLaunches(mpkEngine e);

/* Failure-path test hooks.  SetWaitLimit bounds every wait of the engine's
 * assignment kernel by `ns` (0: the default 4 s).  InjectStall makes the
 * kernel's producer leave centroid-plane stage `stage` (counted per CTA from
 * 0) unloaded on every later assignment (-1: none), so the MMA issuer's wait
 * on it runs out: the kernel sets MPK_DEV_TIMEOUT (bit 0 of the status that
 * mpkEngineCounters reports), winds down and returns, and the context stays
 * usable.  ClearStatus zeroes the engine's device status word. */
mpkStatus mpkDebugSetWaitLimit(mpkEngine e, unsigned long long ns);
mpkStatus mpkDebugInjectStall(mpkEngine e, int stage);
mpkStatus mpkDebugClearStatus(mpkEngine e);

/* Assignment kernel choice.  The CTA-pair kernel processes row tiles in pairs
 * on two SMs that share each tensor-core MMA; it applies when k > 128 and is
 * the default there.  mode 0: one CTA per row tile instead;
 * non-zero: the default.  Both give the same labels. */
mpkStatus mpkDebugAssignPair(mpkEngine e, int mode);

/* Refinement order.  By default mpkEngineIterate, mpkEngineStep and the Lloyd
 * drivers (without verify or verbose) run the FP32 refinement on a second
 * stream beside the update's segmented sum, which sums the assignment's
 * labels and then moves the refined rows between clusters; mode 0 refines
 * first and updates after.  Both give the same labels and sums, bit for bit. */
mpkStatus mpkDebugOverlapRefine(mpkEngine e, int mode);

/* Failure injection on the host: the nth device allocation the library makes
 * from now on (engine scratch, driver buffers) fails once, as if the device
 * were out of memory; 0 disables.  Every entry point must then return
 * MPK_ERR_ALLOC and free what it had allocated. */
mpkStatus mpkDebugFailAlloc(int nth);

/* Failure injection for mpkMeansMixedMG: its next wait on the devices, once
 * they are idle, reports an asynchronous NCCL error, so the driver aborts its
 * communicators and returns MPK_ERR_CUDA (no collective is in flight then). */
mpkStatus mpkDebugMGFailNextWait(void);

/* The emulated GEMM's device status word on the current device (bit 0: a
 * bounded wait inside the kernel ran out and the call's output is invalid);
 * synchronises the device; clears the word when `clear` is non-zero.
 * Returns -1 when the word cannot be read.  No reference counterpart. */
int mpkDebugGemmStatus(int clear);

/* Test hook: process the queued wide rows in rounds of at most `rows` (down
 * from the engine's capacity), to exercise several rounds on small inputs
 * (k >= 4096; with smaller k there is one round and the rows past it rescan
 * their classes, which this also exercises). */
mpkStatus mpkDebugWideRoundRows(mpkEngine e, long long rows);

/* While enabled, the engine records a CUDA event pair on its stream around
 * three steps of every iteration: the tensor-core assignment (the kernel
 * alone when launched directly; the centroid split and the kernel when
 * replayed by mpkEngineIterate), the refinement (k_refine and the wide and
 * full-scan passes) and the accumulation (the sorted update; with
 * mpkEngineIterate, also the finalisation). */
mpkStatus mpkDebugProfile(mpkEngine e, int enable);

/* Synchronises; summed device milliseconds and event-pair counts of the three
 * steps since profiling was enabled; clears the record. */
mpkStatus mpkDebugProfileRead(mpkEngine e, double* assign_ms, long long* assign_launches, double* refine_ms,
                              long long* refine_launches, double* accum_ms, long long* accum_launches);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#endif /* MPKMEANS_B200_DEBUG_H */
