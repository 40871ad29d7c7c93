/* kernels.cu -- SIMT kernels of the B200 k-means engine: operand preparation,
 * near-tie refinement, the fixed-point centroid update and bookkeeping.
 *
 * All FP32 arithmetic whose result must match the reference bit for bit is
 * written with explicit fmaf() and compiled with -fmad=false, so no other
 * operation is contracted.
 */
#include "engine.cuh"

#include <cmath>

namespace mpk {
namespace {

constexpr unsigned FULL = 0xffffffffu;

/* ------------------------------------------------------------- max |A| --- */

__global__ void k_maxabs(const float* __restrict__ A, long long count, float* out) {
    float m = 0.f;
    const long long stride = (long long)gridDim.x * blockDim.x;
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long n4 = (((uintptr_t)A & 15) == 0) ? count / 4 : 0;
    const float4* A4 = reinterpret_cast<const float4*>(A);
    for (long long t = i; t < n4; t += stride) {
        const float4 v = A4[t];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    for (long long t = 4 * n4 + i; t < count; t += stride) m = fmaxf(m, fabsf(A[t]));
    m = warp_max(m);   /* NaN entries are dropped by fmaxf */
    if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(reinterpret_cast<unsigned int*>(out), __float_as_uint(m));
}

/* Operand scale and update precision, from the maxima, on the device (no host
 * round trip):
 *   scale s = largest power of two with s * max|P, C0| <= 4096, the rule of
 *             gemm-emulation/src/split_fp16.cu:255-262, so hi words sit well
 *             inside FP16's normal range and lo words keep 11 bits;
 *   frac    = min(100, 62 - E - ceil(log2 n)) with max|P| < 2^E, so that n
 *             quantised coordinates of magnitude < 2^(E+frac) sum below 2^62. */
__global__ void k_set_scale(DevParams* prm, long long n_total) {
    const float m = fmaxf(prm->pmax, prm->c0max);
    float s = 1.f;
    if (m > 0.f && isfinite(m)) {
        int e = 0;
        frexpf(4096.0f / m, &e);
        s = ldexpf(1.0f, e - 1);
        if (!(s > 0.f) || !isfinite(s)) s = 1.f;
    }
    prm->scale = s;
    prm->neg2_inv_s2 = -2.0f / (s * s);
    prm->eta = ldexpf(1.0f, -25) / s;
    int E = 0;
    if (prm->pmax > 0.f && isfinite(prm->pmax)) frexpf(prm->pmax, &E);
    int lg = 0;
    while ((1ll << lg) < n_total && lg < 62) ++lg;
    int frac = 62 - E - lg;
    if (frac > 100) frac = 100;   /* 2^frac stays a finite FP32 scale */
    prm->frac = frac;
}

/* ------------------------------------------------------------- splits ---- */

/* One warp per row: hi = fp16(s*x), lo = fp16(s*x - hi); both planes row major
 * with leading dimension dp (zero padded past d).  norms[i] = ||x_i|| (FP32,
 * any order: it only feeds the error bound, which inflates it). */
__global__ void k_split_rows(const float* __restrict__ src, long long rows, int d, int dp,
                             const DevParams* __restrict__ prm, __half* __restrict__ planes,
                             long long plane_stride, float* __restrict__ norms) {
    const int lane = threadIdx.x & 31;
    const long long wstride = (long long)gridDim.x * (blockDim.x >> 5);
    const float s = prm->scale;
    for (long long i = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < rows; i += wstride) {
        const float* x = src + (size_t)i * d;
        __half* hi = planes + (size_t)i * dp;
        __half* lo = hi + plane_stride;
        float acc = 0.f;
        for (int t = lane; t < dp; t += 32) {
            const float v = t < d ? x[t] : 0.f;
            acc = fmaf(v, v, acc);
            const float a = v * s;
            const __half h = __float2half_rn(a);
            const float r = a - __half2float(h);
            hi[t] = h;
            lo[t] = __float2half_rn(r);
        }
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL, acc, o);
        if (norms && lane == 0) norms[i] = sqrtf(acc);
    }
}

/* Centroid preparation, one 256-thread block per centroid row:
 *   cn[j]   = ||c_j||^2 in exactly the order of the reference's k_row_norms
 *             (kmeans/src/kernels.cu:83-92): thread t runs an fmaf chain over
 *             t, t+256, ..., then the shared-memory halving tree;
 *   planes  = hi/lo FP16 of s*c_j, as for the points.
 * Blocks j in [k, kpad) write cn[j] = +inf so the assignment epilogue can read
 * whole 32-wide column groups without a bounds test. */
__global__ void k_prep_c(const float* __restrict__ C, int k, int d, int dp, DevParams* __restrict__ prm,
                         __half* __restrict__ planes, long long plane_stride, float* __restrict__ cn) {
    __shared__ float sh[256];
    const int j = blockIdx.x;
    const int t = threadIdx.x;
    if (j >= k) {                        /* padding rows: zero planes, infinite norm */
        for (int f = t; f < dp; f += 256) {
            planes[(size_t)j * dp + f] = __float2half_rn(0.f);
            planes[(size_t)j * dp + plane_stride + f] = __float2half_rn(0.f);
        }
        if (t == 0) cn[j] = INFINITY;
        return;
    }
    if (j == 0 && t == 0) {              /* the assignment that follows counts from zero */
        prm->nflag = 0;
        prm->nwide = 0;
        prm->nscan = 0;
    }
    const float* c = C + (size_t)j * d;
    const float s = prm->scale;
    float acc = 0.f;
    for (int f = t; f < d; f += 256) acc = fmaf(c[f], c[f], acc);
    __half* hi = planes + (size_t)j * dp;
    __half* lo = hi + plane_stride;
    bool bad = false;
    for (int f = t; f < dp; f += 256) {
        const float v = f < d ? c[f] : 0.f;
        const float a = v * s;
        bad |= !(fabsf(a) <= 32768.f);
        const __half h = __float2half_rn(a);
        hi[f] = h;
        lo[f] = __float2half_rn(a - __half2float(h));
    }
    if (bad) atomicOr(&prm->status, MPK_DEV_SCALE);
    sh[t] = acc;
    __syncthreads();
    for (int off = 128; off > 0; off >>= 1) {
        if (t < off) sh[t] = sh[t] + sh[t + off];
        __syncthreads();
    }
    if (t == 0) cn[j] = sh[0];
}

/* ------------------------------------------------------------- refine ---- */

/* Up to four candidate distances at once, each exactly as the reference's
 * refinement forms it (kmeans/src/kernels.cu:582-602): lane l runs an fmaf
 * chain over l, l+32, ..., the shfl_down tree sums the lanes, and
 * D = fmaf(-2, dot, ||c||^2).  The best (smaller index on a tie) is folded
 * into (bv, bj), valid in lane 0.  The point row is held in registers,
 * pr[i] = p[lane + 32 i], when d <= 32 * NR; NR == 0 reads it from memory
 * (L1) instead, for any d -- the same chain either way. */
template <int NR>
__device__ __forceinline__ void eval4(const float (&pr)[NR > 0 ? NR : 1], const float* __restrict__ p,
                                      const float* __restrict__ C, const float* __restrict__ cn, int d, int lane,
                                      const int (&j)[4], float& bv, int& bj) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (NR > 0) {
#pragma unroll
        for (int i = 0; i < (NR > 0 ? NR : 1); ++i) {
            const int t = lane + 32 * i;
            if (t < d) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (j[q] >= 0) acc[q] = fmaf(pr[i], __ldg(C + (size_t)j[q] * d + t), acc[q]);
            }
        }
    } else {
#pragma unroll 4
        for (int t = lane; t < d; t += 32) {
            const float pv = __ldg(p + t);
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (j[q] >= 0) acc[q] = fmaf(pv, __ldg(C + (size_t)j[q] * d + t), acc[q]);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] += __shfl_down_sync(FULL, acc[q], off);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (j[q] < 0) continue;
        const float v = fmaf(-2.f, acc[q], cn[j[q]]);
        if (v < bv || (v == bv && j[q] < bj)) { bv = v; bj = j[q]; }
    }
}

/* A warp copies row `row`'s two split-plane rows into slot `slot` of Xw. */
__device__ __forceinline__ void copy_planes(const __half* __restrict__ Xs, long long n, int dp, int row,
                                            const WideScratch& w, long long slot, int lane) {
    const int vec = dp / 8;                              /* 16-byte words per plane row */
    for (int p = 0; p < 2; ++p) {
        const uint4* src = reinterpret_cast<const uint4*>(Xs + (size_t)p * n * dp + (size_t)row * dp);
        uint4* dst = reinterpret_cast<uint4*>(w.Xw + (size_t)p * w.cap * dp + (size_t)slot * dp);
        for (int v = lane; v < vec; v += 32) dst[v] = src[v];
    }
}

/* Rounds after the first: copy queued rows [base, base + per_round) to Xw. */
__global__ void k_wide_gather(const RefineEntry* __restrict__ list, const __half* __restrict__ Xs, long long n,
                              int dp, WideScratch w, long long base, const DevParams* __restrict__ prm) {
    const long long nw = (long long)*reinterpret_cast<const volatile unsigned int*>(&prm->nwide);
    const long long cnt = min(w.per_round, nw - base);
    const int lane = threadIdx.x & 31;
    const long long wstride = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long l = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); l < cnt; l += wstride)
        copy_planes(Xs, n, dp, list[w.went[base + l]].row, w, l, lane);
}

/* One warp per refinement entry: the listed candidates, then every column of
 * each overflowing class, in batches of four; the label is the smallest FP32
 * distance, the smaller index on a tie.  Control flow is warp uniform (every
 * lane reads the same entry).  NR: see eval4. */
template <int NR>
__global__ void k_refine(const float* __restrict__ P, const float* __restrict__ C, const float* __restrict__ cn,
                         int d, int k, int bn, const RefineEntry* __restrict__ list, DevParams* __restrict__ prm,
                         int* __restrict__ labels, long long cap, unsigned long long* hist, int hist_cap,
                         const __half* __restrict__ Xs, long long n, int dp, WideScratch w) {
    constexpr int R = NR > 0 ? NR : 1;
    const int lane = threadIdx.x & 31;
    const long long nf = prm->nflag < (unsigned long long)cap ? (long long)prm->nflag : cap;
    const long long wstride = (long long)gridDim.x * (blockDim.x >> 5);
    const long long w0 = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int halfw = bn / 2;
    unsigned long long ncand = 0, novf = 0;
    for (long long e = w0; e < nf; e += wstride) {
        const RefineEntry E = list[e];
        if (w.cap > 0 && (E.ovf[0] | E.ovf[1])) {
            const int classes = __popc((unsigned)E.ovf[0]) + __popc((unsigned)E.ovf[1]);
            if ((long long)classes * ((k + 15) / 16) > w.rescan_limit) {
                unsigned slot = 0;
                if (lane == 0) {
                    slot = atomicAdd(&prm->nwide, 1u);
                    w.went[slot] = (int)e;                       /* slot < n: one entry per row at most */
                }
                slot = __shfl_sync(FULL, slot, 0);
                if ((long long)slot < w.per_round) copy_planes(Xs, n, dp, E.row, w, slot, lane);  /* round 0 */
                if ((long long)slot < w.per_round * w.rounds) continue;
                /* past the last round: rescan its classes here */
            }
        }
        const float* p = P + (size_t)E.row * d;
        float pr[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const int t = lane + 32 * i;
            pr[i] = (NR > 0 && t < d) ? p[t] : 0.f;
        }
        float bv = INFINITY;
        int bj = k;
        int batch[4] = {-1, -1, -1, -1};
        int nb = 0;
        auto push = [&](int j) {
            batch[nb++] = j;
            if (nb == 4) {
                eval4<NR>(pr, p, C, cn, d, lane, batch, bv, bj);
                batch[0] = batch[1] = batch[2] = batch[3] = -1;
                nb = 0;
            }
        };
#pragma unroll 1
        for (int q = 0; q < 16; ++q)
            if (E.c[q] >= 0) { push(E.c[q]); ++ncand; }
        if (E.ovf[0] | E.ovf[1]) {
            ++novf;
#pragma unroll 1
            for (int h = 0; h < 2; ++h)
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    if (!((E.ovf[h] >> c) & 1)) continue;
#pragma unroll 1
                    for (int base = h * halfw + c; base < k; base += bn)
#pragma unroll 1
                        for (int m = 0; m < halfw; m += 8) {
                            const int j = base + m;
                            if (j >= k) break;
                            push(j);
                            ++ncand;
                        }
                }
        }
        if (nb) eval4<NR>(pr, p, C, cn, d, lane, batch, bv, bj);
        if (lane == 0) labels[E.row] = bj;   /* lane 0 holds the reduced dots */
    }
    if (lane == 0 && ncand) {
        atomicAdd(&prm->ncand_total, ncand);
        if (novf) atomicAdd(&prm->novf_total, novf);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&prm->nflag_total, (unsigned long long)nf);
        if (hist) {                       /* slot from the device counter: a graph replay records too */
            const unsigned it = prm->hist_next;
            if (it < (unsigned)hist_cap) hist[it] = (unsigned long long)nf;
            prm->hist_next = it + 1;
        }
    }
}

/* One warp per wide row: the FP32 evaluation (same order, same tie rule) of
 * the columns the emit pass listed, or of all k when a tile half found more
 * than its kWideCand / 2 slots hold. */
template <int NR>
__global__ void k_refine_wide(const float* __restrict__ P, const float* __restrict__ C, const float* __restrict__ cn,
                              int d, int k, const RefineEntry* __restrict__ list, WideScratch w, long long base,
                              DevParams* __restrict__ prm, int* __restrict__ labels) {
    constexpr int R = NR > 0 ? NR : 1;
    const int lane = threadIdx.x & 31;
    const long long nw0 = (long long)*reinterpret_cast<volatile unsigned int*>(&prm->nwide) - base;
    const long long nw = nw0 < w.per_round ? (nw0 > 0 ? nw0 : 0) : w.per_round;
    const long long wstride = (long long)gridDim.x * (blockDim.x >> 5);
    const long long w0 = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    unsigned long long ncand = 0, nfull = 0;
    for (long long s = w0; s < nw; s += wstride) {
        const int row = list[w.went[base + s]].row;
        const float* p = P + (size_t)row * d;
        float pr[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const int t = lane + 32 * i;
            pr[i] = (NR > 0 && t < d) ? p[t] : 0.f;
        }
        float bv = INFINITY;
        int bj = k;
        int batch[4] = {-1, -1, -1, -1};
        int nb = 0;
        auto push = [&](int j) {
            batch[nb++] = j;
            if (nb == 4) {
                eval4<NR>(pr, p, C, cn, d, lane, batch, bv, bj);
                batch[0] = batch[1] = batch[2] = batch[3] = -1;
                nb = 0;
            }
        };
        const int c0 = w.ccount[2 * s], c1 = w.ccount[2 * s + 1];
        constexpr int H = kWideCand / 2;
        if (c0 > H || c1 > H) {
            ++nfull;
            ncand += (unsigned long long)k;
            if (w.scan) {                 /* all k: queued for the tiled scan (k_full_scan) */
                if (lane == 0) w.scan[atomicAdd(&prm->nscan, 1u)] = row;
                continue;
            }
#pragma unroll 1
            for (int j = 0; j < k; ++j) push(j);
        } else {
            const int* cl = w.cand + (size_t)s * kWideCand;
#pragma unroll 1
            for (int i = 0; i < c0; ++i) push(cl[i]);
#pragma unroll 1
            for (int i = 0; i < c1; ++i) push(cl[H + i]);
            ncand += (unsigned long long)(c0 + c1);
        }
        if (nb) eval4<NR>(pr, p, C, cn, d, lane, batch, bv, bj);
        if (lane == 0) labels[row] = bj;
    }
    if (lane == 0 && ncand) {
        atomicAdd(&prm->ncand_total, ncand);
        if (nfull) atomicAdd(&prm->novf_total, nfull);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && nw > 0) atomicAdd(&prm->nwide_total, (unsigned long long)nw);
}

/* The full FP32 scan of the wide rows whose candidate lists overflowed: every
 * centroid, in exactly eval4's arithmetic, but tiled.  A block stages
 * 32 * NC centroids at a time in shared memory for 16 rows (two per warp), so
 * a centroid is read from L2 once per 16 rows instead of once per row, and
 * the scan is arithmetic rather than a chain of dependent loads.
 *
 * Lane j owns NC of the tile's centroids.  For each (centroid, row) it forms
 * the dot eval4 spreads over a warp -- chain u sums fmaf(p[t], c[t], .) over
 * t = u, u+32, ... < d in increasing t; the 32 chains are added by eval4's
 * shfl_down tree (offsets 16, 8, 4, 2, 1) -- inside one thread: the chains
 * are computed one at a time in 5-bit bit-reversed order of u (0, 16, 8, 24,
 * 4, ...), in which that tree is the left-to-right binary tree over the
 * leaves, so a stack of five partial sums reproduces its additions in order.
 * Then fmaf(-2, dot, ||c||^2): the value eval4 leaves in lane 0, bit for bit.
 * Per-lane bests merge by value, then smaller index.  Rows come from w.scan;
 * d <= kScanMaxDim. */
constexpr int kScanRows = 2;           /* rows per warp */
constexpr int kScanWarps = 8;

__host__ __device__ constexpr int bitrev5(int k) {
    return ((k & 1) << 4) | ((k & 2) << 2) | (k & 4) | ((k & 8) >> 2) | ((k & 16) >> 4);
}

template <int NC>
__global__ void __launch_bounds__(32 * kScanWarps)
k_full_scan(const float* __restrict__ P, const float* __restrict__ C, const float* __restrict__ cn, int d, int dpad,
            int k, const int* __restrict__ rows, const DevParams* __restrict__ prm, int* __restrict__ labels) {
    constexpr int TILE = 32 * NC;                      /* centroids per shared-memory tile */
    extern __shared__ float sm[];
    float* tile = sm;                                  /* TILE x dpad */
    float* prow = sm + (size_t)TILE * dpad;            /* kScanWarps x kScanRows x dpad */
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long cnt = (long long)*reinterpret_cast<const volatile unsigned int*>(&prm->nscan);
    constexpr long long per_block = (long long)kScanWarps * kScanRows;
    const int nch = (d + 31) / 32;                     /* products in the longest chain */
    for (long long g0 = (long long)blockIdx.x * per_block; g0 < cnt; g0 += (long long)gridDim.x * per_block) {
        int myrow[kScanRows];
        const float* pr[kScanRows];
#pragma unroll
        for (int r = 0; r < kScanRows; ++r) {
            const long long idx = g0 + warp * kScanRows + r;
            myrow[r] = idx < cnt ? rows[idx] : -1;
            float* dst = prow + (size_t)(warp * kScanRows + r) * dpad;
            for (int t = lane; t < d; t += 32) dst[t] = myrow[r] >= 0 ? P[(size_t)myrow[r] * d + t] : 0.f;
            pr[r] = dst;
        }
        float bv[kScanRows];
        int bj[kScanRows];
#pragma unroll
        for (int r = 0; r < kScanRows; ++r) { bv[r] = INFINITY; bj[r] = k; }
        for (int j0 = 0; j0 < k; j0 += TILE) {
            __syncthreads();                           /* the previous tile is consumed; rows are staged */
            for (int jj = warp; jj < TILE; jj += kScanWarps) {
                const int j = j0 + jj;
                for (int t = lane; t < d; t += 32) tile[(size_t)jj * dpad + t] = j < k ? C[(size_t)j * d + t] : 0.f;
            }
            __syncthreads();
            float stk[NC][kScanRows][5];               /* pending left operands, by tree level */
#pragma unroll
            for (int leaf = 0; leaf < 32; ++leaf) {
                const int u = bitrev5(leaf);
                float a[NC][kScanRows];
#pragma unroll
                for (int c = 0; c < NC; ++c)
#pragma unroll
                    for (int r = 0; r < kScanRows; ++r) a[c][r] = 0.f;
#pragma unroll 4
                for (int i = 0; i < nch; ++i) {             /* unrolled: the next loads overlap these FMAs */
                    const int t = u + 32 * i;
                    if (t < d) {
                        float pv[kScanRows];
#pragma unroll
                        for (int r = 0; r < kScanRows; ++r) pv[r] = pr[r][t];
#pragma unroll
                        for (int c = 0; c < NC; ++c) {
                            const float cv = tile[(size_t)(c * 32 + lane) * dpad + t];
#pragma unroll
                            for (int r = 0; r < kScanRows; ++r) a[c][r] = fmaf(pv[r], cv, a[c][r]);
                        }
                    }
                }
                /* binary-counter merge: a completed subtree at level l combines with the
                 * pending left sibling stk[l] (the earlier leaves), left + right */
#pragma unroll
                for (int c = 0; c < NC; ++c)
#pragma unroll
                    for (int r = 0; r < kScanRows; ++r) {
                        float v = a[c][r];
#pragma unroll
                        for (int l = 0; l < 5; ++l) {
                            if (((leaf >> l) & 1) == 0) { stk[c][r][l] = v; break; }
                            v = stk[c][r][l] + v;
                            if (l == 4) stk[c][r][0] = v;   /* leaf 31: the root, kept in slot 0 */
                        }
                    }
            }
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int j = j0 + c * 32 + lane;
                if (j < k) {
                    const float cj = cn[j];
#pragma unroll
                    for (int r = 0; r < kScanRows; ++r) {
                        const float v = fmaf(-2.f, stk[c][r][0], cj);
                        if (v < bv[r] || (v == bv[r] && j < bj[r])) { bv[r] = v; bj[r] = j; }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kScanRows; ++r) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_xor_sync(FULL, bv[r], off);
                const int oj = __shfl_xor_sync(FULL, bj[r], off);
                if (ov < bv[r] || (ov == bv[r] && oj < bj[r])) { bv[r] = ov; bj[r] = oj; }
            }
            if (lane == 0 && myrow[r] >= 0) labels[myrow[r]] = bj[r];
        }
    }
}

/* The same scan for d <= 256, with the operands laid out by chain: centroid
 * and point rows are staged in shared memory as [u][i] = x[u + 32 i] (chain u,
 * i < 8, zero past d), so a chain's eight operands are two 16-byte loads and
 * every address is a compile-time offset.  The zero padding only adds
 * fmaf(0, 0, acc) = acc + 0 steps, which leave a chain's value unchanged (a
 * -0 chain can turn +0, which no later sum or fmaf(-2, dot, ||c||^2) can
 * tell apart), so the values are eval4's, bit for bit. */
constexpr int kScanChain = 8;          /* d <= 32 * kScanChain */
constexpr int kScanStride = 32 * kScanChain + 4;   /* floats per staged row: 16-byte lanes spread over banks */

template <int NC, int RW>
__global__ void __launch_bounds__(32 * kScanWarps)
k_full_scan_c8(const float* __restrict__ P, const float* __restrict__ C, const float* __restrict__ cn, int d, int k,
               const int* __restrict__ rows, const DevParams* __restrict__ prm, int* __restrict__ labels) {
    constexpr int TILE = 32 * NC;
    extern __shared__ __align__(16) float sm[];
    float* tile = sm;                                          /* TILE x kScanStride */
    float* prow = sm + (size_t)TILE * kScanStride;             /* kScanWarps x RW x kScanStride */
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long cnt = (long long)*reinterpret_cast<const volatile unsigned int*>(&prm->nscan);
    constexpr long long per_block = (long long)kScanWarps * RW;
    /* staging: element x[t] of a row goes to [u][i] with t = u + 32 i */
    auto stage = [&](float* dst, const float* src, bool live) {
        for (int e = lane; e < 32 * kScanChain; e += 32) {      /* e = u * 8 + i */
            const int u = e >> 3, i = e & 7, t = u + 32 * i;
            dst[e] = (live && t < d) ? src[t] : 0.f;
        }
    };
    for (long long g0 = (long long)blockIdx.x * per_block; g0 < cnt; g0 += (long long)gridDim.x * per_block) {
        int myrow[RW];
        const float* pr[RW];
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            const long long idx = g0 + warp * RW + r;
            myrow[r] = idx < cnt ? rows[idx] : -1;
            float* dst = prow + (size_t)(warp * RW + r) * kScanStride;
            stage(dst, P + (size_t)(myrow[r] >= 0 ? myrow[r] : 0) * d, myrow[r] >= 0);
            pr[r] = dst;
        }
        float bv[RW];
        int bj[RW];
#pragma unroll
        for (int r = 0; r < RW; ++r) { bv[r] = INFINITY; bj[r] = k; }
        for (int j0 = 0; j0 < k; j0 += TILE) {
            __syncthreads();                                   /* the previous tile is consumed; rows staged */
            for (int jj = warp; jj < TILE; jj += kScanWarps) {
                const int j = j0 + jj;
                stage(tile + (size_t)jj * kScanStride, C + (size_t)(j < k ? j : 0) * d, j < k);
            }
            __syncthreads();
            float stk[NC][RW][5];
#pragma unroll
            for (int leaf = 0; leaf < 32; ++leaf) {
                const int u = bitrev5(leaf);
                float4 pv[RW][2];
#pragma unroll
                for (int r = 0; r < RW; ++r) {
                    pv[r][0] = *reinterpret_cast<const float4*>(pr[r] + u * kScanChain);
                    pv[r][1] = *reinterpret_cast<const float4*>(pr[r] + u * kScanChain + 4);
                }
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const float* cr = tile + (size_t)(c * 32 + lane) * kScanStride + u * kScanChain;
                    const float4 c0 = *reinterpret_cast<const float4*>(cr);
                    const float4 c1 = *reinterpret_cast<const float4*>(cr + 4);
#pragma unroll
                    for (int r = 0; r < RW; ++r) {
                        float a = fmaf(pv[r][0].x, c0.x, 0.f);
                        a = fmaf(pv[r][0].y, c0.y, a);
                        a = fmaf(pv[r][0].z, c0.z, a);
                        a = fmaf(pv[r][0].w, c0.w, a);
                        a = fmaf(pv[r][1].x, c1.x, a);
                        a = fmaf(pv[r][1].y, c1.y, a);
                        a = fmaf(pv[r][1].z, c1.z, a);
                        a = fmaf(pv[r][1].w, c1.w, a);
                        float v = a;
#pragma unroll
                        for (int l = 0; l < 5; ++l) {
                            if (((leaf >> l) & 1) == 0) { stk[c][r][l] = v; break; }
                            v = stk[c][r][l] + v;
                            if (l == 4) stk[c][r][0] = v;
                        }
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int j = j0 + c * 32 + lane;
                if (j < k) {
                    const float cj = cn[j];
#pragma unroll
                    for (int r = 0; r < RW; ++r) {
                        const float v = fmaf(-2.f, stk[c][r][0], cj);
                        if (v < bv[r] || (v == bv[r] && j < bj[r])) { bv[r] = v; bj[r] = j; }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RW; ++r) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_xor_sync(FULL, bv[r], off);
                const int oj = __shfl_xor_sync(FULL, bj[r], off);
                if (ov < bv[r] || (ov == bv[r] && oj < bj[r])) { bv[r] = ov; bj[r] = oj; }
            }
            if (lane == 0 && myrow[r] >= 0) labels[myrow[r]] = bj[r];
        }
    }
}

/* Verification (params.verify): one warp per row evaluates all k centroids
 * in the refinement's FP32 order (lane-strided fmaf chains, shfl_down tree,
 * fmaf(-2, dot, ||c||^2), smaller index on ties) and compares the argmin
 * with the label the engine produced.  cnt[0] counts rows whose label is not
 * that argmin, *excess adds D(label) - D(argmin).  Both stay 0 when the
 * certified bound holds; this is a check, run only when asked for. */
template <int NR>
__global__ void k_verify(const float* __restrict__ P, const float* __restrict__ C, const float* __restrict__ cn,
                         int d, int k, const int* __restrict__ labels, long long n,
                         unsigned long long* __restrict__ cnt, double* __restrict__ excess) {
    constexpr int R = NR > 0 ? NR : 1;
    const int lane = threadIdx.x & 31;
    const long long wstride = (long long)gridDim.x * (blockDim.x >> 5);
    unsigned long long bad = 0;
    double ex = 0.0;
    for (long long i = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += wstride) {
        const float* p = P + (size_t)i * d;
        float pr[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int t = lane + 32 * r;
            pr[r] = (NR > 0 && t < d) ? p[t] : 0.f;
        }
        const int lab = labels[i];
        float bv = INFINITY, vl = INFINITY;
        int bj = k;
        for (int j0 = 0; j0 < k; j0 += 4) {
            int j[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) j[q] = j0 + q < k ? j0 + q : -1;
            /* the label's own value: a batch holding it is evaluated alone first */
            if (lab >= j0 && lab < j0 + 4) {
                float v1 = INFINITY;
                int b1 = k;
                const int jl[4] = {lab, -1, -1, -1};
                eval4<NR>(pr, p, C, cn, d, lane, jl, v1, b1);
                vl = v1;
            }
            eval4<NR>(pr, p, C, cn, d, lane, j, bv, bj);
        }
        if (lane == 0 && bj != lab) {
            ++bad;
            ex += (double)vl - (double)bv;
        }
    }
    if (lane == 0 && bad) {
        atomicAdd(cnt, bad);
        atomicAdd(excess, ex);
    }
}

/* C_j = (float)((S_j * 2^-frac) / count_j); an empty cluster keeps its old
 * centroid; moved2[j] = ||c_new - c_old||^2 by the reference's 256-wide tree
 * (kmeans/src/kernels.cu:705-723). */
__global__ void k_finalize_fixed(const long long* __restrict__ sums, const long long* __restrict__ counts, int k,
                                 int d, const DevParams* __restrict__ prm, float* __restrict__ C,
                                 float* __restrict__ moved2) {
    __shared__ float sh[256];
    const int j = blockIdx.x;
    const int t = threadIdx.x;
    const long long cnt = counts[j];
    const double inv = ldexp(1.0, -prm->frac);
    float acc = 0.f;
    for (int f = t; f < d; f += 256) {
        const size_t o = (size_t)j * d + f;
        const float old = C[o];
        const float nv = cnt > 0 ? (float)(((double)sums[o] * inv) / (double)cnt) : old;
        C[o] = nv;
        const float dv = nv - old;
        acc = fmaf(dv, dv, acc);
    }
    sh[t] = acc;
    __syncthreads();
    for (int off = 128; off > 0; off >>= 1) {
        if (t < off) sh[t] = sh[t] + sh[t + off];
        __syncthreads();
    }
    if (t == 0 && moved2) moved2[j] = sh[0];
}

/* inertia = sum_i ||p_i - c_a(i)||^2 in FP64, one warp per row. */
__global__ void k_inertia(const float* __restrict__ P, const float* __restrict__ C, const int* __restrict__ labels,
                          long long n, int d, double* out) {
    const int lane = threadIdx.x & 31;
    const long long wstride = (long long)gridDim.x * (blockDim.x >> 5);
    double tot = 0.0;
    for (long long i = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += wstride) {
        const float* p = P + (size_t)i * d;
        const float* c = C + (size_t)labels[i] * d;
        for (int t = lane; t < d; t += 32) {
            const double v = (double)p[t] - (double)c[t];
            tot = fma(v, v, tot);
        }
    }
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(FULL, tot, o);
    if (lane == 0 && tot != 0.0) atomicAdd(out, tot);
}

__global__ void k_count_diff(const int* __restrict__ a, const int* __restrict__ b, long long n,
                             unsigned long long* out) {
    unsigned long long c = 0;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) c += (a[i] != b[i]);
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(FULL, c, o);
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(out, c);
}

__global__ void k_add_const(float* p, long long count, float c) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) p[i] += c;
}

/* Per-feature z-score, FP64 two-pass (kmeans/src/kernels.cu:116-140 semantics):
 * one block per feature; population variance; sd <= 1e-12 divides by 1. */
__global__ void k_standardize(float* P, int n, int d) {
    __shared__ double sh[256];
    const int f = blockIdx.x, t = threadIdx.x;
    double acc = 0.0;
    for (int i = t; i < n; i += 256) acc += (double)P[(size_t)i * d + f];
    sh[t] = acc;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) { if (t < o) sh[t] += sh[t + o]; __syncthreads(); }
    const double mean = sh[0] / (double)n;
    __syncthreads();
    acc = 0.0;
    for (int i = t; i < n; i += 256) { const double v = (double)P[(size_t)i * d + f] - mean; acc = fma(v, v, acc); }
    sh[t] = acc;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) { if (t < o) sh[t] += sh[t + o]; __syncthreads(); }
    const double sd = sqrt(sh[0] / (double)n);
    const double inv = sd > 1e-12 ? 1.0 / sd : 1.0;
    for (int i = t; i < n; i += 256) {
        const size_t o = (size_t)i * d + f;
        P[o] = (float)(((double)P[o] - mean) * inv);
    }
}

inline int grid_for(long long items, int threads, int cap) {
    long long b = (items + threads - 1) / threads;
    if (b < 1) b = 1;
    return (int)(b > cap ? cap : b);
}

}  /* namespace */

/* ------------------------------------------------------------ launchers -- */

void launch_maxabs(const float* A, long long count, float* out, cudaStream_t s) {
    if (count <= 0) return;
    k_maxabs<<<grid_for(count / 4 + 1, 256, 148 * 8), 256, 0, s>>>(A, count, out);
}

void launch_set_scale(DevParams* prm, long long n_total, cudaStream_t s) {
    k_set_scale<<<1, 1, 0, s>>>(prm, n_total);
}

void launch_split_rows(const float* src, long long rows, int d, int dp, const DevParams* prm, __half* planes,
                       long long plane_stride, float* norms, cudaStream_t s) {
    if (rows <= 0) return;
    k_split_rows<<<grid_for(rows, 8, 148 * 16), 256, 0, s>>>(src, rows, d, dp, prm, planes, plane_stride, norms);
}

void launch_prep_c(const float* C, int k, int kpad, int d, int dp, DevParams* prm, __half* planes, float* cn,
                   cudaStream_t s) {
    k_prep_c<<<kpad, 256, 0, s>>>(C, k, d, dp, prm, planes, (long long)kpad * dp, cn);
}

void launch_wide_gather(const RefineEntry* list, const __half* Xs, long long n, int dp, const WideScratch& w,
                        long long base, const DevParams* prm, int num_sms, cudaStream_t s) {
    k_wide_gather<<<num_sms * 4, 256, 0, s>>>(list, Xs, n, dp, w, base, prm);
}

void launch_refine_wide(const float* P, const float* C, const float* cn, int d, int k, const RefineEntry* list,
                        const WideScratch& w, long long base, DevParams* prm, int* labels, int num_sms,
                        cudaStream_t s) {
    if (d <= 256) k_refine_wide<8><<<num_sms * 4, 256, 0, s>>>(P, C, cn, d, k, list, w, base, prm, labels);
    else k_refine_wide<0><<<num_sms * 4, 256, 0, s>>>(P, C, cn, d, k, list, w, base, prm, labels);
}

void launch_refine(const float* P, const float* C, const float* cn, int d, int k, int bn, const RefineEntry* list,
                   DevParams* prm, int* labels, long long n_cap, unsigned long long* hist, int hist_cap,
                   const __half* Xs, long long n, int dp, const WideScratch& w, int num_sms, cudaStream_t s,
                   int blocks_per_sm) {
    /* grid-stride over the entries: any grid works; four blocks a SM fill the register file,
     * one leaves the rest of each SM to a kernel running beside it */
    const int grid = num_sms * (blocks_per_sm > 0 ? blocks_per_sm : 4);
    if (d <= 256)
        k_refine<8><<<grid, 256, 0, s>>>(P, C, cn, d, k, bn, list, prm, labels, n_cap, hist, hist_cap, Xs, n, dp, w);
    else
        k_refine<0><<<grid, 256, 0, s>>>(P, C, cn, d, k, bn, list, prm, labels, n_cap, hist, hist_cap, Xs, n, dp, w);
}

void launch_finalize_fixed(const long long* sums, const long long* counts, int k, int d, const DevParams* prm,
                           float* C, float* moved2, cudaStream_t s) {
    k_finalize_fixed<<<k, 256, 0, s>>>(sums, counts, k, d, prm, C, moved2);
}

void launch_verify(const float* P, const float* C, const float* cn, int d, int k, const int* labels, long long n,
                   unsigned long long* cnt, double* excess, int num_sms, cudaStream_t s) {
    if (n <= 0) return;
    if (d <= 256) k_verify<8><<<num_sms * 4, 256, 0, s>>>(P, C, cn, d, k, labels, n, cnt, excess);
    else k_verify<0><<<num_sms * 4, 256, 0, s>>>(P, C, cn, d, k, labels, n, cnt, excess);
}

void launch_full_scan(const float* P, const float* C, const float* cn, int d, int k, const int* rows,
                      const DevParams* prm, int* labels, int num_sms, cudaStream_t s) {
    const int dpad = ((d + 31) / 32) * 32 + 1;        /* odd stride: lane j's row starts on bank j */
    /* centroids per lane, as many as the 227 KB of shared memory allow */
    const int nc = dpad <= 385 ? 4 : (dpad <= 641 ? 2 : 1);
    const size_t smem = sizeof(float) * (size_t)dpad * (32 * nc + kScanWarps * kScanRows);
    auto go = [&](auto kern) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<num_sms, 32 * kScanWarps, smem, s>>>(P, C, cn, d, dpad, k, rows, prm, labels);
    };
    if (d <= 32 * kScanChain) {                        /* chain-major staging, 16-byte operand loads */
        /* two centroids a lane, four rows a warp: 100 KB of shared memory, 107 registers,
         * two blocks an SM (measured against 1x2, 1x4, 2x2, 4x2 and 2x8) */
        constexpr int RW = 4;
        const size_t sm8 = sizeof(float) * (size_t)kScanStride * (32 * 2 + kScanWarps * RW);
        cudaFuncSetAttribute(k_full_scan_c8<2, RW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm8);
        k_full_scan_c8<2, RW><<<num_sms * 2, 32 * kScanWarps, sm8, s>>>(P, C, cn, d, k, rows, prm, labels);
        return;
    }
    if (nc == 4) go(k_full_scan<4>);
    else if (nc == 2) go(k_full_scan<2>);
    else go(k_full_scan<1>);
}

void launch_inertia(const float* P, const float* C, const int* labels, long long n, int d, double* out,
                    cudaStream_t s) {
    if (n <= 0) return;
    k_inertia<<<grid_for(n, 8, 148 * 16), 256, 0, s>>>(P, C, labels, n, d, out);
}

void launch_count_diff(const int* a, const int* b, long long n, unsigned long long* out, cudaStream_t s) {
    if (n <= 0) return;
    k_count_diff<<<grid_for(n, 256, 148 * 8), 256, 0, s>>>(a, b, n, out);
}

void launch_add_const(float* p, long long count, float c, cudaStream_t s) {
    if (count <= 0) return;
    k_add_const<<<grid_for(count, 256, 8192), 256, 0, s>>>(p, count, c);
}

void launch_standardize(float* P, int n, int d, cudaStream_t s) {
    k_standardize<<<d, 256, 0, s>>>(P, n, d);
}

}  /* namespace mpk */
