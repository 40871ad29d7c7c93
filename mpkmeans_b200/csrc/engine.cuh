/* engine.cuh -- internal interfaces of the B200 k-means engine.
 *
 * HBM layout of one engine (one GPU, one shard of rows):
 *   P      n x d FP32, row major, caller owned, never modified
 *   Xs     2 x n x dp FP16: plane 0 = hi, plane 1 = lo of s*P, dp = d rounded
 *          up to 64 (zero padded); split once per fit
 *   xnorm  n FP32: ||p_i|| (only feeds the error bound)
 *   Cs     2 x kpad x dp FP16: hi/lo of s*C, re-split every iteration; rows
 *          past k are zero (kpad = k rounded up to 256)
 *   cn     kpad FP32: ||c_j||^2 in the reference's tree order; +inf past k
 *   list   refinement entries (row + up to 4 candidates), capacity n
 *   sums   k*d int64 fixed-point coordinate sums, then k int64 counts
 *   prm    DevParams (scales, status word, counters)
 */
#pragma once

#include "common.cuh"

namespace mpk {

struct DevParams {
    float pmax;          /* max |P| over the whole problem (all shards)        */
    float c0max;         /* max |C0| at the start of the fit                   */
    float scale;         /* FP16 operand scale s (a power of two)              */
    float neg2_inv_s2;   /* -2 / s^2, folds the scale out of the products      */
    float eta;           /* 2^-25 / s: absolute floor of a subnormal FP16 word */
    int   frac;          /* fractional bits of the fixed-point update          */
    int   status;        /* MPK_DEV_* bits                                     */
    unsigned int nflag;  /* refinement entries written by the last assign      */
    unsigned long long nflag_total;  /* refinement entries over the run       */
    unsigned long long ncand_total;  /* candidate centroids refined, over run */
    unsigned long long novf_total;   /* rows whose class rescans ran, or whose wide list overflowed */
    unsigned int nwide;              /* rows handed to the wide refinement by the last assign */
    unsigned int hist_next;          /* next survivor-history slot the refinement writes */
    unsigned long long nwide_total;  /* wide rows over the run */
    unsigned long long wait_ns;      /* limit of one wait in the assignment kernel (0: 4 s) */
    unsigned int nscan;              /* wide rows queued for the tiled full FP32 scan */
    unsigned int pad1;
};

/* A row to re-decide in FP32.  The assignment epilogue tracks, per column
 * class (tile half h, column mod 8 = c), the best column and the runner-up
 * value; c[8h + c] is that class's best when it lies within the bound of the
 * row's best, and bit c of ovf[h] is set when the class's runner-up does too
 * (the class may then hold more candidates: all its columns are rescanned,
 * or, when that would visit too many columns, the row goes wide).  v0 is the
 * row's best emulated value and T0 the base of its bound. */
struct RefineEntry {
    int row;
    unsigned short ovf[2];
    float v0;
    float T0;
    int c[16];
};
static_assert(sizeof(RefineEntry) == 80, "refinement entry layout");

/* Wide refinement.  A flagged row whose overflowing classes hold more than
 * rescan_limit columns in all is not rescanned class by class: it is queued
 * (went), and in rounds of `cap` rows its split planes are copied to Xw, a
 * second tensor-core pass over those rows emits every column within the
 * row's bound (up to kWideCand / 2 per tile half), and the FP32 evaluation
 * visits just those -- or all k when a half's list overflowed.  Every round
 * sizes itself from prm->nwide on the device; rounds past the queue exit at
 * once. */
constexpr int kWideCand = 512;
/* the wide path's tensor-core pass runs on 256-wide centroid tiles: k > 128 */
constexpr int kWideMinK = 128;
/* Class-rescan columns above which a row goes wide.  The wide pass costs a
 * fixed ~20 us (a tensor-core launch over whole SMs, after the update's
 * join); class rescans cost FP32 dots in the refinement, which runs beside
 * the update's segmented sum and hides there on small shards.  Measured at
 * k = 1024: at 1e7 rows sending every rescan row wide (32 columns) takes
 * 0.09 ms off an iteration; at 1.25e6 rows it adds 0.02 ms, so small shards
 * keep 256.  Either way the labels are the same, bit for bit. */
inline int wide_rescan_limit(long long n) { return n >= (1LL << 22) ? 32 : 256; }
struct WideScratch {
    __half* Xw;          /* 2 planes x cap x dp FP16: one round's rows */
    int* went;           /* n: refinement-entry index of each queued row */
    int* cand;           /* cap x kWideCand candidate columns */
    int* ccount;         /* cap x 2: columns found by each tile half */
    int* scan;           /* n: rows whose lists overflowed, for the tiled full scan (d <= kScanMaxDim) */
    long long cap;       /* rows Xw holds (its plane stride); 0: no wide path (small k) */
    long long per_round; /* rows per round, <= cap */
    int rounds;          /* rounds per assignment; queued rows past them rescan their classes */
    int rescan_limit;    /* class-rescan columns above which a row goes wide (wide_rescan_limit) */
};

/* Widest row the tiled full scan (k_full_scan) stages in shared memory. */
constexpr int kScanMaxDim = 1024;

/* Error-bound constants of the assignment filter (host computed). */
struct BoundConsts {
    float c1;            /* multiplies ||x|| * max_j ||c_j||                */
    float c2;            /* multiplies eta * (||x|| + max_j ||c_j||)        */
};

/* ---- prep (kernels.cu) ---- */
void launch_maxabs(const float* A, long long count, float* out, cudaStream_t s);
void launch_set_scale(DevParams* prm, long long n_total, cudaStream_t s);
void launch_split_rows(const float* src, long long rows, int d, int dp, const DevParams* prm,
                       __half* planes, long long plane_stride, float* norms, cudaStream_t s);
void launch_prep_c(const float* C, int k, int kpad, int d, int dp, DevParams* prm,
                   __half* planes, float* cn, cudaStream_t s);

/* ---- assign (assign_tc.cu) ---- */
struct AssignArgs {
    const CUtensorMap* tmX;   /* host copies, passed by value to the kernel */
    const CUtensorMap* tmC;
    const CUtensorMap* tmCh;  /* centroid planes in 128-row boxes: the CTA-pair kernel */
    int pair;                 /* CTA-pair kernel where it applies (0: one CTA per tile) */
    int pair_clusters;        /* resident clusters of two for it (0: not available) */
    long long n;
    int k, d, dp;
    const float* xnorm;
    const float* cn;
    const DevParams* prm_ro;
    DevParams* prm;
    int* labels;
    RefineEntry* list;
    int refine;               /* 0: trust the emulated argmin outright      */
    BoundConsts bc;
    int num_sms;
    float4* dbg;              /* optional: (v0, v1, j0, j1) per row, test hook */
    /* emit pass (wide refinement): rows are the first min(prm->nwide, n) of
     * tmX (then Xw, n = its capacity); candidates go to wide->cand */
    bool emit;
    const WideScratch* wide;
    long long wbase;          /* emit pass: first queued row of this round */
    int stall;                /* test hook: centroid-plane stage the producer leaves unloaded (-1: none) */
};
int  assign_bn_for(int k);                   /* N tile width chosen for k     */
int  assign_supported(int d);                /* 1 when d fits the kernel      */
int  assign_pair_clusters(int k, int dp, int num_sms);   /* 0: no CTA-pair kernel */
cudaError_t launch_assign(const AssignArgs& a, cudaStream_t s);

/* ---- refine / update (kernels.cu) ---- */
void launch_refine(const float* P, const float* C, const float* cn, int d, int k, int bn,
                   const RefineEntry* list, DevParams* prm, int* labels, long long n_cap,
                   unsigned long long* hist, int hist_cap, const __half* Xs, long long n, int dp,
                   const WideScratch& w, int num_sms, cudaStream_t s, int blocks_per_sm = 4);
void launch_wide_gather(const RefineEntry* list, const __half* Xs, long long n, int dp, const WideScratch& w,
                        long long base, const DevParams* prm, int num_sms, cudaStream_t s);
void launch_refine_wide(const float* P, const float* C, const float* cn, int d, int k, const RefineEntry* list,
                        const WideScratch& w, long long base, DevParams* prm, int* labels, int num_sms,
                        cudaStream_t s);
/* Scratch of the sorted update: perm n ints, bin_start k+1, cursor k, hist k. */
struct UpdateScratch {
    int* perm;
    int* bin_start;
    int* cursor;
    int* hist;
};
/* sums (k*d int64) must be zero on entry; counts (k int64) are written.
 * Returns the number of kernels launched. */
int launch_update_sorted(const float* P, long long n, int d, const int* labels, int k, DevParams* prm,
                          long long* sums, long long* counts, UpdateScratch sc, int num_sms, cudaStream_t s);
/* The update in two halves: the counting sort of the rows by label (reads
 * labels; writes perm, bin starts and the counts) and the segmented sum
 * (reads only the points, perm and bin starts).  Same contract as
 * launch_update_sorted, which is the two in turn. */
int launch_update_sort(long long n, const int* labels, int k, DevParams* prm, long long* counts, UpdateScratch sc,
                       int num_sms, cudaStream_t s);
int launch_update_sum(const float* P, long long n, int d, int k, DevParams* prm, long long* sums, UpdateScratch sc,
                      int num_sms, cudaStream_t s, bool leave_room);
/* Overlapping the refinement with the segmented sum: snapshot the listed
 * rows' labels before the refinement (old, capacity cap entries); after it,
 * move every row whose label changed between the clusters' sums and counts
 * (sums: k*d + k int64, the counts after the sums). */
int launch_refine_snapshot(const RefineEntry* list, const DevParams* prm, const int* labels, int* old, long long cap,
                           int num_sms, cudaStream_t s);
int launch_refine_correct(const float* P, int d, const RefineEntry* list, const DevParams* prm, const int* labels,
                          const int* old, long long cap, int k, long long* sums, int num_sms, cudaStream_t s);
void launch_finalize_fixed(const long long* sums, const long long* counts, int k, int d,
                           const DevParams* prm, float* C, float* moved2, cudaStream_t s);
/* FP32 argmin over all k in the refinement's order, checked against labels
 * (params.verify): cnt[0] += rows that differ, *excess += D(label) - D(best). */
void launch_verify(const float* P, const float* C, const float* cn, int d, int k, const int* labels, long long n,
                   unsigned long long* cnt, double* excess, int num_sms, cudaStream_t s);
/* The tiled full FP32 scan of the rows k_refine_wide queued in `rows` (count
 * prm->nscan), d <= kScanMaxDim; labels bit-exact with the per-row scan. */
void launch_full_scan(const float* P, const float* C, const float* cn, int d, int k, const int* rows,
                      const DevParams* prm, int* labels, int num_sms, cudaStream_t s);
void launch_inertia(const float* P, const float* C, const int* labels, long long n, int d,
                    double* out, cudaStream_t s);
void launch_count_diff(const int* a, const int* b, long long n, unsigned long long* out, cudaStream_t s);
void launch_add_const(float* p, long long count, float c, cudaStream_t s);
void launch_standardize(float* P, int n, int d, cudaStream_t s);

/* ---- combining the ranks' sums over peer memory (peer.cu) ---- */
constexpr int kPeerMax = 64;                     /* ranks a group can hold */
struct PeerBases {
    void* p[kPeerMax];                           /* every rank's exchange block, as this GPU addresses it */
};
size_t peer_block_bytes(int k, int d);
size_t peer_sums_offset();
/* The fused combine + finalisation of one iteration on this rank (one launch):
 * C (k x d, this rank's centroids) and moved2 (k, optional) become the
 * finalised values of the sums of every rank's exchange block. */
cudaError_t launch_peer_combine(const PeerBases& bases, int rank, int world, int k, int d, const DevParams* prm,
                                int* status, float* C, float* moved2, int num_sms, cudaStream_t s);

/* ---- device memory (mpkmeans_api.cu) ----
 * Engine scratch comes from one stream-ordered memory pool per device whose
 * release threshold keeps freed blocks cached, so a second fit of the same
 * size allocates nothing new from the driver. */
cudaError_t dev_alloc(void** p, size_t bytes, cudaStream_t s);
void dev_free(void* p, cudaStream_t s);

/* ---- tensor maps (engine host code) ---- */
bool make_tmap_planes(CUtensorMap* map, const __half* base, long long rows, int dp, int box_rows);

}  /* namespace mpk */
