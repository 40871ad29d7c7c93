/* mpkmeans_api.cu -- the C ABI of libmpkmeans_b200: engine handle, Lloyd
 * drivers and data helpers.  Declarations and the reference interface each one
 * replaces are in include/mpkmeans.h.
 */
#include "engine.cuh"
#include "mpkmeans.h"
#include "mpkmeans_debug.h"

#include <cublas_v2.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <random>
#include <string>
#include <vector>

using namespace mpk;

/* ----------------------------------------------------------- helpers ---- */

#define MPK_TRY(call)                                                                    \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess) {                                                         \
            fprintf(stderr, "mpkmeans_b200 %s:%d CUDA: %s\n", __FILE__, __LINE__,         \
                    cudaGetErrorString(e_));                                             \
            return MPK_ERR_CUDA;                                                         \
        }                                                                                \
    } while (0)

namespace {

constexpr double U16 = 1.0 / 2048.0;
constexpr double U24 = 1.0 / 16777216.0;
constexpr double U22 = 1.0 / 4194304.0;

cudaStream_t stream_of(cublasHandle_t blas) {
    cudaStream_t s = nullptr;
    if (blas) cublasGetStream(blas, &s);
    return s;
}

long long round_up(long long a, long long b) { return (a + b - 1) / b * b; }

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

/* Error-bound constants of the assignment filter, for inner dimension d (dp
 * padded).  A pair (i, j) is excluded only when
 *     D~_j - D~_best > c1 ||x|| cmax + c2 eta (||x|| + cmax) + 2^-22 (|D~_j| + |D~_best|)
 * where D~ is the tensor-core distance.  The terms:
 *   split    3 * 2^-22 ||x|| ||c||: the lo words carry the residual to 2^-22
 *            relative and the dropped lo*lo product is below 2^-22;
 *   accum    (3 dp / 16 + 16) * 2^-22 ||x|| ||c||: one truncating FP32 add per
 *            16-deep MMA step of the three-product chain, plus slack;
 *   fp32     gamma_d ||x|| ||c||: the FP32 evaluation the labels must agree
 *            with (any summation order);
 *   floor    2^-25/s per coordinate for lo words that fall subnormal (c2);
 * each appears once for the best and once for the candidate (factor 2) and as
 * a distance (factor 2 on the dot).  The norms ||x||, ||c|| are FP32 values,
 * inflated here by their own rounding. */
BoundConsts bound_consts(int d, int dp) {
    const double eps_split = 3.2 * U22;
    const double eps_acc = (3.0 * dp / 16.0 + 16.0) * U22;
    const double g = d * U24;
    const double gamma_d = g / (1.0 - g);
    const double infl = 1.0 + 4.0 * d * U24 + 1.0 / 65536.0;
    BoundConsts bc;
    bc.c1 = (float)(4.0 * (eps_split + eps_acc + gamma_d) * infl);
    bc.c2 = (float)(4.0 * std::sqrt((double)d) * 1.01);
    return bc;
}

int current_sm_count(int* dev_out, int* cc_major) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cc_major) cudaDeviceGetAttribute(cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    if (dev_out) *dev_out = dev;
    return sms;
}

}  /* namespace */

/* ------------------------------------------------------ memory pool ---- */

namespace mpk {

/* peer.cu: the group behind mpkPeerCombine */
bool peer_ready(mpkPeerGroup g, int k, int d);
const PeerBases& peer_bases(mpkPeerGroup g);
int peer_rank(mpkPeerGroup g);
int peer_world(mpkPeerGroup g);

static cudaMemPool_t engine_pool(int dev) {
    static std::mutex m;
    static cudaMemPool_t pools[64] = {};
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(m);
    if (!pools[dev]) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.handleTypes = cudaMemHandleTypeNone;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) return nullptr;
        unsigned long long keep = ~0ull;   /* never return freed blocks to the driver early */
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        pools[dev] = pool;
    }
    return pools[dev];
}

/* Test hook (mpkDebugFailAlloc): n > 0 makes the n-th device allocation from
 * now fail, once. */
static std::atomic<int> g_fail_alloc{0};

cudaError_t dev_alloc(void** p, size_t bytes, cudaStream_t s) {
    for (int f = g_fail_alloc.load(); f > 0;) {
        if (g_fail_alloc.compare_exchange_weak(f, f - 1)) {
            if (f == 1) {
                *p = nullptr;
                return cudaErrorMemoryAllocation;
            }
            break;
        }
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    cudaMemPool_t pool = engine_pool(dev);
    if (!pool) return cudaErrorMemoryAllocation;
    return cudaMallocFromPoolAsync(p, bytes, pool, s);
}

void dev_free(void* p, cudaStream_t s) {
    if (p) cudaFreeAsync(p, s);
}

}  /* namespace mpk */

extern "C" mpkStatus mpkTrimMemoryPool(int device) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return MPK_ERR_CUDA;
    if (device < 0) device = prev;
    cudaMemPool_t pool = mpk::engine_pool(device);
    if (!pool) return MPK_ERR_INVALID;
    if (cudaSetDevice(device) != cudaSuccess) return MPK_ERR_INVALID;
    const cudaError_t e1 = cudaDeviceSynchronize();
    const cudaError_t e2 = cudaMemPoolTrimTo(pool, 0);
    cudaSetDevice(prev);
    return (e1 == cudaSuccess && e2 == cudaSuccess) ? MPK_OK : MPK_ERR_CUDA;
}

/* ------------------------------------------------------------ engine ---- */

struct mpkEngine_s {
    int dev = 0, num_sms = 0;
    cudaStream_t s = nullptr;
    const float* P = nullptr;
    long long n = 0;
    int d = 0, k = 0, dp = 0, kpad = 0;
    bool can_assign = false;
    __half* Xs = nullptr;
    float* xnorm = nullptr;
    __half* Cs = nullptr;
    float* cn = nullptr;
    RefineEntry* list = nullptr;
    DevParams* prm = nullptr;
    double* dInertia = nullptr;
    unsigned long long* hist = nullptr;   /* MPK_MAX_HIST slots */
    UpdateScratch us{nullptr, nullptr, nullptr, nullptr};
    CUtensorMap tmX, tmC, tmCh, tmXw;   /* tmCh: centroid planes in 128-row halves (CTA pairs) */
    WideScratch wide{nullptr, nullptr, nullptr, nullptr, nullptr, 0, 0, 0, 256};
    BoundConsts bc;
    float4* dbg = nullptr;                /* test hook, set by mpkDebugSetAssignTrace */
    int stall = -1;                       /* test hook, set by mpkDebugInjectStall */
    int pair = 1;                         /* CTA-pair assignment kernel (mpkDebugAssignPair) */
    /* the refinement beside the segmented sum (mpkDebugOverlapRefine): it runs on
     * s2 between a fork and a join event, with the listed rows' labels before it
     * in old_lab (n ints) */
    int overlap = 1;
    cudaStream_t s2 = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join2 = nullptr;
    int* old_lab = nullptr;
    int pair_clusters = 0;                /* resident clusters of two for it */
    long long launches = 0;               /* kernels this engine has launched */
    bool prof = false;                    /* bench hook: events around the hot kernels */
    std::vector<cudaEvent_t> ev_assign, ev_refine, ev_accum;
    /* mpkEngineIterate / mpkEngineStep: one iteration as three graphs (the
     * tensor-core assignment; its refinement; the update -- with the
     * finalisation for Iterate, without it for Step), captured for these
     * buffers, this refine flag and that choice */
    struct {
        cudaGraphExec_t assign = nullptr, refine_g = nullptr, update = nullptr;
        const float* C = nullptr;
        const int* A = nullptr;
        const long long* S = nullptr;
        int refine = -1;
        int finalize = -1;
        int overlap = -1;
        long long n_assign = 0, n_refine = 0, n_update = 0;   /* kernels per replay */
        bool failed = false;                    /* a capture failed: launch directly from then on */
    } g;
};

static void graphs_release(mpkEngine e) {
    if (e->g.assign) cudaGraphExecDestroy(e->g.assign);
    if (e->g.refine_g) cudaGraphExecDestroy(e->g.refine_g);
    if (e->g.update) cudaGraphExecDestroy(e->g.update);
    e->g.assign = e->g.refine_g = e->g.update = nullptr;
    e->g.C = nullptr;
    e->g.A = nullptr;
    e->g.S = nullptr;
    e->g.refine = -1;
    e->g.finalize = -1;
    e->g.overlap = -1;
}

static void prof_mark(mpkEngine e, std::vector<cudaEvent_t>& v, cudaStream_t s) {
    if (!e->prof) return;
    cudaEvent_t ev = nullptr;
    if (cudaEventCreate(&ev) == cudaSuccess) {
        cudaEventRecord(ev, s);
        v.push_back(ev);
    }
}

static void prof_mark(mpkEngine e, std::vector<cudaEvent_t>& v) { prof_mark(e, v, e->s); }

static void prof_clear(mpkEngine e) {
    for (auto x : e->ev_assign) cudaEventDestroy(x);
    for (auto x : e->ev_refine) cudaEventDestroy(x);
    for (auto x : e->ev_accum) cudaEventDestroy(x);
    e->ev_assign.clear();
    e->ev_refine.clear();
    e->ev_accum.clear();
}

static void engine_free(mpkEngine e) {
    if (!e) return;
    prof_clear(e);
    graphs_release(e);
    void* bufs[] = {e->Xs, e->xnorm, e->Cs, e->cn, e->list, e->prm, e->dInertia, e->hist,
                    e->us.perm, e->us.bin_start, e->us.cursor, e->us.hist, e->old_lab,
                    e->wide.Xw, e->wide.went, e->wide.cand, e->wide.ccount, e->wide.scan};
    for (void* b : bufs) dev_free(b, e->s);
    if (e->ev_fork) cudaEventDestroy(e->ev_fork);
    if (e->ev_join2) cudaEventDestroy(e->ev_join2);
    if (e->s2) {
        cudaStreamSynchronize(e->s2);
        cudaStreamDestroy(e->s2);
    }
    delete e;
}

static mpkStatus engine_create(mpkEngine* out, const float* dP, long long n, int d, int k, const float* dC0,
                               float pmax_global, long long n_global, cudaStream_t s, bool need_assign) {
    if (!out || n < 0 || d <= 0 || k <= 0 || (n > 0 && !dP)) return MPK_ERR_INVALID;
    if (n > INT_MAX) {
        fprintf(stderr, "mpkmeans_b200: a shard holds at most %d rows (got %lld)\n", INT_MAX, n);
        return MPK_ERR_INVALID;
    }
    *out = nullptr;
    int cc = 0;
    mpkEngine e = new mpkEngine_s();
    e->num_sms = current_sm_count(&e->dev, &cc);
    if (cc != 10) {
        fprintf(stderr, "mpkmeans_b200: needs an sm_100 GPU (B200); device %d is compute capability %d.x\n",
                e->dev, cc);
        delete e;
        return MPK_ERR_CUDA;
    }
    if (need_assign && !assign_supported(d)) {
        fprintf(stderr, "mpkmeans_b200: d = %d is above the assignment kernel's limit of 65536\n", d);
        delete e;
        return MPK_ERR_INVALID;
    }
    e->s = s;
    e->P = dP;
    e->n = n;
    e->d = d;
    e->k = k;
    e->dp = (int)round_up(d, 64);
    e->kpad = (int)round_up(k, 256);
    e->can_assign = need_assign;
    e->bc = bound_consts(d, e->dp);
    const long long ng = n_global > 0 ? n_global : (n > 0 ? n : 1);

#define ALLOC(ptr, bytes)                                                      \
    if (dev_alloc((void**)&(ptr), (size_t)(bytes), s) != cudaSuccess) {        \
        fprintf(stderr, "mpkmeans_b200: allocation of %lld bytes failed\n", (long long)(bytes)); \
        engine_free(e);                                                        \
        return MPK_ERR_ALLOC;                                                  \
    }
    ALLOC(e->prm, sizeof(DevParams));
    ALLOC(e->dInertia, sizeof(double));
    ALLOC(e->hist, sizeof(unsigned long long) * MPK_MAX_HIST);
    ALLOC(e->us.perm, sizeof(int) * (size_t)(n > 0 ? n : 1));
    ALLOC(e->us.bin_start, sizeof(int) * ((size_t)k + 1));
    ALLOC(e->us.cursor, sizeof(int) * (size_t)k);
    ALLOC(e->us.hist, sizeof(int) * (size_t)k);
    if (need_assign) {
        ALLOC(e->Xs, (size_t)2 * (n > 0 ? n : 1) * e->dp * sizeof(__half));
        ALLOC(e->xnorm, (size_t)(n > 0 ? n : 1) * sizeof(float));
        ALLOC(e->Cs, (size_t)2 * e->kpad * e->dp * sizeof(__half));
        ALLOC(e->cn, (size_t)e->kpad * sizeof(float));
        ALLOC(e->list, (size_t)(n > 0 ? n : 1) * sizeof(RefineEntry));
        ALLOC(e->old_lab, (size_t)(n > 0 ? n : 1) * sizeof(int));
        /* the wide path (rows whose class rescans would visit more than
         * wide.rescan_limit columns): its tensor-core pass needs 256-wide centroid
         * tiles, k > kWideMinK */
        /* (16 classes of ceil(k/16) columns: a row can exceed the limit only when they do) */
        if (k > kWideMinK && n > 0 && 16LL * ((k + 15) / 16) > wide_rescan_limit(n)) {
            const long long cap = std::min<long long>(n, std::max<long long>(65536, (n + 7) / 8));
            e->wide.cap = cap;
            e->wide.per_round = cap;
            /* every queued row gets a round when classes are wide (k >= 4096: 256+ columns a
             * class); below that one round, and rows past it rescan their classes */
            e->wide.rounds = k >= 4096 ? (int)((n + cap - 1) / cap) : 1;
            e->wide.rescan_limit = wide_rescan_limit(n);
            ALLOC(e->wide.Xw, (size_t)2 * cap * e->dp * sizeof(__half));
            ALLOC(e->wide.went, (size_t)n * sizeof(int));
            ALLOC(e->wide.cand, (size_t)cap * kWideCand * sizeof(int));
            ALLOC(e->wide.ccount, (size_t)cap * 2 * sizeof(int));
            if (d <= kScanMaxDim) ALLOC(e->wide.scan, (size_t)n * sizeof(int));
        }
    }
#undef ALLOC
    /* the refinement's stream at the highest priority: as the update's blocks
     * retire, the block scheduler places the latency-bound refinement first */
    int prio_lo = 0, prio_hi = 0;
    cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi);
    if (need_assign && (cudaStreamCreateWithPriority(&e->s2, cudaStreamNonBlocking, prio_hi) != cudaSuccess ||
                        cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
                        cudaEventCreateWithFlags(&e->ev_join2, cudaEventDisableTiming) != cudaSuccess)) {
        fprintf(stderr, "mpkmeans_b200: cannot create the engine's second stream\n");
        engine_free(e);
        return MPK_ERR_CUDA;
    }
    cudaMemsetAsync(e->prm, 0, sizeof(DevParams), s);
    cudaMemsetAsync(e->hist, 0, sizeof(unsigned long long) * MPK_MAX_HIST, s);
    if (pmax_global > 0.f) {
        DevParams h{};
        h.pmax = pmax_global;
        h.c0max = 0.f;
        cudaMemcpyAsync(e->prm, &h, sizeof(float) * 2, cudaMemcpyHostToDevice, s);
        cudaStreamSynchronize(s);   /* h is on the stack */
    } else {
        launch_maxabs(dP, n * d, &e->prm->pmax, s);
        if (dC0) launch_maxabs(dC0, (long long)k * d, &e->prm->c0max, s);
    }
    launch_set_scale(e->prm, ng, s);
    if (need_assign) {
        if (n > 0) launch_split_rows(dP, n, d, e->dp, e->prm, e->Xs, n * e->dp, e->xnorm, s);
        auto fn = encode_fn();
        if (!fn) {
            fprintf(stderr, "mpkmeans_b200: cuTensorMapEncodeTiled is unavailable\n");
            engine_free(e);
            return MPK_ERR_CUDA;
        }
        if ((n > 0 && !make_tmap_planes(&e->tmX, e->Xs, n, e->dp, 128)) ||
            !make_tmap_planes(&e->tmC, e->Cs, e->kpad, e->dp, assign_bn_for(k)) ||
            (assign_bn_for(k) == 256 && !make_tmap_planes(&e->tmCh, e->Cs, e->kpad, e->dp, 128)) ||
            (e->wide.cap > 0 && !make_tmap_planes(&e->tmXw, e->wide.Xw, e->wide.cap, e->dp, 128))) {
            fprintf(stderr, "mpkmeans_b200: tensor map encoding failed\n");
            engine_free(e);
            return MPK_ERR_CUDA;
        }
        e->pair_clusters = assign_pair_clusters(k, e->dp, e->num_sms);
    }
    if (cudaGetLastError() != cudaSuccess) {
        engine_free(e);
        return MPK_ERR_CUDA;
    }
    *out = e;
    return MPK_OK;
}

namespace mpk {
bool make_tmap_planes(CUtensorMap* map, const __half* base, long long rows, int dp, int box_rows) {
    auto fn = encode_fn();
    if (!fn || rows <= 0) return false;
    cuuint64_t dims[3] = {(cuuint64_t)dp, (cuuint64_t)rows, 2};
    cuuint64_t strides[2] = {(cuuint64_t)dp * 2, (cuuint64_t)rows * (cuuint64_t)dp * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  /* namespace mpk */

/* The assignment proper: the centroid split and the tensor-core pass, whose
 * labels are final for every row it does not list for refinement. */
/* Arguments of the engine's tensor-core pass over its own rows. */
static AssignArgs assign_args(mpkEngine e, int* dAssign, int refine) {
    AssignArgs a;
    a.tmX = &e->tmX;
    a.tmC = &e->tmC;
    a.tmCh = &e->tmCh;
    a.pair = e->pair;
    a.pair_clusters = e->pair_clusters;
    a.n = e->n;
    a.k = e->k;
    a.d = e->d;
    a.dp = e->dp;
    a.xnorm = e->xnorm;
    a.cn = e->cn;
    a.prm_ro = e->prm;
    a.prm = e->prm;
    a.labels = dAssign;
    a.list = e->list;
    a.refine = refine;
    a.bc = e->bc;
    a.num_sms = e->num_sms;
    a.dbg = e->dbg;
    a.emit = false;
    a.wide = &e->wide;
    a.wbase = 0;
    a.stall = e->stall;
    return a;
}

/* The assignment proper: the centroid split and the tensor-core pass, whose
 * labels are final for every row it does not list for refinement. */
static mpkStatus engine_assign_tc(mpkEngine e, const float* dC, int* dAssign, int refine) {
    if (!e->can_assign) return MPK_ERR_INVALID;
    launch_prep_c(dC, e->k, e->kpad, e->d, e->dp, e->prm, e->Cs, e->cn, e->s);
    ++e->launches;
    if (e->n == 0) return cudaGetLastError() == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
    const AssignArgs a = assign_args(e, dAssign, refine);
    prof_mark(e, e->ev_assign);
    cudaError_t err = launch_assign(a, e->s);
    prof_mark(e, e->ev_assign);
    ++e->launches;
    if (err != cudaSuccess) {
        fprintf(stderr, "mpkmeans_b200: assignment launch failed: %s\n", cudaGetErrorString(err));
        return MPK_ERR_CUDA;
    }
    return cudaGetLastError() == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
}

/* The FP32 refinement of the rows the last engine_assign_tc listed.
 * record_hist: the refinement writes its entry count to the next slot of the
 * engine's survivor history (prm->hist_next counts the slots used). */
/* Which part of the refinement to launch: all of it; the per-row FP32 pass
 * (k_refine: small blocks that can run beside other kernels); or the wide
 * rounds and the tiled full scan that follow it (tensor-core and shared-memory
 * heavy kernels that occupy whole SMs). */
enum RefinePart { REFINE_ALL, REFINE_ROWS, REFINE_WIDE };

static mpkStatus engine_refine(mpkEngine e, const float* dC, int* dAssign, bool record_hist,
                               cudaStream_t rs = nullptr, RefinePart part = REFINE_ALL) {
    if (e->n == 0) return MPK_OK;
    if (!rs) rs = e->s;
    if (part != REFINE_WIDE) prof_mark(e, e->ev_refine, rs);
    if (part != REFINE_WIDE) {
        /* beside the segmented sum (REFINE_ROWS), the sum's one wave keeps three block slots a
         * SM and the refinement's first blocks take the fourth; the rest start as the sum's
         * blocks retire (a heavy refinement, as at config 5, then still gets the whole GPU) */
        launch_refine(e->P, dC, e->cn, e->d, e->k, assign_bn_for(e->k), e->list, e->prm, dAssign, e->n,
                      record_hist ? e->hist : nullptr, MPK_MAX_HIST, e->Xs, e->n, e->dp,
                      e->wide, e->num_sms, rs);
        ++e->launches;
    }
    if (part == REFINE_ROWS) {
        prof_mark(e, e->ev_refine, rs);
        return cudaGetLastError() == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
    }
    /* rows the refinement queued: per round, a tensor-core pass that lists their
     * candidates, then the FP32 evaluation of just those (every launch sizes itself from
     * prm->nwide; rounds past the queue exit at once) */
    for (int r = 0; r < e->wide.rounds; ++r) {
        const long long base = (long long)r * e->wide.per_round;
        if (r > 0) {
            launch_wide_gather(e->list, e->Xs, e->n, e->dp, e->wide, base, e->prm, e->num_sms, rs);
            ++e->launches;
        }
        AssignArgs w = assign_args(e, nullptr, 1);
        w.tmX = &e->tmXw;
        w.n = e->wide.per_round;
        w.dbg = nullptr;
        w.emit = true;
        w.wbase = base;
        const cudaError_t err = launch_assign(w, rs);
        if (err != cudaSuccess) {
            fprintf(stderr, "mpkmeans_b200: wide assignment launch failed: %s\n", cudaGetErrorString(err));
            return MPK_ERR_CUDA;
        }
        launch_refine_wide(e->P, dC, e->cn, e->d, e->k, e->list, e->wide, base, e->prm, dAssign, e->num_sms, rs);
        e->launches += 2;                 /* the emit pass and the FP32 evaluation */
    }
    if (e->wide.scan) {                   /* rows whose lists overflowed: all k, tiled */
        launch_full_scan(e->P, dC, e->cn, e->d, e->k, e->wide.scan, e->prm, dAssign, e->num_sms, rs);
        ++e->launches;
    }
    if (part != REFINE_WIDE) prof_mark(e, e->ev_refine, rs);
    return cudaGetLastError() == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
}

static mpkStatus engine_assign(mpkEngine e, const float* dC, int* dAssign, int refine, bool record_hist) {
    const mpkStatus st = engine_assign_tc(e, dC, dAssign, refine);
    if (st != MPK_OK || !refine) return st;
    return engine_refine(e, dC, dAssign, record_hist);
}

/* Capture body() on gs (a non-default stream) into an executable graph.
 * false, with no graph, when the capture or the instantiation fails. */
template <typename F>
static bool capture_graph(cudaStream_t gs, F&& body, cudaGraphExec_t* exec) {
    *exec = nullptr;
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(gs, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    const mpkStatus st = body();
    const cudaError_t ec = cudaStreamEndCapture(gs, &g);
    const bool ok = st == MPK_OK && ec == cudaSuccess && g != nullptr &&
                    cudaGraphInstantiate(exec, g, cudaGraphInstantiateFlagUseNodePriority) == cudaSuccess;
    if (g) cudaGraphDestroy(g);
    if (!ok) {
        if (*exec) cudaGraphExecDestroy(*exec);
        *exec = nullptr;
        cudaGetLastError();
    }
    return ok;
}

static mpkStatus engine_accumulate(mpkEngine e, const int* dAssign, long long* dSums) {
    const long long len = (long long)e->k * e->d + e->k;
    cudaMemsetAsync(dSums, 0, (size_t)len * sizeof(long long), e->s);
    prof_mark(e, e->ev_accum);
    e->launches += launch_update_sorted(e->P, e->n, e->d, dAssign, e->k, e->prm, dSums,
                                        dSums + (long long)e->k * e->d, e->us, e->num_sms, e->s);
    prof_mark(e, e->ev_accum);
    return cudaGetLastError() == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
}

static mpkStatus engine_finalize(mpkEngine e, const long long* dSums, float* dC, float* dMoved2) {
    launch_finalize_fixed(dSums, dSums + (long long)e->k * e->d, e->k, e->d, e->prm, dC, dMoved2, e->s);
    ++e->launches;
    return cudaGetLastError() == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
}

/* The refinement of the rows the last engine_assign_tc listed and the update,
 * overlapped (finalize: then the finalisation too, into dMoved2 if given).
 * The counting sort reads the assignment's labels; then the latency-bound
 * per-row refinement runs on the second stream beside the bandwidth-bound
 * segmented sum of those labels (which leaves each SM room for it), after
 * snapshotting the listed rows' labels.  After the join come the wide rounds
 * and the full scan (kernels that need whole SMs; they exit at once when no row
 * needs them), and then every listed row whose label changed moves from its old
 * cluster's sums and count to the new one's.  The integer sums come out
 * exactly as an update of the refined labels would give them. */
static mpkStatus engine_refine_update(mpkEngine e, float* dC, int* dAssign, long long* dSums, bool record_hist,
                                      bool finalize, float* dMoved2) {
    const long long kd = (long long)e->k * e->d;
    cudaMemsetAsync(dSums, 0, (size_t)(kd + e->k) * sizeof(long long), e->s);
    prof_mark(e, e->ev_accum);
    e->launches += launch_update_sort(e->n, dAssign, e->k, e->prm, dSums + kd, e->us, e->num_sms, e->s);
    cudaEventRecord(e->ev_fork, e->s);
    cudaStreamWaitEvent(e->s2, e->ev_fork, 0);
    e->launches += launch_refine_snapshot(e->list, e->prm, dAssign, e->old_lab, e->n, e->num_sms, e->s2);
    mpkStatus st = engine_refine(e, dC, dAssign, record_hist, e->s2, REFINE_ROWS);
    /* small shards keep their class rescans in the refinement (wide_rescan_limit): the sum runs
     * as one wave that leaves each SM a block slot for it; on large shards the rescans go wide,
     * the refinement is light, and the sum's two full waves are faster (config 3: update window
     * 1.10 against 1.16 ms; at 1.25e6 rows 0.184 against 0.205 ms the other way) */
    const bool room = wide_rescan_limit(e->n) > 32;
    e->launches += launch_update_sum(e->P, e->n, e->d, e->k, e->prm, dSums, e->us, e->num_sms, e->s, room);
    cudaEventRecord(e->ev_join2, e->s2);
    cudaStreamWaitEvent(e->s, e->ev_join2, 0);       /* always joined, so a capture can end */
    if (st == MPK_OK) st = engine_refine(e, dC, dAssign, record_hist, e->s, REFINE_WIDE);
    e->launches += launch_refine_correct(e->P, e->d, e->list, e->prm, dAssign, e->old_lab, e->n, e->k, dSums,
                                         e->num_sms, e->s);
    prof_mark(e, e->ev_accum);
    if (st == MPK_OK && finalize) st = engine_finalize(e, dSums, dC, dMoved2);
    if (st != MPK_OK) return st;
    return cudaGetLastError() == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
}

namespace mpk {
/* The exclusion attribution of the reference's mpkStats (mpkmeans.h:147-156,
 * filled at mpkmeans.cu:655-676), from S->tested and the engine's counters.
 * This engine has one exclusion test: the certified bound on the tensor-core
 * distances, formed from those values and the norms alone -- the role of the
 * reference's condition (3).  It computes no exact reference entry per row
 * before excluding, so condition (6) and hp_reference have no counterpart and
 * stay 0, as in the reference's own (3)-only scheme.  Every row the bound does
 * not settle has its incumbent evaluated in FP32 together with its candidates
 * (all counted in hp_update), so the pairs the bound excluded are the tested
 * pairs less the non-incumbent candidates evaluated:
 *     excl = tested - (hp_update - rows refined).
 * The count goes to excl_cond3, or to excl_cond6 when the caller enabled only
 * condition (6); excl_both stays 0. */
void fill_exclusions(mpkStats* S, const mpkParams& P, long long rows_refined, long long cands) {
    const long long excl = S->tested - (cands - rows_refined);
    if (P.use_cond3 || !P.use_cond6) S->excl_cond3 = excl;
    else S->excl_cond6 = excl;
}
}  /* namespace mpk */

extern "C" {

mpkStatus mpkEngineCreate(mpkEngine* out, const float* dP, long long n, int d, int k, const float* dC0,
                          float pmax_global, long long n_global, cudaStream_t stream) {
    return engine_create(out, dP, n, d, k, dC0, pmax_global, n_global, stream, true);
}

mpkStatus mpkEngineDestroy(mpkEngine e) {
    if (!e) return MPK_ERR_INVALID;
    cudaStreamSynchronize(e->s);
    engine_free(e);
    return MPK_OK;
}

mpkStatus mpkEngineAssign(mpkEngine e, const float* dC, int* dAssign, int refine) {
    if (!e || !dC || (e->n > 0 && !dAssign)) return MPK_ERR_INVALID;
    return engine_assign(e, dC, dAssign, refine, false);
}

mpkStatus mpkEngineAccumulate(mpkEngine e, const int* dAssign, long long* dSums) {
    if (!e || !dSums || (e->n > 0 && !dAssign)) return MPK_ERR_INVALID;
    return engine_accumulate(e, dAssign, dSums);
}

mpkStatus mpkEngineFinalize(mpkEngine e, const long long* dSums, float* dC, float* dMoved2) {
    if (!e || !dSums || !dC) return MPK_ERR_INVALID;
    return engine_finalize(e, dSums, dC, dMoved2);
}

}  /* extern "C" */

/* iters iterations (finalize) or one step without the finalisation, replayed
 * from the engine's three graphs where the stream allows */
static mpkStatus engine_replay(mpkEngine e, float* dC, int* dAssign, long long* dSums, int iters, int refine,
                               bool finalize) {
    auto assign = [&] { return engine_assign_tc(e, dC, dAssign, refine); };
    auto refine_step = [&] { return engine_refine(e, dC, dAssign, false); };
    auto update = [&] {
        const mpkStatus a = engine_accumulate(e, dAssign, dSums);
        return (a != MPK_OK || !finalize) ? a : engine_finalize(e, dSums, dC, nullptr);
    };
    /* the refinement beside the update's segmented sum (one graph for both) */
    const bool ov = e->overlap && refine && e->n > 0;
    auto refine_update = [&] { return engine_refine_update(e, dC, dAssign, dSums, false, finalize, nullptr); };
    /* graphs need a capturable stream, and no test hook that a replay would freeze */
    const bool graphable = e->s != nullptr && e->s != cudaStreamLegacy && e->s != cudaStreamPerThread &&
                           e->dbg == nullptr && e->stall < 0 && !e->g.failed;
    bool have = e->g.assign && e->g.C == dC && e->g.A == dAssign && e->g.S == dSums && e->g.refine == refine &&
                e->g.finalize == (int)finalize && e->g.overlap == (int)ov;
    if (graphable && !have && iters > 0) {
        graphs_release(e);
        const bool prof = e->prof;
        const long long l0 = e->launches;
        e->prof = false;
        /* three graphs rather than one so that the profiling hook can time the
         * tensor-core pass, the refinement and the update apart */
        bool ok = capture_graph(e->s, assign, &e->g.assign);
        const long long l1 = e->launches;
        ok = ok && (!refine || ov || capture_graph(e->s, refine_step, &e->g.refine_g));
        const long long l2 = e->launches;
        ok = ok && (ov ? capture_graph(e->s, refine_update, &e->g.update) : capture_graph(e->s, update, &e->g.update));
        const long long l3 = e->launches;
        e->prof = prof;
        e->launches = l0;                         /* captured, not yet run */
        if (ok) {
            e->g.C = dC;
            e->g.A = dAssign;
            e->g.S = dSums;
            e->g.refine = refine;
            e->g.finalize = (int)finalize;
            e->g.overlap = (int)ov;
            e->g.n_assign = l1 - l0;
            e->g.n_refine = l2 - l1;
            e->g.n_update = l3 - l2;
            have = true;
        } else {
            graphs_release(e);
            e->g.failed = true;
        }
    }
    for (int i = 0; i < iters; ++i) {
        if (have && graphable) {
            prof_mark(e, e->ev_assign);
            if (cudaGraphLaunch(e->g.assign, e->s) != cudaSuccess) return MPK_ERR_CUDA;
            prof_mark(e, e->ev_assign);
            if (e->g.refine_g) {
                prof_mark(e, e->ev_refine);
                if (cudaGraphLaunch(e->g.refine_g, e->s) != cudaSuccess) return MPK_ERR_CUDA;
                prof_mark(e, e->ev_refine);
            }
            prof_mark(e, e->ev_accum);
            if (cudaGraphLaunch(e->g.update, e->s) != cudaSuccess) return MPK_ERR_CUDA;
            prof_mark(e, e->ev_accum);
            e->launches += e->g.n_assign + e->g.n_refine + e->g.n_update;
        } else {
            mpkStatus st = assign();
            if (st == MPK_OK && ov) {
                st = refine_update();
            } else {
                if (st == MPK_OK && refine) st = refine_step();
                if (st == MPK_OK) st = update();
            }
            if (st != MPK_OK) return st;
        }
    }
    return cudaGetLastError() == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
}

extern "C" {

mpkStatus mpkEngineIterate(mpkEngine e, float* dC, int* dAssign, long long* dSums, int iters, int refine) {
    if (!e || !dC || !dAssign || !dSums || iters < 0 || !e->can_assign) return MPK_ERR_INVALID;
    return engine_replay(e, dC, dAssign, dSums, iters, refine, true);
}

mpkStatus mpkEngineStep(mpkEngine e, const float* dC, int* dAssign, long long* dSums, int refine) {
    if (!e || !dC || (e->n > 0 && !dAssign) || !dSums || !e->can_assign) return MPK_ERR_INVALID;
    return engine_replay(e, const_cast<float*>(dC), dAssign, dSums, 1, refine, false);
}

mpkStatus mpkPeerCombine(mpkPeerGroup g, mpkEngine e, float* dC, float* dMoved2) {
    if (!e || !dC || !mpk::peer_ready(g, e->k, e->d)) return MPK_ERR_INVALID;
    const cudaError_t err = launch_peer_combine(mpk::peer_bases(g), mpk::peer_rank(g), mpk::peer_world(g), e->k,
                                                e->d, e->prm, &e->prm->status, dC, dMoved2, e->num_sms, e->s);
    ++e->launches;
    return err == cudaSuccess ? MPK_OK : MPK_ERR_CUDA;
}

mpkStatus mpkEngineInertia(mpkEngine e, const float* dC, const int* dAssign, double* out) {
    if (!e || !dC || !out) return MPK_ERR_INVALID;
    MPK_TRY(cudaMemsetAsync(e->dInertia, 0, sizeof(double), e->s));
    launch_inertia(e->P, dC, dAssign, e->n, e->d, e->dInertia, e->s);
    MPK_TRY(cudaMemcpyAsync(out, e->dInertia, sizeof(double), cudaMemcpyDeviceToHost, e->s));
    MPK_TRY(cudaStreamSynchronize(e->s));
    return MPK_OK;
}

int mpkEngineFracBits(mpkEngine e) {
    if (!e) return -1;
    int f = 0;
    cudaMemcpyAsync(&f, &e->prm->frac, sizeof(int), cudaMemcpyDeviceToHost, e->s);
    cudaStreamSynchronize(e->s);
    return f;
}

mpkStatus mpkEngineCounters(mpkEngine e, long long* rows_refined, long long* cand_refined, long long* rows_full_scan,
                            int* status) {
    if (!e) return MPK_ERR_INVALID;
    DevParams h;
    MPK_TRY(cudaMemcpyAsync(&h, e->prm, sizeof(DevParams), cudaMemcpyDeviceToHost, e->s));
    MPK_TRY(cudaStreamSynchronize(e->s));
    if (rows_refined) *rows_refined = (long long)h.nflag_total;
    if (cand_refined) *cand_refined = (long long)h.ncand_total;
    if (rows_full_scan) *rows_full_scan = (long long)h.novf_total;
    if (status) *status = h.status;
    return MPK_OK;
}

long long mpkEngineSumsLength(mpkEngine e) { return e ? (long long)e->k * e->d + e->k : 0; }

/* Test hook: while set, every assignment writes (v0, v1, j0, j1) per row --
 * the emulated best and runner-up distances and their centroids -- to dOut4
 * (n float4, device).  Pass NULL to stop.  No reference counterpart. */
mpkStatus mpkDebugSetAssignTrace(mpkEngine e, float* dOut4) {
    if (!e) return MPK_ERR_INVALID;
    e->dbg = reinterpret_cast<float4*>(dOut4);
    return MPK_OK;
}

/* Bench hook: while enabled, the engine records a CUDA event pair on its
 * stream around every tensor-core assignment, refinement and accumulation
 * step (include/mpkmeans_debug.h says what each pair covers). */
mpkStatus mpkDebugProfile(mpkEngine e, int enable) {
    if (!e) return MPK_ERR_INVALID;
    cudaStreamSynchronize(e->s);
    prof_clear(e);
    e->prof = enable != 0;
    return MPK_OK;
}

/* Synchronises, returns the summed device time and launch counts of the
 * three profiled steps since mpkDebugProfile(e, 1), and clears the record. */
mpkStatus mpkDebugProfileRead(mpkEngine e, double* assign_ms, long long* assign_launches, double* refine_ms,
                              long long* refine_launches, double* accum_ms, long long* accum_launches) {
    if (!e) return MPK_ERR_INVALID;
    MPK_TRY(cudaStreamSynchronize(e->s));
    auto total = [](const std::vector<cudaEvent_t>& v) {
        double t = 0.0;
        for (size_t i = 0; i + 1 < v.size(); i += 2) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, v[i], v[i + 1]);
            t += ms;
        }
        return t;
    };
    if (assign_ms) *assign_ms = total(e->ev_assign);
    if (assign_launches) *assign_launches = (long long)(e->ev_assign.size() / 2);
    if (refine_ms) *refine_ms = total(e->ev_refine);
    if (refine_launches) *refine_launches = (long long)(e->ev_refine.size() / 2);
    if (accum_ms) *accum_ms = total(e->ev_accum);
    if (accum_launches) *accum_launches = (long long)(e->ev_accum.size() / 2);
    prof_clear(e);
    return MPK_OK;
}

/* Test hook: the operand scale, eta, fixed-point bits and bound constants. */
mpkStatus mpkDebugEngineInfo(mpkEngine e, float* scale, float* eta, int* frac, float* c1, float* c2) {
    if (!e) return MPK_ERR_INVALID;
    DevParams h;
    MPK_TRY(cudaMemcpyAsync(&h, e->prm, sizeof(DevParams), cudaMemcpyDeviceToHost, e->s));
    MPK_TRY(cudaStreamSynchronize(e->s));
    if (scale) *scale = h.scale;
    if (eta) *eta = h.eta;
    if (frac) *frac = h.frac;
    if (c1) *c1 = e->bc.c1;
    if (c2) *c2 = e->bc.c2;
    return MPK_OK;
}

long long mpkDebugEngineLaunches(mpkEngine e) { return e ? e->launches : -1; }

mpkStatus mpkDebugSetWaitLimit(mpkEngine e, unsigned long long ns) {
    if (!e) return MPK_ERR_INVALID;
    MPK_TRY(cudaMemcpyAsync(&e->prm->wait_ns, &ns, sizeof(ns), cudaMemcpyHostToDevice, e->s));
    MPK_TRY(cudaStreamSynchronize(e->s));
    return MPK_OK;
}

mpkStatus mpkDebugInjectStall(mpkEngine e, int stage) {
    if (!e) return MPK_ERR_INVALID;
    e->stall = stage < 0 ? -1 : stage;
    return MPK_OK;
}

mpkStatus mpkDebugAssignPair(mpkEngine e, int mode) {
    if (!e) return MPK_ERR_INVALID;
    e->pair = mode != 0;
    graphs_release(e);                    /* captured iterations name the old kernel */
    return MPK_OK;
}

mpkStatus mpkDebugOverlapRefine(mpkEngine e, int mode) {
    if (!e) return MPK_ERR_INVALID;
    e->overlap = mode != 0;
    graphs_release(e);                    /* captured iterations hold the old order */
    return MPK_OK;
}

mpkStatus mpkDebugClearStatus(mpkEngine e) {
    if (!e) return MPK_ERR_INVALID;
    MPK_TRY(cudaMemsetAsync(&e->prm->status, 0, sizeof(int), e->s));
    MPK_TRY(cudaStreamSynchronize(e->s));
    return MPK_OK;
}

mpkStatus mpkDebugFailAlloc(int nth) {
    g_fail_alloc.store(nth > 0 ? nth : 0);
    return MPK_OK;
}

mpkStatus mpkDebugWideRoundRows(mpkEngine e, long long rows) {
    if (!e || rows < 1 || e->wide.cap == 0) return MPK_ERR_INVALID;
    e->wide.per_round = std::min(rows, e->wide.cap);
    e->wide.rounds = e->k >= 4096 ? (int)((e->n + e->wide.per_round - 1) / e->wide.per_round) : 1;
    graphs_release(e);                    /* captured iterations hold the old rounds */
    return MPK_OK;
}

mpkStatus mpkDebugWideCounters(mpkEngine e, long long* wide_rows, long long* full_scans, long long* capacity) {
    if (!e) return MPK_ERR_INVALID;
    DevParams h;
    MPK_TRY(cudaMemcpyAsync(&h, e->prm, sizeof(DevParams), cudaMemcpyDeviceToHost, e->s));
    MPK_TRY(cudaStreamSynchronize(e->s));
    if (wide_rows) *wide_rows = (long long)h.nwide_total;
    if (full_scans) *full_scans = (long long)h.novf_total;
    if (capacity) *capacity = e->wide.cap;
    return MPK_OK;
}

/* ------------------------------------------------------------ params ---- */

void mpkParamsInit(mpkParams* p) {
    if (!p) return;
    std::memset(p, 0, sizeof(*p));
    p->max_iter = 100;
    p->tol = 0.f;
    p->use_cond3 = 1;
    p->use_cond6 = 1;
    p->accum = MPK_ACCUM_FP32;
    p->mw_macs = 3;
}

double mpkEpsilon(int d, int accum) {
    const double u = (accum == MPK_ACCUM_FP16) ? U16 : U24;
    const double g = (double)d * u;
    if (g >= 1.0) return -1.0;
    return 2.0 * U16 + g / (1.0 - g);
}

double mpkMultiwordEpsilon(int d, int macs) {
    if (macs < 1 || macs > 3) return -1.0;
    const int m = d + (macs == 1 ? 0 : (macs == 2 ? 1 : 3));
    const double g = (double)m * U24;
    if (g >= 1.0) return -1.0;
    const double gamma = g / (1.0 - g);
    const double dropped = macs == 1 ? 2.0 * U16 + U16 * U16 : (macs == 2 ? U16 + U16 * U16 : 3.0 * U16 * U16);
    const double eps = (1.0 + dropped) * (1.0 + gamma) - 1.0;
    return eps >= 1.0 ? -1.0 : eps;
}

/* ------------------------------------------------------- preprocessing -- */

mpkStatus mpkShiftNonNegative(float* dP, int n, int d, float* out_shift) {
    if (!dP || n <= 0 || d <= 0) return MPK_ERR_INVALID;
    float* dmax = nullptr;
    if (cudaMalloc(&dmax, sizeof(float)) != cudaSuccess) return MPK_ERR_ALLOC;
    cudaMemset(dmax, 0, sizeof(float));
    launch_maxabs(dP, (long long)n * d, dmax, nullptr);
    float M = 0.f;
    cudaError_t e = cudaMemcpy(&M, dmax, sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(dmax);
    if (e != cudaSuccess) return MPK_ERR_CUDA;
    launch_add_const(dP, (long long)n * d, M, nullptr);
    MPK_TRY(cudaGetLastError());
    if (out_shift) *out_shift = M;
    return MPK_OK;
}

mpkStatus mpkStandardize(float* dP, int n, int d) {
    if (!dP || n <= 0 || d <= 0) return MPK_ERR_INVALID;
    launch_standardize(dP, n, d, nullptr);
    MPK_TRY(cudaGetLastError());
    return MPK_OK;
}

mpkStatus mpkShiftCentroids(float* dC, int k, int d, float delta) {
    if (!dC || k <= 0 || d <= 0) return MPK_ERR_INVALID;
    launch_add_const(dC, (long long)k * d, delta, nullptr);
    MPK_TRY(cudaGetLastError());
    return MPK_OK;
}

/* ------------------------------------------------------------ drivers --- */



static mpkStatus lloyd(cublasHandle_t blas, const float* dP, int n, int d, int k, float* dC, int* dAssign,
                       const mpkParams* params, mpkStats* stats, bool force_refine, bool exclusion_stats,
                       const char* tag) {
    if (n <= 0 || d <= 0 || k <= 0 || k > n || !dP || !dC || !dAssign) return MPK_ERR_INVALID;
    mpkParams P;
    if (params) P = *params; else mpkParamsInit(&P);
    mpkStats local;
    mpkStats* S = stats ? stats : &local;
    std::memset(S, 0, sizeof(*S));
    const int refine = (force_refine || P.use_cond3 || P.use_cond6) ? 1 : 0;
    cudaStream_t s = stream_of(blas);

    cudaEvent_t ev_all0, ev_all1, ev_x;
    cudaEventCreate(&ev_all0);
    cudaEventCreate(&ev_all1);
    cudaEventCreate(&ev_x);
    cudaEventRecord(ev_all0, s);

    mpkEngine e = nullptr;
    mpkStatus st = engine_create(&e, dP, n, d, k, dC, 0.f, n, s, true);
    if (st != MPK_OK) {
        cudaEventDestroy(ev_all0); cudaEventDestroy(ev_all1); cudaEventDestroy(ev_x);
        return st;
    }
    cudaEventRecord(ev_x, s);
    long long* sums = nullptr;
    float* moved2 = nullptr;
    std::vector<float> h_moved((size_t)k);
    const int iters_cap = P.max_iter > 0 ? P.max_iter : 0;
    std::vector<cudaEvent_t> ev((size_t)iters_cap * 4, nullptr);
    int it = 0;
    cudaStream_t gs = nullptr;
    cudaEvent_t ev_join = nullptr;
    cudaGraphExec_t g_assign = nullptr, g_update = nullptr;
    bool try_graphs = true;
    /* params.verify: every iteration's labels checked against the FP32 argmin over all k */
    const bool verify = P.verify != 0;
    unsigned long long* vbuf = nullptr;   /* [0] rows that differ, [1] excess (a double) */
    /* params.verbose: the previous labels and a changed-label counter, for the
     * per-iteration line the reference prints (mpkmeans.cu:598-603) */
    int* prev_lab = nullptr;
    unsigned long long* dchanged = nullptr;
    /* Without the per-iteration label checks (verify, verbose), the refinement
     * runs beside the update's segmented sum (engine_refine_update): the
     * "assignment" below is then the tensor-core pass alone, and the update
     * holds the refinement. */
    const bool ov = refine && e->overlap && !verify && !P.verbose;
    auto assign_step = [&] { return ov ? engine_assign_tc(e, dC, dAssign, refine)
                                       : engine_assign(e, dC, dAssign, refine, true); };
    auto update_step = [&] {
        if (ov) return engine_refine_update(e, dC, dAssign, sums, true, true, moved2);
        const mpkStatus a = engine_accumulate(e, dAssign, sums);
        return a != MPK_OK ? a : engine_finalize(e, sums, dC, moved2);
    };
    if (dev_alloc((void**)&sums, ((size_t)k * d + k) * sizeof(long long), s) != cudaSuccess ||
        dev_alloc((void**)&moved2, (size_t)k * sizeof(float), s) != cudaSuccess ||
        (verify && dev_alloc((void**)&vbuf, 2 * sizeof(unsigned long long), s) != cudaSuccess) ||
        (P.verbose && (dev_alloc((void**)&prev_lab, (size_t)n * sizeof(int), s) != cudaSuccess ||
                       dev_alloc((void**)&dchanged, sizeof(unsigned long long), s) != cudaSuccess))) {
        st = MPK_ERR_ALLOC;
        goto done;
    }
    if (verify) cudaMemsetAsync(vbuf, 0, 2 * sizeof(unsigned long long), s);
    if (P.verbose) cudaMemsetAsync(prev_lab, 0xff, (size_t)n * sizeof(int), s);
    for (auto& x : ev) cudaEventCreate(&x);

    /* The iterations run on a private stream gs, ordered after the caller's
     * stream and before it again at the end.  Iteration 0 launches its
     * kernels directly; from iteration 1 on, the assignment and the update
     * are two CUDA graphs captured once and replayed, so that a small problem
     * is not held to the host's kernel-launch rate.  (If a capture fails the
     * iterations keep launching directly.) */
    if (cudaStreamCreateWithFlags(&gs, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_join, cudaEventDisableTiming) != cudaSuccess) {
        st = MPK_ERR_CUDA;
        goto done;
    }
    cudaEventRecord(ev_join, s);
    cudaStreamWaitEvent(gs, ev_join, 0);
    e->s = gs;
    for (it = 0; it < iters_cap; ++it) {
        cudaEventRecord(ev[4 * it + 0], gs);
        if (it == 1 && try_graphs)
            try_graphs = capture_graph(gs, assign_step, &g_assign) && capture_graph(gs, update_step, &g_update);
        const bool replay = it >= 1 && try_graphs;
        if (replay) {
            if (cudaGraphLaunch(g_assign, gs) != cudaSuccess) { st = MPK_ERR_CUDA; goto done; }
        } else if ((st = assign_step()) != MPK_OK) {
            goto done;
        }
        cudaEventRecord(ev[4 * it + 1], gs);
        if (P.verbose) {                  /* labels that changed since the last iteration */
            cudaMemsetAsync(dchanged, 0, sizeof(unsigned long long), gs);
            launch_count_diff(dAssign, prev_lab, n, dchanged, gs);
            cudaMemcpyAsync(prev_lab, dAssign, (size_t)n * sizeof(int), cudaMemcpyDeviceToDevice, gs);
        }
        if (verify) {                     /* untimed: between the assignment and the update */
            launch_verify(e->P, dC, e->cn, d, k, dAssign, n, vbuf, reinterpret_cast<double*>(vbuf + 1),
                          e->num_sms, gs);
            cudaEventRecord(ev[4 * it + 3], gs);
        }
        if (replay) {
            if (cudaGraphLaunch(g_update, gs) != cudaSuccess) { st = MPK_ERR_CUDA; goto done; }
        } else if ((st = update_step()) != MPK_OK) {
            goto done;
        }
        cudaEventRecord(ev[4 * it + 2], gs);
        S->hp_baseline += (long long)n * k;
        if (exclusion_stats) S->tested += (long long)n * (k - 1);
        if (P.tol > 0.f || P.verbose) {
            unsigned long long hv[2] = {0, 0};   /* changed labels, rows refined this iteration */
            cudaMemcpyAsync(h_moved.data(), moved2, (size_t)k * sizeof(float), cudaMemcpyDeviceToHost, gs);
            if (P.verbose) {
                cudaMemcpyAsync(&hv[0], dchanged, sizeof(unsigned long long), cudaMemcpyDeviceToHost, gs);
                if (refine && it < MPK_MAX_HIST)
                    cudaMemcpyAsync(&hv[1], e->hist + it, sizeof(unsigned long long), cudaMemcpyDeviceToHost, gs);
            }
            if (cudaStreamSynchronize(gs) != cudaSuccess) { st = MPK_ERR_CUDA; goto done; }
            double fro2 = 0.0;
            for (int j = 0; j < k; ++j) fro2 += (double)h_moved[j];
            if (P.verbose)
                fprintf(stderr, "[%s] iter %3d  changed %8llu  refined %9llu / %lld  ||dC||_F^2 %.6e\n", tag, it,
                        hv[0], hv[1], (long long)n, fro2);
            if (P.tol > 0.f && fro2 < (double)P.tol * (double)P.tol) { ++it; break; }
        }
    }
    S->iters = it;
    cudaEventRecord(ev_join, gs);
    cudaStreamWaitEvent(s, ev_join, 0);
    e->s = s;
    cudaEventRecord(ev_all1, s);
    if (cudaStreamSynchronize(s) != cudaSuccess) { st = MPK_ERR_CUDA; goto done; }
    {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, ev_all0, ev_all1);
        S->t_total_ms = ms;
        double prep_x = 0.0;
        cudaEventElapsedTime(&ms, ev_all0, ev_x);
        prep_x = ms;
        for (int t = 0; t < it; ++t) {
            cudaEventElapsedTime(&ms, ev[4 * t + 0], ev[4 * t + 1]);
            S->t_gemm_lo_ms += ms;
            cudaEventElapsedTime(&ms, ev[4 * t + (verify ? 3 : 1)], ev[4 * t + 2]);
            S->t_update_ms += ms;
        }
        S->t_prep_ms = prep_x;
        S->t_dist_ms = prep_x + S->t_gemm_lo_ms;
        long long rows = 0, cands = 0, full = 0;
        int status = 0;
        mpkEngineCounters(e, &rows, &cands, &full, &status);
        S->hp_update = cands;
        if (exclusion_stats && refine) fill_exclusions(S, P, rows, cands);
        S->n_hist = it < MPK_MAX_HIST ? it : MPK_MAX_HIST;
        cudaMemcpy(S->hist_survivors, e->hist, sizeof(long long) * S->n_hist, cudaMemcpyDeviceToHost);
        if (verify) {
            unsigned long long hv[2] = {0, 0};
            cudaMemcpy(hv, vbuf, sizeof(hv), cudaMemcpyDeviceToHost);
            /* with the refinement on, a label off the FP32 argmin is a violation of the
             * certified bound; without it (no exclusion test, as in the reference's
             * raw scheme) nothing was excluded and the differences are near-tie misses */
            S->verify_excluded_best = refine ? (long long)hv[0] : 0;
            S->verify_label_diff = (long long)hv[0];
            std::memcpy(&S->verify_excess, &hv[1], sizeof(double));
            S->stats_built = 1;
        }
        if (status) {
            fprintf(stderr, "mpkmeans_b200: device status 0x%x (1 timeout, 2 scale, 4 label, 8 list)\n", status);
            st = MPK_ERR_CUDA;
            goto done;
        }
        if (mpkEngineInertia(e, dC, dAssign, &S->inertia) != MPK_OK) st = MPK_ERR_CUDA;
    }
done:
    if (gs) {
        cudaStreamSynchronize(gs);
        if (e) e->s = s;
    }
    cudaStreamSynchronize(s);
    if (g_assign) cudaGraphExecDestroy(g_assign);
    if (g_update) cudaGraphExecDestroy(g_update);
    if (ev_join) cudaEventDestroy(ev_join);
    if (gs) cudaStreamDestroy(gs);
    for (auto& x : ev) if (x) cudaEventDestroy(x);
    cudaEventDestroy(ev_all0);
    cudaEventDestroy(ev_all1);
    cudaEventDestroy(ev_x);
    dev_free(sums, s);
    dev_free(moved2, s);
    dev_free(vbuf, s);
    dev_free(prev_lab, s);
    dev_free(dchanged, s);
    engine_free(e);
    cudaStreamSynchronize(s);
    return st;
}

mpkStatus mpkMeansMixed(cublasHandle_t blas, const float* dP, int n, int d, int k, float* dC, int* dAssign,
                        const mpkParams* params, mpkStats* stats) {
    return lloyd(blas, dP, n, d, k, dC, dAssign, params, stats, false, true, "mixed");
}

mpkStatus mpkMeansFP32(cublasHandle_t blas, const float* dP, int n, int d, int k, float* dC, int* dAssign,
                       const mpkParams* params, mpkStats* stats) {
    return lloyd(blas, dP, n, d, k, dC, dAssign, params, stats, true, false, "fp32");
}

/* The reference's double-fp16 driver (kmeans/src/multiword.cu:245-645) refuses
 * to run with both exclusion conditions off (multiword.cu:256-259); so does
 * this one.  Otherwise it is the engine: its FP16 hi/lo split is the
 * double-fp16 scheme, every row's label is the exact FP32 argmin, and the
 * three cross products are counted in mw_products. */
mpkStatus mpkMeansMultiword(cublasHandle_t blas, const float* dP, int n, int d, int k, float* dC, int* dAssign,
                            const mpkParams* params, mpkStats* stats) {
    mpkStats local;
    mpkStats* S = stats ? stats : &local;
    if (params && !params->use_cond3 && !params->use_cond6) {
        fprintf(stderr, "mpkMeansMultiword: at least one condition must be on\n");
        return MPK_ERR_INVALID;
    }
    mpkStatus st = lloyd(blas, dP, n, d, k, dC, dAssign, params, S, true, true, "mw");
    if (st == MPK_OK) {
        S->mw_products = 3LL * S->iters;
        S->mw_refine_rows = 0;
    }
    return st;
}

mpkStatus mpkMeansBaselineRT(cublasHandle_t, const float*, int, int, int, float*, int*, const mpkParams*,
                             mpkStats*) {
    fprintf(stderr, "mpkmeans_b200: the arXiv:2407.12208 reliability-test baseline is not part of this engine\n");
    return MPK_ERR_INVALID;
}

int mpkHaveCuvs(void) { return 0; }

mpkStatus mpkMeansCuvs(cublasHandle_t, const float*, int, int, int, float*, int*, const mpkParams*, mpkStats*) {
    return MPK_ERR_INVALID;
}

mpkStatus mpkAssign(cublasHandle_t blas, const float* dP, int n, int d, int k, const float* dC, int* dAssign,
                    const mpkParams* params, mpkStats* stats) {
    if (n <= 0 || d <= 0 || k <= 0 || !dP || !dC || !dAssign) return MPK_ERR_INVALID;
    mpkParams P;
    if (params) P = *params; else mpkParamsInit(&P);
    const int refine = (P.use_cond3 || P.use_cond6) ? 1 : 0;
    cudaStream_t s = stream_of(blas);
    mpkEngine e = nullptr;
    mpkStatus st = engine_create(&e, dP, n, d, k, dC, 0.f, n, s, true);
    if (st != MPK_OK) return st;
    st = engine_assign(e, dC, dAssign, refine, false);
    if (st == MPK_OK && stats) {
        std::memset(stats, 0, sizeof(*stats));
        long long rows = 0, cands = 0, full = 0;
        int status = 0;
        mpkEngineCounters(e, &rows, &cands, &full, &status);
        stats->iters = 1;
        stats->hp_baseline = (long long)n * k;
        stats->tested = (long long)n * (k - 1);
        stats->hp_update = cands;
        if (refine) fill_exclusions(stats, P, rows, cands);
        stats->n_hist = 1;
        stats->hist_survivors[0] = rows;
        if (status) st = MPK_ERR_CUDA;
    }
    cudaStreamSynchronize(s);
    engine_free(e);
    return st;
}

mpkStatus mpkUpdate(cublasHandle_t blas, const float* dP, int n, int d, int k, const int* dAssign, float* dC,
                    float* dMoved2) {
    if (n <= 0 || d <= 0 || k <= 0 || !dP || !dC || !dAssign) return MPK_ERR_INVALID;
    cudaStream_t s = stream_of(blas);
    mpkEngine e = nullptr;
    mpkStatus st = engine_create(&e, dP, n, d, k, nullptr, 0.f, n, s, false);
    if (st != MPK_OK) return st;
    long long* sums = nullptr;
    if (dev_alloc((void**)&sums, ((size_t)k * d + k) * sizeof(long long), s) != cudaSuccess) {
        engine_free(e);
        return MPK_ERR_ALLOC;
    }
    st = engine_accumulate(e, dAssign, sums);
    if (st == MPK_OK) st = engine_finalize(e, sums, dC, dMoved2);
    int status = 0;
    if (st == MPK_OK && mpkEngineCounters(e, nullptr, nullptr, nullptr, &status) == MPK_OK && status) {
        fprintf(stderr, "mpkmeans_b200: mpkUpdate: device status 0x%x\n", status);
        st = MPK_ERR_INVALID;
    }
    dev_free(sums, s);
    engine_free(e);
    cudaStreamSynchronize(s);
    return st;
}

/* ----------------------------------------------------------- data ------ */

void mpkMakeBlobs(int n, int d, int k, float stdv, float center_box, unsigned seed, float* hP, int* hLabels) {
    /* Same engine, distributions and draw order as the reference's generator
     * (kmeans/src/data.cu:12-28), so a seed reproduces its points exactly. */
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> box(-center_box, center_box);
    std::normal_distribution<float> noise(0.f, stdv);
    std::vector<float> centre((size_t)k * d);
    for (auto& v : centre) v = box(rng);
    for (int i = 0; i < n; ++i) {
        const int c = (int)((long long)i * k / n);
        if (hLabels) hLabels[i] = c;
        if (!hP) continue;
        float* row = hP + (size_t)i * d;
        const float* cc = centre.data() + (size_t)c * d;
        for (int t = 0; t < d; ++t) row[t] = cc[t] + noise(rng);
    }
}

mpkStatus mpkInitRandomPoints(const float* dP, int n, int d, int k, unsigned seed, float* dC) {
    /* k distinct rows, chosen by the reference's partial Fisher-Yates under
     * mt19937(seed ^ 0x9e3779b9) and taken in ascending row order
     * (kmeans/src/data.cu:30-51), then gathered with one copy per row. */
    if (!dP || !dC || k <= 0 || d <= 0 || k > n) return MPK_ERR_INVALID;
    std::mt19937 rng(seed ^ 0x9e3779b9u);
    std::vector<int> perm(n);
    for (int i = 0; i < n; ++i) perm[i] = i;
    for (int i = 0; i < k; ++i) {
        std::uniform_int_distribution<int> pick(i, n - 1);
        std::swap(perm[i], perm[pick(rng)]);
    }
    std::sort(perm.begin(), perm.begin() + k);
    for (int j = 0; j < k; ++j)
        MPK_TRY(cudaMemcpy(dC + (size_t)j * d, dP + (size_t)perm[j] * d, (size_t)d * sizeof(float),
                           cudaMemcpyDeviceToDevice));
    return MPK_OK;
}

mpkStatus mpkLoadBin(const char* path, int d, long long max_rows, int* out_n, float** out_P) {
    if (!path || d <= 0 || !out_n || !out_P) return MPK_ERR_INVALID;
    FILE* f = fopen(path, "rb");
    if (!f) { fprintf(stderr, "mpkLoadBin: cannot open %s\n", path); return MPK_ERR_INVALID; }
    if (fseeko(f, 0, SEEK_END) != 0) { fclose(f); return MPK_ERR_INVALID; }
    const long long bytes = (long long)ftello(f);
    rewind(f);
    const long long row = (long long)d * (long long)sizeof(float);
    if (bytes <= 0 || bytes % row != 0) {
        fprintf(stderr, "mpkLoadBin: %s holds %lld bytes, not a whole number of %d-float rows\n", path, bytes, d);
        fclose(f);
        return MPK_ERR_INVALID;
    }
    long long rows = bytes / row;
    if (max_rows > 0 && max_rows < rows) rows = max_rows;
    if (rows > INT_MAX) { fclose(f); return MPK_ERR_INVALID; }
    float* P = (float*)malloc((size_t)rows * d * sizeof(float));
    if (!P) { fclose(f); return MPK_ERR_ALLOC; }
    const size_t want = (size_t)rows * d;
    const size_t got = fread(P, sizeof(float), want, f);
    fclose(f);
    if (got != want) { free(P); return MPK_ERR_INVALID; }
    *out_n = (int)rows;
    *out_P = P;
    return MPK_OK;
}

/* LIBSVM text: "<label> <index>:<value> ..." with 1-based indices, '#'
 * comments and "qid:" tokens skipped.  Two passes: shape, then fill.  Labels
 * are renumbered 0.. in order of first appearance. */
mpkStatus mpkLoadLibsvm(const char* path, int* out_n, int* out_d, float** out_P, int** out_labels,
                        int* out_nclasses) {
    if (!path || !out_n || !out_d || !out_P) return MPK_ERR_INVALID;
    auto scan = [&](bool fill, long long* rows, long long* maxidx, float* P, int* L, std::vector<double>* cls,
                    int d) -> bool {
        FILE* f = fopen(path, "r");
        if (!f) return false;
        char* line = nullptr;
        size_t cap = 0;
        long long r = 0;
        while (getline(&line, &cap, f) != -1) {
            if (char* h = strchr(line, '#')) *h = '\0';
            char* p = line;
            while (*p == ' ' || *p == '\t' || *p == '\r' || *p == '\n') ++p;
            if (!*p) continue;
            char* end = nullptr;
            const double lab = strtod(p, &end);
            p = end ? end : p;
            while (*p && *p != ' ' && *p != '\t') ++p;
            if (fill) {
                size_t c = 0;
                while (c < cls->size() && (*cls)[c] != lab) ++c;
                if (c == cls->size()) cls->push_back(lab);
                L[r] = (int)c;
            }
            while (*p) {
                while (*p == ' ' || *p == '\t' || *p == '\r' || *p == '\n') ++p;
                if (!*p) break;
                char* colon = nullptr;
                const long idx = strtol(p, &colon, 10);
                if (colon == p || *colon != ':') {
                    while (*p && *p != ' ' && *p != '\t') ++p;
                    continue;
                }
                char* vend = nullptr;
                const double v = strtod(colon + 1, &vend);
                if (!fill && idx > *maxidx) *maxidx = idx;
                if (fill && idx >= 1 && idx <= d) P[(size_t)r * d + (idx - 1)] = (float)v;
                p = (vend && vend > colon + 1) ? vend : colon + 1;
            }
            ++r;
        }
        free(line);
        fclose(f);
        if (rows) *rows = r;
        return true;
    };
    long long rows = 0, maxidx = 0;
    if (!scan(false, &rows, &maxidx, nullptr, nullptr, nullptr, 0)) {
        fprintf(stderr, "mpkLoadLibsvm: cannot open %s\n", path);
        return MPK_ERR_INVALID;
    }
    if (rows == 0 || maxidx == 0 || rows > INT_MAX || maxidx > INT_MAX ||
        (double)rows * (double)maxidx * sizeof(float) > 6e10)
        return MPK_ERR_INVALID;
    const int n = (int)rows, d = (int)maxidx;
    float* P = (float*)calloc((size_t)n * d, sizeof(float));
    int* L = (int*)calloc((size_t)n, sizeof(int));
    if (!P || !L) { free(P); free(L); return MPK_ERR_ALLOC; }
    std::vector<double> cls;
    if (!scan(true, nullptr, nullptr, P, L, &cls, d)) { free(P); free(L); return MPK_ERR_INVALID; }
    *out_n = n;
    *out_d = d;
    *out_P = P;
    if (out_labels) *out_labels = L; else free(L);
    if (out_nclasses) *out_nclasses = (int)cls.size();
    return MPK_OK;
}

}  /* extern "C" */
