/* init.cu -- k-means++ seeding on the GPU (mpkInitKMeansPP).
 *
 * The reference has no k-means++ (its seeding is mpkInitRandomPoints,
 * kmeans/src/data.cu:30-51); configuration 1 asks for k-means++ from a seed.
 * This is the definition, chosen so that a parallel implementation and a
 * sequential one agree bit for bit:
 *   - squared distances in FP64, warp order: lane l sums (p_t - c_t)^2 over
 *     t = l, l+32, ... (separate multiply and add), a shfl_down tree folds
 *     the lanes; D2_i = min over the chosen centres;
 *   - weights w_i = floor(D2_i * 2^q), q = 62 - L - e with n < 2^L and
 *     max D2 < 2^e, so W = sum w_i < 2^62 is exact in any order;
 *   - step c draws u = h3(seed, 41, c) >> 11 (53 bits, splitmix64-based
 *     counter hash) and picks the first row whose inclusive prefix of w
 *     exceeds floor(u * W / 2^53); the first centre, and any step with W = 0,
 *     takes row floor(u * n / 2^53).
 * Per centre: one pass over P (the D2 update with a block max), one pass over
 * D2 (block sums of w), and a single-block pick that scans the block sums and
 * then the 4096 rows of the chosen block.
 */
#include "engine.cuh"
#include "mpkmeans.h"

#include <cstdio>

namespace mpk {
namespace {

constexpr int kRowsPerBlock = 4096;   /* partition of the weight sums */
constexpr int kPickThreads = 1024;
static_assert(kRowsPerBlock % kPickThreads == 0, "rows per pick thread");
constexpr unsigned FULL = 0xffffffffu;

__host__ __device__ inline uint64_t sm64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
__host__ __device__ inline uint64_t h3(uint64_t seed, uint64_t stream, uint64_t ctr) {
    return sm64(sm64(seed ^ sm64(stream + 0x632BE59BD9B4E019ull)) ^ ctr);
}
/* floor(u * x / 2^53) for u < 2^53, x < 2^63 */
__host__ __device__ inline uint64_t mul_shift53(uint64_t u, uint64_t x) {
#ifdef __CUDA_ARCH__
    const uint64_t lo = u * x, hi = __umul64hi(u, x);
#else
    const unsigned __int128 p = (unsigned __int128)u * x;
    const uint64_t lo = (uint64_t)p, hi = (uint64_t)(p >> 64);
#endif
    return (hi << 11) | (lo >> 53);
}

__device__ inline int weight_shift(double M, int L) {
    int e = 0;
    frexp(M, &e);
    return 62 - L - e;
}

__global__ void k_fill_inf(double* d2, long long n) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) d2[i] = INFINITY;
}

/* One warp per row: D2_i = min(D2_i, |p_i - c|^2) in warp order; the max of
 * the updated D2 goes to *maxbits (non-negative doubles order as integers). */
__global__ void k_kpp_update(const float* __restrict__ P, long long n, int d, const float* __restrict__ c,
                             double* __restrict__ d2, unsigned long long* maxbits) {
    const int lane = threadIdx.x & 31;
    const long long wstride = (long long)gridDim.x * (blockDim.x >> 5);
    double m = 0.0;
    for (long long i = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += wstride) {
        const float* p = P + (size_t)i * d;
        double a = 0.0;
        for (int t = lane; t < d; t += 32) {
            const double v = (double)p[t] - (double)c[t];
            const double sq = v * v;
            a = a + sq;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) a = a + __shfl_down_sync(FULL, a, off);
        if (lane == 0) {
            double cur = d2[i];
            if (a < cur) {
                cur = a;
                d2[i] = a;
            }
            m = fmax(m, cur);
        }
    }
    if (lane == 0 && m > 0.0) atomicMax(maxbits, (unsigned long long)__double_as_longlong(m));
}

__device__ inline unsigned long long block_sum_u64(unsigned long long v, unsigned long long* sh) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[w] = v;
    __syncthreads();
    unsigned long long t = 0;
    for (int i = 0; i < nw; ++i) t += sh[i];
    return t;
}

/* bsum[b] = sum of w_i over rows [b * kRowsPerBlock, ...). */
__global__ void k_kpp_weights(const double* __restrict__ d2, long long n, const unsigned long long* maxbits, int L,
                              unsigned long long* __restrict__ bsum) {
    __shared__ unsigned long long sh[32];
    const double M = __longlong_as_double((long long)*maxbits);
    const long long r0 = (long long)blockIdx.x * kRowsPerBlock;
    const long long r1 = min(n, r0 + kRowsPerBlock);
    unsigned long long s = 0;
    if (M > 0.0) {
        const int q = weight_shift(M, L);
        for (long long i = r0 + threadIdx.x; i < r1; i += blockDim.x) s += (unsigned long long)ldexp(d2[i], q);
    }
    s = block_sum_u64(s, sh);
    if (threadIdx.x == 0) bsum[blockIdx.x] = s;
}

/* One block: the pick of step c, its row copied to C[c]; resets *maxbits. */
__global__ void __launch_bounds__(kPickThreads)
k_kpp_pick(const float* __restrict__ P, long long n, int d, const double* __restrict__ d2,
           unsigned long long* maxbits, int L, const unsigned long long* __restrict__ bsum, int nb, uint64_t seed,
           int c, float* __restrict__ C, long long* pick_out) {
    __shared__ unsigned long long sh[32];
    __shared__ unsigned long long s_before, s_scan[kPickThreads / 32];
    __shared__ int s_blk;
    __shared__ long long s_pick;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const double M = __longlong_as_double((long long)*maxbits);
    const uint64_t u = h3(seed, 41, (uint64_t)c) >> 11;
    long long pick;
    if (!(M > 0.0)) {
        pick = (long long)mul_shift53(u, (uint64_t)n);
    } else {
        unsigned long long part = 0;
        for (int b = tid; b < nb; b += blockDim.x) part += bsum[b];
        const unsigned long long W = block_sum_u64(part, sh);
        const unsigned long long target = mul_shift53(u, W);
        if (tid == 0) {
            unsigned long long run = 0;
            int blk = nb - 1;
            for (int b = 0; b < nb; ++b) {
                if (run + bsum[b] > target) { blk = b; break; }
                run += bsum[b];
            }
            s_blk = blk;
            s_before = run;
            s_pick = n - 1;
        }
        __syncthreads();
        /* rows of the chosen block: 4 consecutive rows per thread */
        constexpr int RPT = kRowsPerBlock / kPickThreads;
        const int q = weight_shift(M, L);
        const long long r0 = (long long)s_blk * kRowsPerBlock + (long long)tid * RPT;
        unsigned long long wv[RPT], loc = 0;
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
            wv[r] = (r0 + r < n) ? (unsigned long long)ldexp(d2[r0 + r], q) : 0ull;
            loc += wv[r];
        }
        /* exclusive prefix of loc over the block's threads */
        unsigned long long inc = loc;
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(FULL, inc, o);
            if (lane >= o) inc += y;
        }
        if (lane == 31) s_scan[w] = inc;
        __syncthreads();
        unsigned long long wbefore = 0;
        for (int i = 0; i < w; ++i) wbefore += s_scan[i];
        unsigned long long run = s_before + wbefore + inc - loc;
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
            run += wv[r];
            if (run > target && r0 + r < n) {
                atomicMin(reinterpret_cast<unsigned long long*>(&s_pick), (unsigned long long)(r0 + r));
                break;
            }
        }
        __syncthreads();
        pick = s_pick;
    }
    for (int t = tid; t < d; t += blockDim.x) C[(size_t)c * d + t] = P[(size_t)pick * d + t];
    __syncthreads();
    if (tid == 0) {
        *maxbits = 0ull;
        if (pick_out) pick_out[c] = pick;
    }
}

}  /* namespace */
}  /* namespace mpk */

using namespace mpk;

extern "C" mpkStatus mpkInitKMeansPP(const float* dP, int n, int d, int k, unsigned long long seed, float* dC) {
    if (!dP || !dC || n <= 0 || d <= 0 || k <= 0 || k > n) return MPK_ERR_INVALID;
    cudaStream_t s = nullptr;
    double* d2 = nullptr;
    unsigned long long *maxbits = nullptr, *bsum = nullptr;
    const int nb = (int)(((long long)n + kRowsPerBlock - 1) / kRowsPerBlock);
    int L = 0;
    while (L < 63 && ((unsigned long long)n >> L) != 0) ++L;
    mpkStatus rc = MPK_OK;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (dev_alloc((void**)&d2, sizeof(double) * (size_t)n, s) != cudaSuccess ||
        dev_alloc((void**)&maxbits, sizeof(unsigned long long), s) != cudaSuccess ||
        dev_alloc((void**)&bsum, sizeof(unsigned long long) * (size_t)nb, s) != cudaSuccess) {
        rc = MPK_ERR_ALLOC;
    } else {
        const long long pick0 = (long long)mul_shift53(h3(seed, 41, 0) >> 11, (uint64_t)n);
        const int ublocks = (int)std::min<long long>(((long long)n + 7) / 8, (long long)sms * 8);
        k_fill_inf<<<sms * 4, 256, 0, s>>>(d2, n);
        cudaMemsetAsync(maxbits, 0, sizeof(unsigned long long), s);
        cudaMemcpyAsync(dC, dP + (size_t)pick0 * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, s);
        for (int c = 1; c < k; ++c) {
            k_kpp_update<<<ublocks, 256, 0, s>>>(dP, n, d, dC + (size_t)(c - 1) * d, d2, maxbits);
            k_kpp_weights<<<nb, 256, 0, s>>>(d2, n, maxbits, L, bsum);
            k_kpp_pick<<<1, kPickThreads, 0, s>>>(dP, n, d, d2, maxbits, L, bsum, nb, seed, c, dC, nullptr);
        }
        if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess) rc = MPK_ERR_CUDA;
    }
    dev_free(d2, s);
    dev_free(maxbits, s);
    dev_free(bsum, s);
    cudaStreamSynchronize(s);
    return rc;
}
