/* noalloc.cu -- mpkUpdateNoAlloc: the centroid update without any allocation.
 *
 * Some callers cannot call cudaMalloc: code that runs while a memory pool or
 * a custom allocator owns the device, an embedding whose allocator may not be
 * re-entered from a library, or a process that must not grow its device
 * footprint after start-up.  For them this entry point runs the same update
 * as mpkUpdate (counting sort by label, exact int64 segmented sum, finalize)
 * with all of its scratch in one fixed array, g_update_scratch below, that is
 * part of the library image: every GPU that loads the library holds these
 * kNoAllocScratchBytes (32 MiB) until the process exits.
 *
 * With CUDA's lazy module loading (the default) the array is only placed on a
 * device when the library's code is first loaded there, which the first call
 * does: that call grows the device footprint by the 32 MiB, so a caller whose
 * footprint must stay fixed makes one call at start-up.
 *
 * Host code cannot use the array's name as a device address, so the first
 * call on each device resolves it with cudaGetSymbolAddress (with that device
 * current) and caches it together with the device's current context; a new
 * context on that device (after cudaDeviceReset, say) makes the next call
 * resolve it again.  That first call should come before any stream capture.
 * The array keeps the contents of the last call: everything that must start
 * from zero is cleared at the start of every call, and two calls that overlap
 * on the GPU (on different streams, or from several host threads) would race
 * on it.
 */
#include "engine.cuh"
#include "mpkmeans.h"

#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = 32u << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_update_scratch[kNoAllocScratchBytes];

std::mutex g_addr_mutex;
void* g_addr[kMaxDevices] = {};
CUcontext g_ctx[kMaxDevices] = {};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

/* The calling thread's current context (the driver's cuCtxGetCurrent, looked up
 * through the runtime so the library does not link the driver library). */
CUcontext current_context() {
    static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 4000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
    });
    CUcontext c = nullptr;
    if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
    return c;
}

/* Device address of g_update_scratch on the current device: resolved on the
 * first call in each of the device's contexts, cached after that. */
void* scratch_address(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return nullptr;
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lock(g_addr_mutex);
    if (!g_addr[dev] || !ctx || g_ctx[dev] != ctx) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_update_scratch);
        if (e != cudaSuccess) {
            fprintf(stderr, "mpkUpdateNoAlloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                    cudaGetErrorString(e));
            g_addr[dev] = nullptr;
            return nullptr;
        }
        g_addr[dev] = p;
        g_ctx[dev] = ctx;
    }
    return g_addr[dev];
}

/* Scratch bytes one call needs: parameters, k*d + k int64 sums and counts,
 * three k+1 int arrays (histogram, bin starts, cursors), n row indices. */
size_t scratch_bytes(int n, int d, int k) {
    return align256(sizeof(mpk::DevParams)) + align256(sizeof(long long) * ((size_t)k * d + k)) +
           3 * align256(sizeof(int) * ((size_t)k + 1)) + align256(sizeof(int) * (size_t)n);
}

}  /* namespace */

extern "C" mpkStatus mpkUpdateNoAlloc(cudaStream_t stream, const float* dP, int n, int d, int k, const int* dAssign,
                                      float* dC, float* dMoved2) {
    if (n <= 0 || d <= 0 || k <= 0 || !dP || !dC || !dAssign) return MPK_ERR_INVALID;
    const size_t need = scratch_bytes(n, d, k);
    if (need > kNoAllocScratchBytes) {
        fprintf(stderr,
                "mpkUpdateNoAlloc: n=%d, d=%d, k=%d needs %zu bytes of scratch; the fixed array holds %zu "
                "(use mpkUpdate)\n",
                n, d, k, need, kNoAllocScratchBytes);
        return MPK_ERR_INVALID;
    }
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MPK_ERR_CUDA;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    unsigned char* base = static_cast<unsigned char*>(scratch_address(dev));
    if (!base) return MPK_ERR_CUDA;

    /* carve the fixed array: params | sums (k*d) + counts (k) | hist | bin starts | cursor | perm */
    size_t off = 0;
    auto take = [&](size_t bytes) {
        unsigned char* p = base + off;
        off += align256(bytes);
        return p;
    };
    mpk::DevParams* prm = reinterpret_cast<mpk::DevParams*>(take(sizeof(mpk::DevParams)));
    long long* sums = reinterpret_cast<long long*>(take(sizeof(long long) * ((size_t)k * d + k)));
    mpk::UpdateScratch us;
    us.hist = reinterpret_cast<int*>(take(sizeof(int) * ((size_t)k + 1)));
    us.bin_start = reinterpret_cast<int*>(take(sizeof(int) * ((size_t)k + 1)));
    us.cursor = reinterpret_cast<int*>(take(sizeof(int) * ((size_t)k + 1)));
    us.perm = reinterpret_cast<int*>(take(sizeof(int) * (size_t)n));

    /* the previous call's values are still there: clear what must start at zero */
    if (cudaMemsetAsync(prm, 0, sizeof(mpk::DevParams), stream) != cudaSuccess ||
        cudaMemsetAsync(sums, 0, sizeof(long long) * ((size_t)k * d + k), stream) != cudaSuccess)
        return MPK_ERR_CUDA;
    mpk::launch_maxabs(dP, (long long)n * d, &prm->pmax, stream);
    mpk::launch_set_scale(prm, n, stream);
    mpk::launch_update_sorted(dP, n, d, dAssign, k, prm, sums, sums + (size_t)k * d, us, sms, stream);
    mpk::launch_finalize_fixed(sums, sums + (size_t)k * d, k, d, prm, dC, dMoved2, stream);
    if (cudaGetLastError() != cudaSuccess) return MPK_ERR_CUDA;
    int status = 0;
    if (cudaMemcpyAsync(&status, &prm->status, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
        return MPK_ERR_CUDA;
    if (status) {
        fprintf(stderr, "mpkUpdateNoAlloc: a label outside [0, %d) was given\n", k);
        return MPK_ERR_INVALID;
    }
    return MPK_OK;
}
