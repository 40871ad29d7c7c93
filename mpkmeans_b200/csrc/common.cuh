/* common.cuh -- shared device helpers for the B200 (sm_100a) k-means engine.
 *
 * Inline PTX for the Blackwell pieces the kernels use: mbarriers with bounded
 * waits, TMA tile loads (each CTA loads its own tiles), tcgen05 TMEM
 * allocation, MMA issue/commit and TMEM loads.  Every wait is bounded by the
 * global timer: a wait that runs out records an error code in the engine's
 * device status word and makes the kernel wind down instead of spinning.
 */
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda.h>

namespace mpk {

/* ------------------------------------------------------------ status ---- */

/* Device status word bits (engine-owned int, read by the host after a run). */
enum : int {
    MPK_DEV_OK          = 0,
    MPK_DEV_TIMEOUT     = 1,   /* an mbarrier wait exceeded its time limit */
    MPK_DEV_SCALE       = 2,   /* an operand left the FP16 range chosen for it */
    MPK_DEV_LABEL_RANGE = 4,   /* a label outside [0, k) reached the update */
    MPK_DEV_LIST        = 8,   /* refinement list overflow */
};

/* Wall-clock bound on any single wait, in ns.  A legitimate wait here is a few
 * microseconds (one tile of MMAs or one TMA load). */
constexpr unsigned long long kWaitLimitNs = 4000000000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

/* ------------------------------------------------------------ mbarrier -- */

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

/* Wait for the phase of `parity` to complete.  Returns false (and raises the
 * timeout bit in *status and the shared abort flag) if the time limit passes
 * or another thread of the CTA has already aborted. */
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, uint32_t limit_us = (uint32_t)(kWaitLimitNs / 1000)) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer() - t0 > 1000ull * limit_us) {
            *abort_flag = 1;
            atomicOr(status, MPK_DEV_TIMEOUT);
            return false;
        }
    }
}

/* ----------------------------------------------------------------- TMA -- */

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

/* 3D tiled load, coordinates innermost first; completes on `bar` with
 * complete_tx into this CTA's shared memory only. */
__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* smem,
                                            int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        :: "r"(smem_u32(smem)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
           "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* smem,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        :: "r"(smem_u32(smem)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
           "r"(x), "r"(y)
        : "memory");
}

/* -------------------------------------------------------------- tcgen05 -- */

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

/* D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (FP16 or BF16 operands, FP32
 * accumulation).  Issued by one thread. */
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* Arrive on `bar` once every tcgen05 op this thread issued so far completes. */
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

/* 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread. */
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32"
        " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

/* 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread. */
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32"
        " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

/* 32 lanes x 32 consecutive 32-bit columns written from registers. */
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
        " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :: "r"(taddr),
           "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
           "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
           "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
           "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

/* ----------------------------------------------------- UMMA descriptors -- */

/* Shared-memory matrix descriptor (sm_100 format, version 1).
 *   bits  0-13  start address >> 4
 *   bits 16-29  leading-dimension byte offset >> 4
 *   bits 32-45  stride-dimension byte offset >> 4
 *   bits 46-47  version = 1
 *   bits 61-63  layout: 2 = 128-byte swizzle
 * For a K-major operand in 128-byte swizzle the 8-row core groups sit 1024 B
 * apart (SBO) and LBO is unused (1).  For an MN-major operand in 128-byte
 * swizzle, LBO is the distance between 64-element MN blocks and SBO the
 * distance between 8-deep K groups. */
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

/* Instruction descriptor, kind::f16: FP32 accumulator, A/B both FP16 (fmt 0)
 * or both BF16 (fmt 1), majors 0 = K, 1 = MN, M>>4 at bit 24, N>>3 at bit 17. */
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int ab_fmt, int a_mn_major, int b_mn_major) {
    return (1u << 4)                                  /* D format F32   */
         | ((uint32_t)ab_fmt << 7) | ((uint32_t)ab_fmt << 10)
         | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16)
         | ((uint32_t)(N >> 3) << 17)
         | ((uint32_t)(M >> 4) << 24);
}

/* ------------------------------------------------------- CTA pairs ---- */
/* A cluster of two CTAs on two SMs sharing one tcgen05.mma (cta_group::2): the
 * even CTA issues every MMA, each CTA supplies its half of the operand tiles
 * from its own shared memory and receives its half of the rows of D in its own
 * TMEM.  Every tcgen05 instruction of such a kernel uses cta_group::2. */

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

/* Address, in the cluster's shared-memory window, of the variable at the
 * same offset as `local` in the shared memory of CTA `rank`. */
__device__ __forceinline__ uint32_t peer_addr(const void* local, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
    return a;
}

/* Arrive on an mbarrier of any CTA of the cluster, with the instruction's
 * default semantics (release at CTA scope): after tcgen05.wait::ld and
 * tcgen05.fence::before_thread_sync this orders a warp's TMEM reads before the
 * MMAs that the barrier's waiter issues next; a cluster-scope release would
 * also wait for the warp's outstanding global stores. */
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

/* Every thread of both CTAs: arrive with release, wait with acquire. */
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

/* 3D tiled load into this CTA's shared memory whose completion is counted on
 * an mbarrier of either CTA of the pair (`bar` is a cluster address). */
__device__ __forceinline__ void tma_load_3d_pair(const CUtensorMap* map, uint32_t bar, void* smem,
                                                 int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        :: "r"(smem_u32(smem)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar),
           "r"(x), "r"(y), "r"(z)
        : "memory");
}

/* Issued by one warp in each CTA of the pair, at the same shared offset. */
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

/* The pair's D (+)= A * B^T: M = 256 rows, 128 from each CTA's A tile, and N
 * columns, the first N/2 from the even CTA's B tile, the rest from the odd
 * CTA's; descriptors name the same shared offsets in both CTAs. */
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* Arrive on the mbarrier at cluster address `bar` (either CTA) once every
 * pair MMA this thread issued so far completes. */
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}

/* --------------------------------------------------------------- misc ---- */

__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  /* namespace mpk */
