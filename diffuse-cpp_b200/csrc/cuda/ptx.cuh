// Thin inline-PTX wrappers for the sm_100a features the kernels use:
// mbarriers, TMA (bulk and tensor loads, never multicast), CTA pairs, tcgen05 MMA/TMEM.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

namespace dfb {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)::"memory");
    return t;
}

// ── mbarrier ──
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps in the instruction until the
// phase completes (it is woken then) or the hint elapses, instead of spinning and
// taking issue slots from busy warps on its scheduler.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait.  Returns false (and raises *abort and the global error code) when
// the phase has not completed within timeout_ns, or when another role of the CTA or
// another CTA of the launch already gave up.  No wait in this library can spin forever.
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;  // 4 s
#ifndef DFB_WAIT_HINT_NS
#define DFB_WAIT_HINT_NS 200000
#endif
constexpr uint32_t kSuspendHintNs = DFB_WAIT_HINT_NS;  // per try_wait, then re-check the flags
// The abort flag, the global error code and the time limit are checked every
// kWaitCheckNs only: a woken waiter whose phase is not complete yet goes straight back to
// sleep instead of loading them (they take issue slots and global loads from the busy
// warps of its scheduler); an abort then reaches the other waits within that period.
constexpr uint64_t kWaitCheckNs = 20000;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                          int *err, int code, uint64_t timeout_ns = kWaitTimeoutNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    uint64_t checked = t0;
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
        const uint64_t now = globaltimer();
        if (now - checked < kWaitCheckNs) continue;
        checked = now;
        if (*abort_flag) return false;
        if (*reinterpret_cast<volatile int *>(err)) {
            *abort_flag = 1;
            return false;
        }
        if (globaltimer() - t0 > timeout_ns) {
            *abort_flag = 1;
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

// Teardown wait: bounded by time only (used after an abort, when the abort flag is set).
__device__ __forceinline__ bool spin_bounded(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() - t0 > kWaitTimeoutNs) return false;
    return true;
}

// ── TMA ──
// 1-D bulk copy global -> shared (addresses 16 B aligned, size multiple of 16).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Generic-proxy accesses (global and shared) before later async-proxy (bulk copy) ones.
__device__ __forceinline__ int ld_acquire_gpu(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait until the global counter *c reaches target (acquire), with the abort
// rules of mbar_wait.  Every CTA of a launch is resident at once (one per SM), so the
// CTAs whose arrivals this waits for are running.
__device__ __forceinline__ bool wait_count(const int *c, int target, volatile int *abort_flag, int *err, int code,
                                           uint64_t timeout_ns = kWaitTimeoutNs) {
    const uint64_t t0 = globaltimer();
    uint64_t checked = t0;
    for (;;) {
        if (ld_acquire_gpu(c) >= target) return true;
        __nanosleep(32);
        const uint64_t now = globaltimer();
        if (now - checked < kWaitCheckNs) continue;  // flags and limit every kWaitCheckNs, as mbar_wait
        checked = now;
        if (*abort_flag) return false;
        if (*reinterpret_cast<volatile int *>(err)) {
            *abort_flag = 1;
            return false;
        }
        if (globaltimer() - t0 > timeout_ns) {
            *abort_flag = 1;
            atomicCAS(err, 0, code);
            return false;
        }
    }
}
// Per-thread asynchronous copies global -> shared (cp.async, through L2; valid = false
// writes zeros), committed as groups and waited for by the issuing thread.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid = true) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    const int sz = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Make generic-proxy shared-memory writes visible to the async proxy (tensor core).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ── clusters (CTA pairs) and programmatic dependent launch ──
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the object at the same offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Every thread of every CTA of the cluster (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier named by its shared::cluster address (this CTA's or the peer's).
// Default (CTA-scope release) semantics: a cluster-scope release would first wait for
// every earlier memory operation of the thread to become visible cluster-wide (about
// 900 cycles per arrival measured here), and the data these arrivals publish is read
// by the tensor core after the writer's proxy fence.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Let the next kernel of the stream be scheduled / wait until the previous one has
// completed and its memory is visible (no-ops without programmatic serialization).
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 2-D tiled tensor load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (cluster address).  Not a multicast load.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}

// 3-D tiled tensor load (coordinates innermost first).
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}


// ── tcgen05, CTA-pair form (every tcgen05 instruction of a kernel uses one cta_group) ──
// Issued by the same warp of both CTAs of the pair.
__device__ __forceinline__ void tmem_alloc2(uint32_t *holder_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A * B^T, kind::f16, cta_group::2, issued by the even CTA of the pair: A
// rows 0-127 come from the even CTA and 128-255 from the odd one (same TMEM column or
// shared-memory offset), B columns [0, N/2) from the even CTA and [N/2, N) from the odd
// one; each CTA's TMEM receives its own 128 rows of D.  A in TMEM: lane = row of A, one
// 32-bit column per two consecutive k elements (lower k in the low half).
// One 64-wide k-slice = four K = 16 MMAs in one statement, few instructions around them
// (every instruction on the issuing thread's path leaves the tensor pipe idle): A from
// TMEM (8 columns per step), B descriptor advanced by 32 bytes per step; only the first
// step's accumulate flag is the caller's, the others always accumulate.
__device__ __forceinline__ void mma2_f16_ts_k64(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p0, p1;\n\t.reg .b32 a1, a2, a3;\n\t.reg .b64 b1, b2, b3;\n\t"
        "setp.ne.b32 p0, %4, 0;\n\t"
        "setp.eq.b32 p1, %4, %4;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
        "add.u64 b1, %2, 2;\n\tadd.u64 b2, %2, 4;\n\tadd.u64 b3, %2, 6;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a1], b1, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a2], b2, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a3], b3, %3, p1;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 128 k-values of 8-bit operands (kind::f8f6f4, E4M3 x E4M3 into the f32 accumulator):
// four K = 32 MMAs, A from TMEM (four 8-bit values per 32-bit column, lower k in the low
// byte: 8 columns per step), B descriptor advanced by 32 bytes per step.  Accumulates.
__device__ __forceinline__ void mma2_f8_ts_k128(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p1;\n\t.reg .b32 a1, a2, a3;\n\t.reg .b64 b1, b2, b3;\n\t"
        "setp.eq.b32 p1, %3, %3;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
        "add.u64 b1, %2, 2;\n\tadd.u64 b2, %2, 4;\n\tadd.u64 b3, %2, 6;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], [%1], %2, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], [a1], b1, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], [a2], b2, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], [a3], b3, %3, p1;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc)
        : "memory");
}
// Same with A from shared memory (128 bytes per row: descriptor advanced by 32 bytes per step).
__device__ __forceinline__ void mma2_f8_ss_k128(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p1;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
        "setp.eq.b32 p1, %3, %3;\n\t"
        "add.u64 a1, %1, 2;\n\tadd.u64 a2, %1, 4;\n\tadd.u64 a3, %1, 6;\n\t"
        "add.u64 b1, %2, 2;\n\tadd.u64 b2, %2, 4;\n\tadd.u64 b3, %2, 6;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], a1, b1, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], a2, b2, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], a3, b3, %3, p1;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc)
        : "memory");
}
// Same with A from shared memory (descriptor advanced by 32 bytes per step).
__device__ __forceinline__ void mma2_f16_ss_k64(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p0, p1;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
        "setp.ne.b32 p0, %4, 0;\n\t"
        "setp.eq.b32 p1, %4, %4;\n\t"
        "add.u64 a1, %1, 2;\n\tadd.u64 a2, %1, 4;\n\tadd.u64 a3, %1, 6;\n\t"
        "add.u64 b1, %2, 2;\n\tadd.u64 b2, %2, 4;\n\tadd.u64 b3, %2, 6;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a1, b1, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a2, b2, %3, p1;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a3, b3, %3, p1;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 lanes x 16 columns of 32-bit: this thread's lane, columns [col, col+16).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
// 32 lanes x 8 columns of 32-bit: this thread's lane, columns [col, col+8).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
// This thread's tcgen05.st have completed.
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive once on the mbarrier at this smem offset in every CTA of cta_mask when all
// previously issued tcgen05.mma of this thread have completed.
__device__ __forceinline__ void mma2_commit_mc(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}
// Same, on this CTA's barrier only.
__device__ __forceinline__ void mma2_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 lanes x 16 columns of 32-bit: this thread's lane, columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same, tying the loaded registers to the wait so no use of them moves above it.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// Shared-memory matrix descriptor, K-major operand, 128-byte swizzle: rows of 128 B,
// 8-row groups 1024 B apart (SBO), version 1 (sm_100), swizzle mode 2 (128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);  // start address
    d |= (uint64_t)1 << 16;                        // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;              // SBO
    d |= (uint64_t)1 << 46;                        // version
    d |= (uint64_t)2 << 61;                        // SWIZZLE_128B
    return d;
}
// Instruction descriptor: kind::f16, A/B f16, D f32, both K-major, M=m, N=n.
__host__ __device__ __forceinline__ uint32_t idesc_f16(uint32_t m, uint32_t n) {
    return (1u << 4)              // D = F32
           | (0u << 7) | (0u << 10)  // A, B = F16
           | ((n >> 3) << 17)     // N >> 3
           | ((m >> 4) << 24);    // M >> 4
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace dfb
