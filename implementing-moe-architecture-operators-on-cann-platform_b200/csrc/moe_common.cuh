// moe_common.cuh -- shared device helpers for the sm_100a MoE kernels.
//
// Thin inline-PTX wrappers for the Blackwell features the kernels use: mbarriers
// with bounded waits, TMA tiled loads (each CTA loads only into its own shared memory),
// and the tcgen05 tensor-core path (TMEM allocation, UMMA issue, commit, TMEM
// loads).  Every wait is bounded: after MOE_WAIT_LIMIT_NS of %globaltimer time it
// records an error code in a device flag and returns false so the caller can
// unwind instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef MOE_WAIT_LIMIT_NS
#define MOE_WAIT_LIMIT_NS 2000000000ull  // 2 s: healthy waits are microseconds
#endif

// Device-side error codes written to the error word of the workspace.
enum MoeDeviceError : int {
    MOE_DEV_OK = 0,
    MOE_DEV_BAD_EXPERT_ID = 1,      // an expert id outside [0, E)
    MOE_DEV_WAIT_TIMEOUT_TMA = 2,   // producer gave up waiting for a free stage
    MOE_DEV_WAIT_TIMEOUT_MMA = 4,   // MMA issuer gave up waiting for data / accumulator
    MOE_DEV_WAIT_TIMEOUT_EPI = 8,   // epilogue gave up waiting for an accumulator
    MOE_DEV_TMEM_ALLOC = 16,        // TMEM allocation returned an unusable address
};

namespace moe {

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (and ORs
// `code` into *err) once MOE_WAIT_LIMIT_NS has passed, or at once if *abort is
// set by another role of the same CTA.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int* err, int code,
                                                  volatile int* abort_flag)
{
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > MOE_WAIT_LIMIT_NS) {
                atomicOr(err, code);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// ------------------------------------------------------------------ cross-GPU flags
// Acquire load of a flag another GPU (or this one) raises with a system-scope
// atomic after its data stores and a system fence.
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p)
{
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait (one thread) until *flag >= target.  Gives up, recording `code` in
// *err, after MOE_WAIT_LIMIT_NS, or at once when *stop (optional) is nonzero or
// already holds `code` (another waiter of this launch gave up: one timeout, not
// one per waiter).
__device__ __forceinline__ bool flag_wait_bounded(const unsigned long long* flag, unsigned long long target,
                                                  int* err, int code, volatile int* stop)
{
    if (ld_acquire_sys(flag) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (ld_acquire_sys(flag) >= target) return true;
        if ((stop && *stop) || (*reinterpret_cast<volatile int*>(err) & code)) return false;
        if (global_timer_ns() - t0 > MOE_WAIT_LIMIT_NS) {
            atomicOr(err, code);
            if (stop) *stop = 1;
            return false;
        }
        __nanosleep(64);
    }
}

// Orders this thread's earlier generic-proxy observations (a flag acquired) before
// its later async-proxy (TMA) reads of global memory.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ------------------------------------------------------------------ dependent launch
// Programmatic dependent launch: a kernel lets the next kernel of the stream start
// its prologue early (pdl_trigger), and that kernel waits for this one's results
// before reading them (pdl_wait).  Both are no-ops without the launch attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// 2-D tiled load of one box into shared memory, completing on `bar`.  The
// inner coordinate c0 is an element index along the contiguous dimension; the
// callers only pass multiples of 64 fp16 elements (128 bytes).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                            int32_t c0, int32_t c1, uint64_t cache_hint)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(bar), "l"(cache_hint)
        : "memory");
}

// L2 eviction-priority policies for TMA loads (createpolicy.fractional).
__device__ __forceinline__ uint64_t l2_policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ------------------------------------------------------------------ tcgen05
// TMEM allocation: executed by one full warp.  Writes the TMEM base address to
// the shared-memory word at `dst_smem`.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 64 fp16, 8-row atoms of 1024 bytes):
// start address >>4 in bits [0,14), leading byte offset 16 B (unused for swizzled
// K-major), stride byte offset 1024 B between 8-row groups, descriptor version 1
// (bits 46-47), layout type 2 = SWIZZLE_128B (bits 61-63).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr)
{
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(16u >> 4) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor for kind::f16 with fp16 A/B, fp32 accumulator, both
// operands K-major: D format bits [4,6) = 1 (F32), A/B format = 0 (F16),
// N>>3 in bits [17,23), M>>4 in bits [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int M, int N)
{
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// One warp reads 32 lanes x 32 consecutive fp32 columns: thread i gets lane
// (row) base_lane+i, columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ CTA pairs
// Helpers for the paired-CTA (cta_group::2) GEMM: two CTAs of a 2-CTA cluster
// share one M=256 UMMA; the even rank (the leader) issues it, each CTA holds half
// of A (its 128 rows) and half of B (128 of the N rows) in its own shared memory,
// and each CTA's TMEM receives its own 128 rows of the accumulator.
__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier of any CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait_bounded with cluster-scope acquire (the phase is completed by arrivals
// or copies from the peer CTA as well).
__device__ __forceinline__ bool mbar_wait_bounded_cluster(uint32_t bar, uint32_t parity, int* err, int code,
                                                          volatile int* abort_flag)
{
    if (mbar_try_wait_cluster(bar, parity)) return true;
    uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > MOE_WAIT_LIMIT_NS) {
                atomicOr(err, code);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// Tiled load into this CTA's shared memory whose completion (bytes) is counted on
// an mbarrier of either CTA of the pair (`cluster_bar`: a shared::cluster address).
// A plain per-CTA load: no broadcast to other CTAs.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* tm, uint32_t cluster_bar,
                                                 int32_t c0, int32_t c1, uint64_t cache_hint)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(cluster_bar), "l"(cache_hint)
        : "memory");
}

// TMEM allocation for a CTA pair: one warp of EACH CTA of the pair executes it.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// M=256 UMMA over the pair, issued by the leader CTA.
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on the mbarrier at `cluster_bar` (either CTA of the pair) once the pair
// UMMAs issued so far by this thread are done.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
                 : "memory");
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b)
{
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace moe
