// routing.cu -- MoeRoutingTopK on sm_100a: gating GEMM on the tensor cores, then
// softmax, top-K and renormalisation per token.
//
// Replaces op_kernel/moe_routing.cpp (Ascend Cube GEMM + scalar softmax/top-2).
// Semantics follow the fp32 naive reference, tests/moe_cpu_sim.cpp:198-243:
//   logits[t,e] = sum_h x[t,h] * w_gate[h,e]      (fp32 accumulation)
//   probs       = exp(logits - max) / sum         (sum in e ascending order)
//   ids         = top-K of probs, descending, equal probs -> lower expert id
//   weights     = probs[ids] / sum_k probs[ids]   -> fp16 (round to nearest even)
//
// The gating product is a skinny GEMM [T,H] x [H,E]; it is HBM-bound (x is read
// once), so it runs as tcgen05.mma with M=128 tokens per CTA, N=E rounded up to a
// multiple of 16, K=16 per instruction and the fp32 accumulator in TMEM.  The
// products of fp16 values are exact; the tensor core's fp32 accumulation order
// differs from the reference's sequential sum, so logits can differ in the last
// bits, and expert ids can only differ at (near-)ties -- the parity tests
// compare ids bit for bit away from ties (top-K logit margin >= 1e-3).
//
// Per CTA: x tiles [128 tokens x 64 h] arrive by TMA (128-byte swizzle, K-major);
// w_gate [H,E] is tiny and L2-resident, so the threads copy its [64 h x E] block
// transposed into the K-major, 128-byte-swizzled B tile; a 4-stage ring keeps
// three k-blocks in flight, and the w_gate loads for a refill are issued a step early.  Afterwards each thread owns one token (one TMEM lane): the E
// logits go through shared memory and the thread runs softmax and top-K in the
// reference's order.
#include <cooperative_groups.h>

#include "moe_common.cuh"
#include "moe_kernels.h"

namespace cg = cooperative_groups;

namespace moe {

constexpr int RT_BM = 128;     // tokens per CTA (UMMA M)
constexpr int RT_BK = 64;      // h per stage (one 128-byte swizzle row)
constexpr int RT_MAX_STAGES = 8;  // ring depth: as many as fit (>= 2)
constexpr int RT_THREADS = 128;
constexpr int RT_A_BYTES = RT_BM * RT_BK * 2;  // 16 KB

struct RoutingSmemTail {
    uint64_t full[RT_MAX_STAGES];   // A tile landed (TMA)
    uint64_t mdone[RT_MAX_STAGES];  // MMAs that read this stage are done
    uint32_t tmem_base;
    int abort_flag;
};

static inline int routing_epad(int E) { return (E + 15) & ~15; }

// Row pitch (floats) of the logits rows in shared memory: E+4 keeps rows 16-byte
// aligned for vector stores when E % 4 == 0, else E+1 (odd: conflict-free scalars).
__host__ __device__ inline int routing_pitch(int E) { return (E % 4 == 0) ? E + 4 : E + 1; }

// Bytes before the barrier tail: the A ring plus either per-stage B tiles or (RESIDENT)
// all of w_gate^T as one B tile per k-block; the logits later reuse the front.
__host__ __device__ inline size_t routing_region_bytes(bool resident, int E, int epad, int nk, int nst, int S)
{
    const size_t ring = resident ? (size_t)nst * RT_A_BYTES + (size_t)nk * epad * 128
                                 : (size_t)nst * (RT_A_BYTES + (size_t)epad * 128);
    const size_t logits = (size_t)S * RT_BM * routing_pitch(E) * 4;  // one slot of partial logits per cluster rank
    return ((ring > logits ? ring : logits) + 15) & ~(size_t)15;
}

static size_t routing_smem_bytes(bool resident, int E, int epad, int nk, int nst, int S)
{
    return 1024 + routing_region_bytes(resident, E, epad, nk, nst, S) + sizeof(RoutingSmemTail) + 64;
}

// Byte offset of element (row n, k) of a K-major tile with 128-byte rows and the
// 128-byte swizzle: 8-row atoms of 1024 bytes, 16-byte chunk index XOR (row % 8).
__device__ __forceinline__ uint32_t sw128_offset(int n, int k)
{
    return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((((k >> 3) ^ (n & 7)) & 7) << 4) + (k & 7) * 2);
}

__device__ int g_routing_err;

#ifdef MOE_ROUTING_PROBE  // development builds only: phase timestamps of CTA 0
__device__ unsigned long long g_rt_probe[8];
#define RT_STAMP(i) \
    if (blockIdx.x == 0 && threadIdx.x == 0) g_rt_probe[i] = global_timer_ns();
#else
#define RT_STAMP(i)
#endif

template <bool RESIDENT>
__global__ void __launch_bounds__(RT_THREADS)
routing_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __half* __restrict__ w_gate,
                  int32_t* __restrict__ expert_ids, __half* __restrict__ weights, int T, int H, int E, int K,
                  int epad, uint32_t tmem_cols, int nst, int nkl_max, int* err, int32_t* __restrict__ tile_counts,
                  int32_t* __restrict__ tile_rank)
{
    // A cluster of S CTAs shares one 128-token tile; CTA rank c handles k-blocks
    // [c*nk/S, (c+1)*nk/S) and rank 0 sums the partial logits in rank order.
    cg::cluster_group cluster = cg::this_cluster();
    const int S = (int)cluster.num_blocks();
    const int crank = (int)cluster.block_rank();
    extern __shared__ uint8_t rt_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(rt_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const size_t stage_bytes = (size_t)RT_A_BYTES + (size_t)epad * 128;  // non-resident stages
    const int nk_all = (H + RT_BK - 1) / RT_BK;
    const int kb0 = crank * nk_all / S, kb1 = (crank + 1) * nk_all / S;
    const int nk = kb1 - kb0;  // this CTA's k-blocks (local index kb <-> global kb0 + kb)
    RoutingSmemTail* tail =
        reinterpret_cast<RoutingSmemTail*>(smem + routing_region_bytes(RESIDENT, E, epad, nkl_max, nst, S));
    const int tid = threadIdx.x, warp = tid >> 5;
    const int t0 = (blockIdx.x / S) * RT_BM;
    volatile int* abort_flag = &tail->abort_flag;
    // MoeRoutingTopK has no workspace: a timed-out wait is recorded in a device
    // global (the waits still end the kernel instead of spinning forever)
    int* errp = err ? err : &g_routing_err;

    RT_STAMP(0)
    pdl_trigger();  // the permutation launch after it may be scheduled now (it waits for this grid)
    if (tid == 0) {
        for (int s = 0; s < nst; s++) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->mdone[s]), 1);
        }
        tail->abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmX);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&tail->tmem_base), tmem_cols);
        tmem_relinquish();
    }
    // B rows >= E stay zero for the whole kernel
    {
        const int ntiles = RESIDENT ? nk : nst;
        for (int tt = 0; tt < ntiles; tt++) {
            uint8_t* bt = RESIDENT ? smem + nst * (size_t)RT_A_BYTES + (size_t)tt * epad * 128
                                   : smem + tt * stage_bytes + RT_A_BYTES;
            for (int i = tid; i < (epad - E) * 8; i += RT_THREADS) {
                const int n = E + i / 8, c = i % 8;
                *reinterpret_cast<uint4*>(bt + sw128_offset(n, c * 8)) = make_uint4(0, 0, 0, 0);
            }
        }
    }

    uint8_t* bres = smem + nst * (size_t)RT_A_BYTES;  // RESIDENT: all of w_gate^T, one tile per k-block
    auto b_tile = [&](int kb, int s) -> uint8_t* {
        return RESIDENT ? bres + (size_t)kb * epad * 128 : smem + s * stage_bytes + RT_A_BYTES;
    };
    // w_gate rows [h_begin, h_end) -> swizzled K-major B tiles.  The rows are one
    // contiguous block of (h_end-h_begin)*E halves: read it with 16-byte loads, 8 in
    // flight per thread, and scatter each half to (row n = expert, k = h % 64) of the
    // tile of k-block h / 64 (tile_of(kb) gives its address).
    auto b_fill_rows = [&](int h_begin, int h_end, auto tile_of) {
        if ((E & 7) == 0 && ((h_end - h_begin) & 7) == 0) {
            // 8 h x 8 experts per step: eight 16-byte loads (one per h row), an 8x8
            // transpose of 16-bit values in registers, eight 16-byte swizzled stores
            const int hg = (h_end - h_begin) >> 3, eg = E >> 3;
            for (int b = tid; b < hg * eg; b += RT_THREADS) {
                const int h0 = h_begin + (b / eg) * 8, e0 = (b % eg) * 8;
                uint4 in[8];
#pragma unroll
                for (int j = 0; j < 8; j++)
                    in[j] = __ldg(reinterpret_cast<const uint4*>(w_gate + (size_t)(h0 + j) * E + e0));
                uint8_t* bt = tile_of(h0 / RT_BK);
                const int k = h0 % RT_BK;
#pragma unroll
                for (int j = 0; j < 8; j++) {  // expert e0+j: halves j of rows h0..h0+7
                    const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;
                    uint32_t w[4];
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const uint32_t* a = reinterpret_cast<const uint32_t*>(&in[2 * q]);
                        const uint32_t* c = reinterpret_cast<const uint32_t*>(&in[2 * q + 1]);
                        w[q] = __byte_perm(a[j >> 1], c[j >> 1], sel);
                    }
                    *reinterpret_cast<uint4*>(bt + sw128_offset(e0 + j, k)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            return;
        }
        const uint4* src = reinterpret_cast<const uint4*>(w_gate + (size_t)h_begin * E);
        const int nvec = ((h_end - h_begin) * E) >> 3;  // H*E and 64*E are multiples of 8
        for (int v0 = tid; v0 < nvec; v0 += 8 * RT_THREADS) {
            uint4 buf[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int v = v0 + u * RT_THREADS;
                buf[u] = v < nvec ? __ldg(src + v) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int v = v0 + u * RT_THREADS;
                if (v >= nvec) break;
                const unsigned short* hv = reinterpret_cast<const unsigned short*>(&buf[u]);
                int f = 8 * v;
                int hh = h_begin + f / E, n = f - (f / E) * E;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    *reinterpret_cast<unsigned short*>(tile_of(hh / RT_BK) + sw128_offset(n, hh % RT_BK)) = hv[j];
                    if (++n == E) { n = 0; ++hh; }
                }
            }
        }
    };
    // one k-block (non-resident stages): rows beyond H are zero
    auto b_fill = [&](int kb, uint8_t* bt) {  // local k-block kb
        const int h0 = (kb0 + kb) * RT_BK, h1 = min(H, h0 + RT_BK);
        if (h1 - h0 < RT_BK)
            for (int i = tid; i < epad * 8; i += RT_THREADS)
                *reinterpret_cast<uint4*>(bt + sw128_offset(i / 8, (i % 8) * 8)) = make_uint4(0, 0, 0, 0);
        if (h1 - h0 < RT_BK) __syncthreads();
        b_fill_rows(h0, h1, [&](int) { return bt; });
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // B is read by the tensor core
    };
    auto a_load = [&](int kb, int s) {  // thread 0
        const uint32_t full = smem_u32(&tail->full[s]);
        mbar_arrive_expect_tx(full, RT_A_BYTES);
        tma_load_2d(smem_u32(smem + s * (RESIDENT ? (size_t)RT_A_BYTES : stage_bytes)), &tmX, full, (kb0 + kb) * RT_BK, t0,
                    l2_policy_evict_first());
    };
    auto a_addr = [&](int s) -> uint32_t {
        return smem_u32(smem + s * (RESIDENT ? (size_t)RT_A_BYTES : stage_bytes));
    };

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tail->tmem_base;
    const uint32_t idesc = umma_idesc_f16_f32(RT_BM, epad);
    bool ok = true;

    if (RESIDENT) {
        // A ring by TMA starts at once; meanwhile every thread transposes w_gate in
        if (tid == 0)
            for (int kb = 0; kb < nk && kb < nst; kb++) a_load(kb, kb);
        if ((H % RT_BK) && kb1 == nk_all) {  // the last tile's rows beyond H are zero
            uint8_t* bt = b_tile(nk - 1, 0);
            for (int i = tid; i < epad * 8; i += RT_THREADS)
                *reinterpret_cast<uint4*>(bt + sw128_offset(i / 8, (i % 8) * 8)) = make_uint4(0, 0, 0, 0);
            __syncthreads();
        }
        RT_STAMP(1)
        b_fill_rows(kb0 * RT_BK, min(H, kb1 * RT_BK), [&](int kbg) { return b_tile(kbg - kb0, 0); });
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        RT_STAMP(2)
        if (tid == 0) {
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % nst;
                if (!mbar_wait_bounded(smem_u32(&tail->full[s]), (kb / nst) & 1u, errp, MOE_DEV_WAIT_TIMEOUT_MMA,
                                       abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a = a_addr(s), b = smem_u32(b_tile(kb, s));
#pragma unroll
                for (int k = 0; k < RT_BK / 16; k++)
                    umma_f16_ss(tmem_base, umma_desc_sw128(a + k * 32), umma_desc_sw128(b + k * 32), idesc,
                                (kb | k) != 0);
                umma_commit(smem_u32(&tail->mdone[s]));
                // refill the stage MMA kb-1 read, once that MMA is done
                const int nb = kb - 1 + nst;
                if (kb >= 1 && nb < nk) {
                    const int sn = nb % nst;
                    if (!mbar_wait_bounded(smem_u32(&tail->mdone[sn]), ((kb - 1) / nst) & 1u, errp,
                                           MOE_DEV_WAIT_TIMEOUT_MMA, abort_flag)) {
                        ok = false;
                        break;
                    }
                    a_load(nb, sn);
                }
            }
        }
    } else {
        const int pro = nk < nst ? nk : nst;
        for (int kb = 0; kb < pro; kb++) {
            if (tid == 0) a_load(kb, kb);
            b_fill(kb, b_tile(kb, kb));
        }
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % nst;
            const uint32_t par = (kb / nst) & 1u;
            __syncthreads();  // every thread's B stores for this stage are in
            if (tid == 0) {
                if (ok && mbar_wait_bounded(smem_u32(&tail->full[s]), par, errp, MOE_DEV_WAIT_TIMEOUT_MMA, abort_flag)) {
                    tc_fence_after();
                    const uint32_t a = a_addr(s), b = smem_u32(b_tile(kb, s));
#pragma unroll
                    for (int k = 0; k < RT_BK / 16; k++)
                        umma_f16_ss(tmem_base, umma_desc_sw128(a + k * 32), umma_desc_sw128(b + k * 32), idesc,
                                    (kb | k) != 0);
                } else {
                    ok = false;
                }
                umma_commit(smem_u32(&tail->mdone[s]));
            }
            if (kb + nst < nk) {  // refill stage s once the MMAs that read it are done
                if (!mbar_wait_bounded(smem_u32(&tail->mdone[s]), par, errp, MOE_DEV_WAIT_TIMEOUT_MMA, abort_flag))
                    ok = false;
                if (tid == 0) a_load(kb + nst, s);
                b_fill(kb + nst, b_tile(kb + nst, s));
            }
        }
    }
    __syncthreads();
    if (!ok && tid == 0) {
        // unwinding after a timeout: wait (bounded) for TMA copies still in flight
        for (int kb = nk > nst ? nk - nst : 0; kb < nk; kb++) {
            const uint64_t w0 = global_timer_ns();
            while (!mbar_try_wait(smem_u32(&tail->full[kb % nst]), (kb / nst) & 1u))
                if (global_timer_ns() - w0 > MOE_WAIT_LIMIT_NS) break;
        }
    }
    // the last commit covers every MMA of this CTA
    {
        const int s = (nk - 1) % nst;
        mbar_wait_bounded(smem_u32(&tail->mdone[s]), ((nk - 1) / nst) & 1u, errp, MOE_DEV_WAIT_TIMEOUT_EPI,
                          abort_flag);
    }
    tc_fence_after();
    __syncthreads();
    RT_STAMP(3)

    // logits: TMEM lane r (this thread's token) -> row r of slot `crank` of the
    // leader's shared memory ([S][128][E+1]; with S == 1 that is this CTA's own)
    const int r = tid;  // warp w reads TMEM lanes 32w..32w+31
    if (S > 1) cluster.sync();  // every CTA of the cluster is done with its ring (the slots overlap it)
    float* lg = reinterpret_cast<float*>(smem);
    const int pitch = routing_pitch(E);
    float* dst = (S > 1 ? cluster.map_shared_rank(lg, 0) : lg) + ((size_t)crank * RT_BM + r) * pitch;
    const uint32_t tbase = tmem_base + ((uint32_t)(warp * 32) << 16);
    for (int c0 = 0; c0 < epad; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + c0, v);
        tmem_ld_wait();
        if ((E & 3) == 0) {  // 16-byte stores (fewer distributed-shared-memory transactions)
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                if (c0 + j < E)
                    *reinterpret_cast<float4*>(dst + c0 + j) =
                        make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                    __uint_as_float(v[j + 3]));
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (c0 + j < E) dst[c0 + j] = __uint_as_float(v[j]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, tmem_cols);
    }
    if (S > 1) {
        RT_STAMP(6)
        cluster.sync();  // all partial slots have landed in the leader
        RT_STAMP(7)
        if (crank != 0) return;
        // rank 0: slot 0 += slot 1 + ... in rank order (deterministic)
        float* mine = lg + (size_t)r * pitch;
        if ((E & 3) == 0) {
            for (int i = 0; i < E; i += 4) {
                float4 a = *reinterpret_cast<const float4*>(mine + i);
                for (int c = 1; c < S; c++) {
                    const float4 o = *reinterpret_cast<const float4*>(lg + ((size_t)c * RT_BM + r) * pitch + i);
                    a.x += o.x;
                    a.y += o.y;
                    a.z += o.z;
                    a.w += o.w;
                }
                *reinterpret_cast<float4*>(mine + i) = a;
            }
        } else {
            for (int c = 1; c < S; c++) {
                const float* o = lg + ((size_t)c * RT_BM + r) * pitch;
                for (int i = 0; i < E; i++) mine[i] += o[i];
            }
        }
    }
    RT_STAMP(4)
    // softmax + top-K for this thread's token (moe_cpu_sim.cpp:211-243) in one pass:
    // the exp-sum in expert order as the reference sums it, and a stable top-8 of the
    // exps kept in registers (strict '>' keeps the lower id ahead on equal values).
    // Only the selected probabilities are divided, p = e / sum, as the reference
    // computes them; ordering by e instead of e / sum can differ only where the
    // division rounds two different exps to one probability (a near tie).
    const int t = t0 + r;
    int ti[8];  // this token's top-K ids (slot order)
#pragma unroll
    for (int j = 0; j < 8; j++) ti[j] = 0;
    if (t < T) {
        const float* l = lg + (size_t)r * pitch;
        float maxv = -1e30f;
        for (int i = 0; i < E; i++) maxv = l[i] > maxv ? l[i] : maxv;
        float sum = 0.0f;
        float tv[8];
#pragma unroll
        for (int j = 0; j < 8; j++) tv[j] = -1.0f;
        for (int i = 0; i < E; i++) {
            float cv = expf(l[i] - maxv);
            sum += cv;
            int ci = i;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (cv > tv[j]) {
                    const float fv = tv[j];
                    const int fi = ti[j];
                    tv[j] = cv;
                    ti[j] = ci;
                    cv = fv;
                    ci = fi;
                }
            }
        }
        float wsum = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (j < K) {
                tv[j] = tv[j] / sum;  // the selected probabilities
                wsum += tv[j];        // selection order, as the reference's wSum (moe_cpu_sim.cpp:236-240)
            }
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (j < K) {
                expert_ids[(size_t)t * K + j] = ti[j];
                weights[(size_t)t * K + j] = __float2half_rn(tv[j] / wsum);
            }
    }
    if (tile_counts) {
        // First pass of the permutation, fused (layer calls): this tile's per-expert
        // histogram, tile_counts[tile][E], and each entry's stable rank among the
        // tile's entries of its expert, tile_rank[t*K+k], in flat order t*K+k (the
        // order of tests/moe_cpu_sim.cpp:412-419).  The 128*K entries go in K rounds
        // of 128 consecutive flat indices; inside a round, a warp match gives the
        // rank among the warp's lanes and per-warp counts give the rest.
        __syncthreads();  // every thread is done with the logits: reuse their space
        int* ids_s = reinterpret_cast<int*>(smem);  // [128*K]
        int* wcnt = ids_s + RT_BM * K;              // [4 warps][E]
        int* base = wcnt + 4 * E;                   // [E] entries of each expert so far
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (j < K) ids_s[r * K + j] = t < T ? ti[j] : -1;
        for (int i = tid; i < 4 * E; i += RT_THREADS) wcnt[i] = 0;
        for (int i = tid; i < E; i += RT_THREADS) base[i] = 0;
        __syncthreads();
        const int lane = tid & 31;
        for (int q = 0; q < K; q++) {
            const int f = q * RT_BM + tid;  // flat index inside the tile
            const int e = ids_s[f];
            const unsigned same = __match_any_sync(0xffffffffu, e);
            const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
            if (e >= 0 && rank_in_warp == 0) wcnt[warp * E + e] = __popc(same);
            __syncthreads();
            for (int ee = tid; ee < E; ee += RT_THREADS) {
                int run = base[ee];
                for (int w = 0; w < 4; w++) {
                    const int c = wcnt[w * E + ee];
                    wcnt[w * E + ee] = run;
                    run += c;
                }
                base[ee] = run;
            }
            __syncthreads();
            if (e >= 0) tile_rank[(size_t)t0 * K + f] = wcnt[warp * E + e] + rank_in_warp;
            __syncthreads();
            for (int i = tid; i < 4 * E; i += RT_THREADS) wcnt[i] = 0;
            __syncthreads();
        }
        for (int i = tid; i < E; i += RT_THREADS) tile_counts[(size_t)(t0 / RT_BM) * E + i] = base[i];
    }
    __syncthreads();
    RT_STAMP(5)
}

static int dev_of_current()
{
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

typedef CUresult (*RtEncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int* routing_error_word()
{
    static int* addr[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_routing_err) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        addr[dev] = static_cast<int*>(p);
    }
    return addr[dev];
}

cudaError_t launch_routing(const __half* x, const __half* w_gate, int32_t* ids, __half* weights, int T, int H,
                           int E, int K, cudaStream_t s, int32_t* tile_counts, int32_t* tile_rank)
{
    if (T == 0) return cudaSuccess;
    static RtEncodeTiledFn enc = nullptr;
    if (!enc) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return cudaErrorInvalidValue;
        enc = reinterpret_cast<RtEncodeTiledFn>(p);
    }
    CUtensorMap tm;
    cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)H * 2};
    cuuint32_t box[2] = {RT_BK, RT_BM};
    cuuint32_t es[2] = {1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    const int epad = routing_epad(E);
    const int nk = (H + RT_BK - 1) / RT_BK;
    uint32_t cols = 32;
    while (cols < (uint32_t)epad) cols <<= 1;
    // all of w_gate^T resident in shared memory when it fits (the benchmark's E=16:
    // 64 KB at H=2048), else per-stage B tiles
    // cluster split along H: enough CTAs to cover the SMs when there are few tiles
    static int sms = 0;
    if (!sms) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev_of_current());
        if (sms <= 0) sms = 148;
    }
    const int tiles = (T + RT_BM - 1) / RT_BM;
    int S = 1;
#ifndef MOE_RT_OVERSUB
#define MOE_RT_OVERSUB 1
#endif
    while (S < 8 && (long long)tiles * S * 2 <= (long long)sms * MOE_RT_OVERSUB && nk / (S * 2) >= 2) S *= 2;
    const size_t cap = 210 * 1024;
    // a wider split when it lets each CTA keep its slice of w_gate^T resident (large E)
    while (S < 8 && routing_smem_bytes(true, E, epad, (nk + S - 1) / S, 4, S) > cap && nk / (S * 2) >= 2) S *= 2;
    const int nkl_max = (nk + S - 1) / S;
    const bool resident = routing_smem_bytes(true, E, epad, nkl_max, 4, S) <= cap;
    int nst = RT_MAX_STAGES;
    while (nst > 2 && routing_smem_bytes(resident, E, epad, nkl_max, nst, S) > cap) nst--;
    const size_t smem = routing_smem_bytes(resident, E, epad, nkl_max, nst, S);
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(routing_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(routing_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(tiles * S);
    lc.blockDim = dim3(RT_THREADS);
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = S;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    int* no_err = nullptr;
    cudaError_t e = resident ? cudaLaunchKernelEx(&lc, routing_tc_kernel<true>, tm, w_gate, ids, weights, T, H, E, K,
                                                  epad, cols, nst, nkl_max, no_err, tile_counts, tile_rank)
                             : cudaLaunchKernelEx(&lc, routing_tc_kernel<false>, tm, w_gate, ids, weights, T, H, E, K,
                                                  epad, cols, nst, nkl_max, no_err, tile_counts, tile_rank);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace moe
