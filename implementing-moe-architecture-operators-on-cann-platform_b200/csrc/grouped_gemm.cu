// grouped_gemm.cu -- the expert FFN as two grouped GEMMs on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA).
//
// Replaces op_kernel/moe_expert_ffn.cpp (Ascend MatmulImpl with a GM workspace
// between a gate/up stage and a down stage, :265-394).  Math, per expert e and
// per permuted row r of that expert (tests/moe_cpu_sim.cpp:262-294):
//   GEMM1 (MODE_SWIGLU): h[r, i]  = silu(xp[r,:] . Wg_e[i,:]) * (xp[r,:] . Wu_e[i,:])
//   GEMM2 (MODE_DOWN)  : out[perm[r], n] = h[r,:] . Wd_e[n,:]
// with Wg_e, Wu_e = [I,H] and Wd_e = [H,I] row-major slices of expert_weights
// [E, 3I, H] (the reference CPU oracle's layout).  Every operand is K-major, so
// no weight is transposed or repacked: TMA reads them in place.
//
// Kernel structure (one persistent CTA per SM, 192 threads):
//   warp 0      : TMA producer -- per k-block, one 128x64 box of A and two
//                 128x64 boxes of B (gate rows + up rows for GEMM1, two halves of
//                 256 down rows for GEMM2) into a STAGES-deep shared-memory ring;
//   warp 1      : TMEM allocator + single-thread UMMA issuer, M=128 N=256 K=16
//                 instructions accumulating in fp32 in TMEM; two accumulator
//                 buffers of 256 columns so the epilogue of tile i overlaps the
//                 main loop of tile i+1;
//   warps 2..5  : epilogue -- tcgen05.ld of the warp's 32 TMEM lanes (= rows),
//                 SwiGLU in fp32 (GEMM1) or plain conversion (GEMM2), fp16 stores;
//                 GEMM2 scatters each row to expert_out[t, k, :] through perm.
// Tiles are (expert, n-tile, m-tile) with m innermost, so the CTAs working at the
// same time share one weight tile in L2 and every weight byte comes from HBM once.
// The tile list is derived on the device from offsets[] (no host sync).
//
// Paired mode (PAIR=1, large experts): a 2-CTA cluster shares M=256 cta_group::2
// UMMAs; the leader CTA issues them and owns the barriers they wait on, and each
// CTA loads its own half of A and B into its own shared memory.  No load is
// broadcast to several CTAs, so the same kernel runs on every rank of the
// expert-parallel path.
#include <cstdio>
#include <cstdlib>

#include "moe_common.cuh"
#include "moe_kernels.h"

namespace moe {

constexpr int GM_BM = 128;        // rows per tile (UMMA M)
constexpr int GM_BN = 256;        // accumulator columns per tile (UMMA N)
constexpr int GM_BK = 64;         // k per stage: 64 fp16 = one 128-byte swizzle row
#ifndef MOE_GEMM_STAGES
#define MOE_GEMM_STAGES 4
#endif
constexpr int GM_STAGES = MOE_GEMM_STAGES;
#ifndef MOE_GEMM_ACCURATE_SILU
#define MOE_GEMM_ACCURATE_SILU 0
#endif
#ifndef MOE_GEMM_EPI_DIRECT
#define MOE_GEMM_EPI_DIRECT 0
#endif
#ifndef MOE_GEMM_NOSTORE
#define MOE_GEMM_NOSTORE 0  // tuning builds only: 1 drops the epilogue's stores
#endif

constexpr int GM_A_BYTES = GM_BM * GM_BK * 2;          // 16 KB
constexpr int GM_BHALF_BYTES = 128 * GM_BK * 2;        // 16 KB
constexpr int GM_STAGE_BYTES = GM_A_BYTES + 2 * GM_BHALF_BYTES;  // 48 KB
constexpr int GM_TMEM_COLS = 512;  // two 256-column fp32 accumulators
constexpr int GM_THREADS = 192;
constexpr int GM_MAX_E = 256;

struct GemmArgs {
    const int32_t* offsets;  // [E+1] permuted-row boundaries per expert
    const int32_t* perm;     // [rows] flat source index t*K+k per permuted row
    __half* out;             // GEMM1: h [rows, I]; GEMM2: expert_out [T*K, H]
    int* err;
    int E;
    int kdim;                // H for GEMM1, I for GEMM2
    int nvalid;              // I for GEMM1, H for GEMM2 (valid output columns)
    int n_tiles;             // N tiles per expert
    int b_rows_per_expert;   // 3I (GEMM1, B view [E*3I, H]) or 3H (GEMM2, B view [E*3H, I])
    int b_seg;               // first B row of the segment inside an expert: 0 or 2H
    int b_nstep;             // B rows advanced per N tile: 128 (GEMM1) or 256 (GEMM2)
    int b_hi_delta;          // row distance of the second B box: I (up rows) or 128
    int out_ld;              // leading dimension of out: I or H
    // MODE_DOWN_PTR only: row r of the tile list goes to row_ptr[r] (a local or a
    // peer GPU's address); when every CTA is done, the last one adds 1 to each
    // *peer_flags[p] (system-scope release) so the owners of those rows know the
    // rows have landed.
    const unsigned long long* row_ptr;
    unsigned int* done_counter;
    unsigned long long* const* peer_flags;
    int npeers;
    // Expert-parallel GEMM1 only (src_flags != nullptr): the A rows arrive from n
    // source ranks while the kernel runs.  Before loading a tile's rows the producer
    // waits (bounded) until every source whose rows the tile covers has raised its
    // flag: src_flags[s] >= src_target.  src_seg[(e*nsrc + s)*3] = {first row, -,
    // rows} of the (local expert e, source s) block of A.
    const unsigned long long* src_flags;
    const int32_t* src_seg;
    int nsrc;
    int src_err_code;
    unsigned long long src_target;
};

// Paired-CTA variant (PAIR=1): a 2-CTA cluster runs one 256-row tile with M=256
// cta_group::2 UMMAs.  Each CTA stages its own 128 rows of A and one half (128
// rows) of the tile's 256 B rows, so every SM reads 32 KB of shared memory per k
// block instead of 48 KB; that leaves room for deeper pipelines.
#ifndef MOE_GEMM_PAIR_STAGES
#define MOE_GEMM_PAIR_STAGES 6
#endif
constexpr int GM_MAX_STAGES = 8;

// Narrow tiles (BN=128, single-CTA, down projection only): one 128-row box of B per
// stage, N=128 UMMAs.  Used when the problem has fewer wide tiles than SMs (few
// rows per launch: expert-parallel ranks, decode); each output element's
// accumulation over k is the same UMMA chain as with wide tiles.
#ifndef MOE_GEMM_NARROW_STAGES
#define MOE_GEMM_NARROW_STAGES 6
#endif

template <int PAIR, int BN = GM_BN>
struct GemmCfg {
    static_assert(BN == GM_BN || (BN == 128 && !PAIR), "narrow tiles are single-CTA only");
    static constexpr int STAGES = PAIR ? MOE_GEMM_PAIR_STAGES : (BN == 128 ? MOE_GEMM_NARROW_STAGES : GM_STAGES);
    static constexpr int STAGE_BYTES =
        PAIR ? GM_A_BYTES + GM_BHALF_BYTES : (BN == 128 ? GM_A_BYTES + GM_BHALF_BYTES : GM_STAGE_BYTES);
    static constexpr int ROWS = PAIR ? 2 * GM_BM : GM_BM;  // rows of one tile (over the pair)
};
static_assert(GemmCfg<0>::STAGES <= GM_MAX_STAGES && GemmCfg<1>::STAGES <= GM_MAX_STAGES &&
                  GemmCfg<0, 128>::STAGES <= GM_MAX_STAGES, "stages");

struct GemmSmemTail {
    uint64_t full[GM_MAX_STAGES];
    uint64_t empty[GM_MAX_STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    int tile_prefix[GM_MAX_E + 1];
};

// Epilogue staging for coalesced stores: per epilogue warp 32 rows x 80 bytes
// (one 32-column fp16 chunk per row, padded by 16 bytes).
constexpr int GM_STG_ROW = 80;
constexpr int GM_STG_BYTES = 4 * 32 * GM_STG_ROW;

template <int PAIR, int BN = GM_BN>
__host__ __device__ constexpr size_t gemm_smem_bytes()
{
    return 1024 + (size_t)GemmCfg<PAIR, BN>::STAGES * GemmCfg<PAIR, BN>::STAGE_BYTES +
           ((sizeof(GemmSmemTail) + 127) & ~(size_t)127) + GM_STG_BYTES;
}
static_assert(gemm_smem_bytes<0>() <= 227 * 1024 && gemm_smem_bytes<1>() <= 227 * 1024 &&
                  gemm_smem_bytes<0, 128>() <= 227 * 1024, "smem");

// Stores one 32-column chunk (64 bytes) of each of the warp's 32 rows.  Each
// thread parks its row's chunk in shared memory (rows padded to 80 bytes so the
// 16-byte pieces of different rows fall in different banks); the warp then reads
// it back transposed so that every store instruction writes 8 whole 64-byte row
// segments (lane l: row 8i + l/4, piece l%4) instead of 32 scattered 16-byte ones.
// dst: this thread's row destination for the chunk (nullptr: row not stored);
// nbytes: valid bytes of the chunk (a multiple of 16), the same for every row.
__device__ __forceinline__ void epi_warp_store(uint8_t* stg_warp, int lane, const uint4 (&v)[4], __half* dst,
                                               int nbytes)
{
#if MOE_GEMM_EPI_DIRECT  // tuning builds: each thread stores its own row's pieces
    if (dst)
        for (int p = 0; p < 4; p++)
            if (p * 16 < nbytes) reinterpret_cast<uint4*>(dst)[p] = v[p];
    return;
#endif
    uint4* mine = reinterpret_cast<uint4*>(stg_warp + lane * GM_STG_ROW);
    mine[0] = v[0];
    mine[1] = v[1];
    mine[2] = v[2];
    mine[3] = v[3];
    __syncwarp();
    const int piece = lane & 3;
    const unsigned long long d = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = 8 * i + (lane >> 2);
        const unsigned long long rd = __shfl_sync(0xffffffffu, d, row);
        const uint4 val = *reinterpret_cast<const uint4*>(stg_warp + row * GM_STG_ROW + piece * 16);
        if (rd != 0ull && piece * 16 < nbytes) *reinterpret_cast<uint4*>(rd + piece * 16) = val;
    }
    __syncwarp();
}

// Maps a tile index to (expert, m tile, n tile); m tiles are `ROWS` rows.  Tile
// indices a CTA visits only grow, so the expert cursor only moves forward.
template <int ROWS>
struct TileCursor {
    int e = 0;
    __device__ __forceinline__ void decode(const int* prefix, const int32_t* offsets, int n_tiles,
                                           int tile, int& e_out, int& mt, int& nt)
    {
        while (tile >= prefix[e + 1]) e++;
        const int cnt = offsets[e + 1] - offsets[e];
        const int mts = (cnt + ROWS - 1) / ROWS;
        const int local = tile - prefix[e];
        nt = local / mts;
        mt = local - nt * mts;
        e_out = e;
    }
};

template <int MODE, int PAIR, int BN>
__global__ void __launch_bounds__(GM_THREADS, 1)
ffn_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const GemmArgs args)
{
    static_assert(BN == GM_BN || MODE != MODE_SWIGLU, "GEMM1 tiles carry 128 gate + 128 up columns");
    using Cfg = GemmCfg<PAIR, BN>;
    constexpr int STAGES = Cfg::STAGES;
    constexpr int STAGE_BYTES = Cfg::STAGE_BYTES;
    constexpr int ROWS = Cfg::ROWS;
    extern __shared__ uint8_t gm_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(gm_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    GemmSmemTail* tail = reinterpret_cast<GemmSmemTail*>(smem + STAGES * STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int E = args.E;
    const int32_t* __restrict__ offsets = args.offsets;
    // Pair mode: rank 0 of the cluster is the leader (issues the UMMAs and owns the
    // barriers the UMMAs wait on); `unit` numbers the pairs.
    const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = crank == 0u;
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int nunits = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(smem_u32(&tail->tfull[a]), 1);
            mbar_init(smem_u32(&tail->tempty[a]), PAIR ? 8 : 4);  // one arrival per epilogue warp
        }
        mbar_init(smem_u32(&tail->drain), 1);
        tail->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    pdl_trigger();
    // offsets, A rows (and perm) come from the previous launches.  Expert-parallel
    // GEMM1 is the exception: it runs alongside the dispatch kernel before it (whose
    // rows it gates on the sources' flags), and its offsets and segment table come
    // from a launch that completed before that kernel started.
    if (!args.src_flags) pdl_wait();
    if (warp == 2) {  // tile prefix: tiles per expert = ceil(rows/ROWS) * n_tiles
        if (lane == 0) {
            int run = 0;
            for (int e = 0; e < E; e++) {
                tail->tile_prefix[e] = run;
                const int cnt = offsets[e + 1] - offsets[e];
                run += ((cnt + ROWS - 1) / ROWS) * args.n_tiles;
            }
            tail->tile_prefix[E] = run;
        }
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(smem_u32(&tail->tmem_base), GM_TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(&tail->tmem_base), GM_TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if (PAIR)
        cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
    else
        __syncthreads();
    tc_fence_after();

    const uint32_t tmem_base = tail->tmem_base;
    const int total_tiles = tail->tile_prefix[E];
    const int nk = (args.kdim + GM_BK - 1) / GM_BK;
    volatile int* abort_flag = &tail->abort_flag;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol_a = l2_policy_evict_last();  // activations: reused by every N tile
#ifndef MOE_GEMM_B_EVICT_FIRST
            const uint64_t pol_b = l2_policy_evict_last();  // weights: shared by the m tiles in flight
#else
            const uint64_t pol_b = l2_policy_evict_first();
#endif
            TileCursor<ROWS> cur;
            uint32_t it = 0;
            bool ok = true;
            uint32_t src_ready = 0;  // sources whose rows have landed (expert-parallel GEMM1)
            for (int tile = unit; ok && tile < total_tiles; tile += nunits) {
                int e, mt, nt;
                cur.decode(tail->tile_prefix, offsets, args.n_tiles, tile, e, mt, nt);
                const int a_row = offsets[e] + mt * ROWS + (int)crank * GM_BM;
                if (args.src_flags) {
                    const int a_end = min(a_row + GM_BM, offsets[e + 1]);
                    for (int sidx = 0; ok && sidx < args.nsrc; sidx++) {
                        if ((src_ready >> sidx) & 1u) continue;
                        const int32_t* g = args.src_seg + 3 * (e * args.nsrc + sidx);
                        const int d0 = g[0], len = g[2];
                        if (len <= 0 || d0 >= a_end || d0 + len <= a_row) continue;
                        if (flag_wait_bounded(args.src_flags + sidx, args.src_target, args.err, args.src_err_code,
                                              abort_flag))
                            src_ready |= 1u << sidx;
                        else
                            ok = false;
                    }
                    if (!ok) break;
                    fence_proxy_async_global();  // the rows were stored by peers' generic stores
                }
                const int b_lo = e * args.b_rows_per_expert + args.b_seg + nt * args.b_nstep;
                const int b_hi = b_lo + args.b_hi_delta;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t par = ((it / STAGES) & 1u) ^ 1u;
                    const bool got = PAIR ? mbar_wait_bounded_cluster(smem_u32(&tail->empty[s]), par, args.err,
                                                                      MOE_DEV_WAIT_TIMEOUT_TMA, abort_flag)
                                          : mbar_wait_bounded(smem_u32(&tail->empty[s]), par, args.err,
                                                              MOE_DEV_WAIT_TIMEOUT_TMA, abort_flag);
                    if (!got) {
                        ok = false;
                        break;
                    }
                    const uint32_t full = smem_u32(&tail->full[s]);
                    uint8_t* st = smem + s * STAGE_BYTES;
                    if (PAIR) {
                        // Both CTAs' copies complete on the leader's barrier; the leader
                        // expects the bytes of both.
                        const uint32_t full_leader = mapa_shared(full, 0);
                        if (leader) mbar_arrive_expect_tx(full, 2 * STAGE_BYTES);
                        tma_load_2d_pair(smem_u32(st), &tmA, full_leader, kb * GM_BK, a_row, pol_a);
                        tma_load_2d_pair(smem_u32(st + GM_A_BYTES), &tmB, full_leader, kb * GM_BK,
                                         leader ? b_lo : b_hi, pol_b);
                    } else {
                        mbar_arrive_expect_tx(full, STAGE_BYTES);
                        tma_load_2d(smem_u32(st), &tmA, full, kb * GM_BK, a_row, pol_a);
                        tma_load_2d(smem_u32(st + GM_A_BYTES), &tmB, full, kb * GM_BK, b_lo, pol_b);
                        if (BN == GM_BN)
                            tma_load_2d(smem_u32(st + GM_A_BYTES + GM_BHALF_BYTES), &tmB, full, kb * GM_BK,
                                        b_hi, pol_b);
                    }
                }
            }
            if (!ok && leader) {
                // Unwinding after a timeout: wait (bounded) until the copies issued into
                // the ring have landed before the CTA exits.  In pair mode the leader's
                // barriers count the copies of both CTAs, and the peer stays resident
                // until the leader reaches the closing cluster barrier.
                const uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
                for (uint32_t j = first; j < it; j++) {
                    const uint64_t t0 = global_timer_ns();
                    while (!(PAIR ? mbar_try_wait_cluster(smem_u32(&tail->full[j % STAGES]), (j / STAGES) & 1u)
                                  : mbar_try_wait(smem_u32(&tail->full[j % STAGES]), (j / STAGES) & 1u)))
                        if (global_timer_ns() - t0 > MOE_WAIT_LIMIT_NS) break;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = umma_idesc_f16_f32(ROWS, BN);
            uint32_t it = 0, lt = 0;
            bool ok = true;
            for (int tile = unit; ok && tile < total_tiles; tile += nunits, lt++) {
                const uint32_t acc = lt & 1u;
                const uint32_t tpar = ((lt >> 1) & 1u) ^ 1u;
                const bool free_acc =
                    PAIR ? mbar_wait_bounded_cluster(smem_u32(&tail->tempty[acc]), tpar, args.err,
                                                     MOE_DEV_WAIT_TIMEOUT_MMA, abort_flag)
                         : mbar_wait_bounded(smem_u32(&tail->tempty[acc]), tpar, args.err, MOE_DEV_WAIT_TIMEOUT_MMA,
                                             abort_flag);
                if (!free_acc) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + acc * GM_BN;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t fpar = (it / STAGES) & 1u;
                    const bool got = PAIR ? mbar_wait_bounded_cluster(smem_u32(&tail->full[s]), fpar, args.err,
                                                                      MOE_DEV_WAIT_TIMEOUT_MMA, abort_flag)
                                          : mbar_wait_bounded(smem_u32(&tail->full[s]), fpar, args.err,
                                                              MOE_DEV_WAIT_TIMEOUT_MMA, abort_flag);
                    if (!got) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * STAGE_BYTES);
                    const uint32_t b_addr = a_addr + GM_A_BYTES;
#pragma unroll
                    for (int k = 0; k < GM_BK / 16; k++) {
                        // advancing K by 16 fp16 = 32 bytes inside the 128-byte swizzle row
                        if (PAIR)
                            umma_f16_ss_pair(d, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                                             idesc, (kb | k) != 0);
                        else
                            umma_f16_ss(d, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                                        idesc, (kb | k) != 0);
                    }
                    // frees the stage (in both CTAs of a pair) when these MMAs finish
                    if (PAIR) {
                        umma_commit_pair(smem_u32(&tail->empty[s]));
                        umma_commit_pair(mapa_shared(smem_u32(&tail->empty[s]), 1));
                    } else {
                        umma_commit(smem_u32(&tail->empty[s]));
                    }
                }
                if (ok) {  // accumulator ready
                    if (PAIR) {
                        umma_commit_pair(smem_u32(&tail->tfull[acc]));
                        umma_commit_pair(mapa_shared(smem_u32(&tail->tfull[acc]), 1));
                    } else {
                        umma_commit(smem_u32(&tail->tfull[acc]));
                    }
                }
            }
            // Make sure no MMA of this CTA (pair) is still running before TMEM is freed.
            if (PAIR)
                umma_commit_pair(smem_u32(&tail->drain));
            else
                umma_commit(smem_u32(&tail->drain));
            const uint64_t t0 = global_timer_ns();
            while (!(PAIR ? mbar_try_wait_cluster(smem_u32(&tail->drain), 0) : mbar_try_wait(smem_u32(&tail->drain), 0)))
                if (global_timer_ns() - t0 > MOE_WAIT_LIMIT_NS) {
                    atomicOr(args.err, MOE_DEV_WAIT_TIMEOUT_MMA);
                    break;
                }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp & 3;            // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;       // row inside this CTA's 128 rows of the tile
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        uint8_t* stg_warp = smem + STAGES * STAGE_BYTES + ((sizeof(GemmSmemTail) + 127) & ~(size_t)127) +
                            (size_t)(warp - 2) * 32 * GM_STG_ROW;
        // In pair mode every epilogue warp of both CTAs releases the leader's accumulator.
        const uint32_t tempty_bar0 = PAIR ? mapa_shared(smem_u32(&tail->tempty[0]), 0) : smem_u32(&tail->tempty[0]);
        TileCursor<ROWS> cur;
        uint32_t lt = 0;
        for (int tile = unit; tile < total_tiles; tile += nunits, lt++) {
            int e, mt, nt;
            cur.decode(tail->tile_prefix, offsets, args.n_tiles, tile, e, mt, nt);
            const uint32_t acc = lt & 1u;
            const uint32_t tpar = (lt >> 1) & 1u;
            const bool ready = PAIR ? mbar_wait_bounded_cluster(smem_u32(&tail->tfull[acc]), tpar, args.err,
                                                                MOE_DEV_WAIT_TIMEOUT_EPI, abort_flag)
                                    : mbar_wait_bounded(smem_u32(&tail->tfull[acc]), tpar, args.err,
                                                        MOE_DEV_WAIT_TIMEOUT_EPI, abort_flag);
            if (!ready) break;
            tc_fence_after();
            const int row0 = offsets[e] + mt * ROWS + (int)crank * GM_BM;
            const int rows = min(GM_BM, offsets[e + 1] - row0);  // <= 0: this CTA's half is empty
            const bool valid = r < rows;
            const uint32_t tbase = tmem_base + acc * GM_BN + lane_off;
            if (MODE == MODE_SWIGLU) {
                const int col0 = nt * 128;
                __half* dst = valid ? args.out + (size_t)(row0 + r) * args.out_ld + col0 : nullptr;
#pragma unroll 1
                for (int j = 0; j < 4; j++) {
                    uint32_t g[32], u[32];
                    tmem_ld_32x32b_x32(tbase + j * 32, g);
                    tmem_ld_32x32b_x32(tbase + 128 + j * 32, u);
                    tmem_ld_wait();
                    {
                        uint32_t pk[16];
#pragma unroll
                        for (int c = 0; c < 16; c++) {
                            const float g0 = __uint_as_float(g[2 * c]), g1 = __uint_as_float(g[2 * c + 1]);
                            const float u0 = __uint_as_float(u[2 * c]), u1 = __uint_as_float(u[2 * c + 1]);
                            // silu(g) = g / (1 + exp(-g)), tests/moe_cpu_sim.cpp:155-158.  The
                            // fast exp / divide intrinsics err by ~1e-6 relative, far below
                            // the fp16 rounding (~5e-4) that h gets next.
#if MOE_GEMM_ACCURATE_SILU
                            const float h0 = g0 / (1.0f + expf(-g0)) * u0;
                            const float h1 = g1 / (1.0f + expf(-g1)) * u1;
#else
                            const float h0 = __fdividef(g0 * u0, 1.0f + __expf(-g0));
                            const float h1 = __fdividef(g1 * u1, 1.0f + __expf(-g1));
#endif
                            pk[c] = pack_half2(h0, h1);
                        }
                        const int cb = col0 + j * 32;
                        const int nb = min(32, args.nvalid - cb) * 2;
                        const uint4 vv[4] = {make_uint4(pk[0], pk[1], pk[2], pk[3]), make_uint4(pk[4], pk[5], pk[6], pk[7]),
                                             make_uint4(pk[8], pk[9], pk[10], pk[11]),
                                             make_uint4(pk[12], pk[13], pk[14], pk[15])};
                        if (nb > 0 && !MOE_GEMM_NOSTORE)
                            epi_warp_store(stg_warp, lane, vv, valid ? dst + j * 32 : nullptr, nb);
                    }
                }
            } else {
                const int col0 = nt * BN;
                __half* dst = nullptr;
                if (valid) {
                    if (MODE == MODE_DOWN_PTR)
                        dst = reinterpret_cast<__half*>(args.row_ptr[row0 + r]) + col0;
                    else
                        dst = args.out + (size_t)args.perm[row0 + r] * args.out_ld + col0;
                }
#pragma unroll 1
                for (int j = 0; j < BN / 32; j++) {
                    uint32_t v32[32];
                    tmem_ld_32x32b_x32(tbase + j * 32, v32);
                    tmem_ld_wait();
                    if (!MOE_GEMM_NOSTORE) {  // warp-collective: local rows or peer rows alike
                        const int cb = col0 + j * 32;
                        const int nb = min(32, args.nvalid - cb) * 2;
                        uint4 vv[4];
#pragma unroll
                        for (int v = 0; v < 4; v++) {
                            vv[v].x = pack_half2(__uint_as_float(v32[8 * v + 0]), __uint_as_float(v32[8 * v + 1]));
                            vv[v].y = pack_half2(__uint_as_float(v32[8 * v + 2]), __uint_as_float(v32[8 * v + 3]));
                            vv[v].z = pack_half2(__uint_as_float(v32[8 * v + 4]), __uint_as_float(v32[8 * v + 5]));
                            vv[v].w = pack_half2(__uint_as_float(v32[8 * v + 6]), __uint_as_float(v32[8 * v + 7]));
                        }
                        if (nb > 0) epi_warp_store(stg_warp, lane, vv, valid ? dst + j * 32 : nullptr, nb);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                const uint32_t bar = tempty_bar0 + acc * (uint32_t)sizeof(uint64_t);
                if (PAIR)
                    mbar_arrive_cluster(bar);
                else
                    mbar_arrive(bar);
            }
        }
    }

    if (MODE == MODE_DOWN_PTR) __threadfence_system();  // this thread's (peer) row stores
    // Pair mode: neither CTA frees TMEM or exits while the other may still address it.
    __syncwarp();
    if (PAIR)
        cluster_sync_all();
    else
        __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if (PAIR)
            tmem_dealloc_pair(tmem_base, GM_TMEM_COLS);
        else
            tmem_dealloc(tmem_base, GM_TMEM_COLS);
    }
    if (MODE == MODE_DOWN_PTR && threadIdx.x == 0) {
        __threadfence_system();
        const unsigned int old = atomicAdd(args.done_counter, 1u);
        if (old == gridDim.x - 1) {  // last CTA: every row of this launch is stored
            *reinterpret_cast<volatile unsigned int*>(args.done_counter) = 0u;
            __threadfence_system();
            for (int p = 0; p < args.npeers; p++) atomicAdd_system(args.peer_flags[p], 1ull);
        }
    }
}

// ---------------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D fp16 tensor [rows, inner] (inner contiguous), 64 x 128 boxes, 128-byte swizzle,
// zero fill outside the tensor.
static bool make_tmap(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t rows)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {GM_BK, 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                     es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

static int sm_count()
{
    static int n[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!n[dev]) {
        cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
        if (n[dev] <= 0) n[dev] = 148;
    }
    return n[dev];
}

template <int MODE, int PAIR, int BN>
static cudaError_t set_gemm_attr()
{
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(ffn_gemm_kernel<MODE, PAIR, BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)gemm_smem_bytes<PAIR, BN>());
    if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
    return e;
}

int grid_for(int rows_cap, int E, int n_tiles, int max_ctas)
{
    long long upper = (long long)n_tiles * ((rows_cap + GM_BM - 1) / GM_BM + E);
    int sms = sm_count();
    if (max_ctas > 0 && max_ctas < sms) sms = max_ctas;
    return (int)(upper < sms ? (upper > 0 ? upper : 1) : sms);
}

// Paired-CTA tiles pay off when experts hold many 256-row tiles: the pair halves
// each SM's shared-memory traffic, but an expert's rows are padded to 256 instead
// of 128.  MOE_GEMM_PAIR=0/1 forces the choice; otherwise pairs are used from
// 1536 rows per expert on average (measured: faster at 1536 and 2048 rows per
// expert, slower at 512).
static bool use_pair(int rows_cap, int E)
{
    static int forced = -2;
    if (forced == -2) {
        const char* v = getenv("MOE_GEMM_PAIR");
        forced = (v && (v[0] == '0' || v[0] == '1')) ? v[0] - '0' : -1;
    }
    if (forced >= 0) return forced == 1;
    return E > 0 && rows_cap / E >= 1536;
}

template <int MODE, int PAIR, int BN = GM_BN>
static cudaError_t launch_ffn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int rows_cap,
                              int max_ctas, bool pdl, cudaStream_t s)
{
    cudaError_t e = set_gemm_attr<MODE, PAIR, BN>();
    if (e != cudaSuccess) return e;
    int grid;
    if (PAIR) {
        constexpr int R = GemmCfg<1>::ROWS;
        const long long upper = (long long)a.n_tiles * ((rows_cap + R - 1) / R + a.E);
        // Co-resident pairs: a pair needs two free SMs of one GPC, so GPCs with an odd
        // number of usable SMs leave one idle; a grid of sms/2 pairs would run a tail.
        static int resident[64] = {0};
        int dev = 0;
        cudaGetDevice(&dev);
        int pairs_cap = (dev >= 0 && dev < 64) ? resident[dev] : 0;
        if (pairs_cap <= 0) {
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3(2 * (sm_count() / 2));
            q.blockDim = dim3(GM_THREADS);
            q.dynamicSmemBytes = gemm_smem_bytes<PAIR, BN>();
            cudaLaunchAttribute ca;
            ca.id = cudaLaunchAttributeClusterDimension;
            ca.val.clusterDim.x = 2;
            ca.val.clusterDim.y = 1;
            ca.val.clusterDim.z = 1;
            q.attrs = &ca;
            q.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, ffn_gemm_kernel<MODE, PAIR, BN>, &q) != cudaSuccess || n <= 0) {
                cudaGetLastError();
                n = sm_count() / 2;
            }
            if (getenv("MOE_GEMM_PAIR_DEBUG")) fprintf(stderr, "moe: %d co-resident CTA pairs\n", n);
            pairs_cap = n;
            if (dev >= 0 && dev < 64) resident[dev] = n;
        }
        if (max_ctas > 0 && max_ctas / 2 < pairs_cap) pairs_cap = max_ctas / 2;
        if (pairs_cap < 1) pairs_cap = 1;
        grid = 2 * (int)(upper < pairs_cap ? (upper > 0 ? upper : 1) : pairs_cap);
    } else {
        grid = grid_for(rows_cap, a.E, a.n_tiles, max_ctas);
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(grid);
    lc.blockDim = dim3(GM_THREADS);
    lc.dynamicSmemBytes = gemm_smem_bytes<PAIR, BN>();
    lc.stream = s;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (PAIR) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = 2;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        na++;
    }
    lc.attrs = at;
    lc.numAttrs = na;
    e = cudaLaunchKernelEx(&lc, ffn_gemm_kernel<MODE, PAIR, BN>, ta, tb, a);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <int MODE>
static cudaError_t launch_ffn_any(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int rows_cap,
                                  int rows_hint, int max_ctas, bool pdl, cudaStream_t s)
{
    if (use_pair(rows_hint >= 0 ? rows_hint : rows_cap, a.E)) return launch_ffn<MODE, 1>(ta, tb, a, rows_cap, max_ctas, pdl, s);
    return launch_ffn<MODE, 0>(ta, tb, a, rows_cap, max_ctas, pdl, s);
}

// Down projection: narrow (BN=128) tiles when all of them fit in one wave (twice the
// wide tiles <= SMs), i.e. when the wide tiles would leave half the SMs idle.
// Measured (one B200): 2 experts x 512 rows, H=2048, I=8192: 53 us narrow against
// 64 us wide; 4 experts x 512 rows (two narrow waves): 96 against 68; decode (16
// experts x 16 rows, HBM-bound): 110 against 106.  rows: the expected permuted
// rows; the m tiles are estimated as rows/128 plus half a tail tile per expert.
// MOE_GEMM_DOWN_BN=128/256 forces the width.
static bool use_narrow_down(int rows, int E, int H, bool pair)
{
    static int forced = -1;
    if (forced == -1) {
        const char* v = getenv("MOE_GEMM_DOWN_BN");
        forced = v ? atoi(v) : 0;
    }
    if (forced == 128) return true;
    if (forced == 256 || pair) return false;
    const long long wide = (long long)((H + GM_BN - 1) / GM_BN) * (rows / GM_BM + (E + 1) / 2);
    return 2 * wide <= sm_count();
}

template <int MODE>
static cudaError_t launch_down_any(const CUtensorMap& ta, const CUtensorMap& tb, GemmArgs a, int rows_cap, int rows_hint, bool allow_pair, int max_ctas,
                                   bool pdl, cudaStream_t s)
{
    const int rows = rows_hint >= 0 ? rows_hint : rows_cap;
    const bool pair = allow_pair && use_pair(rows, a.E);
    if (!pair && use_narrow_down(rows, a.E, a.nvalid, false)) {
        a.n_tiles = (a.nvalid + 127) / 128;
        a.b_nstep = 128;
        return launch_ffn<MODE, 0, 128>(ta, tb, a, rows_cap, max_ctas, pdl, s);
    }
    if (pair) return launch_ffn<MODE, 1>(ta, tb, a, rows_cap, max_ctas, pdl, s);
    return launch_ffn<MODE, 0>(ta, tb, a, rows_cap, max_ctas, pdl, s);
}

// GEMM1: h[rows, I] = SwiGLU(xp @ [Wg; Wu]^T) per expert.
cudaError_t launch_gemm_swiglu(const __half* xp, const __half* expert_weights, const int32_t* offsets,
                               __half* h, int* err, int rows_cap, int H, int E, int I, int max_ctas,
                               cudaStream_t s, int rows_hint, const SourceWait* src)
{
    CUtensorMap ta, tb;
    if (!make_tmap(&ta, xp, (uint64_t)H, (uint64_t)(rows_cap > 0 ? rows_cap : 1)) ||
        !make_tmap(&tb, expert_weights, (uint64_t)H, (uint64_t)E * 3 * I))
        return cudaErrorInvalidValue;
    GemmArgs a = {};
    a.offsets = offsets;
    a.perm = nullptr;
    a.out = h;
    a.err = err;
    a.E = E;
    a.kdim = H;
    a.nvalid = I;
    a.n_tiles = (I + 127) / 128;
    a.b_rows_per_expert = 3 * I;
    a.b_seg = 0;
    a.b_nstep = 128;
    a.b_hi_delta = I;
    a.out_ld = I;
    if (src) {
        if (src->nsrc < 1 || src->nsrc > 32) return cudaErrorInvalidValue;
        a.src_flags = src->flags;
        a.src_seg = src->seg;
        a.nsrc = src->nsrc;
        a.src_err_code = src->err_code;
        a.src_target = src->target;
    }
    return launch_ffn_any<MODE_SWIGLU>(ta, tb, a, rows_cap, rows_hint, max_ctas, true, s);
}

// GEMM2: expert_out[perm[r], :] = h[r, :] @ Wd^T per expert.
cudaError_t launch_gemm_down(const __half* h, const __half* expert_weights, const int32_t* offsets,
                             const int32_t* perm, __half* expert_out, int* err, int rows_cap, int H,
                             int E, int I, int max_ctas, cudaStream_t s, int rows_hint, bool allow_pair)
{
    CUtensorMap ta, tb;
    if (!make_tmap(&ta, h, (uint64_t)I, (uint64_t)(rows_cap > 0 ? rows_cap : 1)) ||
        !make_tmap(&tb, expert_weights, (uint64_t)I, (uint64_t)E * 3 * H))
        return cudaErrorInvalidValue;
    GemmArgs a = {};
    a.offsets = offsets;
    a.perm = perm;
    a.out = expert_out;
    a.err = err;
    a.E = E;
    a.kdim = I;
    a.nvalid = H;
    a.n_tiles = (H + GM_BN - 1) / GM_BN;
    a.b_rows_per_expert = 3 * H;
    a.b_seg = 2 * H;
    a.b_nstep = GM_BN;
    a.b_hi_delta = 128;
    a.out_ld = H;
    return launch_down_any<MODE_DOWN>(ta, tb, a, rows_cap, rows_hint, allow_pair, max_ctas, true, s);
}

}  // namespace moe

namespace moe {

// GEMM2 with a per-row destination pointer table and a completion signal to peers
// (the expert-parallel return path: rows go straight into the source ranks' memory).
cudaError_t launch_gemm_down_ptr(const __half* h, const __half* expert_weights, const int32_t* offsets,
                                 const unsigned long long* row_ptr, unsigned int* done_counter,
                                 unsigned long long* const* peer_flags, int npeers, int* err, int rows_cap,
                                 int H, int E, int I, cudaStream_t s, int rows_hint, bool allow_pair)
{
    CUtensorMap ta, tb;
    if (!make_tmap(&ta, h, (uint64_t)I, (uint64_t)(rows_cap > 0 ? rows_cap : 1)) ||
        !make_tmap(&tb, expert_weights, (uint64_t)I, (uint64_t)E * 3 * H))
        return cudaErrorInvalidValue;
    GemmArgs a = {};
    a.offsets = offsets;
    a.err = err;
    a.E = E;
    a.kdim = I;
    a.nvalid = H;
    a.n_tiles = (H + GM_BN - 1) / GM_BN;
    a.b_rows_per_expert = 3 * H;
    a.b_seg = 2 * H;
    a.b_nstep = GM_BN;
    a.b_hi_delta = 128;
    a.out_ld = H;
    a.row_ptr = row_ptr;
    a.done_counter = done_counter;
    a.peer_flags = peer_flags;
    a.npeers = npeers;
    return launch_down_any<MODE_DOWN_PTR>(ta, tb, a, rows_cap, rows_hint, allow_pair, 0, false, s);
}

}  // namespace moe
