// ep.cu -- the MoE layer expert-parallel over n GPUs.
//
// The reference runs on one device (tests/test_moe.cpp:642-648); the benchmark
// definition asks for the layer partitioned expert-parallel across the GPUs of a
// box.  Rank r owns experts [r*El, (r+1)*El), El = E/n, and routes its own tokens.
//
// Peer-memory path (default, one process per GPU, n <= 8; no host synchronisation):
//   1. routing + stable counting sort of this rank's (token, slot) pairs by expert
//      (experts are owned contiguously, so expert order is also owner order);
//   2. per-expert counts stored into every peer's inbox, then a device-side plan
//      once every source's counts are in;
//   3. fused gather + dispatch: each row goes from x straight into its owner's
//      inbox over NVLink; GEMM1 (gate/up + SwiGLU) runs alongside it, each tile
//      waiting only for the sources whose rows it covers;
//   4. GEMM2 (down) stores every output row straight into its source rank's
//      return inbox and raises this owner's flag there;
//   5. combine on arrival: tokens whose owners have all returned their rows first.
// NCCL path (fallback, or MOE_EP_FORCE_NCCL=1): counts exchange with one bounded
// host wait, grouped ncclSend/ncclRecv dispatch and return, an expert-major reorder,
// the same GEMMs, combine through the inverse permutation.
// Every kernel computes each row exactly as the single-GPU path does, so each row
// of y is bit-identical to MoeLayerForward on the same tokens with all experts.
// No kernel reads peer memory with TMA or with cluster multicast: remote data is
// written with plain stores and read from local HBM.
//
// Failure handling: the communicator is non-blocking; every host wait (communicator
// set-up, group completion, the counts event) polls against a deadline and aborts
// the communicator on timeout, returning MOE_ERR_TIMEOUT instead of hanging.  Every
// device wait on a peer's flag is bounded and records an error bit.
#include <nccl.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <thread>
#include <vector>

#include "../../include/moe_ops.h"
#include "moe_common.cuh"
#include "moe_kernels.h"

struct EpPeersHost;
struct MoeEpContext {
    ncclComm_t comm = nullptr;
    int rank = 0, nranks = 1, device = 0;
    int timeout_ms = 60000;
    bool broken = false;  // a wait timed out or NCCL failed: only MoeEpDestroy is valid
    cudaEvent_t counts_ready = nullptr;
    int32_t* host = nullptr;  // pinned: offsets [E+1], recv counts [n*El], plan tables
    size_t host_ints = 0;
    // peer-memory path (process-per-GPU, up to 8 ranks): IPC-shared inboxes
    int p2p_state = 0;  // 0 not tried, 1 ready, -1 unavailable (NCCL path)
    int64_t p2p_T = 0, p2p_H = 0, p2p_E = 0, p2p_K = 0, p2p_R = 0;
    void* p2p_base = nullptr;      // this rank's allocation
    void* p2p_peer[8] = {};        // opened peer allocations (p2p_peer[rank] = p2p_base)
    void* p2p_dev_peers = nullptr; // device copy of the peer pointer table
    size_t off_cnt = 0, off_rows = 0, off_ret = 0, off_flags = 0;
    unsigned long long epoch = 0;
};

namespace {

using clk = std::chrono::steady_clock;

int check_nccl(MoeEpContext* c, ncclResult_t r)
{
    if (r == ncclSuccess || r == ncclInProgress) return MOE_OK;
    c->broken = true;
    return MOE_ERR_NCCL;
}

// Polls the communicator until no operation is in progress, or the deadline.
int wait_comm(MoeEpContext* c, clk::time_point deadline)
{
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = ncclCommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) {
            c->broken = true;
            return MOE_ERR_NCCL;
        }
        if (st == ncclSuccess) return MOE_OK;
        if (st != ncclInProgress) {
            c->broken = true;
            return MOE_ERR_NCCL;
        }
        if (clk::now() > deadline) {
            ncclCommAbort(c->comm);
            c->comm = nullptr;
            c->broken = true;
            return MOE_ERR_TIMEOUT;
        }
        std::this_thread::yield();  // enqueue completes in microseconds: spin, do not sleep
    }
}

// Waits for a CUDA event while watching the communicator for asynchronous errors.
int wait_event(MoeEpContext* c, cudaEvent_t ev, clk::time_point deadline)
{
    for (;;) {
        cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) return MOE_OK;
        if (q != cudaErrorNotReady) return MOE_ERR_CUDA;
        ncclResult_t st = ncclSuccess;
        if (ncclCommGetAsyncError(c->comm, &st) != ncclSuccess ||
            (st != ncclSuccess && st != ncclInProgress)) {
            c->broken = true;
            return MOE_ERR_NCCL;
        }
        if (clk::now() > deadline) {
            ncclCommAbort(c->comm);
            c->comm = nullptr;
            c->broken = true;
            return MOE_ERR_TIMEOUT;
        }
        std::this_thread::yield();
    }
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }
constexpr int kChunk = 1024;  // permutation chunk (permute.cu)

struct EpLayout {
    size_t err, chunk_counts, chunk_base, offsets, perm, dest, ids, weights, sendcnt, recvcnt,
        expoff, seg, row_src, xp, recv, xr, h, tile_counts, tile_rank, total;
};

// Row hint passed to the grouped GEMM launchers: 0 keeps the expert-parallel GEMMs
// on single-CTA tiles.  Paired tiles measured 3% slower here (4 GPUs, prefill
// shape, about 2048 rows per local expert), although they win on one GPU at that size.
constexpr int kEpRowsHint = 0;

EpLayout ep_layout(int n, int64_t T, int64_t H, int64_t E, int64_t K, int64_t I, int64_t R)
{
    EpLayout L;
    const int64_t TK = T * K > 0 ? T * K : 1;
    const int64_t nch = (T * K + kChunk - 1) / kChunk > 0 ? (T * K + kChunk - 1) / kChunk : 1;
    const int64_t El = E / n;
    const int64_t Rr = R > 0 ? R : 1;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t at = o;
        o += align_up(bytes);
        return at;
    };
    L.err = take(16);
    L.chunk_counts = take(4 * (size_t)nch * E);
    L.chunk_base = take(4 * (size_t)nch * E);
    L.offsets = take(4 * (size_t)(E + 1));
    L.perm = take(4 * (size_t)TK);
    L.dest = take(4 * (size_t)TK);
    L.ids = take(4 * (size_t)TK);
    L.weights = take(2 * (size_t)TK);
    L.sendcnt = take(4 * (size_t)n * El);
    L.recvcnt = take(4 * (size_t)n * El);
    L.expoff = take(4 * (size_t)(El + 1));
    L.seg = take(4 * 3 * (size_t)n * El);
    L.row_src = take(4 * (size_t)Rr);
    L.xp = take(2 * (size_t)TK * H);    // permuted rows out; later the returned rows (ret)
    L.recv = take(2 * (size_t)Rr * H);  // received rows; later GEMM2's output (eo)
    L.xr = take(2 * (size_t)Rr * H);    // received rows, expert-major
    L.h = take(2 * (size_t)Rr * I);
    L.tile_counts = take(4 * (size_t)(moe::routing_tiles((int)T) > 0 ? moe::routing_tiles((int)T) : 1) * E);
    L.tile_rank = take(4 * (size_t)TK);
    L.total = o;
    return L;
}

template <class T>
T* at(void* base, size_t off)
{
    return reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off);
}

// sendcnt[r*El+e] = offsets[r*El+e+1] - offsets[r*El+e]
__global__ void ep_send_counts_kernel(const int32_t* __restrict__ offsets, int nE,
                                      int32_t* __restrict__ sendcnt)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nE; i += gridDim.x * blockDim.x)
        sendcnt[i] = offsets[i + 1] - offsets[i];
}

// row_src[dst + i] = src + i for each (expert, source) segment (one block each)
__global__ void ep_row_map_kernel(const int32_t* __restrict__ seg, int nseg, int32_t* __restrict__ row_src)
{
    for (int sgi = blockIdx.x; sgi < nseg; sgi += gridDim.x) {
        const int dst = seg[3 * sgi], src = seg[3 * sgi + 1], len = seg[3 * sgi + 2];
        for (int i = threadIdx.x; i < len; i += blockDim.x) row_src[dst + i] = src + i;
    }
}


// ============================================================================ peer-memory path
// One allocation per rank, shared with the peers through CUDA IPC:
//   flags [32] u64       per-source epoch counters, each raised by one rank once per
//                        call: [s] counts of source s are in, [8+s] rows of source s
//                        have landed, [16+o] owner o's returned rows have landed;
//                        [24]/[25]: local completion counters (u32) of the dispatch
//                        kernel and the down GEMM
//   cnt   [2][n][E] int32  row s of buffer (call & 1): source s's per-expert counts
//   rows  [R][H] fp16    rows for this rank's experts, expert-major (written by sources)
//   ret   [T*K][H] fp16  this rank's rows back from their experts, in permuted order
// Call c waits for flag >= c.  A counter only grows, and it is per source, so a fast
// rank's call c+1 never satisfies a wait for a slow rank's call c.  The counts are
// double-buffered by call parity: a rank can run one call ahead of a peer's plan
// (its combine waits only for the owners its own tokens used), never two, because
// its next plan needs that peer's next counts.
constexpr int EP_MAX_PEERS = 8;
constexpr int F_CNT = 0, F_ROWS = 8, F_RET = 16, F_DONE1 = 24, F_DONE2 = 25, F_WORDS = 32;

struct EpPeers {
    int32_t* cnt[EP_MAX_PEERS];
    __half* rows[EP_MAX_PEERS];
    __half* ret[EP_MAX_PEERS];
    unsigned long long* flags[EP_MAX_PEERS];
    unsigned long long* ret_flag[EP_MAX_PEERS];  // &flags[p][F_RET + me], for the GEMM2 signal
};

enum EpDevError { EP_ERR_WAIT_COUNTS = 64, EP_ERR_WAIT_ROWS = 128, EP_ERR_WAIT_RET = 256, EP_ERR_OVERFLOW = 512 };

// Bounded wait (one thread) until *flag >= target; on timeout records `code`.
__device__ bool ep_wait_flag(const unsigned long long* flag, unsigned long long target, int* err, int code)
{
    return moe::flag_wait_bounded(flag, target, err, code, nullptr);
}

// Counts exchange and plan in one block.  First this rank's per-expert counts go
// into row `me` of buffer `par` of every peer's cnt inbox, and its counts flag is
// raised there; then, once every source's counts are in:
// for each global expert e the row in its owner's inbox where this rank's rows
// start (disp_base[e]); this rank's expert-major offsets (expoff[El+1]); for each
// (local expert, source) {first inbox row, row index in the source's permuted
// order, rows} (seg); and the return address of every inbox row (row_ptr: the
// source's ret inbox, at the row's index in the source's permuted order).
__global__ void __launch_bounds__(256)
ep_p2p_plan_kernel(const EpPeers* __restrict__ peers, const int32_t* __restrict__ offsets,
                   const int32_t* __restrict__ cnt_all, const unsigned long long* flags, int E, int El, int me,
                   int n, int par, int R, int H, unsigned long long target, int* err,
                   int32_t* __restrict__ disp_base, int32_t* __restrict__ expoff, int32_t* __restrict__ seg,
                   int32_t* __restrict__ overflow, unsigned long long* __restrict__ row_ptr)
{
    __shared__ int ok;
    __shared__ int over;
    extern __shared__ int32_t pl_tot[];  // [E] rows per global expert over all sources
    for (int p = 0; p < n; p++)
        for (int e = threadIdx.x; e < E; e += blockDim.x)
            peers->cnt[p][((size_t)par * n + me) * E + e] = offsets[e + 1] - offsets[e];
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < n) {
        __threadfence_system();
        atomicAdd_system(&peers->flags[threadIdx.x][F_CNT + me], 1ull);
    }
    if (threadIdx.x == 0) {
        int good = 1;
        for (int s = 0; s < n && good; s++) good = ep_wait_flag(&flags[F_CNT + s], target, err, EP_ERR_WAIT_COUNTS);
        ok = good;
        over = 0;
    }
    __syncthreads();
    const int32_t* cnt = cnt_all + (size_t)par * n * E;
    if (!ok) {  // counts never arrived: plan nothing, move nothing
        for (int i = threadIdx.x; i <= El; i += blockDim.x) expoff[i] = 0;
        for (int i = threadIdx.x; i < El * n; i += blockDim.x) seg[3 * i + 2] = 0;
        if (threadIdx.x == 0) *overflow = 1;
        return;
    }
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int t = 0;
        for (int s = 0; s < n; s++) t += cnt[s * E + e];
        pl_tot[e] = t;
    }
    __syncthreads();
    // per owner p: expert-major prefix over its experts; capacity check
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        long long run = 0;
        for (int el = 0; el < El; el++) {
            const int e = p * El + el;
            long long before = 0;
            for (int s = 0; s < me; s++) before += cnt[s * E + e];
            disp_base[e] = (int32_t)(run + before);
            if (p == me) expoff[el] = (int32_t)run;
            run += pl_tot[e];
        }
        if (p == me) expoff[El] = (int32_t)run;
        if (run > R) atomicOr(&over, 1);
    }
    __syncthreads();
    if (over) {
        if (threadIdx.x == 0) {
            atomicOr(err, EP_ERR_OVERFLOW);
            *overflow = 1;
        }
        for (int i = threadIdx.x; i <= El; i += blockDim.x) expoff[i] = 0;
        for (int i = threadIdx.x; i < El * n; i += blockDim.x) seg[3 * i + 2] = 0;
        return;
    }
    if (threadIdx.x == 0) *overflow = 0;
    for (int i = threadIdx.x; i < El * n; i += blockDim.x) {
        const int el = i / n, s = i - el * n;
        const int e = me * El + el;
        long long d0 = 0;
        for (int s2 = 0; s2 < s; s2++) d0 += cnt[s2 * E + e];
        long long rb = 0;
        for (int e2 = 0; e2 < e; e2++) rb += cnt[s * E + e2];
        seg[3 * i] = expoff[el] + (int32_t)d0;  // expoff written above by the same block
        seg[3 * i + 1] = (int32_t)rb;
        seg[3 * i + 2] = cnt[s * E + e];
    }
    __syncthreads();
    for (int i = 0; i < El * n; i++) {  // return address of every inbox row
        const int s = i % n;
        const int d0 = seg[3 * i], rb = seg[3 * i + 1], len = seg[3 * i + 2];
        __half* base = peers->ret[s];
        for (int j = threadIdx.x; j < len; j += blockDim.x)
            row_ptr[d0 + j] = reinterpret_cast<unsigned long long>(base + (size_t)(rb + j) * H);
    }
}

// Fused gather + dispatch: row r of this rank's permuted order (expert e) goes from
// x[perm[r]/K] straight to its owner's inbox row disp_base[e] + (r - offsets[e]),
// over NVLink for remote owners.  The last block to finish raises this rank's
// rows flag at every peer.  It lets the GEMM1 launch after it start at once (that
// kernel reads the rows only behind their flags) and runs on a small grid, so the
// GEMM1 CTAs fit on the SMs beside its blocks.
__global__ void __launch_bounds__(256)
ep_p2p_dispatch_kernel(const __half* __restrict__ x, const int32_t* __restrict__ perm,
                       const int32_t* __restrict__ offsets, const int32_t* __restrict__ disp_base,
                       const int32_t* __restrict__ overflow, const EpPeers* __restrict__ peers, int TK, int E,
                       int El, int K, int H, int me, int n, unsigned int* done)
{
    moe::pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int nv = H >> 3;
    if (!*overflow) {
        for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < TK; r += gridDim.x * 8) {
            int lo = 0, hi = E;  // expert e with offsets[e] <= r < offsets[e+1]
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (offsets[mid] <= r) lo = mid; else hi = mid;
            }
            const int e = lo;
            const int p = e / El;
            const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(perm[r] / K) * H);
            uint4* dst = reinterpret_cast<uint4*>(peers->rows[p] + (size_t)(disp_base[e] + r - offsets[e]) * H);
            // all of a lane's loads of a chunk first, then its stores: one memory latency
            // per 4 KB of row instead of one per 16 bytes (the grid is small by design)
            constexpr int VPL = 8;
            for (int v0 = lane; v0 < nv; v0 += 32 * VPL) {
                uint4 buf[VPL];
#pragma unroll
                for (int u = 0; u < VPL; u++)
                    if (v0 + 32 * u < nv) buf[u] = __ldg(src + v0 + 32 * u);
#pragma unroll
                for (int u = 0; u < VPL; u++)
                    if (v0 + 32 * u < nv) dst[v0 + 32 * u] = buf[u];
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned int old = atomicAdd(done, 1u);
        if (old == gridDim.x - 1) {
            *reinterpret_cast<volatile unsigned int*>(done) = 0u;
            __threadfence_system();
            for (int p = 0; p < n; p++) atomicAdd_system(&peers->flags[p][F_ROWS + me], 1ull);
        }
    }
}

// Waits (bounded) until *flag >= target (the failure-detection self-test).
__global__ void ep_p2p_wait_kernel(const unsigned long long* flag, unsigned long long target, int* err, int code)
{
    if (threadIdx.x == 0) ep_wait_flag(flag, target, err, code);
}

// Combine on arrival.  Block b owns tokens [b*CH, b*CH+CH).  Slot (t,k) comes back
// from owner ids[t,k]/El, whose rows are all in once ret_flags[owner] >= target.
// Two phases, each spread over all the block's threads: first the tokens whose
// owners have all signalled, then -- after one thread has waited (bounded) for the
// missing owners -- the rest; so tokens that do not need a slow owner are not held
// up by it.  Each token is the same fp32 sum in slot order as
// combine_indexed_kernel (tests/moe_cpu_sim.cpp:298-305), so y is bit-identical.
constexpr int EP_COMBINE_CH = 8;

__device__ __forceinline__ void ep_combine_vec(const __half* __restrict__ ret, const int32_t* __restrict__ dest,
                                               const __half* __restrict__ weights, __half* __restrict__ y, int t,
                                               int c, int H, int K)
{
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; q++) acc[q] = 0.0f;
    for (int k = 0; k < K; k++) {
        const float w = __half2float(weights[(size_t)t * K + k]);
        const int r = dest[(size_t)t * K + k];
        const uint4 qv = __ldcg(reinterpret_cast<const uint4*>(ret + (size_t)r * H + c));  // stored by peers
        const __half2* q2 = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float2 f = __half22float2(q2[q]);
            acc[2 * q] = fmaf(w, f.x, acc[2 * q]);
            acc[2 * q + 1] = fmaf(w, f.y, acc[2 * q + 1]);
        }
    }
    uint4 o;
    o.x = moe::pack_half2(acc[0], acc[1]);
    o.y = moe::pack_half2(acc[2], acc[3]);
    o.z = moe::pack_half2(acc[4], acc[5]);
    o.w = moe::pack_half2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(y + (size_t)t * H + c) = o;
}

__global__ void __launch_bounds__(256)
ep_combine_arrival_kernel(const __half* __restrict__ ret, const int32_t* __restrict__ dest,
                          const int32_t* __restrict__ ids, const __half* __restrict__ weights,
                          __half* __restrict__ y, int T, int H, int K, int El, int n,
                          const unsigned long long* ret_flags, unsigned long long target, int* err)
{
    __shared__ uint32_t need[EP_COMBINE_CH];
    __shared__ int order[EP_COMBINE_CH];
    __shared__ int n_ready;
    const int t0 = blockIdx.x * EP_COMBINE_CH;
    const int cnt = min(EP_COMBINE_CH, T - t0);
    if (threadIdx.x < cnt) {
        uint32_t m = 0;
        for (int k = 0; k < K; k++) {
            const int e = ids[(size_t)(t0 + threadIdx.x) * K + k];
            if (e >= 0 && e < El * n) m |= 1u << (e / El);  // a bad id was reported by the permutation
        }
        need[threadIdx.x] = m;
    }
    __syncthreads();
    uint32_t late = 0;  // thread 0: owners not yet in at the first look
    if (threadIdx.x == 0) {
        uint32_t all = 0, rd = 0;
        for (int i = 0; i < cnt; i++) all |= need[i];
        for (int o = 0; o < n; o++)  // one look at each owner this block needs
            if (((all >> o) & 1u) && moe::ld_acquire_sys(&ret_flags[o]) >= target) rd |= 1u << o;
        int j = 0;
        for (int i = 0; i < cnt; i++)
            if (!(need[i] & ~rd)) order[j++] = i;
        n_ready = j;
        for (int i = 0; i < cnt; i++)
            if (need[i] & ~rd) order[j++] = i;
        late = all & ~rd;
    }
    __syncthreads();
    const int vpr = H >> 3;
    const int nr = n_ready;
    for (int it = threadIdx.x; it < nr * vpr; it += blockDim.x) {  // tokens with every owner in
        const int j = it / vpr;
        ep_combine_vec(ret, dest, weights, y, t0 + order[j], (it - j * vpr) << 3, H, K);
    }
    if (nr == cnt) return;  // block-uniform
    if (threadIdx.x == 0)
        for (int o = 0; late; o++, late >>= 1)
            if (late & 1u) ep_wait_flag(&ret_flags[o], target, err, EP_ERR_WAIT_RET);
    __syncthreads();
    for (int it = nr * vpr + threadIdx.x; it < cnt * vpr; it += blockDim.x) {  // the rest
        const int j = it / vpr;
        ep_combine_vec(ret, dest, weights, y, t0 + order[j], (it - j * vpr) << 3, H, K);
    }
}

}  // namespace

namespace {
void p2p_release(MoeEpContext* c);
int p2p_setup(MoeEpContext* c, int64_t T, int64_t H, int64_t E, int64_t K, int64_t R, cudaStream_t s);
int p2p_forward(MoeEpContext* c, const void* x, const void* w_gate, const void* ewl, void* y, int64_t T,
                int64_t H, int64_t E, int64_t K, int64_t I, int64_t R, void* ws, const EpLayout& L,
                cudaStream_t s);
}  // namespace

extern "C" {

int MoeEpPlan(const int32_t* sendCounts, const int32_t* recvCounts, int n, int El, int32_t* sendOff,
              int32_t* recvOff, int32_t* expertOff, int32_t* segments)
{
    if (!sendCounts || !recvCounts || !sendOff || !recvOff || !expertOff || !segments)
        return MOE_ERR_NULL_POINTER;
    if (n < 1 || El < 1) return MOE_ERR_BAD_SHAPE;
    int64_t so = 0, ro = 0;
    for (int r = 0; r < n; r++) {
        sendOff[r] = (int32_t)so;
        recvOff[r] = (int32_t)ro;
        for (int e = 0; e < El; e++) {
            if (sendCounts[r * El + e] < 0 || recvCounts[r * El + e] < 0) return MOE_ERR_BAD_SHAPE;
            so += sendCounts[r * El + e];
            ro += recvCounts[r * El + e];
        }
    }
    if (so >= (int64_t(1) << 31) || ro >= (int64_t(1) << 31)) return MOE_ERR_BAD_SHAPE;
    sendOff[n] = (int32_t)so;
    recvOff[n] = (int32_t)ro;
    // expert-major destination: expert e's rows from source 0, then source 1, ...
    int64_t d = 0;
    for (int e = 0; e < El; e++) {
        expertOff[e] = (int32_t)d;
        for (int s = 0; s < n; s++) {
            int64_t src = recvOff[s];
            for (int e2 = 0; e2 < e; e2++) src += recvCounts[s * El + e2];
            int32_t* g = segments + 3 * (e * n + s);
            g[0] = (int32_t)d;
            g[1] = (int32_t)src;
            g[2] = recvCounts[s * El + e];
            d += recvCounts[s * El + e];
        }
    }
    expertOff[El] = (int32_t)d;
    return MOE_OK;
}

int MoeEpGetUniqueId(void* uniqueId)
{
    if (!uniqueId) return MOE_ERR_NULL_POINTER;
    static_assert(sizeof(ncclUniqueId) == MOE_EP_UNIQUE_ID_BYTES, "unique id size");
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return MOE_ERR_NCCL;
    memcpy(uniqueId, &id, sizeof(id));
    return MOE_OK;
}

int MoeEpInit(const void* uniqueId, int rank, int nranks, int timeoutMs, MoeEpContext** out)
{
    if (!uniqueId || !out) return MOE_ERR_NULL_POINTER;
    if (nranks < 1 || rank < 0 || rank >= nranks) return MOE_ERR_BAD_SHAPE;
    MoeEpContext* c = new MoeEpContext;
    c->rank = rank;
    c->nranks = nranks;
    c->timeout_ms = timeoutMs > 0 ? timeoutMs : 60000;
    if (cudaGetDevice(&c->device) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->counts_ready, cudaEventDisableTiming) != cudaSuccess) {
        delete c;
        return MOE_ERR_CUDA;
    }
    ncclUniqueId id;
    memcpy(&id, uniqueId, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&c->comm, nranks, id, rank, &cfg);
    int rc = check_nccl(c, r);
    if (rc == MOE_OK) rc = wait_comm(c, clk::now() + std::chrono::milliseconds(c->timeout_ms));
    if (rc != MOE_OK) {
        if (c->comm) ncclCommAbort(c->comm);
        cudaEventDestroy(c->counts_ready);
        delete c;
        return rc;
    }
    *out = c;
    return MOE_OK;
}

int MoeEpDestroy(MoeEpContext* c)
{
    if (!c) return MOE_ERR_NULL_POINTER;
    int rc = MOE_OK;
    if (c->comm) {
        if (c->broken) {
            ncclCommAbort(c->comm);
        } else {
            ncclResult_t r = ncclCommFinalize(c->comm);
            if (r == ncclSuccess || r == ncclInProgress)
                rc = wait_comm(c, clk::now() + std::chrono::milliseconds(c->timeout_ms));
            if (c->comm) ncclCommDestroy(c->comm);
        }
    }
    if (c->counts_ready) cudaEventDestroy(c->counts_ready);
    if (c->host) cudaFreeHost(c->host);
    p2p_release(c);
    delete c;
    return rc;
}

size_t MoeEpWorkspaceSize(int n, int64_t T, int64_t H, int64_t E, int64_t K, int64_t I, int64_t R)
{
    if (n < 1 || T < 0 || H < 8 || (H & 7) || I < 8 || (I & 7) || E < 1 || E > 256 || E % n ||
        K < 1 || K > 8 || K > E || T * K >= (int64_t(1) << 31))
        return 0;
    if (R <= 0) R = (int64_t)n * T * K;
    if (R >= (int64_t(1) << 31)) return 0;
    return ep_layout(n, T, H, E, K, I, R).total;
}

int MoeEpLayerForward(MoeEpContext* c, const void* x, const void* w_gate,
                      const void* expert_weights_local, void* y, int64_t T, int64_t H, int64_t E,
                      int64_t K, int64_t I, int64_t R, void* ws, size_t ws_bytes, void* stream)
{
    if (!c || !ws) return MOE_ERR_NULL_POINTER;
    if (c->broken || !c->comm) return MOE_ERR_NCCL;
    const int n = c->nranks;
    if (R <= 0) R = (int64_t)n * T * K;
    const size_t need = MoeEpWorkspaceSize(n, T, H, E, K, I, R);
    if (need == 0) return MOE_ERR_BAD_SHAPE;
    if (ws_bytes < need) return MOE_ERR_WORKSPACE_TOO_SMALL;
    if (T > 0 && (!x || !w_gate || !expert_weights_local || !y)) return MOE_ERR_NULL_POINTER;
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!a16(ws) || (T > 0 && (!a16(x) || !a16(w_gate) || !a16(expert_weights_local) || !a16(y))))
        return MOE_ERR_MISALIGNED;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != c->device) return MOE_ERR_UNSUPPORTED;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int El = (int)(E / n);
    const EpLayout L = ep_layout(n, T, H, E, K, I, R);
    // peer-memory path: set up (collectively) on the first call and whenever the
    // shapes change; every rank must call with the same shapes
    if (n <= 8 && !getenv("MOE_EP_FORCE_NCCL") && c->p2p_state >= 0 &&
        (c->p2p_state == 0 || c->p2p_T != T || c->p2p_H != H || c->p2p_E != E || c->p2p_K != K || c->p2p_R != R)) {
        int src = p2p_setup(c, T, H, E, K, R, s);
        if (src != MOE_OK) return src;
    }
    if (c->p2p_state == 1) return p2p_forward(c, x, w_gate, expert_weights_local, y, T, H, E, K, I, R, ws, L, s);
    const auto deadline = clk::now() + std::chrono::milliseconds(c->timeout_ms);
    int* err = at<int>(ws, L.err);
    int32_t* offsets = at<int32_t>(ws, L.offsets);
    int32_t* perm = at<int32_t>(ws, L.perm);
    int32_t* dest = at<int32_t>(ws, L.dest);
    int32_t* ids = at<int32_t>(ws, L.ids);
    __half* wts = at<__half>(ws, L.weights);
    int32_t* sendcnt = at<int32_t>(ws, L.sendcnt);
    int32_t* recvcnt = at<int32_t>(ws, L.recvcnt);
    int32_t* expoff = at<int32_t>(ws, L.expoff);
    int32_t* row_src = at<int32_t>(ws, L.row_src);
    __half* xp = at<__half>(ws, L.xp);
    __half* recv = at<__half>(ws, L.recv);
    __half* xr = at<__half>(ws, L.xr);
    __half* hbuf = at<__half>(ws, L.h);
    const int TK = (int)(T * K);
    cudaError_t e;

    // host tables (pinned): offsets [E+1] | recvcnt [n*El] | sendOff [n+1] | recvOff [n+1]
    //                       | expOff [El+1] | segments [El*n*3]
    const size_t hints = (size_t)(E + 1) + (size_t)n * El + 2 * (size_t)(n + 1) + (El + 1) + 3 * (size_t)El * n;
    if (c->host_ints < hints) {
        if (c->host) cudaFreeHost(c->host);
        c->host = nullptr;
        c->host_ints = 0;
        if (cudaMallocHost(&c->host, hints * sizeof(int32_t)) != cudaSuccess) return MOE_ERR_CUDA;
        c->host_ints = hints;
    }
    int32_t* h_off = c->host;
    int32_t* h_recv = h_off + (E + 1);
    int32_t* h_sendoff = h_recv + (size_t)n * El;
    int32_t* h_recvoff = h_sendoff + (n + 1);
    int32_t* h_expoff = h_recvoff + (n + 1);
    int32_t* h_seg = h_expoff + (El + 1);

    // stage events (MoeTraceStart): routing | permute | gather + counts + dispatch + reorder
    //                               | gate/up GEMM | down GEMM | return + combine
    cudaEvent_t* ev = moe::trace_begin_call();
    moe::trace_mark(ev, 0, s);
    // 1-2. routing, permutation (with its inverse), gather
    // the error word is cleared by the permutation launch below
    int32_t* tcounts = at<int32_t>(ws, L.tile_counts);
    int32_t* trank = at<int32_t>(ws, L.tile_rank);
    if (T > 0) {
        if ((e = moe::launch_routing(static_cast<const __half*>(x), static_cast<const __half*>(w_gate), ids,
                                     wts, (int)T, (int)H, (int)E, (int)K, s, tcounts, trank)) != cudaSuccess)
            return MOE_ERR_CUDA;
    }
    moe::trace_mark(ev, 1, s);
    if ((e = moe::launch_permute_tiles(ids, tcounts, trank, (int)T, (int)K, (int)E, offsets, perm, dest, err,
                                       moe::routing_error_word(), s)) != cudaSuccess)
        return MOE_ERR_CUDA;
    moe::trace_mark(ev, 2, s);
    if (T > 0 && (e = moe::launch_gather_rows(static_cast<const __half*>(x), perm, offsets, (int)E, (int)K,
                                              (int)H, TK, xp, s)) != cudaSuccess)
        return MOE_ERR_CUDA;
    ep_send_counts_kernel<<<1, 256, 0, s>>>(offsets, n * El, sendcnt);
    if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;

    // 3. counts exchange, one bounded host wait
    int rc = check_nccl(c, ncclGroupStart());
    for (int p = 0; rc == MOE_OK && p < n; p++) {
        rc = check_nccl(c, ncclSend(sendcnt + p * El, El, ncclInt32, p, c->comm, s));
        if (rc == MOE_OK) rc = check_nccl(c, ncclRecv(recvcnt + p * El, El, ncclInt32, p, c->comm, s));
    }
    if (rc == MOE_OK) rc = check_nccl(c, ncclGroupEnd());
    if (rc == MOE_OK) rc = wait_comm(c, deadline);
    if (rc != MOE_OK) return rc;
    if (cudaMemcpyAsync(h_off, offsets, sizeof(int32_t) * (E + 1), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(h_recv, recvcnt, sizeof(int32_t) * n * El, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaEventRecord(c->counts_ready, s) != cudaSuccess)
        return MOE_ERR_CUDA;
    if ((rc = wait_event(c, c->counts_ready, deadline)) != MOE_OK) return rc;
    std::vector<int32_t> h_send((size_t)n * El);
    for (int i = 0; i < n * El; i++) h_send[i] = h_off[i + 1] - h_off[i];
    if ((rc = MoeEpPlan(h_send.data(), h_recv, n, El, h_sendoff, h_recvoff, h_expoff, h_seg)) != MOE_OK)
        return rc;
    const int rows = h_recvoff[n];
    // Too many rows for this rank's workspace: it stops here, and its peers' next
    // exchange times out, so the call fails on every rank (by MOE_ERR_TIMEOUT there).
    if (rows > R) return MOE_ERR_WORKSPACE_TOO_SMALL;
    if (cudaMemcpyAsync(expoff, h_expoff, sizeof(int32_t) * (El + 1), cudaMemcpyHostToDevice, s) != cudaSuccess)
        return MOE_ERR_CUDA;
    int32_t* d_seg = at<int32_t>(ws, L.seg);
    if (rows > 0 &&
        cudaMemcpyAsync(d_seg, h_seg, sizeof(int32_t) * 3 * El * n, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return MOE_ERR_CUDA;

    // 4. dispatch
    const size_t Hs = (size_t)H;
    rc = check_nccl(c, ncclGroupStart());
    for (int p = 0; rc == MOE_OK && p < n; p++) {
        rc = check_nccl(c, ncclSend(xp + (size_t)h_sendoff[p] * Hs, (size_t)(h_sendoff[p + 1] - h_sendoff[p]) * Hs,
                                    ncclFloat16, p, c->comm, s));
        if (rc == MOE_OK)
            rc = check_nccl(c, ncclRecv(recv + (size_t)h_recvoff[p] * Hs,
                                        (size_t)(h_recvoff[p + 1] - h_recvoff[p]) * Hs, ncclFloat16, p, c->comm, s));
    }
    if (rc == MOE_OK) rc = check_nccl(c, ncclGroupEnd());
    if (rc == MOE_OK) rc = wait_comm(c, deadline);
    if (rc != MOE_OK) return rc;

    // 5. expert-major reorder, grouped GEMMs on the local experts
    if (rows > 0) {
        ep_row_map_kernel<<<El * n < 1024 ? El * n : 1024, 256, 0, s>>>(d_seg, El * n, row_src);
        if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;
        if (moe::launch_copy_rows(recv, row_src, rows, (int)H, xr, s) != cudaSuccess) return MOE_ERR_CUDA;
        moe::trace_mark(ev, 3, s);
        e = moe::launch_gemm_swiglu(xr, static_cast<const __half*>(expert_weights_local), expoff, hbuf, err, rows,
                                    (int)H, El, (int)I, 0, s, kEpRowsHint);
        if (e == cudaErrorInvalidValue) return MOE_ERR_UNSUPPORTED;
        if (e != cudaSuccess) return MOE_ERR_CUDA;
        moe::trace_mark(ev, 4, s);
        // GEMM2 writes row r of expert order to recv[row_src[r]] (source-major order)
        e = moe::launch_gemm_down(hbuf, static_cast<const __half*>(expert_weights_local), expoff, row_src, recv, err,
                                  rows, (int)H, El, (int)I, 0, s, rows, false);
        if (e == cudaErrorInvalidValue) return MOE_ERR_UNSUPPORTED;
        if (e != cudaSuccess) return MOE_ERR_CUDA;
    }

    if (rows == 0) {
        moe::trace_mark(ev, 3, s);
        moe::trace_mark(ev, 4, s);
    }
    moe::trace_mark(ev, 5, s);
    // 6. return rows to their sources, into xp's space (this rank's permuted order)
    rc = check_nccl(c, ncclGroupStart());
    for (int p = 0; rc == MOE_OK && p < n; p++) {
        rc = check_nccl(c, ncclSend(recv + (size_t)h_recvoff[p] * Hs, (size_t)(h_recvoff[p + 1] - h_recvoff[p]) * Hs,
                                    ncclFloat16, p, c->comm, s));
        if (rc == MOE_OK)
            rc = check_nccl(c, ncclRecv(xp + (size_t)h_sendoff[p] * Hs,
                                        (size_t)(h_sendoff[p + 1] - h_sendoff[p]) * Hs, ncclFloat16, p, c->comm, s));
    }
    if (rc == MOE_OK) rc = check_nccl(c, ncclGroupEnd());
    if (rc == MOE_OK) rc = wait_comm(c, deadline);
    if (rc != MOE_OK) return rc;

    // 7. combine through the inverse permutation
    if (T > 0 && moe::launch_combine_indexed(xp, dest, wts, static_cast<__half*>(y), (int)T, (int)H, (int)K, s) !=
                     cudaSuccess)
        return MOE_ERR_CUDA;
    moe::trace_mark(ev, 6, s);
    return MOE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------- peer-memory host side
namespace {

void p2p_release(MoeEpContext* c)
{
    for (int p = 0; p < c->nranks && p < 8; p++)
        if (c->p2p_peer[p] && c->p2p_peer[p] != c->p2p_base) cudaIpcCloseMemHandle(c->p2p_peer[p]);
    for (auto& q : c->p2p_peer) q = nullptr;
    if (c->p2p_base) cudaFree(c->p2p_base);
    if (c->p2p_dev_peers) cudaFree(c->p2p_dev_peers);
    c->p2p_base = nullptr;
    c->p2p_dev_peers = nullptr;
    c->p2p_state = 0;
}

// Collective: allocates and zeroes this rank's inboxes, exchanges IPC handles with
// NCCL, opens the peers' allocations, agrees (all ranks) whether every step worked,
// and ends with a barrier so no peer signals a flag before it is zeroed.
int p2p_setup(MoeEpContext* c, int64_t T, int64_t H, int64_t E, int64_t K, int64_t R, cudaStream_t s)
{
    const auto deadline = clk::now() + std::chrono::milliseconds(c->timeout_ms);
    const int n = c->nranks;
    if (c->p2p_base) {  // shapes changed: the previous call's kernels must be done first
        if (cudaDeviceSynchronize() != cudaSuccess) return MOE_ERR_CUDA;
        p2p_release(c);
    }
    size_t o = 0;
    c->off_cnt = o;
    o += align_up(sizeof(int32_t) * 2 * n * E);  // double-buffered by call parity
    c->off_flags = o;
    o += align_up(sizeof(unsigned long long) * F_WORDS);
    c->off_rows = o;
    o += align_up((size_t)R * H * 2);
    c->off_ret = o;
    o += align_up((size_t)(T * K > 0 ? T * K : 1) * H * 2);
    int ok = 1;
    cudaIpcMemHandle_t mine;
    memset(&mine, 0, sizeof(mine));
    if (cudaMalloc(&c->p2p_base, o) != cudaSuccess) {
        c->p2p_base = nullptr;
        ok = 0;
    }
    if (ok && (cudaMemset(c->p2p_base, 0, o) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
               cudaIpcGetMemHandle(&mine, c->p2p_base) != cudaSuccess))
        ok = 0;
    cudaGetLastError();
    // all-gather of the handles (and of `ok`) through NCCL
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    uint8_t* d_h = nullptr;
    int* d_ok = nullptr;
    if (cudaMalloc(&d_h, hb * n) != cudaSuccess || cudaMalloc(&d_ok, sizeof(int)) != cudaSuccess) return MOE_ERR_CUDA;
    cudaMemcpy(d_h + hb * c->rank, &mine, hb, cudaMemcpyHostToDevice);
    cudaMemcpy(d_ok, &ok, sizeof(int), cudaMemcpyHostToDevice);
    int rc = check_nccl(c, ncclGroupStart());
    if (rc == MOE_OK) rc = check_nccl(c, ncclAllGather(d_h + hb * c->rank, d_h, hb, ncclUint8, c->comm, s));
    if (rc == MOE_OK) rc = check_nccl(c, ncclAllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, c->comm, s));
    if (rc == MOE_OK) rc = check_nccl(c, ncclGroupEnd());
    if (rc == MOE_OK) rc = wait_comm(c, deadline);
    if (rc == MOE_OK && cudaEventRecord(c->counts_ready, s) != cudaSuccess) rc = MOE_ERR_CUDA;
    if (rc == MOE_OK) rc = wait_event(c, c->counts_ready, deadline);
    std::vector<uint8_t> handles(hb * n);
    if (rc == MOE_OK) {
        cudaMemcpy(handles.data(), d_h, hb * n, cudaMemcpyDeviceToHost);
        cudaMemcpy(&ok, d_ok, sizeof(int), cudaMemcpyDeviceToHost);
    }
    if (rc != MOE_OK) {
        cudaFree(d_h);
        cudaFree(d_ok);
        return rc;
    }
    // open the peers' allocations; then agree again on success
    int opened = ok;
    for (int p = 0; opened && p < n; p++) {
        if (p == c->rank) {
            c->p2p_peer[p] = c->p2p_base;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, handles.data() + hb * p, hb);
        if (cudaIpcOpenMemHandle(&c->p2p_peer[p], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            c->p2p_peer[p] = nullptr;
            opened = 0;
        }
    }
    cudaGetLastError();
    cudaMemcpy(d_ok, &opened, sizeof(int), cudaMemcpyHostToDevice);
    rc = check_nccl(c, ncclAllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, c->comm, s));
    if (rc == MOE_OK) rc = wait_comm(c, deadline);
    if (rc == MOE_OK && cudaEventRecord(c->counts_ready, s) != cudaSuccess) rc = MOE_ERR_CUDA;
    if (rc == MOE_OK) rc = wait_event(c, c->counts_ready, deadline);
    if (rc == MOE_OK) cudaMemcpy(&opened, d_ok, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(d_h);
    cudaFree(d_ok);
    if (rc != MOE_OK) return rc;
    if (!opened) {
        p2p_release(c);
        c->p2p_state = -1;  // every rank falls back to the NCCL path together
        return MOE_OK;
    }
    EpPeers hp;
    memset(&hp, 0, sizeof(hp));
    for (int p = 0; p < n; p++) {
        uint8_t* b = static_cast<uint8_t*>(c->p2p_peer[p]);
        hp.cnt[p] = reinterpret_cast<int32_t*>(b + c->off_cnt);
        hp.rows[p] = reinterpret_cast<__half*>(b + c->off_rows);
        hp.ret[p] = reinterpret_cast<__half*>(b + c->off_ret);
        hp.flags[p] = reinterpret_cast<unsigned long long*>(b + c->off_flags);
        hp.ret_flag[p] = hp.flags[p] + F_RET + c->rank;
    }
    if (cudaMalloc(&c->p2p_dev_peers, sizeof(EpPeers)) != cudaSuccess ||
        cudaMemcpy(c->p2p_dev_peers, &hp, sizeof(hp), cudaMemcpyHostToDevice) != cudaSuccess)
        return MOE_ERR_CUDA;
    c->p2p_T = T;
    c->p2p_H = H;
    c->p2p_E = E;
    c->p2p_K = K;
    c->p2p_R = R;
    c->epoch = 0;
    c->p2p_state = 1;
    return MOE_OK;
}

}  // namespace

namespace {

int p2p_forward(MoeEpContext* c, const void* x, const void* w_gate, const void* ewl, void* y, int64_t T,
                int64_t H, int64_t E, int64_t K, int64_t I, int64_t R, void* ws, const EpLayout& L,
                cudaStream_t s)
{
    const int n = c->nranks, me = c->rank, El = (int)(E / n);
    const int TK = (int)(T * K);
    const unsigned long long target = ++c->epoch;  // call number: every flag is raised once per call
    const int par = (int)(target & 1u);              // counts buffer of this call
    const EpPeers* dp = static_cast<const EpPeers*>(c->p2p_dev_peers);
    uint8_t* base = static_cast<uint8_t*>(c->p2p_base);
    const int32_t* cnt_local = reinterpret_cast<const int32_t*>(base + c->off_cnt);
    unsigned long long* flags = reinterpret_cast<unsigned long long*>(base + c->off_flags);
    const __half* rows_local = reinterpret_cast<const __half*>(base + c->off_rows);
    const __half* ret_local = reinterpret_cast<const __half*>(base + c->off_ret);
    int* err = at<int>(ws, L.err);
    int32_t* offsets = at<int32_t>(ws, L.offsets);
    int32_t* perm = at<int32_t>(ws, L.perm);
    int32_t* dest = at<int32_t>(ws, L.dest);
    int32_t* ids = at<int32_t>(ws, L.ids);
    __half* wts = at<__half>(ws, L.weights);
    int32_t* disp_base = at<int32_t>(ws, L.sendcnt);  // [E]
    int32_t* overflow = at<int32_t>(ws, L.recvcnt);   // [1]
    int32_t* expoff = at<int32_t>(ws, L.expoff);
    int32_t* seg = at<int32_t>(ws, L.seg);
    unsigned long long* row_ptr = at<unsigned long long>(ws, L.xr);  // R entries fit: H*2 >= 8
    __half* hbuf = at<__half>(ws, L.h);
    unsigned int* done1 = reinterpret_cast<unsigned int*>(flags + F_DONE1);
    unsigned int* done2 = reinterpret_cast<unsigned int*>(flags + F_DONE2);
    cudaEvent_t* ev = moe::trace_begin_call();
    moe::trace_mark(ev, 0, s);
    // the error word is cleared by the permutation launch below
    int32_t* tcounts = at<int32_t>(ws, L.tile_counts);
    int32_t* trank = at<int32_t>(ws, L.tile_rank);
    if (T > 0 && moe::launch_routing(static_cast<const __half*>(x), static_cast<const __half*>(w_gate), ids, wts,
                                     (int)T, (int)H, (int)E, (int)K, s, tcounts, trank) != cudaSuccess)
        return MOE_ERR_CUDA;
    moe::trace_mark(ev, 1, s);
    if (moe::launch_permute_tiles(ids, tcounts, trank, (int)T, (int)K, (int)E, offsets, perm, dest, err,
                                  moe::routing_error_word(), s) != cudaSuccess)
        return MOE_ERR_CUDA;
    moe::trace_mark(ev, 2, s);
    ep_p2p_plan_kernel<<<1, 256, sizeof(int32_t) * E, s>>>(dp, offsets, cnt_local, flags, (int)E, El, me, n, par,
                                                           (int)R, (int)H, target, err, disp_base, expoff, seg,
                                                           overflow, row_ptr);
    // two blocks (16 warps, one row each at a time) per SM: enough to keep NVLink busy
    int dgrid = (TK + 7) / 8;
    if (dgrid > 2 * 148) dgrid = 2 * 148;
    if (dgrid < 1) dgrid = 1;
    ep_p2p_dispatch_kernel<<<dgrid, 256, 0, s>>>(static_cast<const __half*>(x), perm, offsets, disp_base, overflow, dp,
                                                 TK, (int)E, El, (int)K, (int)H, me, n, done1);
    if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;
    moe::trace_mark(ev, 3, s);
    // GEMM1 starts as soon as this rank's own dispatch is issued; its producer waits,
    // per tile, only for the sources whose rows the tile covers (dispatch overlapped
    // with the first tiles).  MOE_EP_SERIAL=1: one wait for every source first
    // (no overlap; for comparisons).
    static const bool serial = getenv("MOE_EP_SERIAL") && getenv("MOE_EP_SERIAL")[0] == '1';
    if (serial)
        for (int src = 0; src < n; src++)
            ep_p2p_wait_kernel<<<1, 32, 0, s>>>(flags + F_ROWS + src, target, err, EP_ERR_WAIT_ROWS);
    const moe::SourceWait sw = {flags + F_ROWS, seg, n, EP_ERR_WAIT_ROWS, target};
    cudaError_t e = moe::launch_gemm_swiglu(rows_local, static_cast<const __half*>(ewl), expoff, hbuf, err, (int)R,
                                            (int)H, El, (int)I, 0, s, kEpRowsHint, serial ? nullptr : &sw);
    if (e == cudaErrorInvalidValue) return MOE_ERR_UNSUPPORTED;
    if (e != cudaSuccess) return MOE_ERR_CUDA;
    moe::trace_mark(ev, 4, s);
    // the down GEMM stores each row straight into its source rank's ret inbox and,
    // when the launch is done, bumps every rank's ret flag
    e = moe::launch_gemm_down_ptr(hbuf, static_cast<const __half*>(ewl), expoff, row_ptr, done2,
                                  reinterpret_cast<unsigned long long* const*>(
                                      reinterpret_cast<const uint8_t*>(dp) + offsetof(EpPeers, ret_flag)),
                                  n, err, (int)R, (int)H, El, (int)I, s, (int)(T * K), false);
    if (e == cudaErrorInvalidValue) return MOE_ERR_UNSUPPORTED;
    if (e != cudaSuccess) return MOE_ERR_CUDA;
    moe::trace_mark(ev, 5, s);
    // combine on arrival: tokens whose owners have returned their rows first; a
    // timed-out wait leaves stale rows, and the error word says so
    if (T > 0)
        ep_combine_arrival_kernel<<<(int)((T + EP_COMBINE_CH - 1) / EP_COMBINE_CH), 256, 0, s>>>(
            ret_local, dest, ids, wts, static_cast<__half*>(y), (int)T, (int)H, (int)K, El, n, flags + F_RET, target,
            err);
    if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;
    moe::trace_mark(ev, 6, s);
    return MOE_OK;
}

}  // namespace

extern "C" int MoeEpSelfTestWaitTimeout(int* code)
{
    // The expert-parallel kernels' bounded wait, on a flag that nothing sets: after
    // its time limit the kernel records the error bit and returns, and the context
    // stays usable.  Used by the failure-detection test; no GPU fault involved.
    if (!code) return MOE_ERR_NULL_POINTER;
    unsigned long long* flag = nullptr;
    int* err = nullptr;
    if (cudaMalloc(&flag, sizeof(*flag)) != cudaSuccess) return MOE_ERR_CUDA;
    if (cudaMalloc(&err, sizeof(int)) != cudaSuccess) {
        cudaFree(flag);
        return MOE_ERR_CUDA;
    }
    cudaMemset(flag, 0, sizeof(*flag));
    cudaMemset(err, 0, sizeof(int));
    ep_p2p_wait_kernel<<<1, 32>>>(flag, 1ull, err, EP_ERR_WAIT_ROWS);
    cudaError_t e = cudaDeviceSynchronize();
    int v = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(flag);
    cudaFree(err);
    if (e != cudaSuccess) return MOE_ERR_CUDA;
    *code = v;
    return MOE_OK;
}
