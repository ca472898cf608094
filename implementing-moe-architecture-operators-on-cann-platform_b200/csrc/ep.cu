// ep.cu -- the MoE layer expert-parallel over n GPUs with NCCL send/recv.
//
// The reference runs on one device (tests/test_moe.cpp:642-648); the benchmark
// definition asks for the layer partitioned expert-parallel across the GPUs of a
// box.  Rank r owns experts [r*El, (r+1)*El), El = E/n, and routes its own tokens:
//
//   1. routing + stable counting sort of this rank's (token, slot) pairs by expert
//      (experts are owned contiguously, so expert order is also owner order);
//   2. gather of the permuted rows xp [T*K, H];
//   3. exchange of per-(owner, expert) row counts (NCCL send/recv of El ints per
//      peer), one bounded host wait on them, host plan (MoeEpPlan);
//   4. dispatch: grouped ncclSend/ncclRecv of row blocks, into recv [R, H] in
//      source-major order;
//   5. reorder to expert-major (copy_rows), grouped GEMM1 (gate/up + SwiGLU) and
//      GEMM2 (down) on the local experts; GEMM2 scatters each row back to its
//      source-major slot, so no second reorder is needed;
//   6. return: the mirrored send/recv into ret [T*K, H] (this rank's permuted order);
//   7. combine through the permutation's inverse (combine_indexed).
// Every kernel is the single-GPU one, so each row of y is bit-identical to
// MoeLayerForward on the same tokens with all experts.  Remote rows reach local
// HBM through NCCL before any kernel reads them; no kernel reads peer memory.
//
// Failure handling: the communicator is non-blocking; every wait (communicator
// set-up, group completion, the counts event) polls against a deadline and aborts
// the communicator on timeout, returning MOE_ERR_TIMEOUT instead of hanging.
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <thread>
#include <vector>

#include "../../include/moe_ops.h"
#include "moe_common.cuh"
#include "moe_kernels.h"

struct MoeEpContext {
    ncclComm_t comm = nullptr;
    int rank = 0, nranks = 1, device = 0;
    int timeout_ms = 60000;
    bool broken = false;  // a wait timed out or NCCL failed: only MoeEpDestroy is valid
    cudaEvent_t counts_ready = nullptr;
    int32_t* host = nullptr;  // pinned: offsets [E+1], recv counts [n*El], plan tables
    size_t host_ints = 0;
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
        std::this_thread::sleep_for(std::chrono::microseconds(20));
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
        std::this_thread::sleep_for(std::chrono::microseconds(5));
    }
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }
constexpr int kChunk = 1024;  // permutation chunk (permute.cu)

struct EpLayout {
    size_t err, chunk_counts, chunk_base, offsets, perm, dest, ids, weights, sendcnt, recvcnt,
        expoff, seg, row_src, xp, recv, xr, h, total;
};

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
    if ((e = cudaMemsetAsync(err, 0, sizeof(int), s)) != cudaSuccess) return MOE_ERR_CUDA;
    if (T > 0) {
        if ((e = moe::launch_routing(static_cast<const __half*>(x), static_cast<const __half*>(w_gate), ids,
                                     wts, (int)T, (int)H, (int)E, (int)K, s)) != cudaSuccess)
            return MOE_ERR_CUDA;
    }
    moe::trace_mark(ev, 1, s);
    if ((e = moe::launch_permute(ids, TK, (int)E, at<int32_t>(ws, L.chunk_counts),
                                 at<int32_t>(ws, L.chunk_base), offsets, perm, dest, err, s)) != cudaSuccess)
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
                                    (int)H, El, (int)I, 0, s);
        if (e == cudaErrorInvalidValue) return MOE_ERR_UNSUPPORTED;
        if (e != cudaSuccess) return MOE_ERR_CUDA;
        moe::trace_mark(ev, 4, s);
        // GEMM2 writes row r of expert order to recv[row_src[r]] (source-major order)
        e = moe::launch_gemm_down(hbuf, static_cast<const __half*>(expert_weights_local), expoff, row_src, recv, err,
                                  rows, (int)H, El, (int)I, 0, s);
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
