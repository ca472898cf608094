// moe_ops.cu -- C-ABI host layer: argument validation, workspace layout, launches.
//
// Mirrors the host side of the reference operators (op_host/moe_ops.cpp): shape
// checks of the TilingFuncs (:71-90, :241-258, :412-428), topK / intermediateSize
// attribute defaults (:97-105, :270-278), InferShape (:181-214, :364-388,
// :495-515) and InferDataType (:219-226, :393-398, :520-525).  The Ascend tiling
// (tileS, blockDim = AI-core count) has no counterpart: grid sizes come from the
// SM count and the shapes.
#include <stdio.h>

#include <vector>

#include "../../include/moe_ops.h"
#include "moe_common.cuh"
#include "moe_kernels.h"

namespace moe {

// ---- stage tracing: events[call][0..MOE_TRACE_STAGES] at stage boundaries
struct Trace {
    bool on = false;
    int max_calls = 0;
    int next = 0;
    std::vector<cudaEvent_t> ev;  // max_calls * (MOE_TRACE_STAGES + 1)
};
thread_local Trace g_trace;
constexpr int kTraceEv = MOE_TRACE_STAGES + 1;

cudaEvent_t* trace_begin_call()
{
    if (!g_trace.on || g_trace.next >= g_trace.max_calls) return nullptr;
    return &g_trace.ev[(size_t)g_trace.next++ * kTraceEv];
}
void trace_mark(cudaEvent_t* ev, int boundary, cudaStream_t s)
{
    if (ev) cudaEventRecord(ev[boundary], s);
}

}  // namespace moe

using moe::g_trace;
using moe::kTraceEv;
using moe::trace_begin_call;
using moe::trace_mark;

namespace {

thread_local int g_last_cuda_error = 0;

int cuda_status(cudaError_t e)
{
    if (e == cudaSuccess) return MOE_OK;
    g_last_cuda_error = (int)e;
    return MOE_ERR_CUDA;
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kChunk = 1024;  // flat entries per permutation chunk (permute.cu)

struct PermLayout {
    size_t err, chunk_counts, chunk_base, offsets, perm, total;
};

PermLayout perm_layout(int64_t T, int64_t K, int64_t E)
{
    PermLayout L;
    const int64_t n = T * K;
    const int64_t nchunks = (n + kChunk - 1) / kChunk;
    size_t o = 0;
    L.err = o;
    o += align_up(sizeof(int) * 4);
    L.chunk_counts = o;
    o += align_up(sizeof(int32_t) * (size_t)(nchunks > 0 ? nchunks : 1) * E);
    L.chunk_base = o;
    o += align_up(sizeof(int32_t) * (size_t)(nchunks > 0 ? nchunks : 1) * E);
    L.offsets = o;
    o += align_up(sizeof(int32_t) * (size_t)(E + 1));
    L.perm = o;
    o += align_up(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    L.total = o;
    return L;
}

struct FfnLayout {
    PermLayout p;
    size_t xp, h, total;
};

FfnLayout ffn_layout(int64_t T, int64_t H, int64_t E, int64_t K, int64_t I)
{
    FfnLayout L;
    L.p = perm_layout(T, K, E);
    size_t o = L.p.total;
    const size_t n = (size_t)(T * K > 0 ? T * K : 1);
    L.xp = o;
    o += align_up(n * (size_t)H * 2);
    L.h = o;
    o += align_up(n * (size_t)I * 2);
    L.total = o;
    return L;
}

struct LayerLayout {
    FfnLayout f;
    size_t ids, weights, expert_out, tile_counts, tile_rank, total;
};

LayerLayout layer_layout(int64_t T, int64_t H, int64_t E, int64_t K, int64_t I)
{
    LayerLayout L;
    L.f = ffn_layout(T, H, E, K, I);
    size_t o = L.f.total;
    const size_t n = (size_t)(T * K > 0 ? T * K : 1);
    L.ids = o;
    o += align_up(n * 4);
    L.weights = o;
    o += align_up(n * 2);
    L.expert_out = o;
    o += align_up(n * (size_t)H * 2);
    L.tile_counts = o;  // routing's per-tile expert histograms and in-tile ranks
    o += align_up(sizeof(int32_t) * (size_t)(moe::routing_tiles((int)T) > 0 ? moe::routing_tiles((int)T) : 1) * E);
    L.tile_rank = o;
    o += align_up(n * 4);
    L.total = o;
    return L;
}

bool shapes_ok(int64_t T, int64_t H, int64_t E, int64_t K)
{
    if (T < 0 || H < 8 || (H & 7) || E < 1 || E > 256 || K < 1 || K > 8 || K > E) return false;
    if (T * K >= (int64_t(1) << 31) || T * H >= (int64_t(1) << 40)) return false;
    return true;
}

bool ffn_shapes_ok(int64_t T, int64_t H, int64_t E, int64_t K, int64_t I)
{
    if (!shapes_ok(T, H, E, K)) return false;
    if (I < 8 || (I & 7)) return false;
    if (E * 3 * I >= (int64_t(1) << 31) || E * 3 * H >= (int64_t(1) << 31)) return false;
    return true;
}

template <class T>
T* at(void* base, size_t off)
{
    return reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off);
}

// fold: the routing error word when a routing launch precedes (layer calls), else nullptr
int run_permute(const int32_t* ids, int64_t T, int64_t K, int64_t E, void* ws, const PermLayout& L,
                int32_t* perm, int32_t* offsets, cudaStream_t s, int* fold = nullptr)
{
    int* err = at<int>(ws, L.err);  // cleared (or set to the folded routing error) by the permutation launch
    cudaError_t e = moe::launch_permute(ids, (int)(T * K), (int)E, at<int32_t>(ws, L.chunk_counts),
                            at<int32_t>(ws, L.chunk_base), offsets, perm, nullptr, err, fold, s);
    return cuda_status(e);
}

// tiles: the routing kernel's tile histograms / ranks {tile_counts, tile_rank} when
// it ran just before (layer calls): the permutation then takes one plain launch.
int run_ffn(const void* x, const int32_t* ids, const void* ew, void* out, int64_t T, int64_t H,
            int64_t E, int64_t K, int64_t I, void* ws, const FfnLayout& L, cudaStream_t s,
            cudaEvent_t* ev, int* fold = nullptr, int32_t* const* tiles = nullptr)
{
    int32_t* perm = at<int32_t>(ws, L.p.perm);
    int32_t* offsets = at<int32_t>(ws, L.p.offsets);
    int rc = tiles ? cuda_status(moe::launch_permute_tiles(ids, tiles[0], tiles[1], (int)T, (int)K, (int)E, offsets,
                                                           perm, nullptr, at<int>(ws, L.p.err), fold, s))
                   : run_permute(ids, T, K, E, ws, L.p, perm, offsets, s, fold);
    if (rc != MOE_OK) return rc;
    trace_mark(ev, 2, s);
    if (T == 0) return MOE_OK;
    const int rows = (int)(T * K);
    int* err = at<int>(ws, L.p.err);
    __half* xp = at<__half>(ws, L.xp);
    __half* h = at<__half>(ws, L.h);
    cudaError_t e = moe::launch_gather_rows(static_cast<const __half*>(x), perm, offsets, (int)E,
                                            (int)K, (int)H, rows, xp, s);
    if (e != cudaSuccess) return cuda_status(e);
    trace_mark(ev, 3, s);
    e = moe::launch_gemm_swiglu(xp, static_cast<const __half*>(ew), offsets, h, err, rows, (int)H,
                                (int)E, (int)I, 0, s);
    if (e == cudaErrorInvalidValue) return MOE_ERR_UNSUPPORTED;  // tensor map rejected
    if (e != cudaSuccess) return cuda_status(e);
    trace_mark(ev, 4, s);
    e = moe::launch_gemm_down(h, static_cast<const __half*>(ew), offsets, perm,
                              static_cast<__half*>(out), err, rows, (int)H, (int)E, (int)I, 0, s);
    if (e == cudaErrorInvalidValue) return MOE_ERR_UNSUPPORTED;
    trace_mark(ev, 5, s);
    return cuda_status(e);
}

}  // namespace

extern "C" {

int MoeRoutingTopK(const void* x, const void* w_gate, int32_t* expert_ids, void* weights,
                   int64_t T, int64_t H, int64_t E, int64_t K, void* stream)
{
    if (K <= 0) K = 2;  // attr default, moe_ops.cpp:98-105
    if (!shapes_ok(T, H, E, K)) return MOE_ERR_BAD_SHAPE;
    if (T == 0) return MOE_OK;
    if (!x || !w_gate || !expert_ids || !weights) return MOE_ERR_NULL_POINTER;
    if (!aligned16(x) || !aligned16(w_gate)) return MOE_ERR_MISALIGNED;
    return cuda_status(moe::launch_routing(static_cast<const __half*>(x),
                                           static_cast<const __half*>(w_gate), expert_ids,
                                           static_cast<__half*>(weights), (int)T, (int)H, (int)E,
                                           (int)K, static_cast<cudaStream_t>(stream)));
}

size_t MoeExpertFFNWorkspaceSize(int64_t T, int64_t H, int64_t E, int64_t K, int64_t I)
{
    if (!ffn_shapes_ok(T, H, E, K, I)) return 0;
    return ffn_layout(T, H, E, K, I).total;
}

int MoeExpertFFN(const void* x, const int32_t* expert_ids, const void* weights,
                 const void* expert_weights, void* expert_out, int64_t T, int64_t H, int64_t E,
                 int64_t K, int64_t I, void* workspace, size_t ws_bytes, void* stream)
{
    (void)weights;  // accepted and unused, as in op_kernel/moe_expert_ffn.cpp:89-90
    if (!ffn_shapes_ok(T, H, E, K, I)) return MOE_ERR_BAD_SHAPE;
    if (!workspace) return MOE_ERR_NULL_POINTER;
    FfnLayout L = ffn_layout(T, H, E, K, I);
    if (ws_bytes < L.total) return MOE_ERR_WORKSPACE_TOO_SMALL;
    if (T > 0 && (!x || !expert_ids || !expert_weights || !expert_out)) return MOE_ERR_NULL_POINTER;
    if (!aligned16(workspace) || (T > 0 && (!aligned16(x) || !aligned16(expert_weights) ||
                                            !aligned16(expert_out))))
        return MOE_ERR_MISALIGNED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaEvent_t* ev = trace_begin_call();
    trace_mark(ev, 0, s);
    trace_mark(ev, 1, s);
    int rc = run_ffn(x, expert_ids, expert_weights, expert_out, T, H, E, K, I, workspace, L, s, ev);
    trace_mark(ev, 5, s);
    trace_mark(ev, 6, s);
    return rc;
}

int MoeCombine(const void* expert_out, const int32_t* expert_ids, const void* weights, void* y,
               int64_t T, int64_t H, int64_t K, void* stream)
{
    (void)expert_ids;  // accepted and unused, as in op_kernel/moe_combine.cpp:6
    if (T < 0 || H < 8 || (H & 7) || K < 1 || K > 8 || T * K >= (int64_t(1) << 31))
        return MOE_ERR_BAD_SHAPE;
    if (T == 0) return MOE_OK;
    if (!expert_out || !weights || !y) return MOE_ERR_NULL_POINTER;
    if (!aligned16(expert_out) || !aligned16(y)) return MOE_ERR_MISALIGNED;
    return cuda_status(moe::launch_combine(static_cast<const __half*>(expert_out),
                                           static_cast<const __half*>(weights),
                                           static_cast<__half*>(y), (int)T, (int)H, (int)K,
                                           static_cast<cudaStream_t>(stream)));
}

size_t MoeLayerWorkspaceSize(int64_t T, int64_t H, int64_t E, int64_t K, int64_t I)
{
    if (!ffn_shapes_ok(T, H, E, K, I)) return 0;
    return layer_layout(T, H, E, K, I).total;
}

int MoeLayerForward(const void* x, const void* w_gate, const void* expert_weights, void* y,
                    int32_t* expert_ids, void* weights, void* expert_out, int64_t T, int64_t H,
                    int64_t E, int64_t K, int64_t I, void* workspace, size_t ws_bytes, void* stream)
{
    if (!ffn_shapes_ok(T, H, E, K, I)) return MOE_ERR_BAD_SHAPE;
    if (!workspace) return MOE_ERR_NULL_POINTER;
    LayerLayout L = layer_layout(T, H, E, K, I);
    if (ws_bytes < L.total) return MOE_ERR_WORKSPACE_TOO_SMALL;
    if (T > 0 && (!x || !w_gate || !expert_weights || !y)) return MOE_ERR_NULL_POINTER;
    if (!expert_ids) expert_ids = at<int32_t>(workspace, L.ids);
    if (!weights) weights = at<void>(workspace, L.weights);
    if (!expert_out) expert_out = at<void>(workspace, L.expert_out);
    if (!aligned16(workspace) ||
        (T > 0 && (!aligned16(x) || !aligned16(w_gate) || !aligned16(expert_weights) || !aligned16(y) ||
                   !aligned16(expert_out))))
        return MOE_ERR_MISALIGNED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (T == 0) return run_ffn(x, expert_ids, expert_weights, expert_out, T, H, E, K, I, workspace,
                               L.f, s, nullptr);
    cudaEvent_t* ev = trace_begin_call();
    trace_mark(ev, 0, s);
    int32_t* tiles[2] = {at<int32_t>(workspace, L.tile_counts), at<int32_t>(workspace, L.tile_rank)};
    int rc = cuda_status(moe::launch_routing(static_cast<const __half*>(x),
                                             static_cast<const __half*>(w_gate), expert_ids,
                                             static_cast<__half*>(weights), (int)T, (int)H, (int)E,
                                             (int)K, s, tiles[0], tiles[1]));
    if (rc != MOE_OK) return rc;
    trace_mark(ev, 1, s);
    // the permutation (from the routing kernel's tile histograms) moves a routing
    // wait timeout into this call's error word
    rc = run_ffn(x, expert_ids, expert_weights, expert_out, T, H, E, K, I, workspace, L.f, s, ev,
                 moe::routing_error_word(), tiles);
    if (rc != MOE_OK) return rc;
    rc = cuda_status(moe::launch_combine(static_cast<const __half*>(expert_out),
                                         static_cast<const __half*>(weights),
                                         static_cast<__half*>(y), (int)T, (int)H, (int)K, s));
    trace_mark(ev, 6, s);
    return rc;
}

size_t MoePermuteWorkspaceSize(int64_t T, int64_t K, int64_t E)
{
    if (T < 0 || K < 1 || E < 1 || E > 256 || T * K >= (int64_t(1) << 31)) return 0;
    return perm_layout(T, K, E).total;
}

int MoePermute(const int32_t* expert_ids, int32_t* perm, int32_t* expert_offsets, int64_t T,
               int64_t K, int64_t E, void* workspace, size_t ws_bytes, void* stream)
{
    if (T < 0 || K < 1 || E < 1 || E > 256 || T * K >= (int64_t(1) << 31)) return MOE_ERR_BAD_SHAPE;
    if (!workspace || !expert_offsets || (T > 0 && (!expert_ids || !perm))) return MOE_ERR_NULL_POINTER;
    PermLayout L = perm_layout(T, K, E);
    if (ws_bytes < L.total) return MOE_ERR_WORKSPACE_TOO_SMALL;
    return run_permute(expert_ids, T, K, E, workspace, L, perm, expert_offsets,
                       static_cast<cudaStream_t>(stream));
}

int MoeGetDeviceError(const void* workspace, int* code, void* stream)
{
    if (!workspace || !code) return MOE_ERR_NULL_POINTER;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e);
    *code = v;
    return MOE_OK;
}

int MoeRoutingGetDeviceError(int* code, void* stream)
{
    if (!code) return MOE_ERR_NULL_POINTER;
    int* word = moe::routing_error_word();
    if (!word) return cuda_status(cudaErrorInvalidSymbol);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, word, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(word, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e);
    *code = v;
    return MOE_OK;
}

const char* MoeStatusString(int status)
{
    switch (status) {
        case MOE_OK: return "MOE_OK";
        case MOE_ERR_NULL_POINTER: return "MOE_ERR_NULL_POINTER: a required pointer is NULL";
        case MOE_ERR_BAD_SHAPE: return "MOE_ERR_BAD_SHAPE: unsupported or inconsistent shape";
        case MOE_ERR_WORKSPACE_TOO_SMALL: return "MOE_ERR_WORKSPACE_TOO_SMALL";
        case MOE_ERR_CUDA: return "MOE_ERR_CUDA: a CUDA call failed (see MoeLastCudaError)";
        case MOE_ERR_UNSUPPORTED: return "MOE_ERR_UNSUPPORTED: configuration not supported";
        case MOE_ERR_MISALIGNED: return "MOE_ERR_MISALIGNED: a buffer is not 16-byte aligned";
        case MOE_ERR_NCCL: return "MOE_ERR_NCCL: an NCCL call failed";
        case MOE_ERR_TIMEOUT: return "MOE_ERR_TIMEOUT: an operation exceeded its deadline";
        case MOE_ERR_DEVICE: return "MOE_ERR_DEVICE: the device reported an error";
        default: return "unknown MoE status";
    }
}

int MoeLastCudaError(void) { return g_last_cuda_error; }

int MoeTraceStart(int maxCalls)
{
    if (maxCalls < 1) return MOE_ERR_BAD_SHAPE;
    if (g_trace.on) return MOE_ERR_UNSUPPORTED;
    g_trace.ev.assign((size_t)maxCalls * kTraceEv, nullptr);
    for (auto& e : g_trace.ev) {
        cudaError_t r = cudaEventCreate(&e);
        if (r != cudaSuccess) {
            for (auto& d : g_trace.ev)
                if (d) cudaEventDestroy(d);
            g_trace.ev.clear();
            return cuda_status(r);
        }
    }
    g_trace.max_calls = maxCalls;
    g_trace.next = 0;
    g_trace.on = true;
    return MOE_OK;
}

int MoeTraceStop(float* stageMs, int maxCalls, int* numCalls)
{
    if (!g_trace.on) return MOE_ERR_UNSUPPORTED;
    int n = g_trace.next;
    int rc = MOE_OK;
    for (int c = 0; c < n && c < maxCalls; c++) {
        cudaEvent_t* ev = &g_trace.ev[(size_t)c * kTraceEv];
        for (int st = 0; st < MOE_TRACE_STAGES; st++) {
            float ms = 0.0f;
            cudaError_t r = cudaEventSynchronize(ev[st + 1]);
            if (r == cudaSuccess) r = cudaEventElapsedTime(&ms, ev[st], ev[st + 1]);
            if (r != cudaSuccess) {
                rc = cuda_status(r);
                ms = 0.0f;
            }
            if (stageMs) stageMs[(size_t)c * MOE_TRACE_STAGES + st] = ms;
        }
    }
    for (auto& e : g_trace.ev) cudaEventDestroy(e);
    g_trace.ev.clear();
    g_trace.on = false;
    if (numCalls) *numCalls = n;
    return rc;
}

// ------------------------------------------------------------------ shape inference
int MoeRoutingInferShape(const int64_t* xDims, int xRank, const int64_t* wGateDims, int wGateRank,
                         int64_t topK, int64_t* expertIdsDims, int64_t* weightsDims,
                         int* expertIdsDtype, int* weightsDtype)
{
    if (!xDims || !wGateDims) return MOE_ERR_NULL_POINTER;
    if (xRank != 2 || wGateRank != 2) return MOE_ERR_BAD_SHAPE;  // moe_ops.cpp:80-85
    if (xDims[1] != wGateDims[0]) return MOE_ERR_BAD_SHAPE;       // moe_ops.cpp:86-90
    if (topK <= 0) topK = 2;                                       // moe_ops.cpp:194-203
    if (expertIdsDims) { expertIdsDims[0] = xDims[0]; expertIdsDims[1] = topK; }
    if (weightsDims) { weightsDims[0] = xDims[0]; weightsDims[1] = topK; }
    if (expertIdsDtype) *expertIdsDtype = MOE_DT_INT32;            // moe_ops.cpp:222
    if (weightsDtype) *weightsDtype = MOE_DT_FLOAT16;              // moe_ops.cpp:224
    return MOE_OK;
}

int MoeExpertFFNInferShape(const int64_t* xDims, int xRank, const int64_t* eidDims, int eidRank,
                           const int64_t* ewDims, int ewRank, int64_t intermediateSize,
                           int64_t* outDims, int* outDtype, int64_t* rE, int64_t* rK, int64_t* rI)
{
    if (!xDims || !eidDims) return MOE_ERR_NULL_POINTER;
    if (xRank != 2 || eidRank != 2) return MOE_ERR_BAD_SHAPE;  // moe_ops.cpp:251-254, :375-377
    int64_t E = 0, I = 0;
    if (ewDims) {
        if (ewRank != 3) return MOE_ERR_BAD_SHAPE;  // moe_ops.cpp:255-258
        E = ewDims[0];
        I = ewDims[1] / 3;                          // moe_ops.cpp:264
    }
    if (intermediateSize > 0) I = intermediateSize;  // moe_ops.cpp:270-278
    if (outDims) { outDims[0] = xDims[0]; outDims[1] = eidDims[1]; outDims[2] = xDims[1]; }
    if (outDtype) *outDtype = MOE_DT_FLOAT16;
    if (rE) *rE = E;
    if (rK) *rK = eidDims[1];
    if (rI) *rI = I;
    return MOE_OK;
}

int MoeCombineInferShape(const int64_t* outDims, int outRank, const int64_t* eidDims, int eidRank,
                         int64_t* yDims, int* yDtype)
{
    if (!outDims) return MOE_ERR_NULL_POINTER;
    if (outRank != 3) return MOE_ERR_BAD_SHAPE;              // moe_ops.cpp:421-424
    if (eidDims && eidRank != 2) return MOE_ERR_BAD_SHAPE;   // moe_ops.cpp:425-428
    if (yDims) { yDims[0] = outDims[0]; yDims[1] = outDims[2]; }
    if (yDtype) *yDtype = MOE_DT_FLOAT16;
    return MOE_OK;
}

}  // extern "C"
