/*
 * moe_ops.h -- C ABI of the B200 (sm_100a) MoE layer operators.
 *
 * Drop-in for the three CANN operators of
 * Lu-Yu-Zhen/Implementing-MoE-Architecture-Operators-on-CANN-Platform:
 *   MoeRoutingTopK  op_host/moe_ops.cpp:537-579, kernel op_kernel/moe_routing.cpp:434-440
 *   MoeExpertFFN    op_host/moe_ops.cpp:584-632, kernel op_kernel/moe_expert_ffn.cpp:613-621
 *   MoeCombine      op_host/moe_ops.cpp:637-679, kernel op_kernel/moe_combine.cpp:136-143
 * The reference's host test binds the kernels as
 *   extern "C" void MoeRoutingTopK(void* x, void* wGate, void* expertIds, void* weights, void* tiling);
 * (tests/test_moe.cpp:33-41) and launches them with aclrtLaunchKernel(fn, stream, blockDim, ...).
 * Here the serialized tiling struct is replaced by explicit shape arguments and
 * the launch by the stream argument; everything else keeps its meaning:
 *   - inputs first, then outputs; all tensors ND (row-major, contiguous);
 *   - x, w_gate, weights, expert_weights, expert_out, y are IEEE fp16
 *     (passed as void*, 2 bytes per element); expert_ids is int32;
 *   - attrs: topK (default 2, moe_ops.cpp:566-567) and intermediateSize
 *     (default 8192, moe_ops.cpp:619-620) are the K and I arguments;
 *   - the caller owns every buffer, including the workspace whose size the
 *     *WorkspaceSize query returns (moe_ops.cpp:340-349 sets it in the reference);
 *   - calls are asynchronous on `stream` (a cudaStream_t, NULL = legacy default
 *     stream) and keep no host state between calls.
 * Status: 0 on success, a negative MOE_ERR_* code otherwise (the reference's
 * tiling functions return ge::GRAPH_FAILED, moe_ops.cpp:71-90).  Nothing aborts
 * or exits.  Errors only detectable on the device (an expert id outside [0,E),
 * a bounded wait that timed out) are recorded in the workspace and read back with
 * MoeGetDeviceError.
 *
 * Supported shapes: E in [1,256], K in [1, min(8,E)], H and I multiples of 8,
 * T*K < 2^31.  x, w_gate, expert_weights, expert_out, y and the workspace must be
 * 16-byte aligned.
 */
#ifndef MOE_OPS_H
#define MOE_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_OK 0
#define MOE_ERR_NULL_POINTER (-1)
#define MOE_ERR_BAD_SHAPE (-2)
#define MOE_ERR_WORKSPACE_TOO_SMALL (-3)
#define MOE_ERR_CUDA (-4)
#define MOE_ERR_UNSUPPORTED (-5)
#define MOE_ERR_MISALIGNED (-6)
#define MOE_ERR_NCCL (-7)
#define MOE_ERR_TIMEOUT (-8)
#define MOE_ERR_DEVICE (-9)

/* Data-type codes of the shape/dtype inference mirror (ge::DataType values). */
#define MOE_DT_FLOAT16 1
#define MOE_DT_INT32 3

/* ------------------------------------------------------------------ operators */

/* Replaces MoeRoutingTopK (op_kernel/moe_routing.cpp:434-440, moe_ops.cpp:63-226).
 * x [T,H] fp16, w_gate [H,E] fp16 -> expert_ids [T,K] int32, weights [T,K] fp16.
 * Slot 0 holds the most probable expert; equal probabilities keep the lower id. */
int MoeRoutingTopK(const void* x, const void* w_gate, int32_t* expert_ids, void* weights,
                   int64_t numTokens, int64_t hiddenSize, int64_t numExperts, int64_t topK,
                   void* stream);

/* Workspace of MoeExpertFFN in bytes (replaces the workspace sizing of
 * moe_ops.cpp:340-349; no per-expert token cap). */
size_t MoeExpertFFNWorkspaceSize(int64_t numTokens, int64_t hiddenSize, int64_t numExperts,
                                 int64_t topK, int64_t intermediateSize);

/* Replaces MoeExpertFFN (op_kernel/moe_expert_ffn.cpp:613-621, moe_ops.cpp:231-398).
 * x [T,H], expert_ids [T,K], weights [T,K] (accepted, unused, as in the reference),
 * expert_weights [E, 3I, H] = per expert W_gate [I,H], W_up [I,H], W_down [H,I]
 * -> expert_out [T,K,H] with expert_out[t,k] = FFN_{expert_ids[t,k]}(x[t]). */
int MoeExpertFFN(const void* x, const int32_t* expert_ids, const void* weights,
                 const void* expert_weights, void* expert_out, int64_t numTokens,
                 int64_t hiddenSize, int64_t numExperts, int64_t topK, int64_t intermediateSize,
                 void* workspace, size_t workspaceBytes, void* stream);

/* Replaces MoeCombine (op_kernel/moe_combine.cpp:136-143, moe_ops.cpp:403-525).
 * expert_out [T,K,H], expert_ids [T,K] (accepted, unused), weights [T,K] -> y [T,H]. */
int MoeCombine(const void* expert_out, const int32_t* expert_ids, const void* weights, void* y,
               int64_t numTokens, int64_t hiddenSize, int64_t topK, void* stream);

/* MoeExpertFFN for callers that cannot allocate device memory (a host framework
 * that owns every allocation through its own pool, a runtime that forbids
 * cudaMalloc after start-up, a service with a fixed memory budget).  This entry
 * point has no counterpart in the reference.  The caller still passes inputs and
 * outputs; the scratch is a static device array of MOE_NO_ALLOC_SCRATCH_BYTES
 * inside the library, held by every GPU that loads it until the process exits.
 * Problems whose MoeExpertFFNWorkspaceSize exceeds that limit are rejected with
 * MOE_ERR_WORKSPACE_TOO_SMALL.  The first call on a device looks up the array's
 * device address (make it before any stream capture).  All calls share the one
 * array: calls that overlap on the GPU race and must be serialised by the caller.
 * Calls no cudaMalloc, cudaFree or allocating library routine. */
#define MOE_NO_ALLOC_SCRATCH_BYTES (64u << 20)
int MoeExpertFFNNoAlloc(const void* x, const int32_t* expert_ids, const void* weights,
                        const void* expert_weights, void* expert_out, int64_t numTokens,
                        int64_t hiddenSize, int64_t numExperts, int64_t topK,
                        int64_t intermediateSize, void* stream);

/* The device error word of MoeExpertFFNNoAlloc (it has no caller workspace for
 * MoeGetDeviceError to read): synchronises `stream` and writes the code the last
 * call recorded (same codes as MoeGetDeviceError) into *code.  Each call of the
 * entry point starts with the word cleared.  No counterpart in the reference. */
int MoeNoAllocGetDeviceError(int* code, void* stream);

/* ------------------------------------------------------------------ whole layer */

/* The three operators in sequence (the flow of tests/test_moe.cpp:446-463), with
 * the intermediates in the workspace.  expert_ids / weights / expert_out may be
 * NULL (then they live in the workspace) or caller buffers to receive them. */
size_t MoeLayerWorkspaceSize(int64_t numTokens, int64_t hiddenSize, int64_t numExperts,
                             int64_t topK, int64_t intermediateSize);
int MoeLayerForward(const void* x, const void* w_gate, const void* expert_weights, void* y,
                    int32_t* expert_ids, void* weights, void* expert_out, int64_t numTokens,
                    int64_t hiddenSize, int64_t numExperts, int64_t topK,
                    int64_t intermediateSize, void* workspace, size_t workspaceBytes,
                    void* stream);

/* ------------------------------------------------------------------ expert parallel
 * The layer partitioned expert-parallel over n GPUs (one process or thread per
 * GPU).  Rank r owns experts [r*E/n, (r+1)*E/n) -- a contiguous slice
 * expert_weights_local [E/n, 3I, H] of the [E,3I,H] tensor -- and routes its own
 * T tokens.  Token rows travel to their experts' owners and back with NCCL
 * send/recv over NVLink.  The reference is single-device (tests/test_moe.cpp:642-648
 * pins device 0); this has no counterpart there and follows the same operator
 * semantics, so rank r's y equals MoeLayerForward on its tokens with all weights. */
#define MOE_EP_UNIQUE_ID_BYTES 128
typedef struct MoeEpContext MoeEpContext;

/* Writes an NCCL unique id (MOE_EP_UNIQUE_ID_BYTES bytes); one rank calls it and
 * the caller distributes the bytes to every rank. */
int MoeEpGetUniqueId(void* uniqueId);

/* Joins the communicator on the current CUDA device.  Non-blocking NCCL: every
 * wait is bounded by timeoutMs (<= 0: 60 s); on timeout the communicator is
 * aborted and MOE_ERR_TIMEOUT returned. */
int MoeEpInit(const void* uniqueId, int rank, int nranks, int timeoutMs, MoeEpContext** ctx);
int MoeEpDestroy(MoeEpContext* ctx);

/* Workspace of MoeEpLayerForward.  maxRecvRows bounds the (token, slot) rows this
 * rank's experts may receive in one call (<= 0: the worst case nranks*T*K). */
size_t MoeEpWorkspaceSize(int nranks, int64_t numTokens, int64_t hiddenSize, int64_t numExperts,
                          int64_t topK, int64_t intermediateSize, int64_t maxRecvRows);

/* Every rank makes the same sequence of calls with the same shapes: call c of one
 * rank exchanges rows with call c of every other rank.  A call whose device error
 * word reports a timed-out wait (64/128/256) leaves the ranks' call counters out of
 * step; destroy the context and build a new one.
 * x [T,H] (this rank's tokens), w_gate [H,E] (all experts), expert_weights_local
 * [E/n, 3I, H] -> y [T,H].  Synchronises the host once per call, on the exchanged
 * row counts (bounded by the context's timeout).  Returns MOE_ERR_WORKSPACE_TOO_SMALL
 * if more rows than maxRecvRows arrive (nothing is written past the workspace). */
int MoeEpLayerForward(MoeEpContext* ctx, const void* x, const void* w_gate,
                      const void* expert_weights_local, void* y, int64_t numTokens,
                      int64_t hiddenSize, int64_t numExperts, int64_t topK,
                      int64_t intermediateSize, int64_t maxRecvRows, void* workspace,
                      size_t workspaceBytes, void* stream);

/* The host-side exchange plan of one rank (pure host code).  sendCounts[r][e]: rows
 * this rank sends to rank r for r's local expert e; recvCounts[s][e]: rows it
 * receives from rank s for its local expert e (both [nranks][expertsPerRank]).
 * Outputs: sendOff[nranks+1], recvOff[nranks+1] (row offsets of each peer's block),
 * expertOff[expertsPerRank+1] (offsets after the expert-major reorder) and
 * segments[expertsPerRank*nranks][3] = {dst row, src row, rows} for each
 * (expert e, source s) at index e*nranks+s. */
int MoeEpPlan(const int32_t* sendCounts, const int32_t* recvCounts, int nranks, int expertsPerRank,
              int32_t* sendOff, int32_t* recvOff, int32_t* expertOff, int32_t* segments);

/* Failure-detection self-test (no reference counterpart): runs the expert-parallel
 * kernels' bounded flag wait on a flag that nothing sets.  The wait gives up after
 * its limit (about 2 s) and records its error bit (128) in *code; the context stays
 * usable.  Returns MOE_OK or MOE_ERR_CUDA. */
int MoeEpSelfTestWaitTimeout(int* code);

/* ------------------------------------------------------------------ permutation */

/* The token permutation inside MoeExpertFFN, exposed on its own.  Replaces the
 * per-expert scan of op_kernel/moe_expert_ffn.cpp:186-195 (same order: experts
 * ascending, flat index t*K+k ascending within an expert).
 * perm [T*K] int32 <- flat source indices, expert_offsets [E+1] int32. */
size_t MoePermuteWorkspaceSize(int64_t numTokens, int64_t topK, int64_t numExperts);
int MoePermute(const int32_t* expert_ids, int32_t* perm, int32_t* expert_offsets,
               int64_t numTokens, int64_t topK, int64_t numExperts, void* workspace,
               size_t workspaceBytes, void* stream);

/* ------------------------------------------------------------------ diagnostics */

/* MoeRoutingTopK has no workspace: a bounded wait inside the routing kernel that
 * gave up (never expected; 4/8 = a tensor-core or epilogue wait) is recorded in a
 * per-device word of the library.  This synchronises `stream`, writes that word to
 * *code and clears it.  Layer calls (MoeLayerForward, MoeEpLayerForward) move the
 * word into their own error word instead.  Concurrent routing calls on one device
 * share the word.  No counterpart in the reference (its kernels return void). */
int MoeRoutingGetDeviceError(int* code, void* stream);

/* Synchronises `stream` and reads the device error word of a MoeExpertFFN,
 * MoeLayerForward, MoePermute or MoeEpLayerForward workspace into *code (0 = none;
 * 1 = expert id out of range; 2/4/8 = a grouped-GEMM wait timed out; expert
 * parallel: 64/128/256 = the counts / rows / returned-rows flag wait timed out,
 * 512 = more rows than the workspace's maxRecvRows).  Returns MOE_OK or
 * MOE_ERR_CUDA. */
int MoeGetDeviceError(const void* workspace, int* code, void* stream);

/* Stage tracing (the profiling hook of this library; the reference only has
 * host wall-clock timers, tests/test_moe.cpp:592-605).  Between MoeTraceStart
 * and MoeTraceStop, every MoeLayerForward / MoeExpertFFN call made on this host
 * thread records CUDA events at its stage boundaries on its stream, for up to
 * maxCalls calls.  MoeTraceStop synchronises on those events and writes, per
 * call, MOE_TRACE_STAGES durations in milliseconds (routing, permute, gather (in
 * MoeEpLayerForward: gather, count exchange, dispatch and reorder),
 * gate/up GEMM + SwiGLU, down GEMM, combine (with the EP return exchange); stages a
 * call does not run read 0).  MoeEpLayerForward calls are traced too. */
#define MOE_TRACE_STAGES 6
int MoeTraceStart(int maxCalls);
int MoeTraceStop(float* stageMs, int maxCalls, int* numCalls);

/* Text for a MOE_* status code. */
const char* MoeStatusString(int status);

/* The cudaError_t of the most recent MOE_ERR_CUDA returned on this thread. */
int MoeLastCudaError(void);

/* ------------------------------------------------------------------ shape inference
 * Mirrors of the InferShape / InferDataType / TilingFunc checks of
 * op_host/moe_ops.cpp.  Return MOE_OK or MOE_ERR_BAD_SHAPE. */

/* moe_ops.cpp:63-90 and :181-226: x [T,H], w_gate [H,E]; topK <= 0 means the default 2.
 * Writes expert_ids / weights dims ({T, topK}) and dtypes (INT32, FLOAT16). */
int MoeRoutingInferShape(const int64_t* xDims, int xRank, const int64_t* wGateDims, int wGateRank,
                         int64_t topK, int64_t* expertIdsDims, int64_t* weightsDims,
                         int* expertIdsDtype, int* weightsDtype);

/* moe_ops.cpp:231-398: x [T,H], expert_ids [T,K], expert_weights [E,3I,H];
 * intermediateSize <= 0 means I = expert_weights dim 1 / 3.  Writes expert_out
 * dims {T, K, H} and dtype FLOAT16, and the resolved E, K, I. */
int MoeExpertFFNInferShape(const int64_t* xDims, int xRank, const int64_t* expertIdsDims,
                           int expertIdsRank, const int64_t* expertWeightsDims,
                           int expertWeightsRank, int64_t intermediateSize, int64_t* expertOutDims,
                           int* expertOutDtype, int64_t* resolvedE, int64_t* resolvedK,
                           int64_t* resolvedI);

/* moe_ops.cpp:403-525: expert_out [T,K,H], expert_ids [T,K] -> y dims {T, H}, FLOAT16. */
int MoeCombineInferShape(const int64_t* expertOutDims, int expertOutRank,
                         const int64_t* expertIdsDims, int expertIdsRank, int64_t* yDims,
                         int* yDtype);

#ifdef __cplusplus
}
#endif

#endif /* MOE_OPS_H */
