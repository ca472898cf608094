// moe_kernels.h -- internal launch wrappers shared by the kernel files and the
// C-ABI host layer (moe_ops.cu).  Not part of the public interface.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

// Launches `kernel` with programmatic stream serialisation allowed: it may start
// while the previous kernel of the stream drains, and waits for it with pdl_wait().
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args)
{
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, kernel, static_cast<KArgs>(args)...);
}

enum GemmMode { MODE_SWIGLU = 0, MODE_DOWN = 1, MODE_DOWN_PTR = 2 };

// tile_counts [ceil(T/128)][E] / tile_rank [T*K] (both or neither): the routing
// kernel also writes each 128-token tile's expert histogram and each entry's stable
// rank inside its tile, for launch_permute_tiles.
cudaError_t launch_routing(const __half* x, const __half* w_gate, int32_t* ids, __half* weights,
                           int T, int H, int E, int K, cudaStream_t s, int32_t* tile_counts = nullptr,
                           int32_t* tile_rank = nullptr);

// The permutation from the routing kernel's tile histograms and ranks (layer calls;
// the ids are the routing kernel's own, so no id is out of range).
cudaError_t launch_permute_tiles(const int32_t* ids, const int32_t* tile_counts, const int32_t* tile_rank, int T,
                                 int K, int E, int32_t* offsets, int32_t* perm, int32_t* dest, int* err, int* fold,
                                 cudaStream_t s);
inline int routing_tiles(int T) { return (T + 127) / 128; }

cudaError_t launch_permute(const int32_t* ids, int n, int E, int32_t* chunk_counts,
                           int32_t* chunk_base, int32_t* offsets, int32_t* perm, int32_t* dest,
                           int* err, int* fold, cudaStream_t s);

// Device address of the routing kernel's error word on the current device (the
// word its bounded waits record into; MoeRoutingTopK has no workspace).  Layer
// calls pass it to launch_permute as `fold`, which moves it into the call's error
// word.  nullptr if the lookup fails.
int* routing_error_word();

cudaError_t launch_gather_rows(const __half* x, const int32_t* perm, const int32_t* offsets, int E,
                               int K, int H, int rows_cap, __half* xp, cudaStream_t s);

// Grouped GEMM launchers.  rows_cap bounds the permuted rows (the A tensor's
// extent); rows_hint, when >= 0, is the expected number of rows actually present
// (used only to choose the tile shape: single-CTA or paired-CTA tiles, and for the
// down projection wide or narrow ones); allow_pair = false keeps single-CTA tiles.
// Expert-parallel GEMM1: A rows that arrive from `nsrc` source ranks while the
// kernel runs (see GemmArgs::src_flags).  seg: [E][nsrc][3] {first row, -, rows}.
struct SourceWait {
    const unsigned long long* flags;  // [nsrc], raised by each source when its rows have landed
    const int32_t* seg;
    int nsrc;
    int err_code;                     // recorded in *err when a wait gives up
    unsigned long long target;
};

cudaError_t launch_gemm_swiglu(const __half* xp, const __half* expert_weights,
                               const int32_t* offsets, __half* h, int* err, int rows_cap, int H,
                               int E, int I, int max_ctas, cudaStream_t s, int rows_hint = -1,
                               const SourceWait* src = nullptr);

cudaError_t launch_gemm_down(const __half* h, const __half* expert_weights, const int32_t* offsets,
                             const int32_t* perm, __half* expert_out, int* err, int rows_cap,
                             int H, int E, int I, int max_ctas, cudaStream_t s, int rows_hint = -1,
                             bool allow_pair = true);

cudaError_t launch_combine_indexed(const __half* rows, const int32_t* dest, const __half* weights,
                                   __half* y, int T, int H, int K, cudaStream_t s);

cudaError_t launch_copy_rows(const __half* src, const int32_t* idx, int rows, int H, __half* dst,
                             cudaStream_t s);

// Stage tracing (MoeTraceStart/Stop): the event array of the call being traced
// (nullptr when tracing is off) and a record at stage boundary `boundary` (0..6).
cudaEvent_t* trace_begin_call();
void trace_mark(cudaEvent_t* ev, int boundary, cudaStream_t s);

cudaError_t launch_gemm_down_ptr(const __half* h, const __half* expert_weights, const int32_t* offsets,
                                 const unsigned long long* row_ptr, unsigned int* done_counter,
                                 unsigned long long* const* peer_flags, int npeers, int* err, int rows_cap,
                                 int H, int E, int I, cudaStream_t s, int rows_hint = -1, bool allow_pair = true);

cudaError_t launch_combine(const __half* expert_out, const __half* weights, __half* y, int T,
                           int H, int K, cudaStream_t s);

}  // namespace moe
