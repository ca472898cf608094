// permute.cu -- bit-exact stable counting sort of (token, slot) pairs by expert id,
// and the row gather that lays the tokens of each expert out contiguously.
//
// Reference behaviour: the Ascend FFN kernel scans expert_ids once per expert
// (op_kernel/moe_expert_ffn.cpp:186-195) and the CPU simulation builds the same
// list (tests/moe_cpu_sim.cpp:412-419): experts ascending, and inside one expert
// the flat index t*K+k ascending.  A stable counting sort over the flat index
// produces exactly that order in O(T*K) instead of O(E*T*K), with no
// 512-per-expert cap (the reference's MAX_TOKENS_PER_EXPERT truncation).
//
// Three passes over the ids (a few microseconds even at T*K = 98304):
//   1. count   : per chunk of PC flat entries, a histogram over experts
//   2. scan    : per expert, exclusive prefix over chunks -> chunk bases and the
//                expert boundaries offsets[E+1]
//   3. scatter : within a chunk, the stable rank of each entry among the entries
//                with the same expert (warp match + per-warp prefix)
// then a gather copies x[perm[r]/K, :] to row r of the permuted activations.
#include <cooperative_groups.h>

#include "moe_common.cuh"
#include "moe_kernels.h"

namespace cg = cooperative_groups;

namespace moe {

constexpr int PC = 1024;  // flat entries per chunk == threads per block

__global__ void __launch_bounds__(PC)
perm_count_kernel(const int32_t* __restrict__ ids, int n, int E, int32_t* __restrict__ chunk_counts,
                  int* __restrict__ err)
{
    extern __shared__ int pc_hist[];
    for (int i = threadIdx.x; i < E; i += PC) pc_hist[i] = 0;
    __syncthreads();
    const int idx = blockIdx.x * PC + threadIdx.x;
    if (idx < n) {
        int e = ids[idx];
        if (e >= 0 && e < E)
            atomicAdd(&pc_hist[e], 1);
        else
            atomicOr(err, MOE_DEV_BAD_EXPERT_ID);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += PC) chunk_counts[(size_t)blockIdx.x * E + i] = pc_hist[i];
}

// One block.  offsets[E+1]: expert row boundaries.  chunk_base[c][e]: first
// permuted row of expert e's entries that live in chunk c.
__global__ void __launch_bounds__(1024)
perm_scan_kernel(const int32_t* __restrict__ chunk_counts, int nchunks, int E,
                 int32_t* __restrict__ chunk_base, int32_t* __restrict__ offsets)
{
    extern __shared__ int ps_tot[];  // [E+1]
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int s = 0;
        for (int c = 0; c < nchunks; c++) s += chunk_counts[(size_t)c * E + e];
        ps_tot[e] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int e = 0; e < E; e++) {
            int c = ps_tot[e];
            ps_tot[e] = run;
            offsets[e] = run;
            run += c;
        }
        offsets[E] = run;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = ps_tot[e];
        for (int c = 0; c < nchunks; c++) {
            chunk_base[(size_t)c * E + e] = run;
            run += chunk_counts[(size_t)c * E + e];
        }
    }
}

__global__ void __launch_bounds__(PC)
perm_scatter_kernel(const int32_t* __restrict__ ids, int n, int E,
                    const int32_t* __restrict__ chunk_base, int32_t* __restrict__ perm,
                    int32_t* __restrict__ dest)
{
    extern __shared__ int sc_wcnt[];  // [32 warps][E]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < 32 * E; i += PC) sc_wcnt[i] = 0;
    __syncthreads();
    const int idx = blockIdx.x * PC + threadIdx.x;
    int e = -1;
    if (idx < n) {
        e = ids[idx];
        if (e < 0 || e >= E) e = -1;  // reported by the count pass; skipped here
    }
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
    if (e >= 0 && rank_in_warp == 0) sc_wcnt[warp * E + e] = __popc(same);
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += PC) {  // exclusive prefix over warps
        int run = 0;
        for (int w = 0; w < 32; w++) {
            int c = sc_wcnt[w * E + ee];
            sc_wcnt[w * E + ee] = run;
            run += c;
        }
    }
    __syncthreads();
    if (e >= 0) {
        int pos = chunk_base[(size_t)blockIdx.x * E + e] + sc_wcnt[warp * E + e] + rank_in_warp;
        perm[pos] = idx;
        if (dest) dest[idx] = pos;
    }
}

// xp[r, :] = x[perm[r] / K, :] for r < offsets[E]; one warp per row, 16-byte moves.
__global__ void __launch_bounds__(256)
gather_rows_kernel(const __half* __restrict__ x, const int32_t* __restrict__ perm,
                   const int32_t* __restrict__ offsets, int E, int K, int H, int rows_cap,
                   __half* __restrict__ xp)
{
    pdl_trigger();
    pdl_wait();  // perm / offsets come from the permutation launch
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows_cap || r >= offsets[E]) return;
    const int src_t = perm[r] / K;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)src_t * H);
    uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)r * H);
    const int nv = H >> 3;
    for (int v = lane; v < nv; v += 32) dst[v] = __ldg(src + v);
}

// The three passes in one cooperative launch (one block per chunk, every block
// resident): histogram | grid sync | each block derives its own per-expert bases
// from all chunk histograms (O(chunks * E) reads) and block 0 writes offsets |
// stable scatter.  Same order as the three-kernel path, one launch instead of three.
__global__ void __launch_bounds__(PC)
perm_fused_kernel(const int32_t* __restrict__ ids, int n, int E, int32_t* __restrict__ chunk_counts,
                  int32_t* __restrict__ offsets, int32_t* __restrict__ perm, int32_t* __restrict__ dest,
                  int* __restrict__ err, int* __restrict__ fold)
{
    extern __shared__ int pf_smem[];
    int* hist = pf_smem;          // [E]
    int* base = pf_smem + E;      // [E]
    int* wcnt = pf_smem + 2 * E;  // [32 warps][E]
    __shared__ int bad;
    pdl_trigger();
    cg::grid_group grid = cg::this_grid();
    const int nchunks = gridDim.x;
    if (threadIdx.x == 0) {
        bad = 0;
        // this call's error word starts clear (set only after the sync), or with the
        // error the routing launch before it left in `fold` (which is cleared)
        if (blockIdx.x == 0) *err = fold ? atomicExch(fold, 0) : 0;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int idx = blockIdx.x * PC + threadIdx.x;
    for (int i = threadIdx.x; i < E; i += PC) hist[i] = 0;
    for (int i = threadIdx.x; i < 32 * E; i += PC) wcnt[i] = 0;
    __syncthreads();
    int e = -1;
    if (idx < n) {
        e = ids[idx];
        if (e >= 0 && e < E)
            atomicAdd(&hist[e], 1);
        else {
            bad = 1;
            e = -1;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += PC) chunk_counts[(size_t)blockIdx.x * E + i] = hist[i];
    grid.sync();
    if (threadIdx.x == 0 && bad) atomicOr(err, MOE_DEV_BAD_EXPERT_ID);
    // bases: offsets[e] (all experts before e) + this expert's rows in earlier chunks
    for (int ee = threadIdx.x; ee < E; ee += PC) {
        int tot = 0, before = 0;
        for (int c = 0; c < nchunks; c++) {
            const int v = chunk_counts[(size_t)c * E + ee];
            tot += v;
            if (c < blockIdx.x) before += v;
        }
        hist[ee] = tot;  // reuse: per-expert totals
        base[ee] = before;
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan of the totals (E <= 256)
        int run = 0;
        for (int ee = 0; ee < E; ee++) {
            const int t = hist[ee];
            hist[ee] = run;
            run += t;
        }
        if (blockIdx.x == 0) offsets[E] = run;
    }
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += PC) {
        base[ee] += hist[ee];
        if (blockIdx.x == 0) offsets[ee] = hist[ee];
    }
    // stable rank within the chunk: warp match + per-warp prefix (as perm_scatter_kernel)
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
    if (e >= 0 && rank_in_warp == 0) wcnt[warp * E + e] = __popc(same);
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += PC) {
        int run = 0;
        for (int w = 0; w < 32; w++) {
            const int c = wcnt[w * E + ee];
            wcnt[w * E + ee] = run;
            run += c;
        }
    }
    __syncthreads();
    if (e >= 0) {
        const int pos = base[e] + wcnt[warp * E + e] + rank_in_warp;
        perm[pos] = idx;
        if (dest) dest[idx] = pos;
    }
}

// dst[r, :] = src[idx[r], :] for r < rows; one warp per row, 16-byte moves.
__global__ void __launch_bounds__(256)
copy_rows_kernel(const __half* __restrict__ src, const int32_t* __restrict__ idx, int rows, int H,
                 __half* __restrict__ dst)
{
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const uint4* s4 = reinterpret_cast<const uint4*>(src + (size_t)idx[r] * H);
    uint4* d4 = reinterpret_cast<uint4*>(dst + (size_t)r * H);
    const int nv = H >> 3;
    for (int v = lane; v < nv; v += 32) d4[v] = __ldg(s4 + v);
}

// Error word of a call: cleared, or set to the routing error `fold` held (then cleared).
__global__ void err_init_kernel(int* err, int* fold)
{
    *err = fold ? atomicExch(fold, 0) : 0;
}

// The permutation of a layer call, after the routing kernel has written each
// 128-token tile's expert histogram (tile_counts [tiles][E]) and each entry's
// stable rank inside its tile (tile_rank [T*K]): block b derives, for tile b, every
// expert's first position (all tiles' totals before that expert, plus the entries of
// the expert in tiles before b) and scatters its entries.  Same order as the
// counting sort (experts ascending, flat index t*K+k ascending), one ordinary
// launch, no grid-wide synchronisation.  Block 0 writes offsets and the call's
// error word (cleared, or the routing error `fold` held).
constexpr int RT_TILE_TOKENS = 128;  // the routing kernel's tile (routing.cu RT_BM)

__global__ void __launch_bounds__(256)
perm_tiles_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ tile_counts,
                  const int32_t* __restrict__ tile_rank, int T, int K, int E, int32_t* __restrict__ offsets,
                  int32_t* __restrict__ perm, int32_t* __restrict__ dest, int* __restrict__ err, int* fold)
{
    extern __shared__ int pt_smem[];
    int* first = pt_smem;  // [E] first position of expert e's entries of this tile
    int* tot = pt_smem + E;  // [E] entries of expert e over all tiles
    pdl_trigger();
    pdl_wait();  // ids, tile_counts, tile_rank come from the routing launch
    const int ntiles = gridDim.x, b = blockIdx.x;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int all = 0, before = 0;
        for (int c = 0; c < ntiles; c++) {
            const int v = tile_counts[(size_t)c * E + e];
            all += v;
            if (c < b) before += v;
        }
        tot[e] = all;
        first[e] = before;
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan of the totals (E <= 256)
        int run = 0;
        for (int e = 0; e < E; e++) {
            const int v = tot[e];
            tot[e] = run;
            run += v;
        }
        if (b == 0) {
            offsets[E] = run;
            *err = fold ? atomicExch(fold, 0) : 0;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        first[e] += tot[e];
        if (b == 0) offsets[e] = tot[e];
    }
    __syncthreads();
    const long long f0 = (long long)b * RT_TILE_TOKENS * K;
    const long long f1 = min((long long)T * K, f0 + (long long)RT_TILE_TOKENS * K);
    for (long long f = f0 + threadIdx.x; f < f1; f += blockDim.x) {
        const int pos = first[ids[f]] + tile_rank[f];
        perm[pos] = (int32_t)f;
        if (dest) dest[f] = pos;
    }
}

cudaError_t launch_permute_tiles(const int32_t* ids, const int32_t* tile_counts, const int32_t* tile_rank, int T,
                                 int K, int E, int32_t* offsets, int32_t* perm, int32_t* dest, int* err, int* fold,
                                 cudaStream_t s)
{
    const int ntiles = (T + RT_TILE_TOKENS - 1) / RT_TILE_TOKENS;
    if (ntiles == 0) {  // empty batch: offsets all zero, error word initialised
        cudaError_t e = cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), s);
        if (e != cudaSuccess) return e;
        err_init_kernel<<<1, 1, 0, s>>>(err, fold);
        return cudaGetLastError();
    }
    cudaError_t e = launch_pdl(perm_tiles_kernel, dim3(ntiles), dim3(256), (size_t)2 * E * sizeof(int), s, ids,
                               tile_counts, tile_rank, T, K, E, offsets, perm, dest, err, fold);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_copy_rows(const __half* src, const int32_t* idx, int rows, int H, __half* dst,
                             cudaStream_t s)
{
    if (rows == 0) return cudaSuccess;
    copy_rows_kernel<<<(rows + 7) / 8, 256, 0, s>>>(src, idx, rows, H, dst);
    return cudaGetLastError();
}

cudaError_t launch_permute(const int32_t* ids, int n, int E, int32_t* chunk_counts,
                           int32_t* chunk_base, int32_t* offsets, int32_t* perm, int32_t* dest,
                           int* err, int* fold, cudaStream_t s)
{
    const int nchunks = (n + PC - 1) / PC;
    // one cooperative launch when every chunk's block can be resident at once
    static int capacity[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t fsmem = (size_t)(34 * E) * sizeof(int);
    if (dev >= 0 && dev < 64 && capacity[dev] == 0) {
        int per_sm = 0, sms = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, perm_fused_kernel, PC, 34 * 256 * sizeof(int));
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        capacity[dev] = per_sm * sms > 0 ? per_sm * sms : -1;
    }
    if (nchunks > 0 && dev >= 0 && dev < 64 && nchunks <= capacity[dev]) {
        void* args[] = {(void*)&ids, (void*)&n, (void*)&E, (void*)&chunk_counts, (void*)&offsets,
                        (void*)&perm, (void*)&dest, (void*)&err, (void*)&fold};
        cudaError_t e = cudaLaunchCooperativeKernel((const void*)perm_fused_kernel, dim3(nchunks), dim3(PC), args,
                                                    fsmem, s);
        if (e == cudaSuccess) return cudaSuccess;
        cudaGetLastError();  // fall back to the three-kernel path
    }
    err_init_kernel<<<1, 1, 0, s>>>(err, fold);
    if (nchunks > 0) {
        perm_count_kernel<<<nchunks, PC, E * sizeof(int), s>>>(ids, n, E, chunk_counts, err);
    }
    perm_scan_kernel<<<1, 1024, (E + 1) * sizeof(int), s>>>(chunk_counts, nchunks, E, chunk_base,
                                                            offsets);
    if (nchunks > 0) {
        perm_scatter_kernel<<<nchunks, PC, 32 * E * sizeof(int), s>>>(ids, n, E, chunk_base, perm,
                                                                      dest);
    }
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(const __half* x, const int32_t* perm, const int32_t* offsets, int E,
                               int K, int H, int rows_cap, __half* xp, cudaStream_t s)
{
    if (rows_cap == 0) return cudaSuccess;
    cudaError_t e = launch_pdl(gather_rows_kernel, dim3((rows_cap + 7) / 8), dim3(256), 0, s, x, perm, offsets, E,
                               K, H, rows_cap, xp);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace moe
