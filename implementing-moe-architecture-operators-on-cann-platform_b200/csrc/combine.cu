// combine.cu -- MoeCombine on sm_100a: y[t,:] = sum_k w[t,k] * expert_out[t,k,:].
//
// Replaces op_kernel/moe_combine.cpp, which accumulates in fp16 (Muls/Add,
// :80-111).  Here the sum runs in fp32 in slot order k = 0..K-1, starting from
// 0 like the reference (tests/moe_cpu_sim.cpp:298-305), and is rounded to fp16
// once.  Each thread owns 8 consecutive hidden elements of one token, so every
// global access is a 16-byte vector; the kernel streams expert_out once and is
// HBM-bound (T*K*H*2 + T*K*2 + T*H*2 bytes).  expert_ids is not needed and not
// read, as in the reference (moe_combine.cpp:6).
#include "moe_common.cuh"
#include "moe_kernels.h"

namespace moe {

__global__ void __launch_bounds__(256)
combine_kernel(const __half* __restrict__ expert_out, const __half* __restrict__ weights,
               __half* __restrict__ y, int T, int H, int K)
{
    pdl_wait();  // expert_out comes from the down GEMM (a no-op when launched plainly)
    const int vpr = H >> 3;  // 16-byte vectors per row
    const long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= (long long)T * vpr) return;
    const int t = (int)(v / vpr);
    const int c = (int)(v - (long long)t * vpr) << 3;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.0f;
    const __half* src = expert_out + (size_t)t * K * H + c;
    for (int k = 0; k < K; k++) {
        const float w = __half2float(weights[(size_t)t * K + k]);
        uint4 q = __ldcs(reinterpret_cast<const uint4*>(src + (size_t)k * H));
        const __half2* q2 = reinterpret_cast<const __half2*>(&q);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float2 f = __half22float2(q2[i]);
            acc[2 * i] = fmaf(w, f.x, acc[2 * i]);
            acc[2 * i + 1] = fmaf(w, f.y, acc[2 * i + 1]);
        }
    }
    uint4 o;
    o.x = pack_half2(acc[0], acc[1]);
    o.y = pack_half2(acc[2], acc[3]);
    o.z = pack_half2(acc[4], acc[5]);
    o.w = pack_half2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(y + (size_t)t * H + c) = o;
}

// Expert-parallel variant: the (t,k) rows come back from the expert owners in
// permuted order, so slot (t,k) is read from rows[dest[t*K+k]] (dest = the
// permutation's inverse).  Same fp32 sum in slot order as combine_kernel.
__global__ void __launch_bounds__(256)
combine_indexed_kernel(const __half* __restrict__ rows, const int32_t* __restrict__ dest,
                       const __half* __restrict__ weights, __half* __restrict__ y, int T, int H, int K)
{
    const int vpr = H >> 3;
    const long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= (long long)T * vpr) return;
    const int t = (int)(v / vpr);
    const int c = (int)(v - (long long)t * vpr) << 3;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.0f;
    for (int k = 0; k < K; k++) {
        const float w = __half2float(weights[(size_t)t * K + k]);
        const int r = dest[(size_t)t * K + k];
        uint4 q = __ldcs(reinterpret_cast<const uint4*>(rows + (size_t)r * H + c));
        const __half2* q2 = reinterpret_cast<const __half2*>(&q);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float2 f = __half22float2(q2[i]);
            acc[2 * i] = fmaf(w, f.x, acc[2 * i]);
            acc[2 * i + 1] = fmaf(w, f.y, acc[2 * i + 1]);
        }
    }
    uint4 o;
    o.x = pack_half2(acc[0], acc[1]);
    o.y = pack_half2(acc[2], acc[3]);
    o.z = pack_half2(acc[4], acc[5]);
    o.w = pack_half2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(y + (size_t)t * H + c) = o;
}

cudaError_t launch_combine_indexed(const __half* rows, const int32_t* dest, const __half* weights,
                                   __half* y, int T, int H, int K, cudaStream_t s)
{
    long long nv = (long long)T * (H >> 3);
    if (nv == 0) return cudaSuccess;
    combine_indexed_kernel<<<(int)((nv + 255) / 256), 256, 0, s>>>(rows, dest, weights, y, T, H, K);
    return cudaGetLastError();
}

cudaError_t launch_combine(const __half* expert_out, const __half* weights, __half* y, int T, int H,
                           int K, cudaStream_t s)
{
    long long nv = (long long)T * (H >> 3);
    if (nv == 0) return cudaSuccess;
    int grid = (int)((nv + 255) / 256);
    cudaError_t e = launch_pdl(combine_kernel, dim3(grid), dim3(256), 0, s, expert_out, weights, y, T, H, K);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace moe
