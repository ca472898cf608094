// routing.cu -- MoeRoutingTopK on sm_100a: gating GEMV, softmax, top-K, renormalise.
//
// Replaces op_kernel/moe_routing.cpp (Ascend Cube GEMM + scalar softmax/top-2).
// Semantics follow the fp32 naive reference, tests/moe_cpu_sim.cpp:198-243:
//   logits[t,e] = sum_h x[t,h] * w_gate[h,e]   (fp32, h ascending)
//   probs       = exp(logits - max) / sum      (sum in e ascending order)
//   ids         = top-K of probs, descending, equal probs -> lower expert id
//   weights     = probs[ids] / sum_k probs[ids]   -> fp16 (round to nearest even)
//
// Why the gating dot product keeps the reference's sequential order: x and w_gate
// are fp16, so each product x*w is exact in fp32 and fmaf(x, w, acc) rounds exactly
// like the reference's `dot += x*w`.  Accumulating h in ascending order per
// (token, expert) therefore reproduces the reference logits bit for bit, and the
// expert ids can only differ from the reference through expf() rounding at
// (near-)ties.  The cost is a dependent FMA chain of length H per (t,e), which
// still finishes in a few microseconds because a block runs 256 such chains and
// 4 tokens/thread at large E give independent chains for ILP.
//
// Data layout: a block owns TT tokens.  The H axis is walked in chunks of HC
// elements; each chunk of x ([TT][HC]) and of w_gate (transposed to [E][HC+8],
// padded so the 16-byte reads of different experts fall in different banks) is
// staged in shared memory with 16-byte global loads; x is read from HBM once.
#include "moe_common.cuh"
#include "moe_kernels.h"

namespace moe {

constexpr int RT_THREADS = 256;
constexpr int RT_MAXP = 16;  // token chains per thread (E up to 256)

struct RoutingPlan {
    int tpe;  // tokens processed in parallel per pass (256 / E)
    int P;    // chains per thread
    int TT;   // tokens per block = tpe * P
    int HC;   // H chunk (multiple of 8)
    size_t smem;
};

static RoutingPlan routing_plan(int H, int E)
{
    RoutingPlan p;
    p.tpe = RT_THREADS / E;
    int want = (16 + p.tpe - 1) / p.tpe;  // >= 16 tokens per block
    p.P = 1;
    while (p.P < want && p.P < RT_MAXP) p.P *= 2;
    p.TT = p.tpe * p.P;
    int hc = 16384 / E;
    if (16384 / p.TT < hc) hc = 16384 / p.TT;
    if (hc > 512) hc = 512;
    hc &= ~7;
    if (hc < 8) hc = 8;
    if (hc > H) hc = (H + 7) & ~7;
    p.HC = hc;
    // xs [TT][HC] fp16, ws [E][HC+8] fp16, logits [TT][E] fp32
    p.smem = (size_t)p.TT * p.HC * 2 + (size_t)E * (p.HC + 8) * 2 + (size_t)p.TT * E * 4;
    return p;
}

// P (token chains per thread) is a template parameter so that the accumulators
// are indexed statically and stay in registers.
template <int P>
__global__ void __launch_bounds__(RT_THREADS)
routing_topk_kernel(const __half* __restrict__ x, const __half* __restrict__ w_gate,
                    int32_t* __restrict__ expert_ids, __half* __restrict__ weights, int T, int H,
                    int E, int K, int tpe, int TT, int HC)
{
    extern __shared__ __align__(16) uint8_t rt_smem[];
    __half* xs = reinterpret_cast<__half*>(rt_smem);                  // [TT][HC]
    __half* ws = xs + (size_t)TT * HC;                                 // [E][HC+8]
    float* lg = reinterpret_cast<float*>(ws + (size_t)E * (HC + 8));   // [TT][E]
    const int wstride = HC + 8;

    const int tid = threadIdx.x;
    const int t_base = blockIdx.x * TT;
    const bool active = tid < tpe * E;
    const int e = tid % E;
    const int tslot = tid / E;

    float acc[P];
#pragma unroll
    for (int j = 0; j < P; j++) acc[j] = 0.0f;

    for (int h0 = 0; h0 < H; h0 += HC) {
        const int hc = min(HC, H - h0);  // multiple of 8 because H is
        const int vec_per_row = hc >> 3;
        // stage x chunk: TT rows x hc halves, 16-byte loads
        for (int v = tid; v < TT * vec_per_row; v += RT_THREADS) {
            int r = v / vec_per_row, c = (v - r * vec_per_row) << 3;
            int t = t_base + r;
            uint4 val = make_uint4(0, 0, 0, 0);
            if (t < T) val = __ldg(reinterpret_cast<const uint4*>(x + (size_t)t * H + h0 + c));
            *reinterpret_cast<uint4*>(xs + (size_t)r * HC + c) = val;
        }
        // stage w_gate chunk transposed: ws[e][h] = w_gate[h0+h][e]; h-fastest so the
        // shared-memory stores of a warp are consecutive (w_gate itself is L2-resident)
        for (int v = tid; v < hc * E; v += RT_THREADS) {
            int ee = v / hc, h = v - ee * hc;
            ws[(size_t)ee * wstride + h] = __ldg(w_gate + (size_t)(h0 + h) * E + ee);
        }
        __syncthreads();
        if (active) {
            const __half* wrow = ws + (size_t)e * wstride;
            for (int h = 0; h < hc; h += 8) {
                uint4 wv = *reinterpret_cast<const uint4*>(wrow + h);
                const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
                float wf[8];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    float2 f = __half22float2(w2[q]);
                    wf[2 * q] = f.x;
                    wf[2 * q + 1] = f.y;
                }
#pragma unroll
                for (int j = 0; j < P; j++) {
                    {
                        const int r = tslot + j * tpe;
                        uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)r * HC + h);
                        const __half2* x2 = reinterpret_cast<const __half2*>(&xv);
                        float a = acc[j];
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            float2 f = __half22float2(x2[q]);
                            a = fmaf(f.x, wf[2 * q], a);      // exact product, one rounding
                            a = fmaf(f.y, wf[2 * q + 1], a);  // == reference `dot += x*w`
                        }
                        acc[j] = a;
                    }
                }
            }
        }
        __syncthreads();
    }
    if (active) {
#pragma unroll
        for (int j = 0; j < P; j++) lg[(size_t)(tslot + j * tpe) * E + e] = acc[j];
    }
    __syncthreads();

    // softmax + top-K: one thread per token, reference order (moe_cpu_sim.cpp:211-243)
    if (tid < TT) {
        const int t = t_base + tid;
        if (t < T) {
            float* l = lg + (size_t)tid * E;
            float maxv = -1e30f;
            for (int i = 0; i < E; i++) maxv = l[i] > maxv ? l[i] : maxv;
            float sum = 0.0f;
            for (int i = 0; i < E; i++) {
                float pe = expf(l[i] - maxv);
                l[i] = pe;  // l now holds unnormalised probs
                sum += pe;
            }
            for (int i = 0; i < E; i++) l[i] = l[i] / sum;
            // top-K selection: K passes, strict '>' keeps the lower id on ties.
            // Selected entries are marked by negating (probs are >= 0; -1 - p < 0).
            int sel[8];
            float ps[8];
            float wsum = 0.0f;
            for (int k = 0; k < K; k++) {
                int best = -1;
                float bv = 0.0f;
                for (int i = 0; i < E; i++) {
                    float v = l[i];
                    if (v < 0.0f) continue;
                    if (best < 0 || v > bv) { best = i; bv = v; }
                }
                sel[k] = best;
                ps[k] = bv;
                l[best] = -1.0f - bv;
                wsum += bv;
            }
            for (int k = 0; k < K; k++) {
                expert_ids[(size_t)t * K + k] = sel[k];
                weights[(size_t)t * K + k] = __float2half_rn(ps[k] / wsum);
            }
        }
    }
}

cudaError_t launch_routing(const __half* x, const __half* w_gate, int32_t* ids, __half* weights,
                           int T, int H, int E, int K, cudaStream_t s)
{
    if (T == 0) return cudaSuccess;
    RoutingPlan p = routing_plan(H, E);
    const int grid = (T + p.TT - 1) / p.TT;
    switch (p.P) {
#define MOE_ROUTING_CASE(PP)                                                                       \
    case PP:                                                                                       \
        routing_topk_kernel<PP><<<grid, RT_THREADS, p.smem, s>>>(x, w_gate, ids, weights, T, H, E, \
                                                                 K, p.tpe, p.TT, p.HC);             \
        break;
        MOE_ROUTING_CASE(1)
        MOE_ROUTING_CASE(2)
        MOE_ROUTING_CASE(4)
        MOE_ROUTING_CASE(8)
        MOE_ROUTING_CASE(16)
#undef MOE_ROUTING_CASE
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace moe
