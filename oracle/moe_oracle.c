/*
 * moe_oracle.c -- CPU restatement of the reference MoE layer (TEST INFRASTRUCTURE).
 *
 * This file is the parity checker for the CUDA path, never part of the product:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg
 * load it.  It restates, loop for loop, the naive fp32 reference of the
 * Lu-Yu-Zhen/Implementing-MoE-Architecture-Operators-on-CANN-Platform project:
 *
 *   gating      tests/moe_cpu_sim.cpp:198-207   logits[t,e] = sum_h x[t,h]*w_gate[h,e]
 *   softmax     tests/moe_cpu_sim.cpp:209-222   max-subtract, expf, sum, divide
 *   top-K       tests/moe_cpu_sim.cpp:224-243   descending prob, renormalise over K
 *   permutation tests/moe_cpu_sim.cpp:412-419   per expert ascending, (t,k) ascending
 *   expert FFN  tests/moe_cpu_sim.cpp:249-296   SwiGLU: silu(x Wg^T) * (x Wu^T), then Wd
 *   combine     tests/moe_cpu_sim.cpp:298-305   y[t] = sum_k w[t,k] * ffn_out[t,k]
 *
 * The summation orders are the reference's, so with the same compiler settings
 * (no FMA contraction, no fast-math) the results are bit-identical to NaiveMoE;
 * oracle/ref_shim.cpp + the reference's own moe_cpu_sim.cpp are used to pin that.
 *
 * One documented deviation: std::partial_sort (moe_cpu_sim.cpp:232-233) leaves
 * the order of exactly-equal probabilities unspecified; this restatement defines
 * it as ascending expert id (the order the Ascend kernel's strict '>' scan gives,
 * op_kernel/moe_routing.cpp:317-335).
 *
 * Build: cc -O2 -std=c11 -ffp-contract=off -fPIC -shared -pthread (see oracle/Makefile).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* SiLU exactly as tests/moe_cpu_sim.cpp:155-158. */
static inline float oracle_silu(float v) { return v / (1.0f + expf(-v)); }

/*
 * Routing: logits, softmax and top-K with renormalised weights.
 * x [T,H], w_gate [H,E] (row-major, values already rounded to fp16).
 * Outputs: ids [T,K] int32, weights [T,K] fp32 (the reference keeps fp32 here;
 * the operator rounds to fp16 when it stores), and optional diagnostics:
 *   logits [T,E] fp32, probs [T,E] fp32,
 *   margin [T]: the smallest gap between consecutive entries of the top-(K+1)
 *   logits sorted descending (how close the token is to changing its ids).
 */
void oracle_routing(const float* x, const float* w_gate, int T, int H, int E, int K,
                    int32_t* ids, float* weights, float* logits_out, float* probs_out,
                    float* margin_out)
{
    float* logits = (float*)malloc(sizeof(float) * (size_t)E);
    float* probs = (float*)malloc(sizeof(float) * (size_t)E);
    unsigned char* used = (unsigned char*)malloc((size_t)E);
    int* order = (int*)malloc(sizeof(int) * (size_t)(K + 1));
    for (int t = 0; t < T; t++) {
        /* moe_cpu_sim.cpp:200-207: sequential fp32 accumulation over h */
        for (int e = 0; e < E; e++) {
            float dot = 0.0f;
            for (int h = 0; h < H; h++) dot += x[(size_t)t * H + h] * w_gate[(size_t)h * E + e];
            logits[e] = dot;
        }
        /* moe_cpu_sim.cpp:211-222 */
        float maxVal = -1e30f;
        for (int e = 0; e < E; e++)
            if (logits[e] > maxVal) maxVal = logits[e];
        float sumExp = 0.0f;
        for (int e = 0; e < E; e++) {
            probs[e] = expf(logits[e] - maxVal);
            sumExp += probs[e];
        }
        for (int e = 0; e < E; e++) probs[e] /= sumExp;
        /* moe_cpu_sim.cpp:225-243: top-K by prob descending (ties: lower id). */
        memset(used, 0, (size_t)E);
        int nsel = (K + 1 <= E) ? K + 1 : E;
        for (int k = 0; k < nsel; k++) {
            int best = -1;
            for (int e = 0; e < E; e++) {
                if (used[e]) continue;
                if (best < 0 || probs[e] > probs[best]) best = e;
            }
            used[best] = 1;
            order[k] = best;
        }
        float wSum = 0.0f;
        for (int k = 0; k < K; k++) {
            ids[(size_t)t * K + k] = order[k];
            wSum += probs[order[k]];
        }
        for (int k = 0; k < K; k++) weights[(size_t)t * K + k] = probs[order[k]] / wSum;
        if (logits_out) memcpy(logits_out + (size_t)t * E, logits, sizeof(float) * (size_t)E);
        if (probs_out) memcpy(probs_out + (size_t)t * E, probs, sizeof(float) * (size_t)E);
        if (margin_out) {
            float m = INFINITY;
            for (int k = 0; k + 1 < nsel; k++) {
                float g = logits[order[k]] - logits[order[k + 1]];
                if (g < m) m = g;
            }
            margin_out[t] = m;
        }
    }
    free(logits);
    free(probs);
    free(used);
    free(order);
}

/*
 * Permutation: the (token, slot) list of each expert, experts ascending, flat
 * index t*K+k ascending inside an expert (moe_cpu_sim.cpp:412-419 and the
 * Ascend scan op_kernel/moe_expert_ffn.cpp:186-195).
 * perm [T*K] receives flat source indices, offsets [E+1] the expert boundaries.
 * Returns 0, or -1 if an id is outside [0,E).
 */
int oracle_permute(const int32_t* ids, int T, int K, int E, int32_t* perm, int32_t* offsets)
{
    size_t n = (size_t)T * K;
    for (size_t i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= E) return -1;
    int32_t r = 0;
    for (int e = 0; e < E; e++) {
        offsets[e] = r;
        for (size_t i = 0; i < n; i++)
            if (ids[i] == e) perm[r++] = (int32_t)i;
    }
    offsets[E] = r;
    return 0;
}

/* Expert FFN of one (token, slot): moe_cpu_sim.cpp:251-294, same loop order. */
static void ffn_one(const float* x_row, const float* ew, int H, int I, int e, float* out,
                    float* gate, float* up, float* hid)
{
    size_t base = (size_t)e * 3 * I * H;
    const float* Wg = ew + base;
    const float* Wu = ew + base + (size_t)I * H;
    const float* Wd = ew + base + (size_t)2 * I * H;
    for (int i = 0; i < I; i++) {
        float dot = 0.0f;
        for (int h = 0; h < H; h++) dot += x_row[h] * Wg[(size_t)i * H + h];
        gate[i] = dot;
    }
    for (int i = 0; i < I; i++) {
        float dot = 0.0f;
        for (int h = 0; h < H; h++) dot += x_row[h] * Wu[(size_t)i * H + h];
        up[i] = dot;
    }
    for (int i = 0; i < I; i++) hid[i] = oracle_silu(gate[i]) * up[i];
    for (int h = 0; h < H; h++) {
        float dot = 0.0f;
        for (int i = 0; i < I; i++) dot += hid[i] * Wd[(size_t)h * I + i];
        out[h] = dot;
    }
}

typedef struct {
    const float* x;
    const float* ew;
    const int32_t* ids;
    int T0, T1, H, K, I;
    float* ffn_out;
} ffn_job;

static void* ffn_worker(void* arg)
{
    ffn_job* j = (ffn_job*)arg;
    float* scratch = (float*)malloc(sizeof(float) * (size_t)j->I * 3);
    for (int t = j->T0; t < j->T1; t++)
        for (int k = 0; k < j->K; k++)
            ffn_one(j->x + (size_t)t * j->H, j->ew, j->H, j->I, j->ids[(size_t)t * j->K + k],
                    j->ffn_out + ((size_t)t * j->K + k) * j->H, scratch, scratch + j->I,
                    scratch + 2 * (size_t)j->I);
    free(scratch);
    return NULL;
}

/*
 * Expert FFN for every (t,k): ffn_out [T,K,H] fp32.  Tokens are split over
 * `nthreads` POSIX threads; each (t,k) row is computed by one thread with the
 * reference's loop order, so the result does not depend on nthreads.
 */
void oracle_expert_ffn(const float* x, const float* ew, const int32_t* ids, int T, int H, int E,
                       int K, int I, float* ffn_out, int nthreads)
{
    (void)E;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > T) nthreads = T > 0 ? T : 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    ffn_job* jobs = (ffn_job*)malloc(sizeof(ffn_job) * (size_t)nthreads);
    for (int i = 0; i < nthreads; i++) {
        jobs[i].x = x;
        jobs[i].ew = ew;
        jobs[i].ids = ids;
        jobs[i].T0 = (int)((long long)T * i / nthreads);
        jobs[i].T1 = (int)((long long)T * (i + 1) / nthreads);
        jobs[i].H = H;
        jobs[i].K = K;
        jobs[i].I = I;
        jobs[i].ffn_out = ffn_out;
        if (nthreads > 1)
            pthread_create(&th[i], NULL, ffn_worker, &jobs[i]);
        else
            ffn_worker(&jobs[i]);
    }
    if (nthreads > 1)
        for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
}

/* Combine: y[t,:] = sum_k w[t,k] * ffn_out[t,k,:], moe_cpu_sim.cpp:299-305. */
void oracle_combine(const float* ffn_out, const float* weights, int T, int H, int K, float* y)
{
    for (size_t i = 0; i < (size_t)T * H; i++) y[i] = 0.0f;
    for (int t = 0; t < T; t++)
        for (int k = 0; k < K; k++) {
            float w = weights[(size_t)t * K + k];
            for (int h = 0; h < H; h++)
                y[(size_t)t * H + h] += w * ffn_out[((size_t)t * K + k) * H + h];
        }
}

/* The whole naive layer (NaiveMoE, moe_cpu_sim.cpp:183-306). */
void oracle_moe_naive(const float* x, const float* w_gate, const float* ew, int T, int H, int E,
                      int K, int I, float* y, int32_t* ids_out, float* weights_out, int nthreads)
{
    int32_t* ids = ids_out ? ids_out : (int32_t*)malloc(sizeof(int32_t) * (size_t)T * K);
    float* w = weights_out ? weights_out : (float*)malloc(sizeof(float) * (size_t)T * K);
    float* ffn = (float*)malloc(sizeof(float) * (size_t)T * K * H);
    oracle_routing(x, w_gate, T, H, E, K, ids, w, NULL, NULL, NULL);
    oracle_expert_ffn(x, ew, ids, T, H, E, K, I, ffn, nthreads);
    oracle_combine(ffn, w, T, H, K, y);
    free(ffn);
    if (!ids_out) free(ids);
    if (!weights_out) free(w);
}

/*
 * Inputs of the reference's NPU end-to-end test (tests/test_moe.cpp:373-381):
 * srand(seed), then x, w_gate and expert_weights filled in that order with
 * rand()/RAND_MAX*2-1 (uniform [-1,1]) from the C library's generator.
 */
void oracle_test_moe_inputs(unsigned seed, float* x, size_t nx, float* wg, size_t nwg, float* ew, size_t new_)
{
    srand(seed);
    for (size_t i = 0; i < nx; i++) x[i] = (rand() / (float)RAND_MAX) * 2.0f - 1.0f;
    for (size_t i = 0; i < nwg; i++) wg[i] = (rand() / (float)RAND_MAX) * 2.0f - 1.0f;
    for (size_t i = 0; i < new_; i++) ew[i] = (rand() / (float)RAND_MAX) * 2.0f - 1.0f;
}
