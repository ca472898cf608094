// ref_shim.cpp -- C entry points around the reference's own CPU simulation
// (TEST INFRASTRUCTURE, built into oracle/_ref/ only, never shipped).
//
// The reference source is not copied: the Makefile passes its path in
// MOE_CPU_SIM_SRC (the project's tests/moe_cpu_sim.cpp, where it lies) and renames
// its main() with -Dmain=moe_cpu_sim_main.  The functions below only marshal
// plain float/int arrays into the std::vector interface of:
//   NaiveMoE        tests/moe_cpu_sim.cpp:183-306 (the fp32 oracle of the layer)
//   TiledRouting    tests/moe_cpu_sim.cpp:315-389 (expert ids + fp32 weights)
//   TiledExpertFFN  tests/moe_cpu_sim.cpp:395-494
//   TiledCombine    tests/moe_cpu_sim.cpp:499-538
//   TiledMoE        tests/moe_cpu_sim.cpp:543-569
// and time a multi-threaded NaiveMoE over token slices (rows are independent, so a
// slice gives the same rows as the whole call).
#include MOE_CPU_SIM_SRC

#include <thread>

namespace {
struct RefCtx {
    std::vector<float> x, w_gate, ew;
    int T, H, E, K, I;
};
std::vector<float> vec(const float* p, size_t n) { return std::vector<float>(p, p + n); }
}  // namespace

namespace {
// Runs `path` (NaiveMoE or TiledMoE) over tokens [t0, t1), split into nthreads
// contiguous token ranges on nthreads threads; y receives (t1-t0) rows.
template <class Path>
void ctx_run(RefCtx* c, int t0, int t1, int nthreads, float* y, Path path)
{
    int n = t1 - t0;
    if (n <= 0) return;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > n) nthreads = n;
    auto work = [&](int a, int b) {
        std::vector<float> xs(c->x.begin() + (size_t)a * c->H, c->x.begin() + (size_t)b * c->H);
        std::vector<float> out;
        path(xs, c->w_gate, c->ew, b - a, c->H, c->E, c->K, c->I, out);
        std::copy(out.begin(), out.end(), y + (size_t)(a - t0) * c->H);
    };
    std::vector<std::thread> th;
    for (int i = 0; i < nthreads; i++) {
        int a = t0 + (int)((long long)n * i / nthreads);
        int b = t0 + (int)((long long)n * (i + 1) / nthreads);
        th.emplace_back(work, a, b);
    }
    for (auto& t : th) t.join();
}
}  // namespace

extern "C" {

void ref_naive_moe(const float* x, const float* wg, const float* ew, int T, int H, int E, int K,
                   int I, float* y)
{
    std::vector<float> out;
    NaiveMoE(vec(x, (size_t)T * H), vec(wg, (size_t)H * E), vec(ew, (size_t)E * 3 * I * H), T, H,
             E, K, I, out);
    std::copy(out.begin(), out.end(), y);
}

void ref_tiled_moe(const float* x, const float* wg, const float* ew, int T, int H, int E, int K,
                   int I, float* y)
{
    std::vector<float> out;
    TiledMoE(vec(x, (size_t)T * H), vec(wg, (size_t)H * E), vec(ew, (size_t)E * 3 * I * H), T, H,
             E, K, I, out);
    std::copy(out.begin(), out.end(), y);
}

void ref_tiled_routing(const float* x, const float* wg, int T, int H, int E, int K, int32_t* ids,
                       float* weights)
{
    auto tiling = ComputeRoutingTiling(T, H, E, K);
    std::vector<int> eid;
    std::vector<float> w;
    TiledRouting(vec(x, (size_t)T * H), vec(wg, (size_t)H * E), T, H, E, K, tiling, eid, w);
    for (size_t i = 0; i < eid.size(); i++) ids[i] = eid[i];
    std::copy(w.begin(), w.end(), weights);
}

void ref_tiled_expert_ffn(const float* x, const float* ew, const int32_t* ids, const float* weights,
                          int T, int H, int E, int K, int I, float* ffn_out)
{
    auto tiling = ComputeExpertFFNTiling(T, H, I, E, K);
    std::vector<int> eid(ids, ids + (size_t)T * K);
    std::vector<float> out;
    TiledExpertFFN(vec(x, (size_t)T * H), vec(ew, (size_t)E * 3 * I * H), eid,
                   vec(weights, (size_t)T * K), T, H, E, K, I, tiling, out);
    std::copy(out.begin(), out.end(), ffn_out);
}

void ref_tiled_combine(const float* ffn_out, const int32_t* ids, const float* weights, int T, int H,
                       int K, float* y)
{
    auto tiling = ComputeCombineTiling(T, H, K);
    std::vector<int> eid(ids, ids + (size_t)T * K);
    std::vector<float> out;
    TiledCombine(vec(ffn_out, (size_t)T * K * H), eid, vec(weights, (size_t)T * K), T, H, K,
                 tiling, out);
    std::copy(out.begin(), out.end(), y);
}

// Context for timing: the fp32 vectors are built once, outside any timed region.
void* ref_ctx_create(const float* x, const float* wg, const float* ew, int T, int H, int E, int K,
                     int I)
{
    RefCtx* c = new RefCtx;
    c->x = vec(x, (size_t)T * H);
    c->w_gate = vec(wg, (size_t)H * E);
    c->ew = vec(ew, (size_t)E * 3 * I * H);
    c->T = T; c->H = H; c->E = E; c->K = K; c->I = I;
    return c;
}

void ref_ctx_destroy(void* h) { delete static_cast<RefCtx*>(h); }

// TiledMoE (tests/moe_cpu_sim.cpp:543-569) over tokens [t0, t1) on nthreads threads.
void ref_ctx_tiled(void* h, int t0, int t1, int nthreads, float* y)
{
    ctx_run(static_cast<RefCtx*>(h), t0, t1, nthreads, y,
            [](const std::vector<float>& x, const std::vector<float>& wg, const std::vector<float>& ew, int T,
               int H, int E, int K, int I, std::vector<float>& out) { TiledMoE(x, wg, ew, T, H, E, K, I, out); });
}

// NaiveMoE over tokens [t0, t1), split over nthreads threads; y receives
// (t1-t0) rows.  Which is what tests/moe_cpu_sim.cpp computes for those rows.
void ref_ctx_naive(void* h, int t0, int t1, int nthreads, float* y)
{
    ctx_run(static_cast<RefCtx*>(h), t0, t1, nthreads, y,
            [](const std::vector<float>& x, const std::vector<float>& wg, const std::vector<float>& ew, int T,
               int H, int E, int K, int I, std::vector<float>& out) { NaiveMoE(x, wg, ew, T, H, E, K, I, out); });
}

}  // extern "C"
