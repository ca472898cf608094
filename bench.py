#!/usr/bin/env python
"""Benchmark of the MoE layer hot path: routing -> permute -> expert FFN -> combine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config prefill] [--impl ours|reference]

Metric: MoE layer tokens/s on the headline configuration T=4096, H=2048, E=16,
K=2, I=8192 (fp16 in/out, fp32 accumulation), synthetic seeded inputs with the
benchmark's distributions.  A step is one full layer forward over one batch.

* ``value``: whole-job tokens/s with inputs resident in HBM, device time of the K
  timed steps (CUDA events, max over ranks), L2 flushed between steps.
* ``e2e``: the same through the public API with the step's x copied host->device
  from pinned memory and y copied back inside the timed region.
* ``roofline``: the dominant kernel (gate/up grouped GEMM + SwiGLU), its FLOP/s
  from the stage events of the timed steps against the measured bf16/fp16 peak.
* ``cpu_baseline``: the reference's own CPU code (tests/moe_cpu_sim.cpp NaiveMoE,
  compiled into oracle/_ref) on a bounded token slice, rank 0 at N=1 only.

``--impl reference`` times that CPU reference alone (all host threads) and prints
the same JSON line with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

METRIC = "MoE layer tokens/s (T=4096,H=2048,E=16,K=2,I=8192); FFN % FP16 TC peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 512 << 20  # > 126 MB L2


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.isfile(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(key):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/)."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    if not os.path.isfile(p):
        return None
    with open(p) as f:
        for line in f:
            parts = line.split()
            if len(parts) >= 2 and parts[0] == key:
                try:
                    return float(parts[1])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def __enter__(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.tmp is None:
            return None
        self.tmp.flush()
        with open(self.tmp.name) as f:
            rows = [r.split(",") for r in f.read().strip().splitlines() if r.strip()]
        os.unlink(self.tmp.name)
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax = max(smax, float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        load = [v for v in sm if v > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ============================================================================ reference arm
def reference_inputs(cfg, moe, tensors=None):
    """The configuration's inputs as fp32 numpy (fp16-rounded values).  `tensors`:
    the GPU arm's own (x, w_gate, expert_weights); otherwise they are drawn the way
    the GPU arm draws them (on the GPU when there is one: torch's generator gives a
    different stream on the CPU)."""
    import numpy as np
    import torch

    T, H, E, K, I, seed = moe.CONFIGS[cfg]
    if tensors is None:
        dev = "cuda" if torch.cuda.is_available() else "cpu"
        tensors = moe.make_inputs_torch(T, H, E, K, I, seed, device=dev, zipf=moe.inputs.ZIPF.get(cfg))
    x, wg, ew = (t.cpu() for t in tensors)
    return (x.float().numpy(), wg.float().numpy(), ew.float().numpy().astype(np.float32, copy=False)), \
        (T, H, E, K, I)


class CpuReference:
    """The reference's CPU layer on token slices: NaiveMoE (tests/moe_cpu_sim.cpp:183-306)
    and TiledMoE (:543-569) from oracle/_ref, or, when that was not built, the C
    restatement of NaiveMoE (oracle/_build; no tiled path)."""

    def __init__(self, cfg, moe, tensors=None):
        from oracle import oracle as O

        (self.x, self.wg, self.ew), self.shape = reference_inputs(cfg, moe, tensors)
        self.O = O
        self.kind = "reference" if O.ref_available() else "port"
        self.t = O.RefTimer(self.x, self.wg, self.ew, self.shape[3]) if self.kind == "reference" else None

    def run(self, path, t0, t1, threads):
        if self.t is not None:
            return (self.t.naive if path == "naive" else self.t.tiled)(t0, t1, threads)
        if path != "naive":
            raise RuntimeError("TiledMoE needs oracle/_ref")
        return self.O.moe_naive(self.x[t0:t1], self.wg, self.ew, self.shape[3], nthreads=threads)[0]

    def close(self):
        if self.t is not None:
            self.t.close()


def cpu_slices(ref, path, chunk, threads, min_seconds=0.0, steps=None):
    """Successive `chunk`-token slices of the batch from token 0 (wrapping), each run
    over `threads` threads; either `steps` slices or whole slices until at least
    min_seconds.  Returns (per-slice tokens/s list, tokens, seconds)."""
    T = ref.shape[0]
    chunk = max(1, min(chunk, T))
    rates, tokens, spent, a, n = [], 0, 0.0, 0, 0
    while (steps is not None and n < steps) or (steps is None and spent < min_seconds):
        b = min(a + chunk, T)
        s = time.perf_counter()
        ref.run(path, a, b, threads)
        dt = time.perf_counter() - s
        rates.append((b - a) / dt)
        spent += dt
        tokens += b - a
        a = b % T
        n += 1
    return rates, tokens, spent


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    moe = __import__("_moe_loader").load()
    ref = CpuReference(args.config, moe)
    T, H, E, K, I = ref.shape
    threads = os.cpu_count() or 1
    sample = min(args.ref_tokens, T)
    cpu_slices(ref, "naive", sample, threads, steps=args.warmup)  # pages the weights in
    rates, tokens, spent = cpu_slices(ref, "naive", sample, threads, steps=args.steps)
    value = tokens / spent
    tiled = None
    if ref.kind == "reference":
        tr, ttok, tsp = cpu_slices(ref, "tiled", sample, threads, steps=max(1, args.steps // 4))
        tiled = {"value": ttok / tsp, "unit": "tokens/s", "steps": len(tr),
                 "sample": f"TiledMoE (tests/moe_cpu_sim.cpp:543-569) on {len(tr)} slices of {sample} tokens"}
    ref.close()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 1, "ranks_used": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * spent / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config} T={T} H={H} E={E} K={K} I={I}; each step = NaiveMoE on a "
                               f"{sample}-token slice of the batch (successive slices from token 0)",
                   "parallelism": "host threads", "same_protocol_as": "the GPU arm's cpu_baseline"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": ref.kind,
                         "sample": f"{tokens} tokens in slices of {sample} from token 0, NaiveMoE "
                                   f"(tests/moe_cpu_sim.cpp:183-306) split over {threads} threads, {spent:.1f} s",
                         "tiled": tiled},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ============================================================================ our arm
def cpu_baseline_sample(args, moe, tensors, ids_gpu=None):
    """The reference's CPU code on a bounded sample of the same workload (rank 0,
    N=1): NaiveMoE on successive slices of the batch until at least --cpu-seconds,
    then TiledMoE for a third of that; tokens/s over each whole sample.  Also the
    near-tie census of the routing: the oracle's ids over the whole batch against the
    GPU's (ids_gpu), tokens whose oracle top-(K+1) logit margin is < 1e-3 counted
    apart (the reference's own tie order is unspecified, tests/moe_cpu_sim.cpp:232-233)."""
    import numpy as np

    ref = CpuReference(args.config, moe, tensors)
    T, H, E, K, I = ref.shape
    threads = os.cpu_count() or 1
    chunk = max(1, min(args.ref_tokens, T))
    ref.run("naive", 0, min(threads, T), threads)  # warm-up: page in the weights
    _, tokens, spent = cpu_slices(ref, "naive", chunk, threads, min_seconds=args.cpu_seconds)
    out = {"value": tokens / spent, "unit": "tokens/s", "cores": threads, "kind": ref.kind,
           "sample": f"{tokens} tokens of the {args.config} batch in slices of {chunk} from token 0, NaiveMoE "
                     f"(tests/moe_cpu_sim.cpp:183-306) over {threads} threads, {spent:.1f} s"}
    if ref.kind == "reference":
        _, ttok, tsp = cpu_slices(ref, "tiled", chunk, threads, min_seconds=args.cpu_seconds / 3)
        out["tiled"] = {"value": ttok / tsp, "unit": "tokens/s",
                        "sample": f"{ttok} tokens in slices of {chunk}, TiledMoE (tests/moe_cpu_sim.cpp:543-569) "
                                  f"over {threads} threads, {tsp:.1f} s"}
    if ids_gpu is not None:
        rid, _, _, _, margin = ref.O.routing(ref.x, ref.wg, K)
        diff = np.any(ids_gpu != rid, axis=1)
        near = margin < 1e-3
        out["routing_parity"] = {"tokens": int(T), "near_ties": int(near.sum()),
                                 "near_ties_differing": int((diff & near).sum()),
                                 "differing_away_from_ties": int((diff & ~near).sum()),
                                 "near_tie_rule": "oracle top-(K+1) logit margin < 1e-3"}
    ref.close()
    return out


def _timed_steps(step, flush, stream, n, world):
    """n steps, each after an L2 flush, bracketed by a barrier and a device sync on
    both sides; -> per-step milliseconds (CUDA events on the launching stream)."""
    import torch
    import torch.distributed as dist

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(n):
        flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return [s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)]


def _max_over_ranks(vals, world, dev):
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    moe = __import__("_moe_loader").load()
    T, H, E, K, I, seed = moe.CONFIGS[args.config]
    dev = torch.device("cuda", local)
    # weak scaling: every rank routes its own batch of T tokens (per-GPU work fixed
    # as N grows); strong scaling: the config's one batch of T tokens is split into
    # N slices of T/N.  The weights are one model (same seed on every rank).
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, seed, device=dev, zipf=moe.inputs.ZIPF.get(args.config))
    x_cfg, ew_full = x, ew  # the config's batch and all experts (parity checks, strong record)
    T_total = T
    if args.scaling == "strong" and world > 1:
        if T % world:
            raise SystemExit(f"T={T} is not divisible by {world} GPUs")
        T = T_total // world
        x = x[rank * T:(rank + 1) * T].contiguous()
    elif rank > 0:
        x = moe.make_inputs_torch(T, H, 1, 1, 8, seed + rank, device=dev)[0]
    y = torch.empty((T, H), dtype=torch.float16, device=dev)
    flush = torch.empty((L2_FLUSH_BYTES,), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ep = None
    if world > 1:
        # expert parallel: rank r keeps experts [r*E/N, (r+1)*E/N) and exchanges
        # token rows with its peers inside MoeEpLayerForward
        if E % world:
            raise SystemExit(f"E={E} is not divisible by {world} GPUs")
        El = E // world
        ew = ew_full[rank * El:(rank + 1) * El].contiguous()
        uid = [moe.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ep = moe.EpContext(uid[0], rank, world, timeout_ms=120000)
        ws = torch.empty((ep.workspace_size(T, H, E, K, I),), dtype=torch.uint8, device=dev)

        def layer(xin, yout):
            ep.forward(xin, wg, ew, K, y=yout, workspace=ws)
    else:
        ws = torch.empty((moe.moe_layer_workspace_size(T, H, E, K, I),), dtype=torch.uint8, device=dev)

        def layer(xin, yout):
            moe.moe_layer_forward(xin, wg, ew, K, y=yout, workspace=ws)

    def step():
        layer(x, y)

    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    if moe.device_error(ws) != 0:
        raise RuntimeError("device error during warm-up")

    with ClockSampler(local) as clk:
        step_ms = _timed_steps(step, flush, stream, args.steps, world)
    total_ms = sum(step_ms)
    # stage times (and the roofline kernel's duration): a second pass of the same K
    # steps with CUDA events at the stage boundaries, kept out of the timed region so
    # the events do not stand between the kernels there
    if world > 1:
        dist.barrier()
    moe.trace_start(args.steps)
    for i in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    stages = moe.trace_stop(args.steps)
    if moe.device_error(ws) != 0:
        raise RuntimeError("device error during the timed steps")

    # ---- expert-parallel parity: rank r's y rows against the single-GPU layer with
    # all experts on the same tokens (bit for bit: every kernel is the same)
    ep_parity = None
    if world > 1:
        # the single-GPU call gets the rank's whole batch: the routing kernel's split of
        # H over a CTA cluster (hence its fp32 sum order) depends on T
        S = min(256, T)
        y_one = moe.moe_layer_forward(x, wg, ew_full, K)[:S]
        torch.cuda.synchronize()
        eq = torch.tensor([float(torch.equal(y_one, y[:S])), float((y_one.float() - y[:S].float()).abs().max())],
                          dtype=torch.float64, device=dev)
        allv = [torch.empty_like(eq) for _ in range(world)]
        dist.all_gather(allv, eq)
        ep_parity = {"tokens_per_rank": S, "ranks_bit_equal": int(sum(v[0].item() for v in allv)),
                     "ranks": world, "max_abs_diff": max(v[1].item() for v in allv),
                     "against": "MoeLayerForward on one GPU with all experts, same tokens"}

    # ---- end to end through the public API, as a serving loop would run it: every
    # step copies its own x from pinned host memory and its y back to pinned host
    # memory; the copies run on two copy streams (H2D, D2H) so that step i+1's input
    # and step i-1's output cross PCIe while step i computes.  The timed region spans
    # the first H2D to the last D2H (inputs > L2: the weights alone are 1.6 GB).  All
    # ranks start together (barrier), and the run lasts at least --e2e-seconds.
    x_host = [x.cpu().pin_memory(), x.cpu().pin_memory()]
    y_host = [torch.empty((T, H), dtype=torch.float16).pin_memory() for _ in range(2)]
    x_dev = [torch.empty_like(x), torch.empty_like(x)]
    y_dev = [torch.empty_like(y), torch.empty_like(y)]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731

    host_ms = [0.0]  # host time to enqueue the last e2e run

    def e2e_run(nsteps, compute=True):
        in_ready = [ev(), ev()]
        x_free = [None, None]   # compute finished reading x_dev[b]
        y_free = [None, None]   # D2H finished reading y_dev[b]
        t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        host0 = time.perf_counter()
        t_start.record(h2d)
        with torch.cuda.stream(h2d):
            x_dev[0].copy_(x_host[0], non_blocking=True)
        in_ready[0].record(h2d)
        for i in range(nsteps):
            b = i & 1
            if i + 1 < nsteps:
                nb = (i + 1) & 1
                if x_free[nb] is not None:
                    h2d.wait_event(x_free[nb])
                with torch.cuda.stream(h2d):
                    x_dev[nb].copy_(x_host[nb], non_blocking=True)
                in_ready[nb] = ev()
                in_ready[nb].record(h2d)
            stream.wait_event(in_ready[b])
            if y_free[b] is not None:
                stream.wait_event(y_free[b])
            if compute:
                layer(x_dev[b], y_dev[b])
            done = ev()
            done.record(stream)
            x_free[b] = done
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                y_host[b].copy_(y_dev[b], non_blocking=True)
            y_free[b] = ev()
            y_free[b].record(d2h)
        h2d.wait_stream(d2h)
        t_end.record(h2d)
        host_ms[0] = (time.perf_counter() - host0) * 1e3
        torch.cuda.synchronize()
        return t_start.elapsed_time(t_end)

    # every rank must make the same number of layer calls (the expert-parallel
    # exchange pairs call c of every rank), so the step counts below come from the
    # step time agreed over the ranks
    mean_ms = _max_over_ranks([total_ms / args.steps], world, dev)[0]
    e2e_steps = max(args.steps, int(args.e2e_seconds * 1000.0 / max(mean_ms, 1e-3)) + 1)
    e2e_run(args.warmup)
    e2e_ms = e2e_run(e2e_steps)
    e2e_host_ms = host_ms[0]
    e2e_err = moe.device_error(ws)
    # the host-copy ceiling: the same copies on the same streams with no layer
    copy_ms = e2e_run(e2e_steps, compute=False)
    h2d_ms = _copy_only(x_host[0], x_dev[0], h2d, e2e_steps, world)
    d2h_ms = _copy_only(y_dev[0], y_host[0], d2h, e2e_steps, world)
    per_rank_copy = [h2d_ms, d2h_ms]

    # ---- sustained: back-to-back layer steps for --sustained-seconds (the serving
    # case under the power cap), clocks sampled over them; then a traced pass of 20
    # steps while the GPU is still hot, for GEMM1's rate at those clocks
    sus_steps = int(args.sustained_seconds * 1000.0 / max(mean_ms, 1e-3)) + 1 if args.sustained_seconds > 0 else 0
    sus = None
    if sus_steps:
        with ClockSampler(local) as clk_sus:
            sus_ms = _timed_steps(step, flush, stream, sus_steps, world)
            moe.trace_start(20)
            for _ in range(20):
                flush.zero_()
                step()
            torch.cuda.synchronize()
            sus_stages = moe.trace_stop(20)
        sus = {"steps": sus_steps, "ms_total": sum(sus_ms), "clk": clk_sus.summary(),
               "g1_ms": statistics.mean(c["gemm_swiglu"] for c in sus_stages),
               "median_step_ms": statistics.median(sus_ms), "max_step_ms": max(sus_ms),
               "steps_over_2x_median": sum(1 for m in sus_ms if m > 2 * statistics.median(sus_ms)),
               "device_error": moe.device_error(ws)}

    # ---- strong scaling record (N>1): the config's one batch of T tokens split over
    # the N ranks, same process; efficiency against rank 0's single-GPU layer on the
    # whole batch with all experts
    strong = None
    if world > 1 and args.scaling == "weak" and not args.no_strong:
        strong = _strong_record(args, moe, x_cfg, wg, ew_full, ew, ep, K, H, E, I, T_total, flush, stream,
                                rank, world, dev)

    r = _max_over_ranks([total_ms, e2e_ms, copy_ms, h2d_ms, d2h_ms] + ([sus["ms_total"]] if sus else []), world, dev)
    total_ms, e2e_ms, copy_ms = r[0], r[1], r[2]
    if sus:
        sus["ms_total"] = r[5]
    copies = [torch.zeros(2, dtype=torch.float64, device=dev) for _ in range(world)]
    if world > 1:
        dist.all_gather(copies, torch.tensor(per_rank_copy, dtype=torch.float64, device=dev))
    else:
        copies = [torch.tensor(per_rank_copy, dtype=torch.float64)]
    # expert load over the whole job: (token, slot) rows per expert, summed over the
    # ranks; with expert parallelism the busiest rank's rows set the step time
    ids_chk, _ = moe.moe_routing_topk(x, wg, K)
    counts = torch.bincount(ids_chk.flatten().long(), minlength=E)
    counts_rank0 = counts.clone()
    if world > 1:
        dist.all_reduce(counts)
    rank_rows = counts.view(world, E // world).sum(1).tolist() if world > 1 else [int(counts.sum())]

    if rank == 0:
        peaks, peak_src = load_peaks()
        ms = total_ms / args.steps
        value = world * T * args.steps / (total_ms / 1e3)
        e2e_value = world * T * e2e_steps / (e2e_ms / 1e3)
        stage_avg = {k: statistics.mean(c[k] for c in stages) for k in moe.TRACE_STAGES}
        # GEMM FLOPs on the rows this rank's experts received (weak: ~T*K per rank)
        rows0 = rank_rows[0] if world > 1 else T * K
        g1_flops = 2.0 * rows0 * H * 2 * I
        g2_flops = 2.0 * rows0 * I * H
        g1_ms = stage_avg["gemm_swiglu"]
        ach = g1_flops / (g1_ms / 1e3) / 1e12
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        peak_sus = float(peaks["bf16_tflops_sustained"]) if "bf16_tflops_sustained" in peaks else None
        ffn_ms = stage_avg["gemm_swiglu"] + stage_avg["gemm_down"]
        ffn_tf = (g1_flops + g2_flops) / (ffn_ms / 1e3) / 1e12
        traffic = load_traffic(f"gemm_swiglu_{args.config}")
        hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        comb_bytes = T * K * H * 2 + T * K * 2 + T * H * 2
        rout_bytes = T * H * 2 + H * E * 2 + T * K * 6
        load = counts_rank0.float() / ids_chk.numel()
        xbytes = T * H * 2
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            # the metric is also quoted as the median step (rank 0's step times); value is the mean
            "ms_per_step_median": statistics.median(step_ms),
            "value_median": world * T / (statistics.median(step_ms) / 1e3), "scaling": args.scaling,
            "vs_baseline": None, "dtype": "fp16 in/out, fp32 accumulate", "data": "synthetic",
            "config": {"workload": (f"{args.config} T={T} H={H} E={E} K={K} I={I} per GPU" if args.scaling == "weak" or world == 1
                                    else f"{args.config} T={T_total} H={H} E={E} K={K} I={I} split over {world} GPUs ({T} per GPU)"),
                       "global_batch": world * T, "parallelism": f"ep{world} (expert parallel, peer-memory row exchange over NVLink)" if world > 1 else "single GPU",
                       "l2": "flushed between timed steps (512 MB write)", "inputs": "seeded N(0,1)/N(0,1/fan_in) fp16" + (
                           ", w_gate columns scaled toward Zipf s=1 expert load" if args.config in moe.inputs.ZIPF else ""),
                       "expert_load_rank0": [round(v, 4) for v in load.tolist()],
                       "rows_per_rank": rank_rows,
                       "load_imbalance": max(rank_rows) / (sum(rank_rows) / len(rank_rows)) if sum(rank_rows) else None},
            "roofline": {"kernel": "gemm_swiglu (gate/up grouped GEMM + SwiGLU epilogue)", "bound": "tensor",
                         "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                         "rows": rows0,
                         "peak_source": f"{peak_src} bf16_tflops (burst cuBLAS)",
                         # the kernel runs inside back-to-back layer steps under the power cap, so
                         # the sustained cuBLAS figure is the other fair denominator
                         "peak_sustained": peak_sus, "frac_of_sustained": ach / peak_sus if peak_sus else None,
                         "traffic": traffic},
            "ffn": {"tflops": ffn_tf, "frac_of_peak": ffn_tf / peak, "ms": ffn_ms,
                    "frac_of_datasheet_2250": ffn_tf / 2250.0},
            "stages_ms": stage_avg,
            "stages_how": "CUDA events at stage boundaries, a second pass of the same steps (rank 0)",
            "hbm_kernels": {"combine_gbs": comb_bytes / (stage_avg["combine"] / 1e3) / 1e9 if stage_avg["combine"] else None,
                            "routing_gbs": rout_bytes / (stage_avg["routing"] / 1e3) / 1e9 if stage_avg["routing"] else None,
                            "hbm_peak_gbs": hbm},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": xbytes,
                    "d2h_bytes_per_step": xbytes, "steps": e2e_steps, "ms": e2e_ms,
                    "how": "pinned host x -> device -> layer -> pinned host y every step; H2D and D2H on "
                           "two copy streams overlapping the neighbouring steps' compute; ranks start "
                           "together (barrier); max over ranks",
                    "copy_only_ceiling": world * T * e2e_steps / (copy_ms / 1e3),
                    "host_enqueue_ms_rank0": e2e_host_ms, "device_error_rank0": e2e_err,
                    "per_rank_copy_gbs": [{"h2d": xbytes * e2e_steps / (c[0].item() / 1e3) / 1e9,
                                           "d2h": xbytes * e2e_steps / (c[1].item() / 1e3) / 1e9} for c in copies]},
            # per step, one GPU: routing, fused permute, gather, gate/up GEMM, down GEMM,
            # combine; expert parallel: routing, permute, counts + plan + return addresses,
            # dispatch, gate/up GEMM (waits per source), down GEMM, combine on arrival
            "gpu_launches": args.steps * (7 if world > 1 else 6),
            "clocks": clk.summary(),
        }
        if ep_parity is not None:
            line["ep_parity"] = ep_parity
        if sus:
            sv = world * T * sus["steps"] / (sus["ms_total"] / 1e3)
            g1s = g1_flops / (sus["g1_ms"] / 1e3) / 1e12
            line["sustained"] = {"value": sv, "unit": "tokens/s", "steps": sus["steps"],
                                 "median_step_ms_rank0": sus["median_step_ms"], "max_step_ms_rank0": sus["max_step_ms"],
                                 "steps_over_2x_median_rank0": sus["steps_over_2x_median"],
                                 "device_error_rank0": sus["device_error"],
                                 "seconds": sus["ms_total"] / 1e3, "clocks": sus["clk"],
                                 "gemm_swiglu_tflops": g1s,
                                 "gemm_swiglu_frac_of_sustained": g1s / peak_sus if peak_sus else None,
                                 "gemm_swiglu_frac_of_burst": g1s / peak,
                                 "how": "back-to-back layer steps (L2 flush between), device time, max over "
                                        "ranks; GEMM1 from a traced pass of 20 steps right after"}
        if strong is not None:
            line["strong"] = strong
        if world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline_sample(args, moe, (x, wg, ew), ids_gpu=ids_chk.cpu().numpy())
            except Exception as exc:  # reported, never fatal for the GPU number
                line["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
        print(json.dumps(line), flush=True)
    if ep is not None:
        ep.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def _copy_only(src, dst, s, n, world):
    """n back-to-back copies src -> dst on stream s, all ranks at once -> ms."""
    import torch
    import torch.distributed as dist

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a.record(s)
    with torch.cuda.stream(s):
        for _ in range(n):
            dst.copy_(src, non_blocking=True)
    b.record(s)
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def _strong_record(args, moe, x_cfg, wg, ew_full, ew_local, ep, K, H, E, I, T_total, flush, stream, rank,
                   world, dev):
    """The config's batch of T_total tokens split into N slices of T_total/N, one per
    rank, through the same expert-parallel context; y checked bit for bit against the
    single-GPU layer on the same tokens; efficiency against rank 0's single-GPU
    layer on the whole batch."""
    import torch
    import torch.distributed as dist

    if T_total % world:
        return {"skipped": f"T={T_total} not divisible by {world}"}
    Tl = T_total // world
    xs = x_cfg[rank * Tl:(rank + 1) * Tl].contiguous()
    ys = torch.empty((Tl, H), dtype=torch.float16, device=dev)
    ws = torch.empty((ep.workspace_size(Tl, H, E, K, I),), dtype=torch.uint8, device=dev)

    def st():
        ep.forward(xs, wg, ew_local, K, y=ys, workspace=ws)

    for _ in range(args.warmup):
        flush.zero_()
        st()
    torch.cuda.synchronize()
    ms = _timed_steps(st, flush, stream, args.steps, world)
    dist.barrier()
    moe.trace_start(args.steps)
    for _ in range(args.steps):
        flush.zero_()
        st()
    torch.cuda.synchronize()
    stages = moe.trace_stop(args.steps)
    err = moe.device_error(ws)
    y_one = moe.moe_layer_forward(xs, wg, ew_full, K)
    torch.cuda.synchronize()
    eq = float(torch.equal(y_one, ys))
    ids, _ = moe.moe_routing_topk(xs, wg, K)
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    dist.all_reduce(counts)
    rank_rows = counts.view(world, E // world).sum(1).tolist()
    # single-GPU reference run on rank 0 (the others wait at the barrier)
    single_ms = 0.0
    if rank == 0:
        y1 = torch.empty((T_total, H), dtype=torch.float16, device=dev)
        ws1 = torch.empty((moe.moe_layer_workspace_size(T_total, H, E, K, I),), dtype=torch.uint8, device=dev)

        def one():
            moe.moe_layer_forward(x_cfg, wg, ew_full, K, y=y1, workspace=ws1)

        for _ in range(args.warmup):
            flush.zero_()
            one()
        single_ms = sum(_timed_steps(one, flush, stream, args.steps, 1))
        del y1, ws1
    dist.barrier()
    t = torch.tensor([sum(ms), float(err != 0), 1.0 - eq], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, any_err, any_diff = t.tolist()
    value = T_total * args.steps / (total_ms / 1e3)
    single = T_total * args.steps / (single_ms / 1e3) if single_ms else None
    return {"value": value, "unit": "tokens/s", "T_total": T_total, "tokens_per_rank": Tl,
            "ms_per_step": total_ms / args.steps, "single_gpu_value": single,
            "efficiency": value / (world * single) if single else None,
            "rows_per_rank": rank_rows, "load_imbalance": max(rank_rows) / (sum(rank_rows) / world),
            "stages_ms_rank0": {k: statistics.mean(c[k] for c in stages) for k in moe.TRACE_STAGES},
            "ranks_bit_equal_to_single_gpu": not any_diff, "device_error": bool(any_err),
            "how": "same process after the weak record; device time, max over ranks; single-GPU value: rank 0, "
                   "MoeLayerForward on the whole batch with all experts"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="prefill")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-tokens", type=int, default=256,
                    help="tokens per CPU reference step (the reference arm) and per cpu_baseline slice")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU time the cpu_baseline sample runs for (whole slices, at least this long)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-seconds", type=float, default=1.0, help="minimum length of the timed e2e run")
    ap.add_argument("--sustained-seconds", type=float, default=3.0,
                    help="length of the sustained record (back-to-back steps); 0 skips it")
    ap.add_argument("--no-strong", action="store_true", help="N>1: skip the strong-scaling record")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="N>1: weak = T tokens per GPU (default); strong = the config's T split over the GPUs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
