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
def reference_inputs(cfg, moe):
    """The configuration's inputs as fp32 numpy (fp16-rounded values), drawn on the CPU."""
    import numpy as np

    T, H, E, K, I, seed = moe.CONFIGS[cfg]
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, seed, device="cpu", zipf=moe.inputs.ZIPF.get(cfg))
    return (x.float().numpy(), wg.float().numpy(), ew.float().numpy().astype(np.float32, copy=False)), \
        (T, H, E, K, I)


def cpu_reference_timer(cfg, moe):
    """(timer object, kind): the reference's NaiveMoE (oracle/_ref) or, when that was
    not built, the C restatement (oracle/_build)."""
    from oracle import oracle as O

    (x, wg, ew), (T, H, E, K, I) = reference_inputs(cfg, moe)
    if O.ref_available():
        t = O.RefTimer(x, wg, ew, K)
        return (lambda t0, t1, th: t.naive(t0, t1, th)), "reference", (T, H, E, K, I), t
    def run(t0, t1, th):
        return O.moe_naive(x[t0:t1], wg, ew, K, nthreads=th)[0]
    return run, "port", (T, H, E, K, I), None


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    moe = __import__("_moe_loader").load()
    run, kind, (T, H, E, K, I), keep = cpu_reference_timer(args.config, moe)
    threads = os.cpu_count() or 1
    sample = args.ref_tokens
    times = []
    t0 = 0
    for step in range(args.warmup + args.steps):
        a = t0 % T
        b = min(a + sample, T)
        s = time.perf_counter()
        run(a, b, threads)
        dt = time.perf_counter() - s
        if step >= args.warmup:
            times.append((b - a) / dt)
        t0 += sample
    value = statistics.mean(times)
    ms_per_step = 1000.0 * sample / value
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config} T={T} H={H} E={E} K={K} I={I}; each step = NaiveMoE on a "
                               f"{sample}-token slice", "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"{sample} tokens of the {args.config} batch per step, NaiveMoE "
                                   f"(tests/moe_cpu_sim.cpp:183-306) split over {threads} threads"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    if keep is not None:
        keep.close()
    return 0


# ============================================================================ our arm
def cpu_baseline_sample(args, moe):
    """The reference's CPU code on a bounded sample of the same workload (rank 0,
    N=1): successive slices of the batch (wrapping at its end) until at least
    --cpu-seconds of CPU time; tokens/s over the whole sample."""
    run, kind, (T, H, E, K, I), keep = cpu_reference_timer(args.config, moe)
    threads = os.cpu_count() or 1
    chunk = max(1, min(args.ref_tokens, T))
    run(0, min(threads, T), threads)  # warm-up: page in the weights
    tokens, spent, a = 0, 0.0, 0
    while spent < args.cpu_seconds:
        b = min(a + chunk, T)
        s = time.perf_counter()
        run(a, b, threads)
        spent += time.perf_counter() - s
        tokens += b - a
        a = b % T
    if keep is not None:
        keep.close()
    return {"value": tokens / spent, "unit": "tokens/s", "cores": threads, "kind": kind,
            "sample": f"{tokens} tokens of the {args.config} batch in slices of {chunk} from token 0, NaiveMoE "
                      f"(tests/moe_cpu_sim.cpp:183-306) over {threads} threads, {spent:.1f} s"}


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
        # token rows with NCCL send/recv inside MoeEpLayerForward
        if E % world:
            raise SystemExit(f"E={E} is not divisible by {world} GPUs")
        El = E // world
        ew = ew[rank * El:(rank + 1) * El].contiguous()
        torch.cuda.empty_cache()
        uid = [moe.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ep = moe.EpContext(uid[0], rank, world, timeout_ms=120000)
        ws = torch.empty((ep.workspace_size(T, H, E, K, I),), dtype=torch.uint8, device=dev)

        def step(xin=None):
            ep.forward(x if xin is None else xin, wg, ew, K, y=y, workspace=ws)
    else:
        ws = torch.empty((moe.moe_layer_workspace_size(T, H, E, K, I),), dtype=torch.uint8, device=dev)

        def step(xin=None):
            moe.moe_layer_forward(x if xin is None else xin, wg, ew, K, y=y, workspace=ws)

    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    if moe.device_error(ws) != 0:
        raise RuntimeError("device error during warm-up")

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    # stage times (and the roofline kernel's duration): a second pass of the same K
    # steps with CUDA events at the stage boundaries, kept out of the timed region so
    # the events do not stand between the kernels there
    moe.trace_start(args.steps)
    for i in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    stages = moe.trace_stop(args.steps)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    if moe.device_error(ws) != 0:
        raise RuntimeError("device error during the timed steps")

    # End to end through the public API, as a serving loop would run it: every step
    # copies its own x from pinned host memory and its y back to pinned host memory;
    # the copies run on two copy streams (H2D, D2H) so that step i+1's input and
    # step i-1's output cross PCIe while step i computes.  The timed region spans
    # the first H2D to the last D2H (inputs > L2: the weights alone are 1.6 GB).
    x_host = [x.cpu().pin_memory(), x.cpu().pin_memory()]
    y_host = [torch.empty((T, H), dtype=torch.float16).pin_memory() for _ in range(2)]
    x_dev = [torch.empty_like(x), torch.empty_like(x)]
    y_dev = [torch.empty_like(y), torch.empty_like(y)]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731

    def e2e_run(nsteps):
        in_ready = [ev(), ev()]
        x_free = [None, None]   # compute finished reading x_dev[b]
        y_free = [None, None]   # D2H finished reading y_dev[b]
        t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
            if ep is not None:
                ep.forward(x_dev[b], wg, ew, K, y=y_dev[b], workspace=ws)
            else:
                moe.moe_layer_forward(x_dev[b], wg, ew, K, y=y_dev[b], workspace=ws)
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
        torch.cuda.synchronize()
        return t_start.elapsed_time(t_end)

    e2e_run(args.warmup)
    e2e_ms = e2e_run(args.steps)

    t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = float(t[0]), float(t[1])
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
        e2e_value = world * T * args.steps / (e2e_ms / 1e3)
        stage_avg = {k: statistics.mean(c[k] for c in stages) for k in moe.TRACE_STAGES}
        g1_flops = 2.0 * T * K * H * 2 * I
        g2_flops = 2.0 * T * K * I * H
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
                         "peak_source": f"{peak_src} bf16_tflops (burst cuBLAS)",
                         # the kernel runs inside back-to-back layer steps under the power cap, so
                         # the sustained cuBLAS figure is the other fair denominator
                         "peak_sustained": peak_sus, "frac_of_sustained": ach / peak_sus if peak_sus else None,
                         "traffic": traffic},
            "ffn": {"tflops": ffn_tf, "frac_of_peak": ffn_tf / peak, "ms": ffn_ms,
                    "frac_of_datasheet_2250": ffn_tf / 2250.0},
            "stages_ms": stage_avg,
            "stages_how": "CUDA events at stage boundaries, a second pass of the same steps",
            "hbm_kernels": {"combine_gbs": comb_bytes / (stage_avg["combine"] / 1e3) / 1e9 if stage_avg["combine"] else None,
                            "routing_gbs": rout_bytes / (stage_avg["routing"] / 1e3) / 1e9 if stage_avg["routing"] else None,
                            "hbm_peak_gbs": hbm},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                    "d2h_bytes_per_step": T * H * 2,
                    "how": "pinned host x -> device -> layer -> pinned host y every step; H2D and D2H on "
                           "two copy streams overlapping the neighbouring steps' compute"},
            # per step, one GPU: routing, fused permute, gather, gate/up GEMM, down GEMM,
            # combine; expert parallel adds the count, plan, dispatch, row-pointer and two
            # wait kernels and replaces gather + combine with the indexed combine
            "gpu_launches": args.steps * (11 if world > 1 else 6),
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline_sample(args, moe)
            except Exception as exc:  # reported, never fatal for the GPU number
                line["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
        print(json.dumps(line), flush=True)
    if ep is not None:
        ep.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


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
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="N>1: weak = T tokens per GPU (default); strong = the config's T split over the GPUs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
