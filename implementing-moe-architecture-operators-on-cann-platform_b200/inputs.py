"""Seeded synthetic inputs of the benchmark configurations.

The reference ships no dataset; its tests draw Gaussian tensors
(tests/moe_cpu_sim.cpp:161-167, :617-625).  The configurations here are the five
of the benchmark definition: x ~ N(0,1); w_gate, W_gate, W_up ~ N(0, 1/H);
W_down ~ N(0, 1/I); all rounded to fp16 (round to nearest even), which is what
both the CUDA path and the CPU checkers consume.
"""
from __future__ import annotations

import numpy as np

# name -> (T, H, E, K, I, seed); the Mixtral-shaped layer's router is skewed so that
# the expert loads follow Zipf s=1 (ZIPF below)
CONFIGS = {
    "small": (8, 64, 4, 2, 256, 42),
    "decode": (128, 2048, 16, 2, 8192, 44),
    "prefill": (4096, 2048, 16, 2, 8192, 44),
    "mixtral": (8192, 4096, 8, 2, 14336, 44),
    "deepseek": (16384, 2048, 64, 6, 1408, 44),
}
ZIPF = {"mixtral": 1.0}


def zipf_gate(x, w_gate, K, s=1.0, iters=60):
    """Scales the columns of w_gate so the realised top-K load over the tokens x
    follows Zipf(s) over the experts (expert e gets a share ~ 1/(e+1)^s of the
    T*K slots).  The operator API has no router bias, so the skew lives in
    w_gate.  Deterministic: plain fp32 torch on the tensors' device.
    Returns (fp16 w_gate, realised per-expert load fractions)."""
    import torch

    E = w_gate.shape[1]
    target = torch.tensor([1.0 / (e + 1) ** s for e in range(E)], device=x.device)
    target = target / target.sum()
    base = x.float() @ w_gate.float()  # [T, E]
    theta = torch.zeros(E, device=x.device)
    for _ in range(iters):
        ids = torch.topk(base * theta.exp(), K, dim=1).indices
        load = torch.bincount(ids.flatten(), minlength=E).float() / ids.numel()
        theta = theta + 0.5 * (target.log() - load.clamp_min(1e-5).log())
    wg = (w_gate.float() * theta.exp()).half()
    ids = torch.topk(x.float() @ wg.float(), K, dim=1).indices
    load = torch.bincount(ids.flatten(), minlength=E).float() / ids.numel()
    return wg, load.cpu().tolist()


def make_inputs(T, H, E, K, I, seed):
    """numpy fp16 arrays: x [T,H], w_gate [H,E], expert_weights [E,3I,H]."""
    r = np.random.default_rng(seed)
    x = r.standard_normal((T, H), np.float32).astype(np.float16)
    wg = (r.standard_normal((H, E), np.float32) / np.sqrt(H)).astype(np.float16)
    ew = np.empty((E, 3 * I, H), np.float16)
    for e in range(E):
        ew[e, : 2 * I] = (r.standard_normal((2 * I, H), np.float32) / np.sqrt(H)).astype(np.float16)
        ew[e, 2 * I:] = (r.standard_normal((H, I), np.float32) / np.sqrt(I)).astype(np.float16).reshape(I, H)
    return x, wg, ew


def make_inputs_torch(T, H, E, K, I, seed, device="cuda", zipf=None):
    """Same distributions drawn with torch's generator on `device` (fast at full size).

    The stream differs from make_inputs; every check copies the very tensors it
    used to the host, so the checkers always see the same values as the GPU.
    """
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((T, H), generator=g, device=device, dtype=torch.float32).half()
    wg = (torch.randn((H, E), generator=g, device=device, dtype=torch.float32) / H ** 0.5).half()
    ew = torch.empty((E, 3 * I, H), device=device, dtype=torch.float16)
    for e in range(E):
        ew[e, : 2 * I] = (torch.randn((2 * I, H), generator=g, device=device) / H ** 0.5).half()
        ew[e, 2 * I:] = (torch.randn((H, I), generator=g, device=device) / I ** 0.5).half().reshape(I, H)
    if zipf:
        wg, _ = zipf_gate(x, wg, K, zipf)
    return x, wg, ew
