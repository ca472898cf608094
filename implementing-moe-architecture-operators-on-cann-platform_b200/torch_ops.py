"""PyTorch custom operators (torch.library) over the C ABI.

The reference keeps a placeholder for framework adapters (framework/CMakeLists.txt:4-9);
this module is that adapter for PyTorch.  It registers

    torch.ops.moe_b200.routing_topk(x, w_gate, topK) -> (expert_ids, weights)
    torch.ops.moe_b200.expert_ffn(x, expert_ids, weights, expert_weights) -> expert_out
    torch.ops.moe_b200.combine(expert_out, expert_ids, weights) -> y
    torch.ops.moe_b200.layer_forward(x, w_gate, expert_weights, topK) -> y

with CUDA implementations that call libmoe_b200.so, and fake (shape-only)
implementations that follow the reference's InferShape / InferDataType
(op_host/moe_ops.cpp:181-226, :364-398, :495-525), so the ops trace under
torch.compile / FakeTensor without running.  There is no CPU kernel.
"""
from __future__ import annotations

import torch

from . import ops as _ops

_NS = "moe_b200"


@torch.library.custom_op(f"{_NS}::routing_topk", mutates_args=(), device_types="cuda")
def routing_topk(x: torch.Tensor, w_gate: torch.Tensor, topK: int) -> tuple[torch.Tensor, torch.Tensor]:
    return _ops.moe_routing_topk(x.contiguous(), w_gate.contiguous(), topK)


@routing_topk.register_fake
def _(x, w_gate, topK):
    K = topK if topK > 0 else 2  # attr default, moe_ops.cpp:194-203
    T = x.shape[0]
    return x.new_empty((T, K), dtype=torch.int32), x.new_empty((T, K), dtype=torch.float16)


@torch.library.custom_op(f"{_NS}::expert_ffn", mutates_args=(), device_types="cuda")
def expert_ffn(x: torch.Tensor, expert_ids: torch.Tensor, weights: torch.Tensor,
               expert_weights: torch.Tensor) -> torch.Tensor:
    return _ops.moe_expert_ffn(x.contiguous(), expert_ids.contiguous(), weights.contiguous(),
                               expert_weights.contiguous())


@expert_ffn.register_fake
def _(x, expert_ids, weights, expert_weights):
    T, H = x.shape
    return x.new_empty((T, expert_ids.shape[1], H), dtype=torch.float16)  # moe_ops.cpp:383-385


@torch.library.custom_op(f"{_NS}::combine", mutates_args=(), device_types="cuda")
def combine(expert_out: torch.Tensor, expert_ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    return _ops.moe_combine(expert_out.contiguous(), expert_ids, weights.contiguous())


@combine.register_fake
def _(expert_out, expert_ids, weights):
    T, K, H = expert_out.shape
    return expert_out.new_empty((T, H), dtype=torch.float16)  # moe_ops.cpp:510-512


@torch.library.custom_op(f"{_NS}::layer_forward", mutates_args=(), device_types="cuda")
def layer_forward(x: torch.Tensor, w_gate: torch.Tensor, expert_weights: torch.Tensor, topK: int) -> torch.Tensor:
    return _ops.moe_layer_forward(x.contiguous(), w_gate.contiguous(), expert_weights.contiguous(), topK)


@layer_forward.register_fake
def _(x, w_gate, expert_weights, topK):
    return x.new_empty(x.shape, dtype=torch.float16)
