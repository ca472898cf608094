"""B200 (sm_100a) MoE layer operators: Python host mirror of the C ABI.

The product is ``libmoe_b200.so`` (include/moe_ops.h).  This package loads it
with ctypes and offers the reference's three operators on torch CUDA tensors,
with the reference's names and argument meaning (op_host/moe_ops.cpp:537-679):

    expert_ids, weights = moe_routing_topk(x, w_gate, topK=2)
    expert_out          = moe_expert_ffn(x, expert_ids, weights, expert_weights)
    y                   = moe_combine(expert_out, expert_ids, weights)

There is no CPU fallback: if the library is missing, or a tensor is not on a
CUDA device, the call raises.
"""
from .ops import (  # noqa: F401
    MoeError,
    lib,
    lib_path,
    moe_combine,
    moe_expert_ffn,
    moe_expert_ffn_workspace_size,
    moe_layer_forward,
    moe_layer_workspace_size,
    moe_permute,
    moe_routing_topk,
    device_error,
    infer_shapes,
    trace_start,
    trace_stop,
    TRACE_STAGES,
    EpContext,
    ep_unique_id,
    ep_plan,
)
from .inputs import make_inputs, make_inputs_torch, CONFIGS  # noqa: F401


def register_torch_ops():
    """Registers torch.ops.moe_b200.* (routing_topk, expert_ffn, combine, layer_forward)."""
    from . import torch_ops  # noqa: F401

    return torch_ops
