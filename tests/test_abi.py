"""CPU: the C-ABI library loads, exports what include/moe_ops.h declares, and its
host-side validation / shape inference behaves like op_host/moe_ops.cpp.
None of these calls reaches the GPU: every one is rejected (or answered) before
the first CUDA call."""
import ctypes

import pytest


def test_library_exports_every_declared_symbol(moe):
    L = moe.lib()
    names = moe.ops.declared_symbols()
    assert len(names) >= 14
    for n in names:
        assert hasattr(L, n), n


def test_status_strings(moe):
    L = moe.lib()
    for code in range(0, -10, -1):
        assert L.MoeStatusString(code).decode().startswith("MOE_")


def test_routing_infer_shape(moe):
    r = moe.infer_shapes("routing", (4096, 2048), (2048, 16), 0)  # topK default 2
    assert r["expert_ids"] == (4096, 2) and r["weights"] == (4096, 2)
    assert r["dtypes"] == (3, 1)  # INT32, FLOAT16 (moe_ops.cpp:219-225)
    assert moe.infer_shapes("routing", (7, 64), (64, 64), 6)["expert_ids"] == (7, 6)
    with pytest.raises(moe.MoeError):
        moe.infer_shapes("routing", (7, 64), (32, 4), 2)  # hidden mismatch (moe_ops.cpp:86-90)
    with pytest.raises(moe.MoeError):
        moe.infer_shapes("routing", (7, 64, 1), (64, 4), 2)  # rank (moe_ops.cpp:80-85)


def test_ffn_and_combine_infer_shape(moe):
    r = moe.infer_shapes("ffn", (128, 2048), (128, 2), (16, 3 * 8192, 2048), 0)
    assert r["expert_out"] == (128, 2, 2048) and (r["E"], r["K"], r["I"]) == (16, 2, 8192)
    assert moe.infer_shapes("ffn", (4, 64), (4, 2), (4, 768, 64), 100)["I"] == 100  # attr wins
    with pytest.raises(moe.MoeError):
        moe.infer_shapes("ffn", (4, 64), (4, 2), (4, 768), 0)
    c = moe.infer_shapes("combine", (9, 2, 64), (9, 2))
    assert c["y"] == (9, 64) and c["dtype"] == 1
    with pytest.raises(moe.MoeError):
        moe.infer_shapes("combine", (9, 64), (9, 2))


def test_workspace_sizes(moe):
    s1 = moe.moe_expert_ffn_workspace_size(128, 2048, 16, 2, 8192)
    s2 = moe.moe_expert_ffn_workspace_size(4096, 2048, 16, 2, 8192)
    assert 0 < s1 < s2
    # permuted activations + intermediate dominate: T*K*(H+I)*2 bytes
    assert s2 >= 4096 * 2 * (2048 + 8192) * 2
    assert moe.moe_layer_workspace_size(4096, 2048, 16, 2, 8192) > s2
    for bad in [(8, 60, 4, 2, 256), (8, 64, 4, 9, 256), (8, 64, 300, 2, 256), (8, 64, 4, 2, 250),
                (8, 64, 4, 5, 256)]:
        assert moe.moe_expert_ffn_workspace_size(*bad) == 0, bad


def test_argument_errors_without_gpu(moe):
    L = moe.lib()
    v = ctypes.c_void_p
    fake = v(0x1000)
    # bad shapes
    assert L.MoeRoutingTopK(fake, fake, fake, fake, 8, 60, 4, 2, None) == -2
    assert L.MoeRoutingTopK(fake, fake, fake, fake, 8, 64, 4, 5, None) == -2
    assert L.MoeCombine(fake, fake, fake, fake, 8, 64, 9, None) == -2
    # null pointers
    assert L.MoeRoutingTopK(None, fake, fake, fake, 8, 64, 4, 2, None) == -1
    assert L.MoeCombine(fake, None, None, fake, 8, 64, 2, None) == -1
    # misaligned
    assert L.MoeRoutingTopK(v(0x1002), fake, fake, fake, 8, 64, 4, 2, None) == -6
    # workspace too small
    need = L.MoeExpertFFNWorkspaceSize(8, 64, 4, 2, 256)
    assert L.MoeExpertFFN(fake, fake, fake, fake, fake, 8, 64, 4, 2, 256, fake, need - 1, None) == -3
    assert L.MoeExpertFFN(fake, fake, fake, fake, fake, 8, 64, 4, 2, 256, None, need, None) == -1
    assert L.MoeLayerForward(fake, fake, fake, fake, None, None, None, 8, 64, 4, 2, 256, fake, 16,
                             None) == -3
    # T == 0 is a valid no-op for routing and combine
    assert L.MoeRoutingTopK(None, None, None, None, 0, 64, 4, 2, None) == 0
    assert L.MoeCombine(None, None, None, None, 0, 64, 2, None) == 0


def test_python_front_end_has_no_cpu_fallback(moe):
    import torch

    x = torch.zeros((4, 64), dtype=torch.float16)
    wg = torch.zeros((64, 4), dtype=torch.float16)
    with pytest.raises(moe.MoeError):
        moe.moe_routing_topk(x, wg, 2)
