"""The torch.library adapter: shape inference on CPU (fake tensors), results on GPU."""
import pytest

torch = pytest.importorskip("torch")


def test_fake_shapes_follow_infershape(moe):
    moe.register_torch_ops()
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode() as m:
        x = m.from_tensor(torch.empty((7, 64), dtype=torch.float16))
        wg = m.from_tensor(torch.empty((64, 8), dtype=torch.float16))
        ew = m.from_tensor(torch.empty((8, 3 * 32, 64), dtype=torch.float16))
        ids, w = torch.ops.moe_b200.routing_topk(x, wg, 3)
        assert ids.shape == (7, 3) and ids.dtype == torch.int32 and w.dtype == torch.float16
        eo = torch.ops.moe_b200.expert_ffn(x, ids, w, ew)
        assert eo.shape == (7, 3, 64)
        y = torch.ops.moe_b200.combine(eo, ids, w)
        assert y.shape == (7, 64)
        assert torch.ops.moe_b200.layer_forward(x, wg, ew, 2).shape == (7, 64)


@pytest.mark.gpu
def test_torch_ops_match_oracle(moe, O):
    """torch.ops.moe_b200.* against the CPU oracle (tests/moe_cpu_sim.cpp:183-306):
    ids bit-exact away from near ties, expert_out and y within the reference's
    tolerance; the fused layer op gives the same bits as the three ops."""
    import numpy as np

    from test_gpu_parity import check_close, check_ids

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    moe.register_torch_ops()
    T, H, E, K, I = 96, 256, 8, 2, 256
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, 3)
    ids, w = torch.ops.moe_b200.routing_topk(x, wg, K)
    eo = torch.ops.moe_b200.expert_ffn(x, ids, w, ew)
    y = torch.ops.moe_b200.combine(eo, ids, w)
    yl = torch.ops.moe_b200.layer_forward(x, wg, ew, K)
    torch.cuda.synchronize()
    xn, wgn, ewn = (a.float().cpu().numpy() for a in (x, wg, ew))
    rid, rw, _, _, margin = O.routing(xn, wgn, K)
    idn = ids.cpu().numpy()
    check_ids(idn, rid, margin)
    ffn = O.expert_ffn(xn, ewn, idn, I)
    check_close(eo.float().cpu().numpy(), ffn, "expert_out")
    ok = np.all(idn == rid, axis=1)
    check_close(y.float().cpu().numpy()[ok], O.combine(ffn, rw)[ok], "y")
    assert torch.equal(yl, y)
