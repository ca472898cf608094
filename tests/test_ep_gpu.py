"""GPU: the expert-parallel layer (MoeEpLayerForward) through the C ABI.

Every kernel on the EP path is the single-GPU one and each output row depends only
on its own token, so rank r's y must equal MoeLayerForward on rank r's tokens with
all experts' weights, bit for bit.  One GPU: a 1-rank communicator.  Two or more
GPUs: one spawned process per GPU, NCCL over NVLink (NVLS off).  The failure test
(a rank that never joins) makes the failure on the host: the communicator set-up
waits for the missing rank, times out, and is aborted; no GPU kernel is involved.
"""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


SHAPES = [(300, 256, 8, 2, 512), (257, 512, 16, 2, 384)]


@pytest.fixture(params=["p2p", "nccl"])
def ep_path(request, monkeypatch):
    """The peer-memory exchange (default) and the NCCL send/recv fallback."""
    if request.param == "nccl":
        monkeypatch.setenv("MOE_EP_FORCE_NCCL", "1")
    else:
        monkeypatch.delenv("MOE_EP_FORCE_NCCL", raising=False)
    return request.param


@pytest.mark.parametrize("shape", SHAPES)
def test_ep_single_rank_matches_layer(moe, shape, ep_path):
    T, H, E, K, I = shape
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, 5)
    ref = moe.moe_layer_forward(x, wg, ew, K)
    ctx = moe.EpContext(moe.ep_unique_id(), 0, 1, timeout_ms=20000)
    try:
        ws = torch.empty((ctx.workspace_size(T, H, E, K, I),), dtype=torch.uint8, device="cuda")
        y = ctx.forward(x, wg, ew, K, workspace=ws)
        y2 = ctx.forward(x, wg, ew, K, workspace=ws)  # a second call reuses the workspace
        torch.cuda.synchronize()
        assert moe.device_error(ws) == 0
    finally:
        ctx.close()
    assert torch.equal(y, ref) and torch.equal(y2, ref)


_NEVER_JOINS = r"""
import sys
sys.path.insert(0, sys.argv[1])
from _moe_loader import load
moe = load()
try:
    moe.EpContext(moe.ep_unique_id(), 0, 2, timeout_ms=3000)
    print("NO-ERROR")
except moe.MoeError as e:
    print("STATUS", e.status)
"""


def test_ep_rank_that_never_joins_times_out():
    # rank 0 of a 2-rank communicator whose rank 1 never starts; run in a child
    # process so that even a stuck host thread cannot outlive the test
    import subprocess
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-c", _NEVER_JOINS, here], capture_output=True, text=True, timeout=120)
    assert "STATUS -8" in r.stdout, r.stdout + r.stderr  # MOE_ERR_TIMEOUT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_rank(rank, n, port, shape, path, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "tests"))
    import torch.distributed as dist
    from _moe_loader import load

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    if path == "nccl":
        os.environ["MOE_EP_FORCE_NCCL"] = "1"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=n)
    moe = load()
    T, H, E, K, I = shape
    El = E // n
    try:
        uid = [moe.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        x, _, _ = moe.make_inputs_torch(T, H, E, K, I, 1000 + rank)
        _, wg, ew = moe.make_inputs_torch(T, H, E, K, I, 7)  # same weights on every rank
        ref = moe.moe_layer_forward(x, wg, ew, K)
        ctx = moe.EpContext(uid[0], rank, n, timeout_ms=30000)
        try:
            local = ew[rank * El:(rank + 1) * El].contiguous()
            ws = torch.empty((ctx.workspace_size(T, H, E, K, I),), dtype=torch.uint8, device="cuda")
            y = ctx.forward(x, wg, local, K, workspace=ws)
            y2 = ctx.forward(x, wg, local, K, workspace=ws)
            torch.cuda.synchronize()
            assert moe.device_error(ws) == 0
        finally:
            ctx.close()
        q.put((rank, bool(torch.equal(y, ref)), bool(torch.equal(y2, ref)), float((y.float() - ref.float()).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("path", ["p2p", "nccl"])
@pytest.mark.parametrize("shape", [(300, 256, 8, 2, 512), (1024, 2048, 16, 2, 1024)])
def test_ep_multi_gpu_matches_layer(shape, path):
    n = min(torch.cuda.device_count(), 4)
    if n < 2:
        pytest.skip("needs 2 GPUs")
    if shape[2] % n:
        pytest.skip("E not divisible by the GPU count")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_rank, args=(r, n, port, shape, path, q)) for r in range(n)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(n)]
    for p in procs:
        p.join(timeout=120)
    for rank, eq1, eq2, err in res:
        assert eq1 and eq2, (rank, err)


def test_bounded_wait_reports_timeout_and_context_survives(moe):
    """A device wait on a flag nothing sets gives up, reports its error bit, and
    the CUDA context keeps working afterwards."""
    import ctypes

    L = moe.lib()
    L.MoeEpSelfTestWaitTimeout.argtypes = [ctypes.POINTER(ctypes.c_int)]
    code = ctypes.c_int(0)
    assert L.MoeEpSelfTestWaitTimeout(ctypes.byref(code)) == 0
    assert code.value == 128  # rows-flag wait timed out
    T, H, E, K, I = 64, 128, 4, 2, 128
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, 1)
    y = moe.moe_layer_forward(x, wg, ew, K)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
