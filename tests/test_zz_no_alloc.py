"""MoeExpertFFNNoAlloc: the expert FFN for callers that cannot allocate.

Some callers cannot call cudaMalloc (a host framework that owns every device
allocation through its own pool, a runtime that forbids allocation after start-up,
a service with a fixed memory budget), so they cannot hand MoeExpertFFN a
workspace.  MoeExpertFFNNoAlloc uses a static scratch array inside the library
instead.  This test calls it through the C ABI and checks it against the
ordinary MoeExpertFFN on the same inputs, twice in a row with different shapes
in both orders (a later call must not see an earlier call's leftovers in the
shared array), checks that a problem too big for the static array is rejected,
and that a bad expert id is reported through MoeNoAllocGetDeviceError and does
not stick to the next, clean call.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL_MAX, TOL_MEAN, TOL_COS = 0.05, 0.01, 0.999


def _no_alloc(moe):
    L = moe.lib()
    f = L.MoeExpertFFNNoAlloc
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 5 + [ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _close(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    err = np.abs(a - b)
    cos = (a * b).sum() / np.sqrt((a * a).sum() * (b * b).sum())
    return err.max() < TOL_MAX and err.mean() < TOL_MEAN and cos > TOL_COS


def _no_alloc_error(moe):
    f = moe.lib().MoeNoAllocGetDeviceError
    f.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    f.restype = ctypes.c_int
    code = ctypes.c_int(-1)
    rc = f(ctypes.byref(code), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    return code.value


@pytest.mark.parametrize("shapes", [[(96, 256, 8, 2, 512), (40, 128, 4, 2, 256)],
                                    [(40, 128, 4, 2, 256), (96, 256, 8, 2, 512)]])
def test_no_alloc_matches_workspace_path(moe, shapes):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    f = _no_alloc(moe)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for i, (T, H, E, K, I) in enumerate(shapes):
        x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, 100 + i)
        ids, w = moe.moe_routing_topk(x, wg, K)
        ref = moe.moe_expert_ffn(x, ids, w, ew)
        out = torch.full((T, K, H), float("nan"), dtype=torch.float16, device="cuda")
        rc = f(x.data_ptr(), ids.data_ptr(), w.data_ptr(), ew.data_ptr(), out.data_ptr(), T, H, E, K, I, stream)
        assert rc == 0, moe.lib().MoeStatusString(rc)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert _close(out, ref)
        assert torch.equal(out, ref)  # same kernels, same inputs: identical bits
        assert _no_alloc_error(moe) == 0


def test_no_alloc_reports_bad_expert_id(moe):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    f = _no_alloc(moe)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    T, H, E, K, I = 16, 64, 4, 2, 64
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, 3)
    ids = torch.tensor([[0, 1]] * T, dtype=torch.int32, device="cuda")
    ids[5, 1] = E  # outside [0, E)
    w = torch.full((T, K), 0.5, dtype=torch.float16, device="cuda")
    out = torch.zeros((T, K, H), dtype=torch.float16, device="cuda")
    assert f(x.data_ptr(), ids.data_ptr(), w.data_ptr(), ew.data_ptr(), out.data_ptr(), T, H, E, K, I, stream) == 0
    assert _no_alloc_error(moe) == 1  # expert id out of range
    assert torch.count_nonzero(out[5, 1]) == 0  # the bad slot is skipped
    ids[5, 1] = 2
    assert f(x.data_ptr(), ids.data_ptr(), w.data_ptr(), ew.data_ptr(), out.data_ptr(), T, H, E, K, I, stream) == 0
    assert _no_alloc_error(moe) == 0  # the next clean call starts with a cleared word
    assert torch.equal(out, moe.moe_expert_ffn(x, ids, w, ew))


def test_no_alloc_rejects_oversized_problem(moe):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    f = _no_alloc(moe)
    T, H, E, K, I = 4096, 2048, 16, 2, 8192  # needs ~160 MiB of scratch, above the 64 MiB array
    assert moe.moe_expert_ffn_workspace_size(T, H, E, K, I) > (64 << 20)
    rc = f(None, None, None, None, None, T, H, E, K, I, None)
    assert rc == -3  # MOE_ERR_WORKSPACE_TOO_SMALL
