"""GPU parity: the sm_100a path, called through the C ABI, against the CPU oracle.

Bars (from the benchmark definition):
  * expert ids and the permutation bit-exact; a token whose top-K logit margin
    in the oracle is < 1e-3 is a near tie, counted and reported, not failed;
  * y (and expert_out) within max abs err < 0.05, mean abs err < 0.01,
    cosine > 0.999 (tests/moe_cpu_sim.cpp:666, tests/test_moe.cpp:486-490);
  * routing weights within 1 fp16 ulp of the oracle's fp32 weights.
"""
import os

import numpy as np
import pytest

from test_oracle import load_golden
from conftest import GOLDEN_DIR, golden_cases, record_near_ties

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

NEAR_TIE = 1e-3
TOL_MAX, TOL_MEAN, TOL_COS = 0.05, 0.01, 0.999


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check_ids(ids_gpu, ids_ref, margin, name=None):
    """Bit-exact ids away from near ties; near ties counted (and recorded under `name`)."""
    diff = np.any(ids_gpu != ids_ref, axis=1)
    near = margin < NEAR_TIE
    bad = diff & ~near
    assert not bad.any(), f"{bad.sum()} tokens differ away from ties: {np.nonzero(bad)[0][:10]}"
    if name:
        record_near_ties(name, len(diff), near.sum(), (diff & near).sum())
    return int(diff.sum()), int(near.sum())


def check_close(actual, expected, what):
    a = np.asarray(actual, np.float64)
    b = np.asarray(expected, np.float64)
    err = np.abs(a - b)
    cos = float((a * b).sum() / (np.sqrt((a * a).sum() * (b * b).sum()) + 1e-300))
    assert err.max() < TOL_MAX and err.mean() < TOL_MEAN and cos > TOL_COS, \
        f"{what}: max {err.max():.3e} mean {err.mean():.3e} cos {cos:.8f}"
    return float(err.max()), float(err.mean()), cos


def run_layer(moe, x, wg, ew, K):
    """Three operators through the C ABI, as tests/test_moe.cpp:446-463 chains them."""
    xd, wgd, ewd = dev(x), dev(wg), dev(ew)
    ids, w = moe.moe_routing_topk(xd, wgd, K)
    eo = moe.moe_expert_ffn(xd, ids, w, ewd)
    y = moe.moe_combine(eo, ids, w)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), w.float().cpu().numpy(), eo.float().cpu().numpy(), y.float().cpu().numpy()


@pytest.mark.parametrize("name", golden_cases())
def test_golden_layer(name, moe, O):
    g, (T, H, E, K, I), x, wg, ew = load_golden(name, moe)
    ids, w, eo, y = run_layer(moe, x, wg, ew, K)
    margin = O.routing(x.astype(np.float32), wg.astype(np.float32), K)[4]
    ndiff, nnear = check_ids(ids, g["ids"], margin)
    assert ndiff == 0, "golden cases have no near ties; ids must match exactly"
    assert np.abs(w - g["weights"]).max() <= 2.0 ** -11 + 1e-7
    check_close(y, g["y"], "y")
    if "ffn_out" in g:
        check_close(eo, g["ffn_out"], "expert_out")


@pytest.mark.parametrize("name", golden_cases())
def test_golden_permutation(name, moe):
    g = dict(np.load(os.path.join(GOLDEN_DIR, name + ".npz")))
    E = int(g["E"])
    perm, offs, ws = moe.moe_permute(dev(g["ids"]), E)
    assert np.array_equal(perm.cpu().numpy(), g["perm"])
    assert np.array_equal(offs.cpu().numpy(), g["offsets"])
    assert moe.device_error(ws) == 0


# shapes exercising tails: H % 256 != 0 (down-GEMM N tail), I % 128 != 0 (gate/up N tail),
# H % 64 != 0 (k tail), T below / above one 128-row tile, top-6, E = 64
SHAPES = [
    (3, 64, 4, 2, 256),
    (17, 136, 8, 2, 200),
    (130, 192, 4, 1, 72),
    (257, 256, 16, 2, 384),
    (64, 512, 64, 6, 1408),
    (300, 1024, 8, 2, 512),
]


@pytest.mark.parametrize("shape", SHAPES)
def test_layer_vs_oracle(shape, moe, O):
    T, H, E, K, I = shape
    x, wg, ew = moe.make_inputs(T, H, E, K, I, 1234 + T)
    xf, wgf, ewf = (a.astype(np.float32) for a in (x, wg, ew))
    ids, w, eo, y = run_layer(moe, x, wg, ew, K)
    rid, rw, _, _, margin = O.routing(xf, wgf, K)
    check_ids(ids, rid, margin, f"shape T={T} H={H} E={E} K={K} I={I}")
    ok = np.all(ids == rid, axis=1)
    # expert_out of (t,k) for the ids the GPU chose, from the oracle FFN
    ffn = O.expert_ffn(xf, ewf, ids, I)
    check_close(eo, ffn, "expert_out")
    yref = O.combine(ffn, rw)
    check_close(y[ok], yref[ok], "y")


def test_decode_config_full(moe, O):
    """The decode config (T=128, H=2048, E=16, K=2, I=8192) in full against the oracle."""
    T, H, E, K, I, seed = moe.CONFIGS["decode"]
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, seed)
    xn, wgn, ewn = (a.float().cpu().numpy() for a in (x, wg, ew))
    ids_d, w_d = moe.moe_routing_topk(x, wg, K)
    eo = moe.moe_expert_ffn(x, ids_d, w_d, ew)
    y = moe.moe_combine(eo, ids_d, w_d)
    ids = ids_d.cpu().numpy()
    rid, rw, _, _, margin = O.routing(xn, wgn, K)
    check_ids(ids, rid, margin, "decode")
    ffn = O.expert_ffn(xn, ewn, ids, I)
    check_close(eo.float().cpu().numpy(), ffn, "expert_out")
    ok = np.all(ids == rid, axis=1)
    check_close(y.float().cpu().numpy()[ok], O.combine(ffn, rw)[ok], "y")


# y / expert_out checked on the whole batch where the threaded C oracle finishes
# in well under a minute (prefill: 8.2e11 FLOP), on a 512-token slice spread over
# the batch for the two largest (rows are independent)
FULL_Y = {"prefill": None, "deepseek": 512, "mixtral": 512}


@pytest.mark.parametrize("cfg", ["prefill", "deepseek", "mixtral"])
def test_full_size_properties(cfg, moe, O):
    """Full benchmark sizes: ids on every token, permutation bit-exact, and y /
    expert_out against the oracle (whole batch at prefill, 512-token slices for the
    Mixtral- and DeepSeek-shaped layers).  The Mixtral-shaped layer runs with its
    Zipf-skewed router (uneven expert groups)."""
    T, H, E, K, I, seed = moe.CONFIGS[cfg]
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, seed, zipf=moe.inputs.ZIPF.get(cfg))
    ws = torch.empty((moe.moe_layer_workspace_size(T, H, E, K, I),), dtype=torch.uint8, device="cuda")
    ids_d = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w_d = torch.empty((T, K), dtype=torch.float16, device="cuda")
    eo = torch.empty((T, K, H), dtype=torch.float16, device="cuda")
    y = moe.moe_layer_forward(x, wg, ew, K, expert_ids=ids_d, weights=w_d, expert_out=eo, workspace=ws)
    torch.cuda.synchronize()
    assert moe.device_error(ws) == 0
    xn, wgn = x.float().cpu().numpy(), wg.float().cpu().numpy()
    ids = ids_d.cpu().numpy()
    rid, rw, _, _, margin = O.routing(xn, wgn, K)
    check_ids(ids, rid, margin, cfg)
    # permutation of the GPU's ids: bit-exact against the oracle's counting order
    perm, offs, _ = moe.moe_permute(ids_d, E)
    operm, ooffs = O.permute(ids, E)
    assert np.array_equal(perm.cpu().numpy(), operm) and np.array_equal(offs.cpu().numpy(), ooffs)
    n = FULL_Y[cfg]
    sl = np.arange(T) if n is None else np.linspace(0, T - 1, n).astype(np.int64)
    ewn = ew.float().cpu().numpy()
    ffn = O.expert_ffn(xn[sl], ewn, ids[sl], I)
    check_close(eo.float().cpu().numpy()[sl], ffn, f"expert_out ({len(sl)} tokens)")
    ok = np.all(ids[sl] == rid[sl], axis=1)
    check_close(y.float().cpu().numpy()[sl][ok], O.combine(ffn, rw[sl])[ok], f"y ({ok.sum()} tokens)")


def test_routing_error_word_reads_clear(moe):
    """MoeRoutingTopK has no workspace; its error word is read (and cleared) with
    MoeRoutingGetDeviceError.  After ordinary calls it reads 0."""
    import ctypes

    T, H, E, K, I = 300, 256, 16, 2, 64
    x, wg, _ = moe.make_inputs_torch(T, H, E, K, I, 8)
    moe.moe_routing_topk(x, wg, K)
    f = moe.lib().MoeRoutingGetDeviceError
    f.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    code = ctypes.c_int(-1)
    assert f(ctypes.byref(code), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    assert code.value == 0


def test_skewed_load_one_expert(moe, O):
    """Every token on one expert (many 128-row tiles in one group), others empty."""
    T, H, E, K, I = 700, 256, 8, 2, 256
    x, wg, ew = moe.make_inputs(T, H, E, K, I, 9)
    ids = np.zeros((T, K), np.int32)
    ids[:, 0] = 5
    ids[:, 1] = 2
    ids[::7, 1] = 6
    xd, ewd = dev(x), dev(ew)
    idd = dev(ids)
    w = torch.full((T, K), 0.5, dtype=torch.float16, device="cuda")
    eo = moe.moe_expert_ffn(xd, idd, w, ewd)
    torch.cuda.synchronize()
    ffn = O.expert_ffn(x.astype(np.float32), ew.astype(np.float32), ids, I)
    check_close(eo.float().cpu().numpy(), ffn, "expert_out")


def test_bad_expert_id_is_reported_not_fatal(moe):
    T, H, E, K, I = 16, 64, 4, 2, 64
    x, wg, ew = moe.make_inputs(T, H, E, K, I, 2)
    ids = np.tile(np.array([[0, 1]], np.int32), (T, 1))
    ids[3, 1] = 7  # out of range
    ws = torch.empty((moe.moe_expert_ffn_workspace_size(T, H, E, K, I),), dtype=torch.uint8, device="cuda")
    eo = torch.zeros((T, K, H), dtype=torch.float16, device="cuda")
    moe.moe_expert_ffn(dev(x), dev(ids), torch.zeros((T, K), dtype=torch.float16, device="cuda"), dev(ew),
                       expert_out=eo, workspace=ws)
    assert moe.device_error(ws) & 1
    assert torch.count_nonzero(eo[3, 1]) == 0  # the bad slot is skipped, not written
    # the context is still usable
    y = moe.moe_combine(eo, dev(ids), torch.ones((T, K), dtype=torch.float16, device="cuda"))
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()


def test_outputs_leave_canaries_untouched(moe):
    T, H, E, K, I = 33, 128, 4, 2, 128
    x, wg, ew = moe.make_inputs(T, H, E, K, I, 5)
    pad = 4096
    buf = torch.full((T * K * H + 2 * pad,), 1234.0, dtype=torch.float16, device="cuda")
    eo = buf[pad:pad + T * K * H].view(T, K, H)
    ids, w = moe.moe_routing_topk(dev(x), dev(wg), K)
    moe.moe_expert_ffn(dev(x), ids, w, dev(ew), expert_out=eo)
    ybuf = torch.full((T * H + 2 * pad,), 1234.0, dtype=torch.float16, device="cuda")
    y = ybuf[pad:pad + T * H].view(T, H)
    moe.moe_combine(eo, ids, w, y=y)
    torch.cuda.synchronize()
    for b in (buf, ybuf):
        assert torch.all(b[:pad] == 1234.0) and torch.all(b[-pad:] == 1234.0)


def test_empty_batch(moe):
    T, H, E, K, I = 0, 64, 4, 2, 64
    x = torch.empty((0, H), dtype=torch.float16, device="cuda")
    wg = torch.zeros((H, E), dtype=torch.float16, device="cuda")
    ew = torch.zeros((E, 3 * I, H), dtype=torch.float16, device="cuda")
    ids, w = moe.moe_routing_topk(x, wg, K)
    eo = moe.moe_expert_ffn(x, ids, w, ew)
    y = moe.moe_combine(eo, ids, w)
    torch.cuda.synchronize()
    assert y.shape == (0, H)


def test_repeatable_bitwise(moe):
    """Two runs of the layer give identical bits (no atomics in the data path)."""
    T, H, E, K, I = 500, 512, 16, 2, 512
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, 77)
    y1 = moe.moe_layer_forward(x, wg, ew, K)
    y2 = moe.moe_layer_forward(x, wg, ew, K)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
