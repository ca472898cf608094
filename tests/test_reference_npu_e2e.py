"""GPU restatement of the reference's NPU end-to-end test (tests/test_moe.cpp:344-512).

Inputs exactly as that test draws them (:373-381): srand(42), then x, w_gate and
expert_weights filled in order with rand()/RAND_MAX*2-1, from the C library's
generator (oracle_test_moe_inputs).  Expected output: the fp32 naive layer on the
*unrounded* inputs (:385); the device path gets the fp16-rounded values (:389-392).
Sizes: the test's small case 8/64/4/2/256 and its target 128/2048/16/2/8192
(:658-660).

Thresholds.  The test's own bars are max abs < 0.05, mean abs < 0.01 and cos > 0.99
(:486-490).  With uniform [-1,1] weights the outputs are large (|y| up to ~156 at the
small size, ~36000 at the target), so the fp16 output's own rounding step (0.125 and
32 respectively) already exceeds the absolute bars for any fp16 implementation,
the Ascend kernels included, and rounding the inputs to fp16 (as the test does
before launching, :389-392) moves y further still.  The test keeps cos > 0.99 as
written and measures that floor instead of a fixed bar: the same fp32 oracle run on
the fp16-rounded inputs.  The device output must stay within 1.5x that floor's
max / mean deviation from the unrounded oracle, plus one fp16 step of max|y|.  Tokens whose expert choice differs only because the
inputs were rounded to fp16 before routing are counted and excluded (the reference
test would meet the same tokens).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("cfg", [(8, 64, 4, 2, 256), (128, 2048, 16, 2, 8192)])
def test_reference_npu_e2e(cfg, moe, O):
    T, H, E, K, I = cfg
    x, wg, ew = O.test_moe_inputs(T, H, E, I, seed=42)
    y_ref, ids_ref, _ = O.moe_naive(x, wg, ew, K)
    xd, wgd, ewd = (torch.from_numpy(a).cuda().half() for a in (x, wg, ew))
    ids, w = moe.moe_routing_topk(xd, wgd, K)
    eo = moe.moe_expert_ffn(xd, ids, w, ewd)
    y = moe.moe_combine(eo, ids, w).float().cpu().numpy()
    ids = ids.cpu().numpy()
    same = np.all(ids == ids_ref, axis=1)
    assert same.mean() > 0.9, f"{(~same).sum()} of {T} tokens route differently"
    assert np.isfinite(y).all()
    a, b = y[same].astype(np.float64), y_ref[same].astype(np.float64)
    err = np.abs(a - b)
    cos = float((a * b).sum() / np.sqrt((a * a).sum() * (b * b).sum()))
    # floor: the fp32 oracle on the fp16-rounded inputs, against the unrounded one
    xr, wgr, ewr = (v.astype(np.float16).astype(np.float32) for v in (x, wg, ew))
    y_round, _, _ = O.moe_naive(xr, wgr, ewr, K)
    floor = np.abs(y_round[same].astype(np.float64) - b)
    ulp = 2.0 ** (np.floor(np.log2(np.abs(b).max())) - 10)
    print(f"T={T}: max|y|={np.abs(b).max():.1f} max_abs={err.max():.4g} mean_abs={err.mean():.4g} "
          f"floor_max={floor.max():.4g} floor_mean={floor.mean():.4g} cos={cos:.8f} rerouted={(~same).sum()}")
    assert cos > 0.99                                   # tests/test_moe.cpp:486-490
    assert err.max() <= 1.5 * floor.max() + ulp
    assert err.mean() <= 1.5 * floor.mean() + ulp / 4
