"""The tile modes of the grouped GEMMs against the oracle.

The expert FFN GEMMs run either one 128-row tile per CTA or one 256-row tile per
2-CTA cluster (paired cta_group::2 UMMAs).  The library picks paired tiles when
experts average 1536 rows or more.  Small test shapes therefore take single-CTA
tiles, and only the full-size deepseek and mixtral configurations take paired
ones.  MOE_GEMM_PAIR=0/1 forces the choice, once per process.  So these tests rerun the
layer parity tests and the single-rank expert-parallel tests in a child process
with each forced mode: both modes meet the same tolerances on the same shapes,
ragged expert tails and empty halves of a pair included.

The down projection also has narrow tiles (128 output columns instead of 256),
taken when the wide tiles would not cover the SMs once (few rows: decode, the
ranks of the expert-parallel layer).  MOE_GEMM_DOWN_BN=128/256 forces the width.
Each output element accumulates over k through the same UMMA chain in both, so
the layer's output must be bit-identical between the two widths.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _run(mode, args, **extra):
    env = dict(os.environ, MOE_GEMM_PAIR=str(mode), MOE_GEMM_PAIR_DEBUG="1", **extra)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-s", "-p", "no:cacheprovider"] + args,
                       cwd=os.path.dirname(HERE), env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    return r


@pytest.mark.parametrize("mode", [0, 1])
def test_layer_parity_in_each_tile_mode(mode):
    r = _run(mode, [os.path.join(HERE, "test_gpu_parity.py"), "-k", "golden or layer_vs_oracle or skewed or empty or repeatable"])
    # the paired kernel reports its co-resident pair count when it is first launched
    assert ("co-resident CTA pairs" in r.stderr) == (mode == 1)


def test_expert_parallel_single_rank_paired_tiles():
    _run(1, [os.path.join(HERE, "test_ep_gpu.py"), "-k", "single_rank"])


def test_layer_parity_with_narrow_down_tiles():
    _run(0, [os.path.join(HERE, "test_gpu_parity.py"), "-k", "golden or layer_vs_oracle or skewed or empty or repeatable"],
         MOE_GEMM_DOWN_BN="128")


_BN_CHILD = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from _moe_loader import load
import torch
moe = load()
out = {}
# H % 128 != 0 (a partial narrow tile), several experts, top-6
for i, (T, H, E, K, I) in enumerate([(300, 512, 8, 2, 384), (128, 2048, 16, 2, 1024), (257, 264, 4, 2, 256),
                                     (96, 384, 64, 6, 256)]):
    x, wg, ew = moe.make_inputs_torch(T, H, E, K, I, 11 + i)
    out[str(i)] = moe.moe_layer_forward(x, wg, ew, K).cpu().numpy()
np.savez(sys.argv[2], **out)
"""


def test_narrow_and_wide_down_tiles_give_identical_bits(tmp_path):
    import numpy as np

    res = {}
    for bn in ("128", "256"):
        f = str(tmp_path / f"y{bn}.npz")
        env = dict(os.environ, MOE_GEMM_DOWN_BN=bn)
        r = subprocess.run([sys.executable, "-c", _BN_CHILD, HERE, f], env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, r.stderr[-3000:]
        res[bn] = dict(np.load(f))
    for k in res["128"]:
        assert np.array_equal(res["128"][k], res["256"][k]), k
