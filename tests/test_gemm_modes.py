"""Both tile modes of the grouped GEMMs against the oracle.

The expert FFN GEMMs run either one 128-row tile per CTA or one 256-row tile per
2-CTA cluster (paired cta_group::2 UMMAs).  The library picks paired tiles when
experts average 1536 rows or more.  Small test shapes therefore take single-CTA
tiles, and only the full-size deepseek and mixtral configurations take paired
ones.  MOE_GEMM_PAIR=0/1 forces the choice, once per process.  So these tests rerun the
layer parity tests and the single-rank expert-parallel tests in a child process
with each forced mode: both modes meet the same tolerances on the same shapes,
ragged expert tails and empty halves of a pair included.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _run(mode, args):
    env = dict(os.environ, MOE_GEMM_PAIR=str(mode), MOE_GEMM_PAIR_DEBUG="1")
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
