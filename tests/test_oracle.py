"""CPU: the oracle restatement is pinned to the reference itself.

(1) against the golden fixtures generated from the reference's own
tests/moe_cpu_sim.cpp (tests/golden/make_golden.py), and (2) when oracle/_ref is
present, against the reference run live on fresh shapes.  Both must match bit
for bit, since the restatement keeps the reference's summation orders.
"""
import hashlib
import os

import numpy as np
import pytest

from conftest import GOLDEN_DIR, golden_cases


def _digest(x, wg, ew):
    h = hashlib.sha256()
    for a in (x, wg, ew):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_golden(name, moe):
    g = dict(np.load(os.path.join(GOLDEN_DIR, name + ".npz")))
    T, H, E, K, I, seed = (int(g[k]) for k in ("T", "H", "E", "K", "I", "seed"))
    if "x" in g:
        x, wg, ew = g["x"], g["w_gate"], g["expert_weights"]
    else:
        x, wg, ew = moe.make_inputs(T, H, E, K, I, seed)
    assert _digest(x, wg, ew) == str(g["digest"]), "input generator drifted from the fixture"
    return g, (T, H, E, K, I), x, wg, ew


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_reference_golden(name, moe, O):
    g, (T, H, E, K, I), x, wg, ew = load_golden(name, moe)
    xf, wgf, ewf = (a.astype(np.float32) for a in (x, wg, ew))
    ids, w, logits, probs, margin = O.routing(xf, wgf, K)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(w, g["weights"])
    perm, offs = O.permute(ids, E)
    assert np.array_equal(perm, g["perm"]) and np.array_equal(offs, g["offsets"])
    y, ids2, _ = O.moe_naive(xf, wgf, ewf, K)
    assert np.array_equal(y, g["y"]), "restated NaiveMoE is not bit-identical to the reference"
    if "ffn_out" in g:
        ffn = O.expert_ffn(xf, ewf, ids, I)
        assert np.array_equal(ffn, g["ffn_out"])
        assert np.array_equal(O.combine(ffn, w), g["y"])


@pytest.mark.parametrize("shape", [(5, 72, 6, 3, 40), (12, 64, 32, 6, 24), (3, 16, 2, 2, 8)])
def test_oracle_matches_reference_live(shape, moe, O):
    if not O.ref_available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    T, H, E, K, I = shape
    x, wg, ew = (a.astype(np.float32) for a in moe.make_inputs(T, H, E, K, I, 11))
    y, ids, w = O.moe_naive(x, wg, ew, K)
    assert np.array_equal(y, O.ref_naive(x, wg, ew, K))
    rid, rw = O.ref_routing(x, wg, K)
    assert np.array_equal(ids, rid) and np.array_equal(w, rw)
    # the reference's own acceptance test: tiled vs naive (moe_cpu_sim.cpp:666)
    mx, mean, cos = O.compare(O.ref_tiled(x, wg, ew, K), y)
    assert mx < 0.05 and cos > 0.999


def test_oracle_tie_rule_lower_id_first(O):
    # two identical gate columns -> identical probabilities; the lower id wins
    H, E, K = 16, 4, 2
    rng = np.random.default_rng(0)
    wg = rng.standard_normal((H, E)).astype(np.float16).astype(np.float32)
    wg[:, 3] = wg[:, 1]
    x = np.tile(np.sign(wg[:, 1:2].T), (3, 1)).astype(np.float32) * 4.0  # make experts 1/3 the best
    ids, w, logits, probs, margin = O.routing(x, wg, K)
    assert (ids[:, 0] == 1).all() and (ids[:, 1] == 3).all()
    assert np.all(margin == 0.0)


def test_oracle_permutation_is_stable_counting_sort(O):
    rng = np.random.default_rng(5)
    for T, K, E in [(1, 1, 1), (37, 3, 5), (500, 6, 64)]:
        ids = rng.integers(0, E, size=(T, K)).astype(np.int32)
        perm, offs = O.permute(ids, E)
        flat = ids.ravel()
        assert sorted(perm.tolist()) == list(range(T * K))  # bijection
        ref = np.argsort(flat, kind="stable")
        assert np.array_equal(perm, ref)
        assert np.array_equal(offs, np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]))
    with pytest.raises(ValueError):
        O.permute(np.array([[0, 9]], np.int32), 4)
