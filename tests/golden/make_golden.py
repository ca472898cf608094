"""Generates the golden fixtures of tests/golden/ from the reference itself.

Runs the reference's own tests/moe_cpu_sim.cpp (compiled unmodified into
oracle/_ref/libmoe_ref.so by oracle/Makefile) on seeded fp16-rounded inputs:
NaiveMoE for y, TiledRouting for expert ids / fp32 weights, TiledExpertFFN for
the per-(t,k) expert outputs.  The permutation is the order the reference's FFN
builds (moe_cpu_sim.cpp:412-419), recomputed here from the reference's ids.

Small cases store their inputs; larger ones store only a SHA-256 of the inputs
make_inputs() regenerates, so a generator change is detected instead of silently
comparing different data.

    python tests/golden/make_golden.py [REFERENCE_CHECKOUT]   # needs the reference sources
    (default: MOE_REFERENCE_DIR, else a "reference" directory beside the repository)
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from oracle import oracle as O  # noqa: E402
from _moe_loader import load  # noqa: E402

# name -> (T, H, E, K, I, seed, store_inputs)
CASES = {
    "small_t8_h64_e4_k2_i256": (8, 64, 4, 2, 256, 42, True),  # the reference's small case
    "odd_t17_h64_e16_k6_i64": (17, 64, 16, 6, 64, 7, True),    # ragged T, top-6
    "one_t1_h64_e8_k2_i64": (1, 64, 8, 2, 64, 3, True),    # a single token
    "mid_t32_h256_e8_k2_i1024": (32, 256, 8, 2, 1024, 43, False),  # the reference's middle case
}


def input_digest(x, wg, ew):
    h = hashlib.sha256()
    for a in (x, wg, ew):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    ref = (sys.argv[1] if len(sys.argv) > 1 else None) or os.environ.get("MOE_REFERENCE_DIR") or \
        os.path.join(os.path.dirname(ROOT), "reference")
    O.build(ref)
    make_inputs = load().make_inputs
    for name, (T, H, E, K, I, seed, store) in CASES.items():
        x, wg, ew = make_inputs(T, H, E, K, I, seed)
        xf, wgf, ewf = (a.astype(np.float32) for a in (x, wg, ew))
        y = O.ref_naive(xf, wgf, ewf, K)
        ids, wts = O.ref_routing(xf, wgf, K)
        ffn = O.ref_expert_ffn(xf, ewf, ids, wts)
        perm, offs = O.permute(ids, E)
        out = dict(T=T, H=H, E=E, K=K, I=I, seed=seed, y=y, ids=ids, weights=wts, ffn_out=ffn, perm=perm,
                   offsets=offs, digest=np.array(input_digest(x, wg, ew)))
        if store:
            out.update(x=x, w_gate=wg, expert_weights=ew)
        else:
            out.pop("ffn_out")
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **out)
        print(name, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
