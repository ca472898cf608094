"""ctypes front end of the two CPU checkers (TEST INFRASTRUCTURE ONLY).

* ``_build/libmoe_oracle.so`` -- moe_oracle.c, the C restatement of the
  reference's naive layer (tests/moe_cpu_sim.cpp:183-306, :412-419).
* ``_ref/libmoe_ref.so``      -- the reference's own tests/moe_cpu_sim.cpp,
  compiled unmodified where it lies, behind ref_shim.cpp.

Both take fp32 arrays holding fp16-rounded values, exactly as the GPU path sees
them.  Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline /
``--impl reference`` legs may use this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libmoe_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmoe_ref.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_c_int = ctypes.c_int


def build(ref_dir: str | None = None) -> None:
    """Compile the restatement, and the reference itself when its sources exist
    (ref_dir: the reference checkout; None builds the restatement only)."""
    subprocess.check_call(["make", "-s", "-C", HERE, "oracle"])
    if ref_dir and os.path.isfile(os.path.join(ref_dir, "tests", "moe_cpu_sim.cpp")):
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", f"REF={ref_dir}"])


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_f32p)


def _i32(a):
    a = np.ascontiguousarray(a, dtype=np.int32)
    return a, a.ctypes.data_as(_i32p)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.isfile(ORACLE_SO):
            build(None)
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_routing.argtypes = [_f32p, _f32p] + [_c_int] * 4 + [_i32p, _f32p, _f32p, _f32p, _f32p]
        L.oracle_permute.argtypes = [_i32p, _c_int, _c_int, _c_int, _i32p, _i32p]
        L.oracle_permute.restype = _c_int
        L.oracle_expert_ffn.argtypes = [_f32p, _f32p, _i32p] + [_c_int] * 5 + [_f32p, _c_int]
        L.oracle_combine.argtypes = [_f32p, _f32p, _c_int, _c_int, _c_int, _f32p]
        L.oracle_test_moe_inputs.argtypes = [ctypes.c_uint, _f32p, ctypes.c_size_t, _f32p, ctypes.c_size_t, _f32p,
                                             ctypes.c_size_t]
        L.oracle_moe_naive.argtypes = [_f32p, _f32p, _f32p] + [_c_int] * 5 + [_f32p, _i32p, _f32p, _c_int]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.isfile(REF_SO)


def ref():
    global _ref
    if _ref is None:
        if not os.path.isfile(REF_SO):
            raise FileNotFoundError(f"{REF_SO} missing: run oracle.build() where the reference sources exist")
        R = ctypes.CDLL(REF_SO)
        R.ref_naive_moe.argtypes = [_f32p, _f32p, _f32p] + [_c_int] * 5 + [_f32p]
        R.ref_tiled_moe.argtypes = [_f32p, _f32p, _f32p] + [_c_int] * 5 + [_f32p]
        R.ref_tiled_routing.argtypes = [_f32p, _f32p] + [_c_int] * 4 + [_i32p, _f32p]
        R.ref_tiled_expert_ffn.argtypes = [_f32p, _f32p, _i32p, _f32p] + [_c_int] * 5 + [_f32p]
        R.ref_tiled_combine.argtypes = [_f32p, _i32p, _f32p] + [_c_int] * 3 + [_f32p]
        R.ref_ctx_create.argtypes = [_f32p, _f32p, _f32p] + [_c_int] * 5
        R.ref_ctx_create.restype = ctypes.c_void_p
        R.ref_ctx_destroy.argtypes = [ctypes.c_void_p]
        R.ref_ctx_naive.argtypes = [ctypes.c_void_p, _c_int, _c_int, _c_int, _f32p]
        R.ref_ctx_tiled.argtypes = [ctypes.c_void_p, _c_int, _c_int, _c_int, _f32p]
        _ref = R
    return _ref


# ----------------------------------------------------------------------------- restatement
def routing(x, w_gate, K):
    """-> ids [T,K] int32, weights [T,K] f32, logits [T,E], probs [T,E], margin [T]."""
    T, H = x.shape
    E = w_gate.shape[1]
    x, px = _f32(x)
    w_gate, pw = _f32(w_gate)
    ids = np.empty((T, K), np.int32)
    wts = np.empty((T, K), np.float32)
    logits = np.empty((T, E), np.float32)
    probs = np.empty((T, E), np.float32)
    margin = np.empty((T,), np.float32)
    lib().oracle_routing(px, pw, T, H, E, K, ids.ctypes.data_as(_i32p), wts.ctypes.data_as(_f32p),
                         logits.ctypes.data_as(_f32p), probs.ctypes.data_as(_f32p),
                         margin.ctypes.data_as(_f32p))
    return ids, wts, logits, probs, margin


def permute(ids, E):
    """-> perm [T*K] int32 (flat source index t*K+k), offsets [E+1] int32."""
    T, K = ids.shape
    ids, pi = _i32(ids)
    perm = np.empty((T * K,), np.int32)
    offs = np.empty((E + 1,), np.int32)
    rc = lib().oracle_permute(pi, T, K, E, perm.ctypes.data_as(_i32p), offs.ctypes.data_as(_i32p))
    if rc != 0:
        raise ValueError("expert id out of range")
    return perm, offs


def expert_ffn(x, ew, ids, I, nthreads=None):
    """-> ffn_out [T,K,H] f32 for the (t,k) pairs in ids; ew is [E,3I,H]."""
    T, H = x.shape
    K = ids.shape[1]
    E = ew.shape[0]
    x, px = _f32(x)
    ew, pe = _f32(ew)
    ids, pi = _i32(ids)
    out = np.empty((T, K, H), np.float32)
    lib().oracle_expert_ffn(px, pe, pi, T, H, E, K, I, out.ctypes.data_as(_f32p),
                            nthreads or os.cpu_count() or 1)
    return out


def combine(ffn_out, weights):
    T, K, H = ffn_out.shape
    ffn_out, pf = _f32(ffn_out)
    weights, pw = _f32(weights)
    y = np.empty((T, H), np.float32)
    lib().oracle_combine(pf, pw, T, H, K, y.ctypes.data_as(_f32p))
    return y


def moe_naive(x, w_gate, ew, K, nthreads=None):
    """The full naive layer: -> y [T,H] f32, ids, weights (f32)."""
    T, H = x.shape
    E = w_gate.shape[1]
    I = ew.shape[1] // 3
    x, px = _f32(x)
    w_gate, pg = _f32(w_gate)
    ew, pe = _f32(ew)
    y = np.empty((T, H), np.float32)
    ids = np.empty((T, K), np.int32)
    wts = np.empty((T, K), np.float32)
    lib().oracle_moe_naive(px, pg, pe, T, H, E, K, I, y.ctypes.data_as(_f32p),
                           ids.ctypes.data_as(_i32p), wts.ctypes.data_as(_f32p),
                           nthreads or os.cpu_count() or 1)
    return y, ids, wts


def test_moe_inputs(T, H, E, I, seed=42):
    """fp32 inputs of tests/test_moe.cpp:373-381 (srand(seed), uniform [-1,1], x, w_gate, weights)."""
    x = np.empty((T, H), np.float32)
    wg = np.empty((H, E), np.float32)
    ew = np.empty((E, 3 * I, H), np.float32)
    lib().oracle_test_moe_inputs(seed, x.ctypes.data_as(_f32p), x.size, wg.ctypes.data_as(_f32p), wg.size,
                                 ew.ctypes.data_as(_f32p), ew.size)
    return x, wg, ew


# ----------------------------------------------------------------------------- reference itself
def ref_naive(x, w_gate, ew, K):
    T, H = x.shape
    E = w_gate.shape[1]
    I = ew.shape[1] // 3
    x, px = _f32(x)
    w_gate, pg = _f32(w_gate)
    ew, pe = _f32(ew)
    y = np.empty((T, H), np.float32)
    ref().ref_naive_moe(px, pg, pe, T, H, E, K, I, y.ctypes.data_as(_f32p))
    return y


def ref_tiled(x, w_gate, ew, K):
    T, H = x.shape
    E = w_gate.shape[1]
    I = ew.shape[1] // 3
    x, px = _f32(x)
    w_gate, pg = _f32(w_gate)
    ew, pe = _f32(ew)
    y = np.empty((T, H), np.float32)
    ref().ref_tiled_moe(px, pg, pe, T, H, E, K, I, y.ctypes.data_as(_f32p))
    return y


def ref_routing(x, w_gate, K):
    T, H = x.shape
    E = w_gate.shape[1]
    x, px = _f32(x)
    w_gate, pg = _f32(w_gate)
    ids = np.empty((T, K), np.int32)
    wts = np.empty((T, K), np.float32)
    ref().ref_tiled_routing(px, pg, T, H, E, K, ids.ctypes.data_as(_i32p), wts.ctypes.data_as(_f32p))
    return ids, wts


def ref_expert_ffn(x, ew, ids, weights):
    T, H = x.shape
    K = ids.shape[1]
    E = ew.shape[0]
    I = ew.shape[1] // 3
    x, px = _f32(x)
    ew, pe = _f32(ew)
    ids, pi = _i32(ids)
    weights, pw = _f32(weights)
    out = np.empty((T, K, H), np.float32)
    ref().ref_tiled_expert_ffn(px, pe, pi, pw, T, H, E, K, I, out.ctypes.data_as(_f32p))
    return out


class RefTimer:
    """Holds the reference's fp32 vectors so NaiveMoE can be timed on token slices."""

    def __init__(self, x, w_gate, ew, K):
        self.T, self.H = x.shape
        E = w_gate.shape[1]
        I = ew.shape[1] // 3
        _, px = _f32(x)
        _, pg = _f32(w_gate)
        _, pe = _f32(ew)
        self.h = ref().ref_ctx_create(px, pg, pe, self.T, self.H, E, K, I)

    def naive(self, t0, t1, nthreads):
        y = np.empty((t1 - t0, self.H), np.float32)
        ref().ref_ctx_naive(self.h, t0, t1, nthreads, y.ctypes.data_as(_f32p))
        return y

    def tiled(self, t0, t1, nthreads):
        """TiledMoE (tests/moe_cpu_sim.cpp:543-569) on tokens [t0, t1)."""
        y = np.empty((t1 - t0, self.H), np.float32)
        ref().ref_ctx_tiled(self.h, t0, t1, nthreads, y.ctypes.data_as(_f32p))
        return y

    def close(self):
        if self.h:
            ref().ref_ctx_destroy(self.h)
            self.h = None

    __del__ = close


def compare(actual, expected):
    """max abs err, mean abs err, cosine -- CompareResults, tests/moe_cpu_sim.cpp:586-604."""
    a = np.asarray(actual, np.float64).ravel()
    b = np.asarray(expected, np.float64).ravel()
    err = np.abs(a - b)
    da, db = float(a @ a), float(b @ b)
    cos = float(a @ b) / (np.sqrt(da) * np.sqrt(db)) if da > 0 and db > 0 else 0.0
    return float(err.max()) if err.size else 0.0, float(err.mean()) if err.size else 0.0, cos
