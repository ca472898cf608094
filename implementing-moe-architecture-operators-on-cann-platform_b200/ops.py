"""ctypes bindings of libmoe_b200.so and torch-tensor front ends.

Names, argument order and meaning follow the reference operators
(op_host/moe_ops.cpp:537-679): inputs first, then outputs, attrs topK and
intermediateSize.  Errors surface as MoeError carrying the C status code, the
analogue of the reference's GRAPH_FAILED (moe_ops.cpp:71-90).
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "libmoe_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "moe_ops.h")

MOE_OK = 0
STATUS = {
    0: "MOE_OK", -1: "MOE_ERR_NULL_POINTER", -2: "MOE_ERR_BAD_SHAPE", -3: "MOE_ERR_WORKSPACE_TOO_SMALL",
    -4: "MOE_ERR_CUDA", -5: "MOE_ERR_UNSUPPORTED", -6: "MOE_ERR_MISALIGNED", -7: "MOE_ERR_NCCL",
    -8: "MOE_ERR_TIMEOUT", -9: "MOE_ERR_DEVICE",
}


class MoeError(RuntimeError):
    def __init__(self, status: int, where: str = ""):
        self.status = status
        name = STATUS.get(status, str(status))
        extra = ""
        if status == -4 and _lib is not None:
            extra = f" (cudaError {_lib.MoeLastCudaError()})"
        super().__init__(f"{where}: {name}{extra}")


_lib = None
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_i64p = ctypes.POINTER(ctypes.c_int64)
_intp = ctypes.POINTER(ctypes.c_int)


def lib_path() -> str:
    return _LIB_PATH


def declared_symbols() -> list[str]:
    """Every function the public header declares."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.findall(r"\b(Moe[A-Za-z0-9_]+)\s*\(", src)


def lib():
    """Loads libmoe_b200.so (raising if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.isfile(_LIB_PATH):
            raise ImportError(f"{_LIB_PATH} not built; run __graft_entry__.build()")
        try:  # resolve libcudart.so.12 through torch's copy when it is importable
            import torch  # noqa: F401
        except Exception:
            pass
        L = ctypes.CDLL(_LIB_PATH)
        L.MoeRoutingTopK.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]
        L.MoeExpertFFNWorkspaceSize.argtypes = [_i64] * 5
        L.MoeExpertFFNWorkspaceSize.restype = _sz
        L.MoeExpertFFN.argtypes = [_vp] * 5 + [_i64] * 5 + [_vp, _sz, _vp]
        L.MoeCombine.argtypes = [_vp] * 4 + [_i64] * 3 + [_vp]
        L.MoeLayerWorkspaceSize.argtypes = [_i64] * 5
        L.MoeLayerWorkspaceSize.restype = _sz
        L.MoeLayerForward.argtypes = [_vp] * 7 + [_i64] * 5 + [_vp, _sz, _vp]
        L.MoePermuteWorkspaceSize.argtypes = [_i64] * 3
        L.MoePermuteWorkspaceSize.restype = _sz
        L.MoePermute.argtypes = [_vp] * 3 + [_i64] * 3 + [_vp, _sz, _vp]
        L.MoeGetDeviceError.argtypes = [_vp, _intp, _vp]
        L.MoeStatusString.argtypes = [ctypes.c_int]
        L.MoeStatusString.restype = ctypes.c_char_p
        L.MoeLastCudaError.argtypes = []
        L.MoeEpGetUniqueId.argtypes = [_vp]
        L.MoeEpInit.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]
        L.MoeEpDestroy.argtypes = [_vp]
        L.MoeEpWorkspaceSize.argtypes = [ctypes.c_int] + [_i64] * 6
        L.MoeEpWorkspaceSize.restype = _sz
        L.MoeEpLayerForward.argtypes = [_vp] * 5 + [_i64] * 6 + [_vp, _sz, _vp]
        _i32p = ctypes.POINTER(ctypes.c_int32)
        L.MoeEpPlan.argtypes = [_i32p, _i32p, ctypes.c_int, ctypes.c_int, _i32p, _i32p, _i32p, _i32p]
        L.MoeTraceStart.argtypes = [ctypes.c_int]
        L.MoeTraceStop.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int, _intp]
        L.MoeRoutingInferShape.argtypes = [_i64p, ctypes.c_int, _i64p, ctypes.c_int, _i64, _i64p, _i64p,
                                           _intp, _intp]
        L.MoeExpertFFNInferShape.argtypes = [_i64p, ctypes.c_int, _i64p, ctypes.c_int, _i64p, ctypes.c_int,
                                             _i64, _i64p, _intp, _i64p, _i64p, _i64p]
        L.MoeCombineInferShape.argtypes = [_i64p, ctypes.c_int, _i64p, ctypes.c_int, _i64p, _intp]
        _lib = L
    return _lib


def _check(rc: int, where: str):
    if rc != MOE_OK:
        raise MoeError(rc, where)


# ----------------------------------------------------------------------------- torch front end
def _torch():
    import torch

    return torch


def _stream_handle(t):
    torch = _torch()
    return _vp(torch.cuda.current_stream(t.device).cuda_stream)


def _cuda(t, name, dtype=None):
    torch = _torch()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise MoeError(-1, f"{name} must be a CUDA tensor (no CPU fallback)")
    if dtype is not None and t.dtype != dtype:
        raise MoeError(-2, f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise MoeError(-2, f"{name} must be contiguous")
    return t


def _ptr(t):
    return _vp(t.data_ptr()) if t is not None else _vp(0)


def moe_routing_topk(x, w_gate, topK: int = 2, expert_ids=None, weights=None):
    """x [T,H] fp16, w_gate [H,E] fp16 -> (expert_ids [T,K] int32, weights [T,K] fp16)."""
    torch = _torch()
    _cuda(x, "x", torch.float16)
    _cuda(w_gate, "w_gate", torch.float16)
    if x.dim() != 2 or w_gate.dim() != 2 or x.shape[1] != w_gate.shape[0]:
        raise MoeError(-2, "MoeRoutingTopK shapes")
    T, H = x.shape
    E = w_gate.shape[1]
    K = topK if topK > 0 else 2
    if expert_ids is None:
        expert_ids = torch.empty((T, K), dtype=torch.int32, device=x.device)
    if weights is None:
        weights = torch.empty((T, K), dtype=torch.float16, device=x.device)
    _check(lib().MoeRoutingTopK(_ptr(x), _ptr(w_gate), _ptr(expert_ids), _ptr(weights), T, H, E, K,
                                _stream_handle(x)), "MoeRoutingTopK")
    return expert_ids, weights


def moe_expert_ffn_workspace_size(T, H, E, K, I) -> int:
    return int(lib().MoeExpertFFNWorkspaceSize(T, H, E, K, I))


def moe_layer_workspace_size(T, H, E, K, I) -> int:
    return int(lib().MoeLayerWorkspaceSize(T, H, E, K, I))


def _workspace(nbytes, device):
    torch = _torch()
    return torch.empty((max(int(nbytes), 1),), dtype=torch.uint8, device=device)


def moe_expert_ffn(x, expert_ids, weights, expert_weights, intermediateSize: int = 0, expert_out=None,
                   workspace=None):
    """-> expert_out [T,K,H] fp16.  expert_weights [E,3I,H]; weights is accepted and unused."""
    torch = _torch()
    _cuda(x, "x", torch.float16)
    _cuda(expert_ids, "expert_ids", torch.int32)
    _cuda(expert_weights, "expert_weights", torch.float16)
    dims = infer_shapes("ffn", x.shape, expert_ids.shape, expert_weights.shape, intermediateSize)
    T, H = x.shape
    E, K, I = dims["E"], dims["K"], dims["I"]
    if expert_out is None:
        expert_out = torch.empty((T, K, H), dtype=torch.float16, device=x.device)
    need = moe_expert_ffn_workspace_size(T, H, E, K, I)
    if need == 0:
        raise MoeError(-2, "MoeExpertFFN shapes")
    if workspace is None:
        workspace = _workspace(need, x.device)
    _check(lib().MoeExpertFFN(_ptr(x), _ptr(expert_ids), _ptr(weights), _ptr(expert_weights), _ptr(expert_out),
                              T, H, E, K, I, _ptr(workspace), workspace.numel(), _stream_handle(x)),
           "MoeExpertFFN")
    return expert_out


def moe_combine(expert_out, expert_ids, weights, y=None):
    """expert_out [T,K,H], weights [T,K] -> y [T,H] fp16 (expert_ids accepted, unused)."""
    torch = _torch()
    _cuda(expert_out, "expert_out", torch.float16)
    _cuda(weights, "weights", torch.float16)
    if expert_out.dim() != 3:
        raise MoeError(-2, "MoeCombine: expert_out must be 3-D")
    T, K, H = expert_out.shape
    if y is None:
        y = torch.empty((T, H), dtype=torch.float16, device=expert_out.device)
    _check(lib().MoeCombine(_ptr(expert_out), _ptr(expert_ids), _ptr(weights), _ptr(y), T, H, K,
                            _stream_handle(expert_out)), "MoeCombine")
    return y


def moe_layer_forward(x, w_gate, expert_weights, topK: int = 2, y=None, expert_ids=None, weights=None,
                      expert_out=None, workspace=None):
    """Routing -> FFN -> combine in one call; returns y [T,H] fp16."""
    torch = _torch()
    _cuda(x, "x", torch.float16)
    _cuda(w_gate, "w_gate", torch.float16)
    _cuda(expert_weights, "expert_weights", torch.float16)
    T, H = x.shape
    E = w_gate.shape[1]
    K = topK
    I = expert_weights.shape[1] // 3
    if y is None:
        y = torch.empty((T, H), dtype=torch.float16, device=x.device)
    if workspace is None:
        workspace = _workspace(moe_layer_workspace_size(T, H, E, K, I), x.device)
    _check(lib().MoeLayerForward(_ptr(x), _ptr(w_gate), _ptr(expert_weights), _ptr(y), _ptr(expert_ids),
                                 _ptr(weights), _ptr(expert_out), T, H, E, K, I, _ptr(workspace),
                                 workspace.numel(), _stream_handle(x)), "MoeLayerForward")
    return y


def moe_permute(expert_ids, numExperts: int, workspace=None):
    """expert_ids [T,K] int32 -> (perm [T*K] int32, expert_offsets [E+1] int32)."""
    torch = _torch()
    _cuda(expert_ids, "expert_ids", torch.int32)
    T, K = expert_ids.shape
    E = numExperts
    perm = torch.empty((T * K,), dtype=torch.int32, device=expert_ids.device)
    offs = torch.empty((E + 1,), dtype=torch.int32, device=expert_ids.device)
    if workspace is None:
        workspace = _workspace(lib().MoePermuteWorkspaceSize(T, K, E), expert_ids.device)
    _check(lib().MoePermute(_ptr(expert_ids), _ptr(perm), _ptr(offs), T, K, E, _ptr(workspace),
                            workspace.numel(), _stream_handle(expert_ids)), "MoePermute")
    return perm, offs, workspace


def device_error(workspace) -> int:
    """Reads the device error word of a workspace (synchronises the current stream)."""
    code = ctypes.c_int(0)
    _check(lib().MoeGetDeviceError(_ptr(workspace), ctypes.byref(code), _stream_handle(workspace)),
           "MoeGetDeviceError")
    return code.value


def infer_shapes(op, *shapes_and_attrs):
    """InferShape/InferDataType mirrors through the C ABI (op_host/moe_ops.cpp)."""
    L = lib()

    def arr(shape):
        shape = tuple(int(s) for s in shape)
        return (ctypes.c_int64 * max(len(shape), 1))(*shape), len(shape)

    if op == "routing":
        xs, ws, topK = shapes_and_attrs
        xa, xr = arr(xs)
        wa, wr = arr(ws)
        ids = (ctypes.c_int64 * 2)()
        wts = (ctypes.c_int64 * 2)()
        d0, d1 = ctypes.c_int(), ctypes.c_int()
        _check(L.MoeRoutingInferShape(xa, xr, wa, wr, topK, ids, wts, ctypes.byref(d0), ctypes.byref(d1)),
               "MoeRoutingInferShape")
        return {"expert_ids": tuple(ids), "weights": tuple(wts), "dtypes": (d0.value, d1.value)}
    if op == "ffn":
        xs, es, ews, inter = shapes_and_attrs
        xa, xr = arr(xs)
        ea, er = arr(es)
        wa, wr = arr(ews)
        out = (ctypes.c_int64 * 3)()
        dt = ctypes.c_int()
        E, K, I = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        _check(L.MoeExpertFFNInferShape(xa, xr, ea, er, wa, wr, inter, out, ctypes.byref(dt), ctypes.byref(E),
                                        ctypes.byref(K), ctypes.byref(I)), "MoeExpertFFNInferShape")
        return {"expert_out": tuple(out), "dtype": dt.value, "E": E.value, "K": K.value, "I": I.value}
    if op == "combine":
        os_, es = shapes_and_attrs
        oa, orank = arr(os_)
        ea, er = arr(es)
        y = (ctypes.c_int64 * 2)()
        dt = ctypes.c_int()
        _check(L.MoeCombineInferShape(oa, orank, ea, er, y, ctypes.byref(dt)), "MoeCombineInferShape")
        return {"y": tuple(y), "dtype": dt.value}
    raise ValueError(op)


TRACE_STAGES = ("routing", "permute", "gather", "gemm_swiglu", "gemm_down", "combine")


def trace_start(max_calls: int):
    """Starts stage tracing of MoeLayerForward / MoeExpertFFN calls on this thread."""
    _check(lib().MoeTraceStart(max_calls), "MoeTraceStart")
    return max_calls


def trace_stop(max_calls: int):
    """-> list of per-call dicts {stage: milliseconds} (synchronises on the events)."""
    buf = (ctypes.c_float * (max_calls * len(TRACE_STAGES)))()
    n = ctypes.c_int(0)
    _check(lib().MoeTraceStop(buf, max_calls, ctypes.byref(n)), "MoeTraceStop")
    out = []
    for c in range(min(n.value, max_calls)):
        out.append({st: float(buf[c * len(TRACE_STAGES) + i]) for i, st in enumerate(TRACE_STAGES)})
    return out


# ----------------------------------------------------------------------------- expert parallel
EP_UNIQUE_ID_BYTES = 128


def ep_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(EP_UNIQUE_ID_BYTES)
    _check(lib().MoeEpGetUniqueId(buf), "MoeEpGetUniqueId")
    return buf.raw


def ep_plan(send_counts, recv_counts):
    """MoeEpPlan on [n, El] int32 arrays -> (sendOff, recvOff, expertOff, segments[El*n, 3])."""
    import numpy as np

    sc = np.ascontiguousarray(send_counts, np.int32)
    rc = np.ascontiguousarray(recv_counts, np.int32)
    n, El = sc.shape
    so = np.empty(n + 1, np.int32)
    ro = np.empty(n + 1, np.int32)
    eo = np.empty(El + 1, np.int32)
    seg = np.empty((El * n, 3), np.int32)
    p = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))  # noqa: E731
    _check(lib().MoeEpPlan(p(sc), p(rc), n, El, p(so), p(ro), p(eo), p(seg)), "MoeEpPlan")
    return so, ro, eo, seg


class EpContext:
    """One rank of the expert-parallel layer (MoeEpInit / MoeEpLayerForward)."""

    def __init__(self, unique_id: bytes, rank: int, nranks: int, timeout_ms: int = 60000):
        self.rank, self.nranks = rank, nranks
        h = _vp()
        _check(lib().MoeEpInit(ctypes.c_char_p(unique_id), rank, nranks, timeout_ms, ctypes.byref(h)), "MoeEpInit")
        self.h = h
        self._ws = None

    def workspace_size(self, T, H, E, K, I, max_recv_rows=0):
        return int(lib().MoeEpWorkspaceSize(self.nranks, T, H, E, K, I, max_recv_rows))

    def forward(self, x, w_gate, expert_weights_local, topK=2, y=None, max_recv_rows=0, workspace=None):
        torch = _torch()
        _cuda(x, "x", torch.float16)
        _cuda(w_gate, "w_gate", torch.float16)
        _cuda(expert_weights_local, "expert_weights_local", torch.float16)
        T, H = x.shape
        E = w_gate.shape[1]
        I = expert_weights_local.shape[1] // 3
        if y is None:
            y = torch.empty((T, H), dtype=torch.float16, device=x.device)
        if workspace is None:
            need = self.workspace_size(T, H, E, topK, I, max_recv_rows)
            if need == 0:
                raise MoeError(-2, "MoeEpWorkspaceSize")
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty((need,), dtype=torch.uint8, device=x.device)
            workspace = self._ws
        _check(lib().MoeEpLayerForward(self.h, _ptr(x), _ptr(w_gate), _ptr(expert_weights_local), _ptr(y), T, H,
                                       E, topK, I, max_recv_rows, _ptr(workspace), workspace.numel(),
                                       _stream_handle(x)), "MoeEpLayerForward")
        return y

    def close(self):
        if self.h:
            rc = lib().MoeEpDestroy(self.h)
            self.h = None
            _check(rc, "MoeEpDestroy")
