"""TEST INFRASTRUCTURE ONLY: ctypes access to the two CPU checkers.

  impl="orc"  my C restatement (oracle/moe_oracle.c -> oracle/liborc.so)
  impl="ref"  glm.c's own infer.c compiled from its sources
              (oracle/ref_harness.c -> oracle/_ref/libglmref.so)

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may import this
module, and only to check or to time the CPU path -- never to produce a
product result.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_SO = os.path.join(HERE, "liborc.so")
REF_SO = os.path.join(HERE, "_ref", "libglmref.so")

MOE_FIELDS = (
    "ffn_norm", "router", "router_bias",
    "gate_sh_q", "gate_sh_s", "up_sh_q", "up_sh_s", "down_sh_q", "down_sh_s",
    "gate_q", "gate_s", "up_q", "up_s", "down_q", "down_s",
)

_libs: dict = {}


def build() -> None:
    """Compile liborc.so (and _ref/libglmref.so where the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def lib(impl: str = "orc") -> ctypes.CDLL:
    if impl in _libs:
        return _libs[impl]
    path = ORC_SO if impl == "orc" else REF_SO
    if not os.path.exists(path):
        if impl == "orc":
            build()
        else:
            raise FileNotFoundError(f"{path} missing: the reference checker was not built")
    L = ctypes.CDLL(path)
    P = ctypes.c_void_p
    I = ctypes.c_int
    if impl == "orc":
        L.orc_moe_layer_ptrs.argtypes = [I, I, I, I, I, P, I, P, P, P, I]
        L.orc_moe_layer_ptrs.restype = I
        L.orc_matvec_q80.argtypes = [P, P, P, P, I, I, I]
        L.orc_matvec_q80.restype = None
        L.orc_rmsnorm.argtypes = [P, P, P, I]
        L.orc_router_logits.argtypes = [P, P, P, I, I]
        L.orc_sigmoid.argtypes = [ctypes.c_float]
        L.orc_sigmoid.restype = ctypes.c_float
    else:
        L.ref_moe_layer.argtypes = [I, I, I, I, I, P, I, P, P, P]
        L.ref_moe_layer.restype = I
        L.ref_time_moe_layer.argtypes = [I, I, I, I, I, P, I, P, I, I, ctypes.POINTER(ctypes.c_double)]
        L.ref_time_moe_layer.restype = I
        L.ref_matvec_q80.argtypes = [P, P, P, P, I, I, I]
        L.ref_matvec_q80.restype = None
        L.ref_time_matvec_q80.argtypes = [P, P, P, P, I, I, I, I, I, ctypes.POINTER(ctypes.c_double)]
        L.ref_time_matvec_q80.restype = I
        L.ref_rmsnorm.argtypes = [P, P, P, I]
        L.ref_omp_max_threads.restype = I
    _libs[impl] = L
    return L


def _ptr(a):
    return None if a is None else a.ctypes.data


def _ptr_table(layer: dict):
    arr = (ctypes.c_void_p * len(MOE_FIELDS))()
    keep = []
    for i, name in enumerate(MOE_FIELDS):
        a = layer.get(name)
        if a is not None:
            a = np.ascontiguousarray(a)
            keep.append(a)
            arr[i] = a.ctypes.data
        else:
            arr[i] = None
    return arr, keep


def moe_layer(layer: dict, x: np.ndarray, impl: str = "orc", routed: bool = True):
    """Run the MoE FFN layer on every row of x ([T, D] or [D]).

    Returns (x_out [T, D], topk_idx int32 [T, K], topk_w fp32 [T, K]).
    With impl="ref", `routed=False` is expressed the reference's own way,
    through GLM_DISABLE_MOE_ROUTED (infer.c:1161-1165).
    """
    x2 = np.array(x, dtype=np.float32, copy=True, order="C").reshape(-1, layer["dim"])
    T, K = x2.shape[0], layer["k_used"]
    idx = np.zeros((T, K), dtype=np.int32)
    w = np.zeros((T, K), dtype=np.float32)
    table, keep = _ptr_table(layer)
    dims = (layer["dim"], layer["ffn"], layer["n_experts"], K, layer["gs"])
    if impl == "orc":
        rc = lib("orc").orc_moe_layer_ptrs(*dims, ctypes.cast(table, ctypes.c_void_p), T,
                                           _ptr(x2), _ptr(idx), _ptr(w), 1 if routed else 0)
    else:
        old = os.environ.get("GLM_DISABLE_MOE_ROUTED")
        try:
            if not routed:
                os.environ["GLM_DISABLE_MOE_ROUTED"] = "1"
            elif old is not None:
                del os.environ["GLM_DISABLE_MOE_ROUTED"]
            rc = lib("ref").ref_moe_layer(*dims, ctypes.cast(table, ctypes.c_void_p), T,
                                          _ptr(x2), _ptr(idx), _ptr(w))
        finally:
            if old is None:
                os.environ.pop("GLM_DISABLE_MOE_ROUTED", None)
            else:
                os.environ["GLM_DISABLE_MOE_ROUTED"] = old
    del keep
    if rc != 0:
        raise RuntimeError(f"{impl} moe_layer failed rc={rc}")
    return x2, idx, w


def time_moe_layer(layer: dict, x: np.ndarray, warmup: int, iters: int) -> float:
    """Reference MoE layer wall time (ms total over `iters` calls), timed in C
    with the reference's own monotonic clock."""
    x2 = np.array(x, dtype=np.float32, copy=True, order="C").reshape(-1, layer["dim"])
    table, keep = _ptr_table(layer)
    out = ctypes.c_double(0.0)
    lib("ref").ref_time_moe_layer(layer["dim"], layer["ffn"], layer["n_experts"], layer["k_used"], layer["gs"],
                                  ctypes.cast(table, ctypes.c_void_p), x2.shape[0], _ptr(x2),
                                  warmup, iters, ctypes.byref(out))
    del keep
    return out.value


def matvec(q: np.ndarray, s: np.ndarray, x: np.ndarray, gs: int, impl: str = "orc") -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(s, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = q.shape
    y = np.zeros(rows, dtype=np.float32)
    fn = lib(impl).orc_matvec_q80 if impl == "orc" else lib("ref").ref_matvec_q80
    fn(_ptr(q), _ptr(s), _ptr(x), _ptr(y), rows, cols, gs)
    return y


def time_matvec(q, s, x, gs: int, warmup: int, iters: int) -> float:
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(s, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(q.shape[0], dtype=np.float32)
    out = ctypes.c_double(0.0)
    lib("ref").ref_time_matvec_q80(_ptr(q), _ptr(s), _ptr(x), _ptr(y), q.shape[0], q.shape[1], gs,
                                   warmup, iters, ctypes.byref(out))
    return out.value


def omp_threads() -> int:
    return int(lib("ref").ref_omp_max_threads())
