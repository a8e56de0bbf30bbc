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
REF_CUDA_SO = os.path.join(HERE, "_ref", "libglmref_cuda.so")  # glm.c patched with the cuda backend

MOE_FIELDS = (
    "ffn_norm", "router", "router_bias",
    "gate_sh_q", "gate_sh_s", "up_sh_q", "up_sh_s", "down_sh_q", "down_sh_s",
    "gate_q", "gate_s", "up_q", "up_s", "down_q", "down_s",
)

_libs: dict = {}


def reference_dir() -> str:
    """Where glm.c's sources are: $GLM_REFERENCE_DIR, else a `reference`
    directory beside this repository ('' when neither holds infer.c)."""
    cand = os.environ.get("GLM_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isfile(os.path.join(cand, "infer.c")) else ""


def build() -> None:
    """Compile liborc.so (and, where the reference sources exist, glm.c's own
    code: _ref/libglmref.so, plus the cuda-patched glm.c of INTEGRATION.md
    once the CUDA library is built)."""
    ref = reference_dir()
    subprocess.run(["make", "-s", "-C", HERE, "all", f"REF_DIR={ref}"], check=True)
    import glm_cuda_patch

    if ref and os.path.exists(os.path.join(glm_cuda_patch.CUDA_LIB_DIR, "libglm_cuda.so")):
        glm_cuda_patch.build(ref)


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def lib(impl: str = "orc") -> ctypes.CDLL:
    if impl in _libs:
        return _libs[impl]
    path = {"orc": ORC_SO, "ref": REF_SO, "refcuda": REF_CUDA_SO}[impl]
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
        L.ref_time_moe_stack.argtypes = [I, I, I, I, I, P, I, I, P, I, I, ctypes.POINTER(ctypes.c_double)]
        L.ref_time_moe_stack.restype = I
        L.ref_matvec_q80.argtypes = [P, P, P, P, I, I, I]
        L.ref_matvec_q80.restype = None
        L.ref_time_matvec_q80.argtypes = [P, P, P, P, I, I, I, I, I, ctypes.POINTER(ctypes.c_double)]
        L.ref_time_matvec_q80.restype = I
        L.ref_rmsnorm.argtypes = [P, P, P, I]
        L.ref_omp_max_threads.restype = I
        L.ref_set_omp_threads.argtypes = [I]
        L.ref_set_omp_threads.restype = None
        if hasattr(L, "ref_decode"):
            L.ref_decode.argtypes = [P, P, P, P, P, I, I, P, P]
            L.ref_decode.restype = I
        if hasattr(L, "ref_decode_bin"):
            L.ref_decode_bin.argtypes = [ctypes.c_char_p, P, I, I, I, P]
            L.ref_decode_bin.restype = I
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


def time_moe_stack(layers: list, x: np.ndarray, warmup: int, steps: int) -> float:
    """glm.c's MoE layer on one token per step through every layer of
    `layers` in turn (distinct weights); total milliseconds of `steps` steps,
    timed in C with the reference's own clock."""
    L0 = layers[0]
    x2 = np.array(x, dtype=np.float32, copy=True, order="C").reshape(-1, L0["dim"])
    n = len(layers)
    tab = (ctypes.c_void_p * (n * len(MOE_FIELDS)))()
    keep = []
    for l, layer in enumerate(layers):
        t, k = _ptr_table(layer)
        keep += k
        for i in range(len(MOE_FIELDS)):
            tab[l * len(MOE_FIELDS) + i] = t[i]
    out = ctypes.c_double(0.0)
    lib("ref").ref_time_moe_stack(L0["dim"], L0["ffn"], L0["n_experts"], L0["k_used"], L0["gs"],
                                  ctypes.cast(tab, ctypes.c_void_p), n, x2.shape[0], _ptr(x2), warmup, steps,
                                  ctypes.byref(out))
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


def set_omp_threads(n: int) -> None:
    lib("ref").ref_set_omp_threads(int(n))


# Table orders of ref_decode: Runtime globals (model.h:87-103) and
# LayerAttnWeights (model.h:46-62).
GLOBAL_FIELDS = ("output_norm", "tok_q", "tok_s", "out_q", "out_s", "l0_ffn_norm", "l0_gate_q", "l0_gate_s",
                 "l0_up_q", "l0_up_s", "l0_down_q", "l0_down_s")
ATTN_FIELDS = ("attn_norm", "q_a_norm", "kv_a_norm", "q_a_q", "q_a_s", "q_b_q", "q_b_s", "kv_a_q", "kv_a_s",
               "k_b_q", "k_b_s", "v_b_q", "v_b_s", "attn_out_q", "attn_out_s")
DECODER_DIMS = ("dim", "hidden_dim", "n_layers", "n_heads", "vocab_size", "rope_dim", "q_lora_rank",
                "kv_lora_rank", "qk_nope_dim", "head_k_dim", "v_head_dim", "n_routed_experts", "n_experts_used",
                "group_size", "moe_ffn_dim", "cache_cap")


def ref_decode(model: dict, prompt, n_gen: int, cache_cap: int, with_logits: bool = False, impl: str = "ref"):
    """Greedy ids from glm.c's own forward pass (compiled from its sources):
    glm_cpu_forward_token per position, argmax at temperature 0, as
    glm_app_main feeds it (infer.c:2190-2228). model is synth.decoder_model's
    dict; returns (ids [n_gen], logits [n_gen, vocab] or None). impl="refcuda"
    runs glm.c patched with the cuda backend (oracle/glm_cuda_patch.py): the
    same loop with every MoE layer and Q8 matvec in libglm_cuda.so."""
    d = dict(model["dims"], cache_cap=cache_cap)
    icfg = np.array([d[k] for k in DECODER_DIMS], dtype=np.int32)
    keep = []

    def table(ptrs):
        arr = (ctypes.c_void_p * len(ptrs))(*[None if p is None else p.ctypes.data for p in ptrs])
        keep.append(arr)
        return ctypes.cast(arr, ctypes.c_void_p)

    g = model["globals"]
    glob = table([np.ascontiguousarray(g[k]) for k in GLOBAL_FIELDS])
    attn = table([np.ascontiguousarray(a[k]) for a in model["attn"] for k in ATTN_FIELDS])
    moe_ptrs = []
    for l, m in enumerate(model["moe"]):
        moe_ptrs += [None] * 15 if m is None else [np.ascontiguousarray(m[k]) for k in MOE_FIELDS]
    moe = table(moe_ptrs)
    p = np.ascontiguousarray(prompt, dtype=np.int32)
    out = np.zeros(n_gen, dtype=np.int32)
    logits = np.zeros((n_gen, d["vocab_size"]), dtype=np.float32) if with_logits else None
    rc = lib(impl).ref_decode(icfg.ctypes.data, glob, attn, moe, p.ctypes.data, len(p), n_gen, out.ctypes.data,
                               None if logits is None else logits.ctypes.data)
    del keep
    if rc != 0:
        raise RuntimeError(f"ref_decode failed ({rc})")
    return out, logits


def ref_decode_bin(path: str, prompt, n_gen: int, cache_cap: int):
    """Greedy ids from glm.c's own loader (runtime_open) and forward pass on a
    .bin checkpoint file."""
    p = np.ascontiguousarray(prompt, dtype=np.int32)
    out = np.zeros(n_gen, dtype=np.int32)
    rc = lib("ref").ref_decode_bin(os.fsencode(path), p.ctypes.data, len(p), n_gen, cache_cap, out.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"ref_decode_bin failed ({rc})")
    return out
