"""ctypes binding of include/glm_cuda.h (the library's C-ABI).

This is how tests, the benchmark and Python callers reach the CUDA path; it
mirrors the C entry points one to one and raises GlmCudaError on any nonzero
return, carrying glm_cuda_last_error(). Loading fails loudly when the built
library is missing: there is no fallback.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

from . import build as _build

LIB_PATH = _build.LIB
HEADER = os.path.join(_build.INCLUDE, "glm_cuda.h")

MOE_FIELDS = (
    "ffn_norm", "router", "router_bias",
    "gate_sh_q", "gate_sh_s", "up_sh_q", "up_sh_s", "down_sh_q", "down_sh_s",
    "gate_q", "gate_s", "up_q", "up_s", "down_q", "down_s",
)


class GlmCudaError(RuntimeError):
    def __init__(self, fn: str, rc: int, msg: str):
        super().__init__(f"{fn} returned {rc}: {msg}")
        self.rc = rc


def declared_functions(header: str = HEADER) -> list[str]:
    """Names of the functions include/glm_cuda.h declares."""
    src = open(header).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(glm_cuda_\w+)\s*\(", src)))


_P = ctypes.c_void_p
_I = ctypes.c_int


def _signatures(L: ctypes.CDLL) -> None:
    L.glm_cuda_init.argtypes = [_I] * 7
    L.glm_cuda_upload_moe_layer.argtypes = [_I] + [_P] * 15
    L.glm_cuda_bind_moe_layer_device.argtypes = [_I] + [_P] * 15
    L.glm_cuda_moe_layer.argtypes = [_I, _P, _I, _P, _P]
    L.glm_cuda_moe_layer_async.argtypes = [_I, _P, _I, _P, _P, _P]
    L.glm_cuda_moe_layer_profile.argtypes = [_I, _P, _P]
    L.glm_cuda_moe_layers_async.argtypes = [_I, _I, _P, _P, _P, _P]
    L.glm_cuda_model_init.argtypes = [_I, _P]
    L.glm_cuda_upload_model_globals.argtypes = [_P] * 12
    L.glm_cuda_bind_model_globals_device.argtypes = [_P] * 12
    L.glm_cuda_upload_attn_layer.argtypes = [_I] + [_P] * 15
    L.glm_cuda_bind_attn_layer_device.argtypes = [_I] + [_P] * 15
    L.glm_cuda_forward_token.argtypes = [_I, _I, _P]
    L.glm_cuda_generate.argtypes = [_P, _I, _I, _P, _P]
    L.glm_cuda_prefill.argtypes = [_P, _I, _I, _P]
    L.glm_cuda_set_model_prefill.argtypes = [_I]
    L.glm_cuda_set_decode_path.argtypes = [_I]
    L.glm_cuda_decode_path.argtypes = []
    L.glm_cuda_set_prefill_tokens.argtypes = [_I]
    L.glm_cuda_ep_setup.argtypes = [_I, _I, _I]
    L.glm_cuda_ep_dispatch.argtypes = [_I, _P, _I, _P, _P, _P, _P]
    L.glm_cuda_ep_experts.argtypes = [_I, _P, _P, _I, _P, _P]
    L.glm_cuda_ep_combine.argtypes = [_I, _P, _P, _P, _P, _P]
    L.glm_cuda_ep_status.argtypes = []
    L.glm_cuda_ep_peer_region.argtypes = [_P, _P]
    L.glm_cuda_ep_peer_open.argtypes = [_P, _P]
    L.glm_cuda_ep_peer_connect.argtypes = [_P]
    L.glm_cuda_ep_p2p_dispatch.argtypes = [_I, _P, _I, _P]
    L.glm_cuda_ep_p2p_experts.argtypes = [_I, _P]
    L.glm_cuda_ep_p2p_combine.argtypes = [_I, _P, _P, _P, _P]
    L.glm_cuda_ep_p2p_counts.argtypes = [_P, _P]
    L.glm_cuda_load_checkpoint.argtypes = [ctypes.c_char_p, _I, _I]
    L.glm_cuda_moe_layer_noalloc.argtypes = [_P] * 15 + [_I] * 5 + [_P, _I, _P, _P, _P]
    L.glm_cuda_moe_layer_noalloc.restype = _I
    L.glm_cuda_matvec_q80.argtypes = [_P, _P, _P, _P, _I, _I, _I]
    L.glm_cuda_matvec_q80_async.argtypes = [_P, _P, _P, _P, _I, _I, _I, _P]
    L.glm_cuda_synchronize.argtypes = []
    L.glm_cuda_route_stats.argtypes = [_P]
    L.glm_cuda_launch_count.argtypes = []
    L.glm_cuda_launch_count.restype = ctypes.c_uint64
    L.glm_cuda_last_error.argtypes = []
    L.glm_cuda_last_error.restype = ctypes.c_char_p
    L.glm_cuda_free.argtypes = []
    L.glm_cuda_free.restype = None
    for name in ("glm_cuda_init", "glm_cuda_upload_moe_layer", "glm_cuda_bind_moe_layer_device",
                 "glm_cuda_moe_layer", "glm_cuda_moe_layer_async", "glm_cuda_moe_layer_profile",
                 "glm_cuda_moe_layers_async", "glm_cuda_set_decode_path", "glm_cuda_decode_path",
                 "glm_cuda_set_prefill_tokens", "glm_cuda_ep_setup", "glm_cuda_ep_dispatch", "glm_cuda_ep_experts",
                 "glm_cuda_ep_combine", "glm_cuda_ep_status", "glm_cuda_load_checkpoint",
                 "glm_cuda_ep_peer_region", "glm_cuda_ep_peer_open", "glm_cuda_ep_peer_connect",
                 "glm_cuda_ep_p2p_dispatch", "glm_cuda_ep_p2p_experts", "glm_cuda_ep_p2p_combine",
                 "glm_cuda_ep_p2p_counts",
                 "glm_cuda_model_init", "glm_cuda_upload_model_globals", "glm_cuda_bind_model_globals_device",
                 "glm_cuda_upload_attn_layer", "glm_cuda_bind_attn_layer_device", "glm_cuda_forward_token",
                 "glm_cuda_generate", "glm_cuda_prefill", "glm_cuda_set_model_prefill",
                 "glm_cuda_matvec_q80",
                 "glm_cuda_matvec_q80_async", "glm_cuda_synchronize", "glm_cuda_route_stats"):
        getattr(L, name).restype = _I


_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libglm_cuda.so (RTLD_GLOBAL so the process records it as loaded)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is missing: run __graft_entry__.build() (no CPU fallback exists)")
    L = ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
    _signatures(L)
    _lib = L
    return L


def _ptr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()  # torch tensor


class GlmCuda:
    """One-to-one wrapper of the C entry points."""

    def __init__(self, path: str = LIB_PATH):
        self.L = load(path)

    def _check(self, fn: str, rc: int) -> None:
        if rc != 0:
            raise GlmCudaError(fn, rc, self.last_error())

    def last_error(self) -> str:
        return (self.L.glm_cuda_last_error() or b"").decode()

    def init(self, device: int, dim: int, ffn: int, n_experts: int, k_used: int, gs: int, n_layers: int) -> None:
        self._check("glm_cuda_init", self.L.glm_cuda_init(device, dim, ffn, n_experts, k_used, gs, n_layers))

    def upload_moe_layer(self, layer: int, L: dict) -> None:
        arrs = [None if L.get(k) is None else np.ascontiguousarray(L[k]) for k in MOE_FIELDS]
        self._check("glm_cuda_upload_moe_layer",
                    self.L.glm_cuda_upload_moe_layer(layer, *[_ptr(a) for a in arrs]))

    def bind_moe_layer_device(self, layer: int, ptrs: dict) -> None:
        """ptrs: field name -> device pointer (int or torch tensor)."""
        self._check("glm_cuda_bind_moe_layer_device",
                    self.L.glm_cuda_bind_moe_layer_device(layer, *[_ptr(ptrs.get(k)) for k in MOE_FIELDS]))

    def moe_layer(self, layer: int, x: np.ndarray, k_used: int):
        x2 = np.array(x, dtype=np.float32, copy=True, order="C")
        T = x2.shape[0] if x2.ndim == 2 else 1
        idx = np.zeros((T, k_used), dtype=np.int32)
        w = np.zeros((T, k_used), dtype=np.float32)
        self._check("glm_cuda_moe_layer", self.L.glm_cuda_moe_layer(layer, _ptr(x2), T, _ptr(idx), _ptr(w)))
        return x2, idx, w

    def moe_layer_host_inplace(self, layer: int, x: np.ndarray, idx=None, w=None) -> None:
        T = x.shape[0] if x.ndim == 2 else 1
        self._check("glm_cuda_moe_layer", self.L.glm_cuda_moe_layer(layer, _ptr(x), T, _ptr(idx), _ptr(w)))

    def moe_layer_async(self, layer: int, x_dev, n_tokens: int, idx_dev=None, w_dev=None, stream=None) -> None:
        self._check("glm_cuda_moe_layer_async",
                    self.L.glm_cuda_moe_layer_async(layer, _ptr(x_dev), n_tokens, _ptr(idx_dev), _ptr(w_dev),
                                                    stream))

    def moe_layers_async(self, first: int, n_layers: int, x_dev, idx_dev=None, w_dev=None, stream=None) -> None:
        """One token through MoE layers first .. first+n_layers-1 in one launch."""
        self._check("glm_cuda_moe_layers_async",
                    self.L.glm_cuda_moe_layers_async(first, n_layers, _ptr(x_dev), _ptr(idx_dev), _ptr(w_dev),
                                                     stream))

    PATH_AUTO, PATH_PERSISTENT, PATH_CHAIN = 0, 1, 2

    # ---- full decoder
    MODEL_DIMS = ("dim", "hidden_dim", "n_layers", "n_heads", "vocab_size", "rope_dim", "q_lora_rank",
                  "kv_lora_rank", "qk_nope_dim", "head_k_dim", "v_head_dim", "n_routed_experts", "n_experts_used",
                  "group_size", "moe_ffn_dim", "cache_cap")
    GLOBAL_FIELDS = ("output_norm", "tok_q", "tok_s", "out_q", "out_s", "l0_ffn_norm", "l0_gate_q", "l0_gate_s",
                     "l0_up_q", "l0_up_s", "l0_down_q", "l0_down_s")
    ATTN_FIELDS = ("attn_norm", "q_a_norm", "kv_a_norm", "q_a_q", "q_a_s", "q_b_q", "q_b_s", "kv_a_q", "kv_a_s",
                   "k_b_q", "k_b_s", "v_b_q", "v_b_s", "attn_out_q", "attn_out_s")

    def model_init(self, device: int, dims: dict) -> None:
        arr = (ctypes.c_int32 * len(self.MODEL_DIMS))(*[int(dims[k]) for k in self.MODEL_DIMS])
        self._check("glm_cuda_model_init", self.L.glm_cuda_model_init(device, ctypes.addressof(arr)))

    def upload_model_globals(self, g: dict, device: bool = False) -> None:
        fn = "glm_cuda_bind_model_globals_device" if device else "glm_cuda_upload_model_globals"
        self._check(fn, getattr(self.L, fn)(*[_ptr(g[k]) for k in self.GLOBAL_FIELDS]))

    def upload_attn_layer(self, layer: int, a: dict, device: bool = False) -> None:
        fn = "glm_cuda_bind_attn_layer_device" if device else "glm_cuda_upload_attn_layer"
        self._check(fn, getattr(self.L, fn)(layer, *[_ptr(a[k]) for k in self.ATTN_FIELDS]))

    def forward_token(self, token: int, pos: int, vocab: int | None = None):
        logits = np.zeros(vocab, dtype=np.float32) if vocab else None
        self._check("glm_cuda_forward_token", self.L.glm_cuda_forward_token(token, pos, _ptr(logits)))
        return logits

    def generate(self, prompt, n_gen: int):
        """Greedy ids and the device milliseconds of all steps."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen, dtype=np.int32)
        ms = ctypes.c_float(0.0)
        self._check("glm_cuda_generate", self.L.glm_cuda_generate(_ptr(p), len(p), n_gen, _ptr(out),
                                                                   ctypes.addressof(ms)))
        return out, float(ms.value)

    def prefill(self, tokens, start_pos: int = 0, vocab: int | None = None):
        """The batched prompt pass over positions start_pos .. + len(tokens) - 1;
        the last token's logits when vocab is given."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.zeros(vocab, dtype=np.float32) if vocab else None
        self._check("glm_cuda_prefill", self.L.glm_cuda_prefill(_ptr(t), len(t), start_pos, _ptr(logits)))
        return logits

    def set_model_prefill(self, min_tokens: int) -> None:
        self._check("glm_cuda_set_model_prefill", self.L.glm_cuda_set_model_prefill(min_tokens))

    def set_decode_path(self, path: int) -> None:
        self._check("glm_cuda_set_decode_path", self.L.glm_cuda_set_decode_path(path))

    def load_checkpoint(self, path: str, device: int, cache_cap: int) -> None:
        """glm_cuda_load_checkpoint: a glm.c .bin file to the device (model init included)."""
        self._check("glm_cuda_load_checkpoint", self.L.glm_cuda_load_checkpoint(os.fsencode(path), device, cache_cap))

    def set_prefill_tokens(self, min_tokens: int) -> int:
        """Route calls with n_tokens >= min_tokens to the batched prefill
        kernels (0 disables); returns the previous threshold."""
        rc = self.L.glm_cuda_set_prefill_tokens(min_tokens)
        if rc < 0:
            self._check("glm_cuda_set_prefill_tokens", rc)
        return rc

    # ---- expert parallelism (stream: a cudaStream_t handle or None)
    def ep_setup(self, n_shards: int, shard: int, max_tokens: int) -> None:
        self._check("glm_cuda_ep_setup", self.L.glm_cuda_ep_setup(n_shards, shard, max_tokens))

    def ep_dispatch(self, layer: int, x_dev, n_tokens: int, send_rows, send_expert, send_counts, stream=None) -> None:
        self._check("glm_cuda_ep_dispatch",
                    self.L.glm_cuda_ep_dispatch(layer, _ptr(x_dev), n_tokens, _ptr(send_rows), _ptr(send_expert),
                                                _ptr(send_counts), stream))

    def ep_experts(self, layer: int, recv_rows, recv_expert, n_recv: int, out_rows, stream=None) -> None:
        self._check("glm_cuda_ep_experts",
                    self.L.glm_cuda_ep_experts(layer, _ptr(recv_rows), _ptr(recv_expert), n_recv, _ptr(out_rows),
                                               stream))

    def ep_combine(self, layer: int, x_dev, back_rows, idx_dev=None, w_dev=None, stream=None) -> None:
        self._check("glm_cuda_ep_combine",
                    self.L.glm_cuda_ep_combine(layer, _ptr(x_dev), _ptr(back_rows), _ptr(idx_dev), _ptr(w_dev),
                                               stream))

    def ep_status(self) -> None:
        self._check("glm_cuda_ep_status", self.L.glm_cuda_ep_status())

    # ---- expert parallelism over peer memory
    IPC_HANDLE_BYTES = 64

    def ep_peer_region(self) -> tuple[int, bytes]:
        """(device address, IPC handle bytes) of this rank's peer region."""
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(self.IPC_HANDLE_BYTES)
        self._check("glm_cuda_ep_peer_region",
                    self.L.glm_cuda_ep_peer_region(ctypes.byref(ptr), ctypes.cast(handle, ctypes.c_void_p)))
        return int(ptr.value), handle.raw

    def ep_peer_open(self, handle: bytes) -> int:
        """Map another rank's region (its IPC handle) into this process."""
        buf = ctypes.create_string_buffer(bytes(handle), self.IPC_HANDLE_BYTES)
        ptr = ctypes.c_void_p()
        self._check("glm_cuda_ep_peer_open",
                    self.L.glm_cuda_ep_peer_open(ctypes.cast(buf, ctypes.c_void_p), ctypes.byref(ptr)))
        return int(ptr.value)

    def ep_peer_connect(self, regions: list[int]) -> None:
        arr = (ctypes.c_void_p * len(regions))(*regions)
        self._check("glm_cuda_ep_peer_connect", self.L.glm_cuda_ep_peer_connect(ctypes.cast(arr, ctypes.c_void_p)))

    def ep_p2p_dispatch(self, layer: int, x_dev, n_tokens: int, stream=None) -> None:
        self._check("glm_cuda_ep_p2p_dispatch", self.L.glm_cuda_ep_p2p_dispatch(layer, _ptr(x_dev), n_tokens, stream))

    def ep_p2p_experts(self, layer: int, stream=None) -> None:
        self._check("glm_cuda_ep_p2p_experts", self.L.glm_cuda_ep_p2p_experts(layer, stream))

    def ep_p2p_combine(self, layer: int, x_dev, idx_dev=None, w_dev=None, stream=None) -> None:
        self._check("glm_cuda_ep_p2p_combine",
                    self.L.glm_cuda_ep_p2p_combine(layer, _ptr(x_dev), _ptr(idx_dev), _ptr(w_dev), stream))

    def ep_p2p_counts(self, n_shards: int) -> tuple[list[int], list[int]]:
        """(rows sent to each rank, rows received from each rank) of the last layer."""
        send = (ctypes.c_int32 * n_shards)()
        recv = (ctypes.c_int32 * n_shards)()
        self._check("glm_cuda_ep_p2p_counts", self.L.glm_cuda_ep_p2p_counts(send, recv))
        return list(send), list(recv)

    def decode_path(self) -> int:
        rc = self.L.glm_cuda_decode_path()
        if rc < 0:
            self._check("glm_cuda_decode_path", rc)
        return rc

    def moe_layer_profile(self, layer: int, x_dev) -> tuple[float, float, float]:
        """(route, gate_up, down) kernel milliseconds for one token, x_dev in place."""
        out = (ctypes.c_float * 3)()
        self._check("glm_cuda_moe_layer_profile",
                    self.L.glm_cuda_moe_layer_profile(layer, _ptr(x_dev), ctypes.addressof(out)))
        return float(out[0]), float(out[1]), float(out[2])

    def moe_layer_noalloc(self, ptrs: dict, dim: int, ffn: int, n_experts: int, k_used: int, gs: int, x_dev,
                          n_tokens: int, idx_dev=None, w_dev=None, stream=None) -> None:
        """glm_cuda_moe_layer_noalloc: device weights in `ptrs` (field -> pointer
        or tensor), x_dev updated in place; needs no glm_cuda_init."""
        self._check("glm_cuda_moe_layer_noalloc",
                    self.L.glm_cuda_moe_layer_noalloc(*[_ptr(ptrs.get(k)) for k in MOE_FIELDS], dim, ffn,
                                                      n_experts, k_used, gs, _ptr(x_dev), n_tokens,
                                                      _ptr(idx_dev), _ptr(w_dev), stream))

    def matvec(self, q: np.ndarray, s: np.ndarray, x: np.ndarray, gs: int) -> np.ndarray:
        rows, cols = q.shape
        y = np.zeros(rows, dtype=np.float32)
        self._check("glm_cuda_matvec_q80", self.L.glm_cuda_matvec_q80(_ptr(q), _ptr(s), _ptr(x), _ptr(y),
                                                                       rows, cols, gs))
        return y

    def matvec_async(self, q_dev, s_dev, x_dev, y_dev, rows: int, cols: int, gs: int, stream=None) -> None:
        self._check("glm_cuda_matvec_q80_async",
                    self.L.glm_cuda_matvec_q80_async(_ptr(q_dev), _ptr(s_dev), _ptr(x_dev), _ptr(y_dev), rows,
                                                     cols, gs, stream))

    def synchronize(self) -> None:
        self._check("glm_cuda_synchronize", self.L.glm_cuda_synchronize())

    def route_stats(self) -> list[int]:
        out = (ctypes.c_uint64 * 4)()
        self._check("glm_cuda_route_stats", self.L.glm_cuda_route_stats(ctypes.addressof(out)))
        return list(out)

    def launch_count(self) -> int:
        return int(self.L.glm_cuda_launch_count())

    def free(self) -> None:
        self.L.glm_cuda_free()
