"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset or checkpoint is involved).

Every tensor comes from its own numpy PCG64 stream keyed by
(seed, layer, tensor id), so a tensor does not change when another tensor's
shape does, and the same call gives the same bytes on every machine with this
numpy. Distributions follow the configuration text:

  x            fp32 [T, D]        N(0, 1)
  router       fp32 [E, D]        N(0, 0.02)       (gate_inp, model.h:67)
  router_bias  fp32 [E]           N(0, 0.01)       (exp_probs_b, model.h:68)
  ffn_norm     fp32 [D]           1
  *_q          int8 [rows, cols]  uniform in [-127, 127]
  *_s          fp32 [rows, cols/gs]  |N(0, 0.02)| / 127   (one scale per group)

Routed expert blocks are expert-major: gate/up q [E, F, D], s [E, F, D/gs];
down q [E, D, F], s [E, D, F/gs] -- the planar layout of glm.c's checkpoint
(infer.c:697-742, glm47_flash_export.py:444-468).
"""
from __future__ import annotations

import hashlib

import numpy as np

# Pointer order shared by the C checkers and the CUDA upload call:
# LayerMoeShared fields (model.h:65-74) then LayerMoeRouted fields (model.h:76-83).
MOE_FIELDS = (
    "ffn_norm", "router", "router_bias",
    "gate_sh_q", "gate_sh_s", "up_sh_q", "up_sh_s", "down_sh_q", "down_sh_s",
    "gate_q", "gate_s", "up_q", "up_s", "down_q", "down_s",
)

_TENSOR_IDS = {name: i for i, name in enumerate(MOE_FIELDS)}
_TENSOR_IDS["x"] = 100
_TENSOR_IDS["matvec_q"] = 200
_TENSOR_IDS["matvec_s"] = 201
_TENSOR_IDS["matvec_x"] = 202

CONFIG0 = dict(dim=2048, ffn=1536, n_experts=64, k_used=4, gs=32)


def _rng(seed: int, layer: int, name: str) -> np.random.Generator:
    return np.random.default_rng([int(seed), int(layer), _TENSOR_IDS[name]])


def q8_weights(rng: np.random.Generator, rows: int, cols: int, gs: int, lead: tuple = ()):
    """int8 uniform [-127,127] and per-group fp32 scales |N(0,0.02)|/127."""
    q = rng.integers(-127, 128, size=lead + (rows, cols), dtype=np.int8)
    s = np.abs(rng.standard_normal(lead + (rows, cols // gs), dtype=np.float32))
    s *= np.float32(0.02)
    s /= np.float32(127.0)
    return q, s


def moe_layer(seed: int = 42, layer: int = 0, dim: int = 2048, ffn: int = 1536,
              n_experts: int = 64, k_used: int = 4, gs: int = 32, routed: bool = True) -> dict:
    """Weights of one MoE FFN layer (shared expert + routed experts + router)."""
    if dim % gs or ffn % gs:
        raise ValueError("dim and ffn must be multiples of the group size")
    L = dict(dim=dim, ffn=ffn, n_experts=n_experts, k_used=k_used, gs=gs)
    L["ffn_norm"] = np.ones(dim, dtype=np.float32)
    L["router"] = _rng(seed, layer, "router").standard_normal((n_experts, dim), dtype=np.float32) * np.float32(0.02)
    L["router_bias"] = _rng(seed, layer, "router_bias").standard_normal(n_experts, dtype=np.float32) * np.float32(0.01)
    for name, (rows, cols) in (("gate_sh", (ffn, dim)), ("up_sh", (ffn, dim)), ("down_sh", (dim, ffn))):
        L[name + "_q"], L[name + "_s"] = q8_weights(_rng(seed, layer, name + "_q"), rows, cols, gs)
    if routed:
        for name, (rows, cols) in (("gate", (ffn, dim)), ("up", (ffn, dim)), ("down", (dim, ffn))):
            L[name + "_q"], L[name + "_s"] = q8_weights(_rng(seed, layer, name + "_q"), rows, cols, gs, (n_experts,))
    else:
        for name in ("gate", "up", "down"):
            L[name + "_q"], L[name + "_s"] = None, None
    return L


def tokens(seed: int, n_tokens: int, dim: int, layer: int = 0) -> np.ndarray:
    """Decode/prefill activations x ~ N(0,1), fp32 [T, D]."""
    return _rng(seed, layer, "x").standard_normal((n_tokens, dim), dtype=np.float32)


def matvec_case(seed: int, rows: int, cols: int, gs: int = 32):
    """Config-1 matvec: Q8 weights as in config 0 and x ~ N(0,1)."""
    q, s = q8_weights(_rng(seed, 0, "matvec_q"), rows, cols, gs)
    x = _rng(seed, 0, "matvec_x").standard_normal(cols, dtype=np.float32)
    return q, s, x


def moe_bytes(dim: int, ffn: int, n_experts: int, k_used: int, gs: int) -> int:
    """Algorithmic HBM bytes of one decode token through one MoE layer:
    (K routed + 1 shared) x 3 Q8 matrices + fp32 router [E,D] + bias [E]
    + x read, x written, ffn_norm read (q80_bytes of infer.c:1464-1470)."""
    q8 = lambda r, c: r * c + r * (c // gs) * 4
    experts = (k_used + 1) * (2 * q8(ffn, dim) + q8(dim, ffn))
    return experts + n_experts * dim * 4 + n_experts * 4 + 3 * dim * 4


def q8_matvec_bytes(rows: int, cols: int, gs: int) -> int:
    """R*C*(1+4/gs) weight bytes + fp32 x read + fp32 y written."""
    return rows * cols + rows * (cols // gs) * 4 + 4 * (rows + cols)


def digest(arrays) -> str:
    """sha256 over the raw bytes of the given arrays (fixture drift check)."""
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()
