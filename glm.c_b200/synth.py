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

# Full GLM-4.7-Flash-shaped decoder: field names of
# GlmCudaModelDims / RuntimeConfig (model.h:7-45).
CONFIG2 = dict(dim=2048, hidden_dim=10240, n_layers=47, n_heads=20, vocab_size=154880, rope_dim=64,
               q_lora_rank=768, kv_lora_rank=512, qk_nope_dim=192, head_k_dim=256, v_head_dim=256,
               n_routed_experts=64, n_experts_used=4, group_size=32, moe_ffn_dim=1536)

# Pointer orders of the decoder tables (C harness and CUDA upload calls):
# Runtime globals (model.h:87-103) and LayerAttnWeights (model.h:46-62).
GLOBAL_FIELDS = ("output_norm", "tok_q", "tok_s", "out_q", "out_s", "l0_ffn_norm", "l0_gate_q", "l0_gate_s",
                 "l0_up_q", "l0_up_s", "l0_down_q", "l0_down_s")
ATTN_FIELDS = ("attn_norm", "q_a_norm", "kv_a_norm", "q_a_q", "q_a_s", "q_b_q", "q_b_s", "kv_a_q", "kv_a_s",
               "k_b_q", "k_b_s", "v_b_q", "v_b_s", "attn_out_q", "attn_out_s")
for _i, _n in enumerate(GLOBAL_FIELDS + ATTN_FIELDS + ("prompt",)):
    _TENSOR_IDS.setdefault(_n, 300 + _i)


def _rng(seed: int, layer: int, name: str) -> np.random.Generator:
    return np.random.default_rng([int(seed), int(layer), _TENSOR_IDS[name]])


def q8_weights(rng: np.random.Generator, rows: int, cols: int, gs: int, lead: tuple = ()):
    """int8 uniform [-127,127] and per-group fp32 scales |N(0,0.02)|/127."""
    q = rng.integers(-127, 128, size=lead + (rows, cols), dtype=np.int8)
    s = np.abs(rng.standard_normal(lead + (rows, cols // gs), dtype=np.float32))
    s *= np.float32(0.02)
    s /= np.float32(127.0)
    return q, s


# Router-bias scale of zipf_bias: with N(0,1) tokens, N(0,0.02) router rows,
# D = 2048, E = 64 and K = 4, bias_e = -ZIPF_BETA * ln(rank_e) makes the
# expert pick counts fall off as rank^-1.1 (least-squares log-log slope over
# 4096 tokens: -1.100).
ZIPF_BETA = 0.0885


def zipf_bias(seed: int, layer: int, n_experts: int, s: float = 1.1) -> np.ndarray:
    """Router bias giving Zipf(s)-like expert popularity (configs 3 and 4):
    each expert gets a popularity rank from a seeded permutation and
    bias = -ZIPF_BETA * (s / 1.1) * ln(rank)."""
    rank = _rng(seed, layer, "router_bias").permutation(n_experts) + 1
    return (-(ZIPF_BETA * s / 1.1) * np.log(rank)).astype(np.float32)


def moe_layer(seed: int = 42, layer: int = 0, dim: int = 2048, ffn: int = 1536,
              n_experts: int = 64, k_used: int = 4, gs: int = 32, routed: bool = True,
              zipf: float | None = None) -> dict:
    """Weights of one MoE FFN layer (shared expert + routed experts + router).
    zipf=s draws the router bias with zipf_bias instead of N(0, 0.01)."""
    if dim % gs or ffn % gs:
        raise ValueError("dim and ffn must be multiples of the group size")
    L = dict(dim=dim, ffn=ffn, n_experts=n_experts, k_used=k_used, gs=gs)
    L["ffn_norm"] = np.ones(dim, dtype=np.float32)
    L["router"] = _rng(seed, layer, "router").standard_normal((n_experts, dim), dtype=np.float32) * np.float32(0.02)
    if zipf is None:
        L["router_bias"] = (_rng(seed, layer, "router_bias").standard_normal(n_experts, dtype=np.float32)
                            * np.float32(0.01))
    else:
        L["router_bias"] = zipf_bias(seed, layer, n_experts, zipf)
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


def decoder_model(seed: int = 42, moe_layers: list | None = None, **dims) -> dict:
    """Weights of a full decoder with the given GlmCudaModelDims fields:
    Q8 linear layers as in config 0, all norms 1; layers 1.. are MoE layers
    of moe_layer(seed, layer), or the prebuilt `moe_layers` (one per layer
    1..n_layers-1) when given. Returns {"dims", "globals", "attn": [..],
    "moe": [None, ..]}."""
    d = dict(dims)
    D, gs, H = d["dim"], d["group_size"], d["n_heads"]
    g = {"output_norm": np.ones(D, np.float32), "l0_ffn_norm": np.ones(D, np.float32)}
    g["tok_q"], g["tok_s"] = q8_weights(_rng(seed, 0, "tok_q"), d["vocab_size"], D, gs)
    g["out_q"], g["out_s"] = q8_weights(_rng(seed, 0, "out_q"), d["vocab_size"], D, gs)
    for name, (rows, cols) in (("l0_gate", (d["hidden_dim"], D)), ("l0_up", (d["hidden_dim"], D)),
                               ("l0_down", (D, d["hidden_dim"]))):
        g[name + "_q"], g[name + "_s"] = q8_weights(_rng(seed, 0, name + "_q"), rows, cols, gs)
    attn = []
    for l in range(d["n_layers"]):
        a = {"attn_norm": np.ones(D, np.float32), "q_a_norm": np.ones(d["q_lora_rank"], np.float32),
             "kv_a_norm": np.ones(d["kv_lora_rank"], np.float32)}
        shapes = {"q_a": ((d["q_lora_rank"], D), ()),
                  "q_b": ((H * d["head_k_dim"], d["q_lora_rank"]), ()),
                  "kv_a": ((d["kv_lora_rank"] + d["rope_dim"], D), ()),
                  "k_b": ((d["kv_lora_rank"], d["qk_nope_dim"]), (H,)),
                  "v_b": ((d["v_head_dim"], d["kv_lora_rank"]), (H,)),
                  "attn_out": ((D, H * d["v_head_dim"]), ())}
        for name, ((rows, cols), lead) in shapes.items():
            a[name + "_q"], a[name + "_s"] = q8_weights(_rng(seed, l, name + "_q"), rows, cols, gs, lead)
        attn.append(a)
    if moe_layers is not None:
        assert len(moe_layers) == d["n_layers"] - 1
        moe = [None] + list(moe_layers)
    else:
        moe = [None] + [moe_layer(seed, l, D, d["moe_ffn_dim"], d["n_routed_experts"], d["n_experts_used"], gs)
                        for l in range(1, d["n_layers"])]
    return {"dims": d, "globals": g, "attn": attn, "moe": moe}


def rolled_moe_layer(base: dict, shift: int) -> dict:
    """A layer with distinct memory and different (still config-0
    distributed) weights, made cheaply from `base`: the routed experts, the
    router rows and the bias rotated by `shift` along the expert axis, and
    the shared expert's rows rotated by `shift`. Used where many distinct
    layers must sit in host memory and generating each one afresh would take
    seconds (CPU baselines)."""
    L = {k: v for k, v in base.items() if not isinstance(v, np.ndarray)}
    for k, v in base.items():
        if isinstance(v, np.ndarray):
            L[k] = v.copy() if k == "ffn_norm" else np.roll(v, shift, axis=0)
    return L


def prompt_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    """Prompt token ids uniform in [0, vocab)."""
    return _rng(seed, 0, "prompt").integers(0, vocab, size=n, dtype=np.int32)


def digest(arrays) -> str:
    """sha256 over the raw bytes of the given arrays (fixture drift check)."""
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()
