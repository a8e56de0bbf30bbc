"""Golden fixtures for the MoE FFN hot path, produced by glm.c's OWN code.

Every expected output here comes from the reference C implementation compiled
from its sources (oracle/_ref/libglmref.so, built by oracle/Makefile from the
reference checkout), called on seeded synthetic inputs. The fixtures store the
reference's outputs and a sha256 digest of the inputs; the inputs themselves
are rebuilt by the functions in CASES (seeded numpy PCG64, plus the crafted
edits below), and tests refuse to compare if the rebuilt inputs' digest
differs from the recorded one.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from __graft_entry__ import load_package  # noqa: E402

synth = load_package().synth

TINY = dict(dim=256, ffn=128, n_experts=16, k_used=4, gs=32)


def _tiny_gs32():
    return synth.moe_layer(seed=1, **TINY), synth.tokens(1, 6, 256), True


def _tiny_gs16():
    return synth.moe_layer(seed=2, dim=256, ffn=128, n_experts=16, k_used=4, gs=16), synth.tokens(2, 3, 256), True


def _ties():
    """Five experts with identical router rows and biases straddling the top-4
    boundary: the reference keeps the four lowest ids (strict '>' at
    infer.c:1123)."""
    L = synth.moe_layer(seed=7, **TINY)
    x = synth.tokens(7, 4, 256)
    r, b = L["router"].copy(), L["router_bias"].copy()
    base = (np.sign(x[0]) * np.float32(0.01)).astype(np.float32)  # strongly selected by token 0
    for e in (2, 5, 6, 12, 14):
        r[e] = base
        b[e] = np.float32(0.005)
    L["router"], L["router_bias"] = r, b
    return L, x, True


def _near_ties():
    """Experts 3, 9, 10, 11 share a router row except for a one-ulp change in
    one weight of 9 (up) and 10 (down): their fp32 logits differ in the last
    bits only, below any fast error bound, so only the reference's own serial
    order ranks them."""
    L = synth.moe_layer(seed=8, **TINY)
    x = synth.tokens(8, 4, 256)
    r, b = L["router"].copy(), L["router_bias"].copy()
    base = (np.sign(x[0]) * np.float32(0.01)).astype(np.float32)
    for e in (3, 9, 10, 11):
        r[e] = base
    r[9, 17] = np.nextafter(r[9, 17], np.float32(1.0))
    r[10, 40] = np.nextafter(r[10, 40], np.float32(-1.0))
    b[3] = b[9] = b[10] = b[11] = np.float32(0.001)
    L["router"], L["router_bias"] = r, b
    return L, x, True


def _nonfinite():
    x = synth.tokens(3, 4, 256)
    x[1, 5] = np.nan
    x[2, 9] = np.inf
    x[3, :] = 0.0
    return synth.moe_layer(seed=3, **TINY), x, True


def _routed_off():
    return synth.moe_layer(seed=4, **TINY), synth.tokens(4, 2, 256), False


def _all_experts():
    return synth.moe_layer(seed=5, dim=256, ffn=128, n_experts=8, k_used=8, gs=32), synth.tokens(5, 2, 256), True


def _config0():
    return synth.moe_layer(seed=42, **synth.CONFIG0), synth.tokens(42, 8, 2048), True


# name -> (builder, note)
CASES = {
    "moe_tiny_gs32": (_tiny_gs32, "small seeded layer, 6 tokens"),
    "moe_tiny_gs16": (_tiny_gs16, "gs=16 as glm.c's real export"),
    "moe_ties": (_ties, "exact sel ties at the top-4 boundary"),
    "moe_near_ties": (_near_ties, "logits one rounding apart"),
    "moe_nonfinite": (_nonfinite, "NaN, inf and all-zero tokens"),
    "moe_routed_off": (_routed_off, "GLM_DISABLE_MOE_ROUTED=1"),
    "moe_all_experts": (_all_experts, "K == E"),
    "moe_config0": (_config0, "BASELINE config 0 shape, seed 42, 8 decode tokens"),
}

MATVEC_SHAPES = ((1536, 2048), (2048, 1536), (4608, 2048), (154880, 2048))
MATVEC_SEED = 11


def input_digest(L: dict, x: np.ndarray) -> str:
    return synth.digest([x] + [L[k] for k in synth.MOE_FIELDS if L.get(k) is not None])


def load_case(name: str):
    """(layer, x, routed, expected dict) with the input digest verified."""
    L, x, routed = CASES[name][0]()
    z = np.load(os.path.join(HERE, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    got = input_digest(L, x)
    if got != meta["digest"]:
        raise AssertionError(f"{name}: regenerated inputs differ from the fixture's (digest {got[:12]} vs "
                             f"{meta['digest'][:12]}); the generator changed")
    return L, x, routed, {k: z[k] for k in ("x_out", "topk_idx", "topk_w")}


def load_matvec(rows: int, cols: int):
    q, s, x = synth.matvec_case(MATVEC_SEED, rows, cols, 32)
    z = np.load(os.path.join(HERE, "matvec_config1.npz"))
    if synth.digest([q, s, x]) != str(z[f"digest_{rows}x{cols}"]):
        raise AssertionError(f"matvec {rows}x{cols}: regenerated inputs differ from the fixture's")
    return q, s, x, z[f"y_{rows}x{cols}"], float(z[f"sum_{rows}x{cols}"])


def main() -> None:
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    oracle.build()
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref/libglmref.so missing: the reference sources are needed to regenerate")
    for name, (fn, note) in CASES.items():
        L, x, routed = fn()
        x_out, idx, w = oracle.moe_layer(L, x, impl="ref", routed=routed)
        meta = {k: L[k] for k in ("dim", "ffn", "n_experts", "k_used", "gs")}
        meta.update(routed=routed, note=note, digest=input_digest(L, x))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), meta=json.dumps(meta), x_out=x_out,
                            topk_idx=idx, topk_w=w)
        print(f"{name}: idx[0]={idx[0].tolist()}")
    out = {}
    for rows, cols in MATVEC_SHAPES:
        q, s, xv = synth.matvec_case(MATVEC_SEED, rows, cols, 32)
        y = oracle.matvec(q, s, xv, 32, impl="ref")
        out[f"y_{rows}x{cols}"] = y if rows < 100000 else y[:4096]
        out[f"sum_{rows}x{cols}"] = np.float64(y.astype(np.float64).sum())
        out[f"digest_{rows}x{cols}"] = synth.digest([q, s, xv])
        print(f"matvec {rows}x{cols} done")
    np.savez_compressed(os.path.join(HERE, "matvec_config1.npz"), **out)


if __name__ == "__main__":
    main()
