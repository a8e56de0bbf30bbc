"""Test infrastructure: write a synth.decoder_model as glm.c's runtime
checkpoint (.bin, format version 4 with every layer's attention), the layout
glm.c's runtime_open reads (infer.c:357-744; header RuntimeConfig,
model.h:7-45). The CPU tests check the file against glm.c's own loader; the
GPU tests load it with glm_cuda_load_checkpoint."""
import struct

import numpy as np

MAGIC, VERSION, HEADER = 0x67343763, 4, 256
GLOBAL_ORDER = ("output_norm", "tok_q", "tok_s", "out_q", "out_s")
L0_FFN_ORDER = ("l0_ffn_norm", "l0_gate_q", "l0_gate_s", "l0_up_q", "l0_up_s", "l0_down_q", "l0_down_s")
ATTN_ORDER = ("attn_norm", "q_a_norm", "kv_a_norm", "q_a_q", "q_a_s", "q_b_q", "q_b_s", "kv_a_q", "kv_a_s",
              "k_b_q", "k_b_s", "v_b_q", "v_b_s", "attn_out_q", "attn_out_s")
SHARED_ORDER = ("ffn_norm", "router", "router_bias", "gate_sh_q", "gate_sh_s", "up_sh_q", "up_sh_s",
                "down_sh_q", "down_sh_s")
ROUTED_ORDER = ("gate_q", "gate_s", "up_q", "up_s", "down_q", "down_s")


def write_runtime_bin(model: dict, path: str, seq_len: int = 64) -> int:
    d, g = model["dims"], model["globals"]
    blobs = [np.ascontiguousarray(g[k]).tobytes() for k in GLOBAL_ORDER + L0_FFN_ORDER]
    offs, o = [], HEADER
    for b in blobs:
        offs.append(o)
        o += len(b)
    body = list(blobs)
    attn0 = [np.ascontiguousarray(model["attn"][0][k]).tobytes() for k in ATTN_ORDER]
    body += attn0  # the layer-0 block of the v4 extension
    for a in model["attn"]:
        body += [np.ascontiguousarray(a[k]).tobytes() for k in ATTN_ORDER]
    for m in model["moe"][1:]:
        body += [np.ascontiguousarray(m[k]).tobytes() for k in SHARED_ORDER]
    for m in model["moe"][1:]:
        body += [np.ascontiguousarray(m[k]).tobytes() for k in ROUTED_ORDER]
    total = HEADER + sum(len(b) for b in body)
    hdr = struct.pack("<II", MAGIC, VERSION)
    hdr += struct.pack("<16i", d["dim"], d["hidden_dim"], d["n_layers"], d["n_heads"], d["n_heads"],
                       d["vocab_size"], seq_len, d["rope_dim"], d["q_lora_rank"], d["kv_lora_rank"],
                       d["kv_lora_rank"] + d["rope_dim"], d["n_routed_experts"], d["n_experts_used"], 1, -1, -1)
    hdr += struct.pack("<14Q", d["group_size"], offs[0], offs[1], offs[2], offs[3], offs[4], total, *offs[5:12])
    hdr += struct.pack("<5i", d["qk_nope_dim"], d["head_k_dim"], d["v_head_dim"], 1, d["moe_ffn_dim"])
    hdr += b"\0" * (HEADER - len(hdr))
    with open(path, "wb") as f:
        f.write(hdr)
        for b in body:
            f.write(b)
    return total
