"""glm.c with the `cuda` backend of INTEGRATION.md, built from its own sources
(oracle/glm_cuda_patch.py): glm_cpu_forward_token's greedy loop runs with
glm_backend_init(BACKEND_CUDA), so every MoE layer goes through the
library's MoE hook and every Q8 matvec (attention, dense layer, LM head)
through its matvec hook. The greedy ids equal those of the unpatched CPU
build; the logits agree within 1e-3 (and differ in the last bits, which shows
that the device ran them)."""
import numpy as np
import pytest

from helpers import rel_l2

pytestmark = pytest.mark.gpu

TOL_LOGITS = 1e-3
SMALL = dict(dim=256, hidden_dim=512, n_layers=3, n_heads=4, vocab_size=1000, rope_dim=64, q_lora_rank=128,
             kv_lora_rank=128, qk_nope_dim=64, head_k_dim=128, v_head_dim=64, n_routed_experts=16,
             n_experts_used=4, group_size=32, moe_ffn_dim=128)


@pytest.fixture(scope="module")
def oracle_cuda(pkg, oracle_mod):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import os

    if not os.path.exists(oracle_mod.REF_CUDA_SO):
        pytest.skip("the cuda-patched glm.c was not built (needs glm.c's sources at build time)")
    pkg.build.build()
    yield oracle_mod
    pkg.glm_cuda.GlmCuda().free()


@pytest.mark.parametrize("dims, n_prompt, n_gen, seed", [(SMALL, 8, 16, 11), ("config2x3", 16, 8, 42)])
def test_patched_backend_greedy_matches_cpu_build(dims, n_prompt, n_gen, seed, pkg, oracle_cuda):
    synth = pkg.synth
    if dims == "config2x3":  # GLM-4.7-Flash shapes, 3 layers
        dims = dict(synth.CONFIG2, n_layers=3)
    model = synth.decoder_model(seed, **dims)
    prompt = synth.prompt_ids(seed, n_prompt, dims["vocab_size"])
    cap = n_prompt + n_gen + 8
    ids_cpu, logits_cpu = oracle_cuda.ref_decode(model, prompt, n_gen, cap, with_logits=True)
    ids_cuda, logits_cuda = oracle_cuda.ref_decode(model, prompt, n_gen, cap, with_logits=True, impl="refcuda")
    np.testing.assert_array_equal(ids_cuda, ids_cpu)
    worst = max(rel_l2(logits_cuda[g], logits_cpu[g], logits_cpu[g]) for g in range(n_gen))
    print(f"patched glm.c --backend cuda: ids {ids_cuda[:8].tolist()}, worst logits rel L2 {worst:.2e}")
    assert worst <= TOL_LOGITS
    assert not np.array_equal(logits_cuda, logits_cpu)  # the device path ran
