"""Parity of the batched prefill path (exact batched routing, tcgen05 grouped
GEMMs over Q8 weights dequantised to bf16 pairs, rank-order combine) with
glm.c's CPU path, through the C-ABI (glm_cuda_moe_layer with n_tokens at or
above the glm_cuda_set_prefill_tokens threshold).

Bar (north star): expert ids bit-identical to the reference; MoE-layer output
within 1e-3 relative L2 of the reference (FFN delta x_out - x_in, per token).
"""
import numpy as np
import pytest

from helpers import assert_routing_exact, check_moe_outputs, routed_env

pytestmark = pytest.mark.gpu

TOL = 1e-3      # north-star relative L2 bound on the MoE-layer output
TOL_W = 1e-4    # normalised routing weights (absolute)
GOLDEN = ["moe_tiny_gs32", "moe_ties", "moe_near_ties", "moe_nonfinite", "moe_routed_off", "moe_all_experts",
          "moe_config0"]


@pytest.fixture(scope="module")
def lib(pkg):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    pkg.build.build()
    L = pkg.glm_cuda.GlmCuda()
    yield L
    L.free()


def run_prefill(lib, L, x, routed=True, min_tokens=1):
    lib.init(0, L["dim"], L["ffn"], L["n_experts"], L["k_used"], L["gs"], 1)
    lib.upload_moe_layer(0, L)
    assert lib.set_prefill_tokens(min_tokens) == 32  # the default threshold
    with routed_env(routed):
        return lib.moe_layer(0, x, L["k_used"])


def check(x, got, ref):
    x_out, idx, w = got
    x_ref, idx_ref, w_ref = ref
    np.testing.assert_array_equal(idx, idx_ref)
    valid = idx_ref >= 0
    np.testing.assert_allclose(w[valid], w_ref[valid], rtol=0, atol=TOL_W)
    return check_moe_outputs(x, x_out, x_ref, TOL)


@pytest.mark.parametrize("name", GOLDEN)
def test_prefill_matches_golden(name, lib, golden):
    L, x, routed, exp = golden.load_case(name)
    got = run_prefill(lib, L, x, routed)
    worst = check(x, got, (exp["x_out"], exp["topk_idx"], exp["topk_w"]))
    print(f"{name}: worst FFN-delta rel L2 {worst:.2e}")


def test_prefill_config3_zipf_512_tokens(lib, pkg, oracle_mod):
    """Config 3: 512 tokens through the config-0 layer with Zipf(1.1) expert
    popularity (uneven groups): ids bit-exact, outputs within 1e-3."""
    synth = pkg.synth
    L = synth.moe_layer(seed=3, zipf=1.1, **synth.CONFIG0)
    x = synth.tokens(3003, 512, 2048)
    got = run_prefill(lib, L, x, min_tokens=32)
    ref = oracle_mod.moe_layer(L, x, impl="orc")
    worst = check(x, got, ref)
    counts = np.bincount(ref[1].ravel(), minlength=64)
    print(f"config3: worst rel L2 {worst:.2e}; group sizes max {counts.max()} min {counts.min()}")
    assert counts.max() > 4 * max(counts.min(), 1)  # the groups really are uneven
    assert_routing_exact(lib)


@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 130])
def test_prefill_ragged_token_counts(T, lib, pkg, oracle_mod):
    """Token counts around the 64-row tile edge, including one token."""
    synth = pkg.synth
    cfg = dict(dim=512, ffn=256, n_experts=32, k_used=4, gs=32)
    L = synth.moe_layer(seed=11, zipf=1.1, **cfg)
    x = synth.tokens(1100 + T, T, 512)
    check(x, run_prefill(lib, L, x), oracle_mod.moe_layer(L, x, impl="orc"))


def test_prefill_many_experts_k8(lib, pkg, oracle_mod):
    """E = 256 routed experts (the group-table limit), top-8."""
    synth = pkg.synth
    cfg = dict(dim=256, ffn=128, n_experts=256, k_used=8, gs=32)
    L = synth.moe_layer(seed=12, **cfg)
    x = synth.tokens(12, 200, 256)
    check(x, run_prefill(lib, L, x), oracle_mod.moe_layer(L, x, impl="orc"))


def test_prefill_routed_off(lib, pkg, oracle_mod):
    synth = pkg.synth
    cfg = dict(dim=512, ffn=256, n_experts=32, k_used=4, gs=32)
    L = synth.moe_layer(seed=13, **cfg)
    x = synth.tokens(13, 70, 512)
    got = run_prefill(lib, L, x, routed=False)
    ref = oracle_mod.moe_layer(L, x, impl="orc", routed=False)
    check(x, got, ref)


def test_prefill_agrees_with_decode_kernels(lib, pkg):
    """Same ids as the per-token decode kernels; routing weights within 1e-4
    (both take the weight from their own estimate of the router logit, so
    they may differ in the last bit); x within 1e-4 relative."""
    synth = pkg.synth
    cfg = dict(dim=1024, ffn=512, n_experts=64, k_used=4, gs=32)
    L = synth.moe_layer(seed=14, zipf=1.1, **cfg)
    x = synth.tokens(14, 96, 1024)
    xp, ip, wp = run_prefill(lib, L, x, min_tokens=64)
    lib.set_prefill_tokens(0)
    xd, idd, wd = lib.moe_layer(0, x, 4)
    np.testing.assert_array_equal(ip, idd)
    np.testing.assert_allclose(wp, wd, rtol=0, atol=TOL_W)
    check_moe_outputs(x, xp, xd, 1e-4)


def test_prefill_device_entry_and_threshold(lib, pkg, oracle_mod):
    """glm_cuda_moe_layer_async on device memory takes the prefill path at the
    threshold and matches the oracle; below it the decode kernels run."""
    import torch

    synth = pkg.synth
    cfg = dict(dim=512, ffn=256, n_experts=32, k_used=4, gs=32)
    L = synth.moe_layer(seed=15, zipf=1.1, **cfg)
    x = synth.tokens(15, 48, 512)
    lib.init(0, 512, 256, 32, 4, 32, 1)
    lib.upload_moe_layer(0, L)
    assert lib.set_prefill_tokens(48) == 32
    assert lib.set_prefill_tokens(48) == 48
    before = lib.launch_count()
    xd = torch.from_numpy(x.copy()).cuda()
    idx_d = torch.zeros((48, 4), dtype=torch.int32, device="cuda")
    w_d = torch.zeros((48, 4), dtype=torch.float32, device="cuda")
    lib.moe_layer_async(0, xd, 48, idx_d, w_d)
    lib.synchronize()
    assert lib.launch_count() - before == 9  # one batched pass, not 48 per-token launches
    check(x, (xd.cpu().numpy(), idx_d.cpu().numpy(), w_d.cpu().numpy()), oracle_mod.moe_layer(L, x, impl="orc"))
