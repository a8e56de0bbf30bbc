"""Parity of the CUDA MoE decode path (through the C-ABI) with glm.c's CPU path.

Bar (north star): expert ids bit-identical to the reference; MoE-layer output
within 1e-3 relative L2 of the reference, measured on the FFN delta
x_out - x_in. The expected values are the golden fixtures produced by the
compiled reference, or the CPU oracle pinned to it.
"""
import numpy as np
import pytest

from helpers import check_moe_outputs, routed_env

pytestmark = pytest.mark.gpu

TOL = 1e-3          # north-star relative L2 bound on the MoE-layer output
TOL_W = 1e-4        # normalised routing weights (absolute)
GPU_CASES = ["moe_tiny_gs32", "moe_ties", "moe_near_ties", "moe_nonfinite", "moe_routed_off",
             "moe_all_experts", "moe_config0"]


@pytest.fixture(scope="module")
def lib(pkg):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    pkg.build.build()
    L = pkg.glm_cuda.GlmCuda()
    yield L
    L.free()


PATHS = {"persistent": 1, "chain": 2}


def run_layer(lib, L, x, routed=True, path="persistent"):
    lib.init(0, L["dim"], L["ffn"], L["n_experts"], L["k_used"], L["gs"], 1)
    lib.upload_moe_layer(0, L)
    lib.set_prefill_tokens(0)  # per-token decode kernels at every n_tokens
    lib.set_decode_path(PATHS[path])
    assert lib.decode_path() == PATHS[path]
    with routed_env(routed):
        return lib.moe_layer(0, x, L["k_used"])


@pytest.mark.parametrize("path", sorted(PATHS))
@pytest.mark.parametrize("name", GPU_CASES)
def test_moe_decode_matches_golden(name, path, lib, golden):
    L, x, routed, exp = golden.load_case(name)
    x_out, idx, w = run_layer(lib, L, x, routed, path)
    np.testing.assert_array_equal(idx, exp["topk_idx"])
    valid = exp["topk_idx"] >= 0
    np.testing.assert_allclose(w[valid], exp["topk_w"][valid], rtol=0, atol=TOL_W)
    worst = check_moe_outputs(x, x_out, exp["x_out"], TOL)
    print(f"{name}: worst FFN-delta rel L2 {worst:.2e}")


@pytest.mark.parametrize("batched", [False, True])
def test_moe_gs16_golden(batched, lib, golden):
    """gs = 16 (glm.c's own export): per-token calls take the persistent
    kernel (16-column scale groups on the integer MMA); with the prefill
    threshold at 1 every call takes the batched kernels. Both as glm.c's."""
    L, x, routed, exp = golden.load_case("moe_tiny_gs16")
    lib.init(0, L["dim"], L["ffn"], L["n_experts"], L["k_used"], L["gs"], 1)
    lib.upload_moe_layer(0, L)
    assert lib.decode_path() == lib.PATH_PERSISTENT
    lib.set_prefill_tokens(1 if batched else 0)
    with routed_env(routed):
        x_out, idx, w = lib.moe_layer(0, x, L["k_used"])
    np.testing.assert_array_equal(idx, exp["topk_idx"])
    valid = exp["topk_idx"] >= 0
    np.testing.assert_allclose(w[valid], exp["topk_w"][valid], rtol=0, atol=TOL_W)
    check_moe_outputs(x, x_out, exp["x_out"], TOL)


def test_moe_gs16_refuses_the_chain(lib, golden):
    import glm_c_b200.glm_cuda as gc

    L, _, _, _ = golden.load_case("moe_tiny_gs16")
    lib.init(0, L["dim"], L["ffn"], L["n_experts"], L["k_used"], L["gs"], 1)
    with pytest.raises(gc.GlmCudaError):
        lib.set_decode_path(PATHS["chain"])


def test_auto_path_is_persistent_at_config0(lib, pkg):
    c = pkg.synth.CONFIG0
    lib.init(0, c["dim"], c["ffn"], c["n_experts"], c["k_used"], c["gs"], 2)
    assert lib.decode_path() == lib.PATH_PERSISTENT


@pytest.mark.parametrize("path", sorted(PATHS))
def test_moe_config0_routing_256_tokens(path, lib, pkg, oracle_mod):
    """256 decode tokens through the config-0 layer: every expert id equals the
    oracle's (pinned to the compiled reference), outputs within 1e-3."""
    synth = pkg.synth
    L = synth.moe_layer(seed=42, **synth.CONFIG0)
    x = synth.tokens(4242, 256, 2048)
    x_out, idx, w = run_layer(lib, L, x, path=path)
    x_ref, idx_ref, w_ref = oracle_mod.moe_layer(L, x, impl="orc")
    np.testing.assert_array_equal(idx, idx_ref)
    np.testing.assert_allclose(w, w_ref, rtol=0, atol=TOL_W)
    worst = check_moe_outputs(x, x_out, x_ref, TOL)
    stats = lib.route_stats()
    print(f"config0 x256: worst rel L2 {worst:.2e}, route stats {stats}")
    assert stats[0] >= 256 and stats[2] == 0


def test_moe_device_path_matches_host_path(lib, pkg):
    """Weights bound from caller-owned device memory, x on the device, the
    stream-ordered entry point: identical results to the host entry point."""
    import torch

    synth = pkg.synth
    cfg = dict(dim=512, ffn=256, n_experts=32, k_used=4, gs=32)
    L = synth.moe_layer(seed=9, **cfg)
    x = synth.tokens(9, 5, 512)
    x_host, idx_host, w_host = run_layer(lib, L, x)

    lib.init(0, 512, 256, 32, 4, 32, 2)
    dev = {k: torch.from_numpy(np.ascontiguousarray(L[k])).cuda() for k in synth.MOE_FIELDS}
    lib.bind_moe_layer_device(1, dev)
    xd = torch.from_numpy(x).cuda()
    idx_d = torch.zeros((5, 4), dtype=torch.int32, device="cuda")
    w_d = torch.zeros((5, 4), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()
    lib.moe_layer_async(1, xd, 5, idx_d, w_d, stream=s.cuda_stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(idx_d.cpu().numpy(), idx_host)
    np.testing.assert_array_equal(xd.cpu().numpy(), x_host)
    np.testing.assert_array_equal(w_d.cpu().numpy(), w_host)
    del dev


def test_moe_two_layers_in_sequence(lib, pkg, oracle_mod):
    synth = pkg.synth
    cfg = dict(dim=256, ffn=128, n_experts=16, k_used=4, gs=32)
    L1 = synth.moe_layer(seed=21, layer=1, **cfg)
    L2 = synth.moe_layer(seed=21, layer=2, **cfg)
    x = synth.tokens(21, 3, 256)
    lib.init(0, 256, 128, 16, 4, 32, 3)
    lib.upload_moe_layer(1, L1)
    lib.upload_moe_layer(2, L2)
    y, i1, _ = lib.moe_layer(1, x, 4)
    y, i2, _ = lib.moe_layer(2, y, 4)
    r, j1, _ = oracle_mod.moe_layer(L1, x, impl="orc")
    r, j2, _ = oracle_mod.moe_layer(L2, r, impl="orc")
    np.testing.assert_array_equal(i1, j1)
    np.testing.assert_array_equal(i2, j2)
    check_moe_outputs(x, y, r, TOL)


@pytest.mark.parametrize("cfg", [dict(dim=512, ffn=256, n_experts=32, k_used=4, gs=32),
                                 dict(dim=2048, ffn=1536, n_experts=64, k_used=4, gs=32)])
def test_moe_layer_stack_one_launch(cfg, lib, pkg, oracle_mod):
    """glm_cuda_moe_layers_async: one token through a stack of MoE layers in
    one persistent launch equals the oracle applied layer by layer (expert
    ids bit-exact per layer, output within 1e-3)."""
    import torch

    synth = pkg.synth
    n = 4 if cfg["dim"] < 2048 else 2
    layers = [synth.moe_layer(seed=31, layer=l, **cfg) for l in range(1, n + 1)]
    x = synth.tokens(31, 1, cfg["dim"])
    lib.init(0, cfg["dim"], cfg["ffn"], cfg["n_experts"], cfg["k_used"], cfg["gs"], n + 1)
    for l, L in enumerate(layers, start=1):
        lib.upload_moe_layer(l, L)
    xd = torch.from_numpy(x.copy()).cuda()
    idx_d = torch.full((n, cfg["k_used"]), -7, dtype=torch.int32, device="cuda")
    w_d = torch.zeros((n, cfg["k_used"]), dtype=torch.float32, device="cuda")
    lib.moe_layers_async(1, n, xd, idx_d, w_d)
    lib.synchronize()
    r = x
    for l, L in enumerate(layers):
        r, j, wr = oracle_mod.moe_layer(L, r, impl="orc")
        np.testing.assert_array_equal(idx_d[l].cpu().numpy(), j[0])
        np.testing.assert_allclose(w_d[l].cpu().numpy(), wr[0], rtol=0, atol=TOL_W)
    check_moe_outputs(x, xd.cpu().numpy(), r, TOL)


def test_moe_layer_not_uploaded_is_an_error(lib):
    import glm_c_b200.glm_cuda as gc

    lib.init(0, 256, 128, 16, 4, 32, 2)
    with pytest.raises(gc.GlmCudaError) as e:
        lib.moe_layer(1, np.zeros((1, 256), np.float32), 4)
    assert e.value.rc == -2
