"""glm_cuda_moe_layer_noalloc, the MoE decode layer for callers that may not
allocate device memory.

Who needs it: a process that plans all of its GPU memory at start-up and
forbids allocation once it serves (an inference server whose request path may
not call cudaMalloc: that call can block on the device, fragment a pool sized
at start-up, or fail under memory pressure in the middle of a request), or an
embedder that hands this library only buffers it already owns. The entry
point keeps its scratch in a fixed static device array instead.

These tests drive it through the C-ABI, on two calls in a row (the second
reuses whatever the first left in the static array). They check it against
the allocating entry point on the same device-resident weights and inputs,
and against the CPU oracle, which is pinned to glm.c: expert ids
bit-identical, routing weights within 1e-4, outputs within the MoE tolerance.
One case runs at the largest sizes the static array admits. Every test sets
up what it needs itself, so the file passes alone in a fresh process and
after the other tests; its name makes pytest collect it last.
"""
import numpy as np
import pytest

from helpers import check_moe_outputs

pytestmark = pytest.mark.gpu

TOL = 1e-3    # same MoE-output bound as tests/test_moe_gpu.py
TOL_W = 1e-4  # normalised routing weights (absolute), as tests/test_moe_gpu.py


def _noalloc(lib, torch, dev, cfg, xh, n):
    xd = torch.from_numpy(xh.copy()).cuda()
    idx = torch.full((n, cfg["k_used"]), -7, dtype=torch.int32, device="cuda")
    w = torch.zeros((n, cfg["k_used"]), dtype=torch.float32, device="cuda")
    lib.moe_layer_noalloc(dev, cfg["dim"], cfg["ffn"], cfg["n_experts"], cfg["k_used"], cfg["gs"], xd, n, idx, w,
                          stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return xd.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()


def test_noalloc_matches_allocating_entry_point_and_oracle_twice(pkg, oracle_mod):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    pkg.build.build()
    synth = pkg.synth
    cfg = dict(dim=1024, ffn=512, n_experts=32, k_used=4, gs=32)
    L = synth.moe_layer(seed=77, **cfg)
    dev = {k: torch.from_numpy(np.ascontiguousarray(L[k])).cuda() for k in synth.MOE_FIELDS}
    x_host = [synth.tokens(77, 3, cfg["dim"]), synth.tokens(78, 3, cfg["dim"])]

    lib = pkg.glm_cuda.GlmCuda()
    # Results of the allocating entry point.
    lib.init(0, cfg["dim"], cfg["ffn"], cfg["n_experts"], cfg["k_used"], cfg["gs"], 1)
    lib.bind_moe_layer_device(0, dev)
    expect = []
    for xh in x_host:
        xd = torch.from_numpy(xh.copy()).cuda()
        idx = torch.zeros((3, 4), dtype=torch.int32, device="cuda")
        w = torch.zeros((3, 4), dtype=torch.float32, device="cuda")
        lib.moe_layer_async(0, xd, 3, idx, w, stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        expect.append((xd.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()))
    lib.free()

    # Two no-alloc calls in a row, no glm_cuda_init.
    for call, xh in enumerate(x_host):
        x_out, idx, w = _noalloc(lib, torch, dev, cfg, xh, 3)
        x_alloc, idx_alloc, w_alloc = expect[call]
        x_ref, idx_ref, w_ref = oracle_mod.moe_layer(L, xh, impl="orc")
        np.testing.assert_array_equal(idx, idx_alloc)
        np.testing.assert_array_equal(idx, idx_ref)
        np.testing.assert_allclose(w, w_alloc, rtol=0, atol=TOL_W)
        np.testing.assert_allclose(w, w_ref, rtol=0, atol=TOL_W)
        check_moe_outputs(xh, x_out, x_alloc, TOL)
        check_moe_outputs(xh, x_out, x_ref, TOL)


def test_noalloc_at_its_maximum_sizes(pkg, oracle_mod):
    """dim = moe_ffn_dim = 4096, 256 experts, top-8: every region of the static
    array at its largest extent; two calls against the oracle. The weights
    (14.5 GB) are generated on the device with the config-0 distributions."""
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    pkg.build.build()
    cfg = dict(dim=4096, ffn=4096, n_experts=256, k_used=8, gs=32)
    D, F, E, gs = cfg["dim"], cfg["ffn"], cfg["n_experts"], cfg["gs"]
    g = torch.Generator(device="cuda")
    g.manual_seed(4096)

    def q8(lead, rows, cols):
        q = torch.randint(-127, 128, lead + (rows, cols), generator=g, device="cuda", dtype=torch.int8)
        s = torch.randn(lead + (rows, cols // gs), generator=g, device="cuda").abs_().mul_(0.02 / 127.0)
        return q, s

    dev = {"ffn_norm": torch.ones(D, device="cuda"),
           "router": torch.randn(E, D, generator=g, device="cuda").mul_(0.02),
           "router_bias": torch.randn(E, generator=g, device="cuda").mul_(0.01)}
    dev["gate_sh_q"], dev["gate_sh_s"] = q8((), F, D)
    dev["up_sh_q"], dev["up_sh_s"] = q8((), F, D)
    dev["down_sh_q"], dev["down_sh_s"] = q8((), D, F)
    dev["gate_q"], dev["gate_s"] = q8((E,), F, D)
    dev["up_q"], dev["up_s"] = q8((E,), F, D)
    dev["down_q"], dev["down_s"] = q8((E,), D, F)
    host = {k: v.cpu().numpy() for k, v in dev.items()}
    host.update(cfg)
    lib = pkg.glm_cuda.GlmCuda()
    try:
        for call in range(2):
            xh = pkg.synth.tokens(4096 + call, 2, D)
            x_out, idx, w = _noalloc(lib, torch, dev, cfg, xh, 2)
            x_ref, idx_ref, w_ref = oracle_mod.moe_layer(host, xh, impl="orc")
            np.testing.assert_array_equal(idx, idx_ref)
            np.testing.assert_allclose(w, w_ref, rtol=0, atol=TOL_W)
            check_moe_outputs(xh, x_out, x_ref, TOL)
    finally:
        del dev, host
        torch.cuda.empty_cache()


def test_noalloc_rejects_sizes_above_its_static_scratch(pkg):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    lib = pkg.glm_cuda.GlmCuda()
    x = torch.zeros(8192, device="cuda")
    with pytest.raises(pkg.glm_cuda.GlmCudaError) as e:
        lib.moe_layer_noalloc({}, 8192, 1536, 64, 4, 32, x, 1)
    assert e.value.rc == -1 and "static scratch limit" in str(e.value)
