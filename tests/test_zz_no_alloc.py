"""glm_cuda_moe_layer_noalloc against the allocating entry point.

The no-alloc entry point exists for callers that may not allocate device
memory when they call the library (a server that sizes all GPU memory at
start-up and forbids cudaMalloc on the request path, or an embedder that only
passes pointers it owns); its scratch is a static device array. This test
drives both entry points through the C-ABI on the same device-resident
weights and inputs and requires the same expert ids and outputs within the
MoE tolerance, on two calls in a row (the second call reuses the static
array the first one left behind). It sets up everything it needs itself, so
it passes alone in a fresh process and after the other tests; the file name
makes pytest collect it last.
"""
import numpy as np
import pytest

from helpers import check_moe_outputs

pytestmark = pytest.mark.gpu

TOL = 1e-3  # same MoE-output bound as tests/test_moe_gpu.py


def test_noalloc_matches_allocating_entry_point_twice(pkg):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    pkg.build.build()
    synth = pkg.synth
    cfg = dict(dim=1024, ffn=512, n_experts=32, k_used=4, gs=32)
    L = synth.moe_layer(seed=77, **cfg)
    dev = {k: torch.from_numpy(np.ascontiguousarray(L[k])).cuda() for k in synth.MOE_FIELDS}
    x_host = [synth.tokens(77, 3, cfg["dim"]), synth.tokens(78, 3, cfg["dim"])]

    lib = pkg.glm_cuda.GlmCuda()
    # Reference results from the allocating entry point.
    lib.init(0, cfg["dim"], cfg["ffn"], cfg["n_experts"], cfg["k_used"], cfg["gs"], 1)
    lib.bind_moe_layer_device(0, dev)
    expect = []
    for xh in x_host:
        xd = torch.from_numpy(xh.copy()).cuda()
        idx = torch.zeros((3, 4), dtype=torch.int32, device="cuda")
        lib.moe_layer_async(0, xd, 3, idx, None, stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        expect.append((xd.cpu().numpy(), idx.cpu().numpy()))
    lib.free()

    # Two no-alloc calls in a row, no glm_cuda_init.
    for call, xh in enumerate(x_host):
        xd = torch.from_numpy(xh.copy()).cuda()
        idx = torch.full((3, 4), -7, dtype=torch.int32, device="cuda")
        w = torch.zeros((3, 4), dtype=torch.float32, device="cuda")
        lib.moe_layer_noalloc(dev, cfg["dim"], cfg["ffn"], cfg["n_experts"], cfg["k_used"], cfg["gs"], xd, 3,
                              idx, w, stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        x_ref, idx_ref = expect[call]
        np.testing.assert_array_equal(idx.cpu().numpy(), idx_ref)
        check_moe_outputs(xh, xd.cpu().numpy(), x_ref, TOL)
        assert np.isfinite(w.cpu().numpy()).all()


def test_noalloc_rejects_sizes_above_its_static_scratch(pkg):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    lib = pkg.glm_cuda.GlmCuda()
    x = torch.zeros(8192, device="cuda")
    with pytest.raises(pkg.glm_cuda.GlmCudaError) as e:
        lib.moe_layer_noalloc({}, 8192, 1536, 64, 4, 32, x, 1)
    assert e.value.rc == -1 and "static scratch limit" in str(e.value)
