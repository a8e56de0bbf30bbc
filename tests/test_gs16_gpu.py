"""Group size 16 (glm.c's own checkpoint export, glm47_flash_export.py:36)
on the GPU: the MoE layer through the persistent kernel (per-token calls)
and the batched kernels (64 tokens), the Q8 matvec on the integer MMA with
16-column scale groups, and the full decoder, against glm.c's CPU path at
gs = 16 (same bars as gs = 32: ids bit-exact, MoE output within 1e-3,
matvec within 1e-5, greedy ids identical and logits within 1e-3)."""
import numpy as np
import pytest

from helpers import check_moe_outputs, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(pkg):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    pkg.build.build()
    L = pkg.glm_cuda.GlmCuda()
    yield L
    L.free()


@pytest.mark.parametrize("T", [1, 3, 64])
def test_gs16_config0_shape(T, lib, pkg, oracle_mod):
    synth = pkg.synth
    cfg = dict(synth.CONFIG0, gs=16)
    L = synth.moe_layer(seed=16, zipf=1.1, **cfg)
    x = synth.tokens(1600 + T, T, cfg["dim"])
    lib.init(0, cfg["dim"], cfg["ffn"], cfg["n_experts"], cfg["k_used"], 16, 1)
    lib.upload_moe_layer(0, L)
    assert lib.decode_path() == lib.PATH_PERSISTENT  # T < 32: per-token calls; T = 64 batched
    x_out, idx, w = lib.moe_layer(0, x, cfg["k_used"])
    ref, ref_idx, ref_w = oracle_mod.moe_layer(L, x, impl="orc")
    np.testing.assert_array_equal(idx, ref_idx)
    np.testing.assert_allclose(w, ref_w, rtol=0, atol=1e-4)
    worst = check_moe_outputs(x, x_out, ref, 1e-3)
    print(f"gs16 T={T}: worst rel L2 {worst:.2e}")


@pytest.mark.parametrize("rows,cols", [(1536, 2048), (2048, 1536), (4608, 2048), (37, 192), (1, 64), (5000, 10240)])
def test_gs16_matvec(rows, cols, lib, pkg, oracle_mod):
    q, s, x = pkg.synth.matvec_case(rows + 16 * cols, rows, cols, 16)
    lib.init(0, 256, 128, 8, 2, 16, 1)
    y = lib.matvec(q, s, x, 16)
    y_ref = oracle_mod.matvec(q, s, x, 16, impl="orc")
    assert rel_l2(y, y_ref, y_ref) < 1e-5


def test_gs16_decoder_small(lib, pkg, oracle_mod):
    from test_decoder_gpu import SMALL, load_model

    synth = pkg.synth
    dims = dict(SMALL, group_size=16)
    model = synth.decoder_model(12, **dims)
    prompt = synth.prompt_ids(12, 8, dims["vocab_size"])
    n_gen, cap = 12, 8 + 12 + 8
    ids_ref, logits_ref = oracle_mod.ref_decode(model, prompt, n_gen, cap, with_logits=True)
    load_model(lib, model, cap)
    ids, _ = lib.generate(prompt, n_gen)
    np.testing.assert_array_equal(ids, ids_ref)
    tok = int(prompt[0])
    feed = list(prompt[1:]) + list(ids_ref)
    worst = 0.0
    for pos in range(len(prompt) + n_gen - 1):
        logits = lib.forward_token(tok, pos, dims["vocab_size"])
        g = pos - (len(prompt) - 1)
        if g >= 0:
            worst = max(worst, rel_l2(logits, logits_ref[g], logits_ref[g]))
        tok = int(feed[pos])
    print(f"gs16 decoder: worst logits rel L2 {worst:.2e}")
    assert worst <= 1e-3


@pytest.mark.parametrize("gs", [32, 16])
def test_checkpoint_file_decodes_like_glm(gs, lib, pkg, oracle_mod, tmp_path):
    """A .bin written in glm.c's format: glm_cuda_load_checkpoint + generate
    gives the greedy ids of glm.c's own loader and forward pass on the file."""
    from bin_writer import write_runtime_bin
    from test_decoder_gpu import SMALL

    synth = pkg.synth
    dims = dict(SMALL, group_size=gs)
    model = synth.decoder_model(23, **dims)
    prompt = synth.prompt_ids(23, 8, dims["vocab_size"])
    path = str(tmp_path / "model.bin")
    write_runtime_bin(model, path)
    ids_ref = oracle_mod.ref_decode_bin(path, prompt, 12, 32)
    lib.load_checkpoint(path, 0, 32)
    ids, _ = lib.generate(prompt, 12)
    np.testing.assert_array_equal(ids, ids_ref)


@pytest.mark.parametrize("gs", [32, 16])
def test_checkpoint_config2_shapes(gs, lib, pkg, oracle_mod, tmp_path):
    """GLM-4.7-Flash shapes (3 layers, vocab 154880) through the .bin path."""
    from bin_writer import write_runtime_bin

    synth = pkg.synth
    dims = dict(synth.CONFIG2, n_layers=3, group_size=gs)
    model = synth.decoder_model(24, **dims)
    prompt = synth.prompt_ids(24, 8, dims["vocab_size"])
    path = str(tmp_path / "model.bin")
    write_runtime_bin(model, path)
    ids_ref = oracle_mod.ref_decode_bin(path, prompt, 6, 24)
    lib.load_checkpoint(path, 0, 24)
    ids, _ = lib.generate(prompt, 6)
    np.testing.assert_array_equal(ids, ids_ref)
