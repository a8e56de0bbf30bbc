"""glm.c's .bin checkpoint format without a GPU: a synthetic model written by
tests/bin_writer.py decodes through glm.c's own loader (runtime_open) to the
same greedy ids as the same model handed over in memory, and the library's
loader refuses malformed files before touching the device."""
import os

import numpy as np
import pytest

from bin_writer import write_runtime_bin

SMALL = dict(dim=256, hidden_dim=512, n_layers=3, n_heads=4, vocab_size=1000, rope_dim=64, q_lora_rank=128,
             kv_lora_rank=128, qk_nope_dim=64, head_k_dim=128, v_head_dim=64, n_routed_experts=16,
             n_experts_used=4, group_size=32, moe_ffn_dim=128)


@pytest.mark.parametrize("gs", [32, 16])
def test_bin_file_matches_in_memory_model_under_glm_loader(gs, pkg, oracle_mod, tmp_path):
    if not oracle_mod.ref_available():
        pytest.skip("the reference harness was not built")
    synth = pkg.synth
    dims = dict(SMALL, group_size=gs)
    model = synth.decoder_model(21, **dims)
    prompt = synth.prompt_ids(21, 6, dims["vocab_size"])
    path = str(tmp_path / "model.bin")
    size = write_runtime_bin(model, path)
    assert os.path.getsize(path) == size
    ids_mem, _ = oracle_mod.ref_decode(model, prompt, 10, 32)
    ids_bin = oracle_mod.ref_decode_bin(path, prompt, 10, 32)
    np.testing.assert_array_equal(ids_bin, ids_mem)


def test_loader_refuses_bad_files(pkg, tmp_path):
    gc = pkg.glm_cuda
    lib = gc.GlmCuda()
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"\0" * 300)
    with pytest.raises(gc.GlmCudaError) as e:
        lib.load_checkpoint(str(bad), 0, 16)
    assert e.value.rc == -1 and "magic" in str(e.value)
    with pytest.raises(gc.GlmCudaError):
        lib.load_checkpoint(str(tmp_path / "missing.bin"), 0, 16)
    model = pkg.synth.decoder_model(22, **SMALL)
    path = str(tmp_path / "trunc.bin")
    write_runtime_bin(model, path)
    with open(path, "r+b") as f:
        f.truncate(os.path.getsize(path) - 4)
    with pytest.raises(gc.GlmCudaError) as e:
        lib.load_checkpoint(path, 0, 16)
    assert "size" in str(e.value)
