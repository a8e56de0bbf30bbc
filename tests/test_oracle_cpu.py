"""The CPU oracle (my restatement, oracle/moe_oracle.c) against glm.c's own
outputs: the golden fixtures (made by the compiled reference) and, where the
reference build is present, the compiled reference itself on fresh seeds."""
import numpy as np
import pytest

from helpers import check_moe_outputs, rel_l2

SMALL_CASES = ["moe_tiny_gs32", "moe_tiny_gs16", "moe_ties", "moe_near_ties", "moe_nonfinite",
               "moe_routed_off", "moe_all_experts"]


@pytest.mark.parametrize("name", SMALL_CASES)
def test_oracle_matches_golden(name, oracle_mod, golden):
    L, x, routed, exp = golden.load_case(name)
    x_out, idx, w = oracle_mod.moe_layer(L, x, impl="orc", routed=routed)
    np.testing.assert_array_equal(idx, exp["topk_idx"])
    np.testing.assert_array_equal(w, exp["topk_w"])  # same serial fp32 arithmetic: bit-exact
    check_moe_outputs(x, x_out, exp["x_out"], tol=1e-5)


def test_oracle_matches_golden_config0(oracle_mod, golden):
    L, x, routed, exp = golden.load_case("moe_config0")
    x_out, idx, w = oracle_mod.moe_layer(L, x, impl="orc", routed=routed)
    np.testing.assert_array_equal(idx, exp["topk_idx"])
    np.testing.assert_array_equal(w, exp["topk_w"])
    check_moe_outputs(x, x_out, exp["x_out"], tol=1e-5)


@pytest.mark.parametrize("gs", [32, 16])
@pytest.mark.parametrize("seed", [100, 101, 102])
def test_oracle_matches_compiled_reference(seed, gs, oracle_mod, pkg):
    if not oracle_mod.ref_available():
        pytest.skip("reference not compiled here (oracle/_ref/libglmref.so absent)")
    synth = pkg.synth
    L = synth.moe_layer(seed=seed, dim=256, ffn=128, n_experts=16, k_used=4, gs=gs)
    x = synth.tokens(seed, 48, 256)
    a = oracle_mod.moe_layer(L, x, impl="orc")
    b = oracle_mod.moe_layer(L, x, impl="ref")
    np.testing.assert_array_equal(a[1], b[1])
    np.testing.assert_array_equal(a[2], b[2])
    check_moe_outputs(x, a[0], b[0], tol=1e-5)


@pytest.mark.parametrize("shape", [(1536, 2048), (2048, 1536), (4608, 2048)])
def test_matvec_oracle_matches_golden(shape, oracle_mod, golden):
    q, s, x, y_ref, _ = golden.load_matvec(*shape)
    y = oracle_mod.matvec(q, s, x, 32, impl="orc")
    assert rel_l2(y, y_ref, y_ref) < 1e-6


def test_matvec_oracle_lm_head_golden(oracle_mod, golden):
    q, s, x, y_head, y_sum = golden.load_matvec(154880, 2048)
    y = oracle_mod.matvec(q, s, x, 32, impl="orc")
    assert rel_l2(y[:4096], y_head, y_head) < 1e-6
    assert abs(float(y.astype(np.float64).sum()) - y_sum) <= 1e-5 * float(np.abs(y).astype(np.float64).sum())


def test_topk_semantics_edge_cases(oracle_mod):
    """Tie to the lower id, NaN and -inf never selected, unused slots -1/-1e30."""
    import ctypes

    lib = oracle_mod.lib("orc")
    lib.orc_topk.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] * 2 + [ctypes.c_void_p] * 2
    p = np.array([0.5, 0.7, 0.7, np.nan, 0.1, -np.inf], dtype=np.float32)
    b = np.zeros(6, dtype=np.float32)
    idx = np.zeros(5, dtype=np.int32)
    w = np.zeros(5, dtype=np.float32)
    lib.orc_topk(p.ctypes.data, b.ctypes.data, 6, 5, idx.ctypes.data, w.ctypes.data)
    assert idx.tolist() == [1, 2, 0, 4, -1]
    assert w[-1] == np.float32(-1e30)
