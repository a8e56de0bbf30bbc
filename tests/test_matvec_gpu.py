"""Parity of the CUDA Q8 matvec (config 1 shapes, LM head included) with
glm.c's matvec_q80_rows, through the C-ABI's glm_backend_try_metal_matvec-
shaped entry point."""
import numpy as np
import pytest

from helpers import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the integer-MMA path is fp32-class; the reference reassociates too


@pytest.fixture(scope="module")
def lib(pkg):
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    L = pkg.glm_cuda.GlmCuda()
    L.init(0, 256, 128, 16, 4, 32, 1)
    yield L
    L.free()


@pytest.mark.parametrize("shape", [(1536, 2048), (2048, 1536), (4608, 2048)])
def test_matvec_config1_matches_golden(shape, lib, golden):
    q, s, x, y_ref, _ = golden.load_matvec(*shape)
    y = lib.matvec(q, s, x, 32)
    r = rel_l2(y, y_ref, y_ref)
    print(f"{shape}: rel L2 {r:.2e}")
    assert r < TOL


def test_matvec_lm_head_matches_golden(lib, golden):
    q, s, x, y_head, y_sum = golden.load_matvec(154880, 2048)
    y = lib.matvec(q, s, x, 32)
    assert rel_l2(y[:4096], y_head, y_head) < TOL
    assert abs(float(y.astype(np.float64).sum()) - y_sum) <= 1e-5 * float(np.abs(y).astype(np.float64).sum())


@pytest.mark.parametrize("rows,cols", [(1, 64), (17, 128), (37, 192), (1000, 64), (300, 4096)])
def test_matvec_ragged_shapes(rows, cols, lib, pkg, oracle_mod):
    q, s, x = pkg.synth.matvec_case(rows * 7 + cols, rows, cols, 32)
    y = lib.matvec(q, s, x, 32)
    y_ref = oracle_mod.matvec(q, s, x, 32, impl="orc")
    assert rel_l2(y, y_ref, y_ref) < TOL


def test_matvec_weight_cache_follows_shape_change(lib, pkg, oracle_mod):
    """The cache is keyed by host address; a new shape at the same address re-uploads."""
    q, s, x = pkg.synth.matvec_case(5, 64, 256, 32)
    y1 = lib.matvec(q, s, x, 32)
    q2 = q.reshape(128, 128)
    s2 = np.ascontiguousarray(s.reshape(64, 8)[:, :].reshape(-1)[: 128 * 4].reshape(128, 4))
    y2 = lib.matvec(q2, s2, x[:128].copy(), 32)
    np.testing.assert_allclose(y1, oracle_mod.matvec(q, s, x, 32), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(y2, oracle_mod.matvec(q2, s2, x[:128].copy(), 32), rtol=1e-5, atol=1e-6)
