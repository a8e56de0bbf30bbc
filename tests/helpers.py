"""Small numeric helpers shared by the tests."""
import contextlib
import os

import numpy as np


def rel_l2(a, b, base) -> float:
    """||a - b|| / ||base|| in float64."""
    den = float(np.linalg.norm(np.asarray(base, dtype=np.float64)))
    return float(np.linalg.norm(np.asarray(a, dtype=np.float64) - np.asarray(b, dtype=np.float64))) / max(den, 1e-30)


def finite_rows(x_out_ref: np.ndarray) -> np.ndarray:
    return np.isfinite(x_out_ref).all(axis=1)


def check_moe_outputs(x_in, x_out, x_out_ref, tol: float) -> float:
    """Finite tokens: relative L2 of the FFN delta (x_out - x_in) within tol.
    Non-finite tokens: the same NaN / inf pattern as the reference."""
    x_in = np.asarray(x_in).reshape(x_out_ref.shape)
    ok = finite_rows(x_out_ref)
    worst = 0.0
    for t in np.nonzero(ok)[0]:
        r = rel_l2(x_out[t] - x_in[t], x_out_ref[t] - x_in[t], x_out_ref[t] - x_in[t])
        worst = max(worst, r)
    assert worst <= tol, f"FFN delta rel L2 {worst:.3e} > {tol:g}"
    for t in np.nonzero(~ok)[0]:
        np.testing.assert_array_equal(np.isnan(x_out[t]), np.isnan(x_out_ref[t]))
        np.testing.assert_array_equal(np.isposinf(x_out[t]), np.isposinf(x_out_ref[t]))
        np.testing.assert_array_equal(np.isneginf(x_out[t]), np.isneginf(x_out_ref[t]))
    return worst


def assert_routing_exact(lib) -> None:
    """Every routing since glm_cuda_init was certified even where its
    intervals needed the exact recompute: glm_cuda_route_stats()[2] == 0. The
    count is conservative (it also counts experts with bit-identical exact
    logits, whose order the id settles exactly as glm.c's does), so it is
    asserted on the benchmark configurations' random data, not on fixtures
    built with exact ties."""
    stats = lib.route_stats()
    assert stats[2] == 0, f"{stats[2]} routings hinged on the last bit of expf (stats {stats})"


@contextlib.contextmanager
def routed_env(routed: bool):
    """Express 'routed experts off' the reference's way (GLM_DISABLE_MOE_ROUTED)."""
    old = os.environ.get("GLM_DISABLE_MOE_ROUTED")
    if routed:
        os.environ.pop("GLM_DISABLE_MOE_ROUTED", None)
    else:
        os.environ["GLM_DISABLE_MOE_ROUTED"] = "1"
    try:
        yield
    finally:
        if old is None:
            os.environ.pop("GLM_DISABLE_MOE_ROUTED", None)
        else:
            os.environ["GLM_DISABLE_MOE_ROUTED"] = old
