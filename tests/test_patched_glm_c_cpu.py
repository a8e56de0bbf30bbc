"""The drop-in binding of INTEGRATION.md applied to glm.c's own sources
(oracle/glm_cuda_patch.py): the patched glm.c compiles and links against
libglm_cuda.so, its CLI accepts `--backend cuda` (and still refuses unknown
backends), and the harness built over it exports the MoE hook."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


@pytest.fixture(scope="module")
def patched():
    import glm_cuda_patch
    import oracle

    ref = oracle.reference_dir()
    if not ref:
        pytest.skip("glm.c's sources are not here (set GLM_REFERENCE_DIR)")
    from __graft_entry__ import load_package

    load_package().build.build()
    return glm_cuda_patch.build(ref)


def test_patched_glm_c_builds_and_links(patched):
    app, harness = patched
    assert os.access(app, os.X_OK) and os.path.exists(harness)
    syms = subprocess.run(["nm", "-D", harness], capture_output=True, text=True, check=True).stdout
    for name in ("glm_backend_try_cuda_moe", "glm_backend_init", "ref_decode"):
        assert f" T {name}" in syms, name
    needed = subprocess.run(["readelf", "-d", harness], capture_output=True, text=True, check=True).stdout
    assert "libglm_cuda.so" in needed


def test_patched_cli_knows_the_cuda_backend(patched):
    app, _ = patched
    r = subprocess.run([app, "/nonexistent.bin", "--backend", "cuda", "-n", "1", "-i", "hi"], capture_output=True,
                       text=True)
    assert "unknown backend" not in r.stderr + r.stdout and "checkpoint" in r.stderr + r.stdout
    r = subprocess.run([app, "/nonexistent.bin", "--backend", "vulkan", "-i", "hi"], capture_output=True, text=True)
    assert r.returncode != 0 and "unknown backend" in r.stderr
