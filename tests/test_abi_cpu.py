"""Host-side checks that need no GPU: the C-ABI library loads, exports every
entry point include/glm_cuda.h declares, and rejects calls cleanly before
initialisation; the algorithmic-byte formulas match glm.c's q80_bytes."""
import os
import subprocess

import pytest


def test_header_declares_entry_points(pkg):
    names = pkg.glm_cuda.declared_functions()
    for must in ("glm_cuda_init", "glm_cuda_upload_moe_layer", "glm_cuda_moe_layer", "glm_cuda_matvec_q80",
                 "glm_cuda_free", "glm_cuda_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol(pkg):
    pkg.build.build()
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.build.LIB], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in pkg.glm_cuda.declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    L = pkg.glm_cuda.load()
    for n in pkg.glm_cuda.declared_functions():
        assert getattr(L, n) is not None


def test_calls_before_init_fail_cleanly(pkg):
    import numpy as np

    lib = pkg.glm_cuda.GlmCuda()
    lib.free()
    x = np.zeros((1, 256), dtype=np.float32)
    with pytest.raises(pkg.glm_cuda.GlmCudaError) as e:
        lib.moe_layer(0, x, 4)
    assert e.value.rc == -2 and "glm_cuda_init" in str(e.value)
    with pytest.raises(pkg.glm_cuda.GlmCudaError) as e:
        lib.matvec(np.zeros((2, 64), np.int8), np.zeros((2, 2), np.float32), np.zeros(64, np.float32), 32)
    assert e.value.rc == -2
    lib.free()  # idempotent


def test_expert_parallel_calls_before_setup_fail_cleanly(pkg):
    """Every expert-parallel entry point, called before glm_cuda_init (or
    before glm_cuda_ep_setup / _peer_connect), returns the state error and
    touches no device."""
    import numpy as np

    gc = pkg.glm_cuda
    lib = gc.GlmCuda()
    lib.free()
    x = np.zeros((4, 256), np.float32)
    calls = [
        lambda: lib.ep_setup(2, 0, 4),
        lambda: lib.ep_peer_region(),
        lambda: lib.ep_peer_open(bytes(64)),
        lambda: lib.ep_peer_connect([16 << 20, 32 << 20]),
        lambda: lib.ep_p2p_dispatch(0, x, 4),
        lambda: lib.ep_p2p_experts(0),
        lambda: lib.ep_p2p_combine(0, x),
        lambda: lib.ep_p2p_counts(2),
        lambda: lib.ep_status(),
    ]
    for call in calls:
        with pytest.raises(gc.GlmCudaError) as e:
            call()
        assert e.value.rc == -2, str(e.value)
    lib.free()


def test_init_rejects_unsupported_shapes(pkg):
    lib = pkg.glm_cuda.GlmCuda()
    for args in ((0, 2048, 1536, 64, 4, 8, 1),    # gs=8 (supported: 32, 16)
                 (0, 2000, 1536, 64, 4, 32, 1),   # dim % 128
                 (0, 2048, 1536, 64, 9, 32, 1),   # K > 8
                 (0, 2048, 1536, 64, 4, 32, 0)):  # no layers
        with pytest.raises(pkg.glm_cuda.GlmCudaError) as e:
            lib.init(*args)
        assert e.value.rc == -1


def test_init_without_gpu_reports_cuda_error(pkg):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = pkg.glm_cuda.GlmCuda()
    with pytest.raises(pkg.glm_cuda.GlmCudaError) as e:
        lib.init(0, 2048, 1536, 64, 4, 32, 1)
    assert e.value.rc in (-3, -1)
    assert lib.last_error()


def test_algorithmic_bytes_match_reference_formula(pkg):
    s = pkg.synth
    # q80_bytes (infer.c:1464-1470) composition used for config 0 / config 1
    assert s.moe_bytes(2048, 1536, 64, 4, 32) == 53_633_280
    assert s.q8_matvec_bytes(1536, 2048, 32) == 3_553_280
    assert s.q8_matvec_bytes(2048, 1536, 32) == 3_553_280
    assert s.q8_matvec_bytes(4608, 2048, 32) == 10_643_456
    assert s.q8_matvec_bytes(154880, 2048, 32) == 357_471_232


def test_header_is_plain_c_and_links(pkg, tmp_path):
    """A C99 translation unit that includes include/glm_cuda.h and takes the
    address of every declared entry point compiles with -Wall -Werror, links
    against the built library and runs (calls only glm_cuda_free and
    glm_cuda_last_error): the boundary needs no C++, CUDA or torch types."""
    import shutil

    gcc = shutil.which("gcc")
    if not gcc:
        pytest.skip("no C compiler")
    pkg.build.build()
    names = pkg.glm_cuda.declared_functions()
    src = tmp_path / "abi_check.c"
    body = "\n".join(f"    table[n++] = (void (*)(void))&{fn};" for fn in names)
    src.write_text(f'''#include <stdio.h>
#include "glm_cuda.h"
int main(void) {{
    void (*table[{len(names) + 1}])(void);
    int n = 0;
{body}
    int linked = 0;
    for (int i = 0; i < n; ++i) linked += table[i] != NULL;
    glm_cuda_free();
    printf("%d entry points\\n", linked);
    return linked == {len(names)} ? 0 : 1;
}}
''')
    exe = tmp_path / "abi_check"
    lib_dir = os.path.dirname(pkg.build.LIB)
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-Wno-pedantic", "-I", pkg.build.INCLUDE, str(src),
                        "-o", str(exe), "-L", lib_dir, "-lglm_cuda", f"-Wl,-rpath,{lib_dir}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"{len(names)} entry points" in r.stdout
