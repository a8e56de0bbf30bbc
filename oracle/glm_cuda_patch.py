"""TEST INFRASTRUCTURE ONLY: glm.c with the `cuda` backend of INTEGRATION.md,
built from glm.c's own sources to show that the drop-in patch compiles, links
and runs.

The recipe copies glm.c's main.c, infer.c, backend.c, backend.h and model.h
from the reference checkout (REF_DIR) into a temporary directory, applies the
maintainer patch of INTEGRATION.md there (each edit is anchored on exact text
of the reference and refuses to apply if that text is missing or ambiguous),
and compiles, with the reference Makefile's flags plus -DGLM_ENABLE_CUDA=1,
against glm.c_b200/libglm_cuda.so:

  _ref/glm_cuda_app       the glm CLI with `--backend cuda` (main.c + infer.c
                          + backend.c, as the reference Makefile builds it)
  _ref/libglmref_cuda.so  oracle/ref_harness.c over the patched sources: its
                          ref_decode runs glm_cpu_forward_token with the cuda
                          backend started (glm_backend_init(BACKEND_CUDA)), so
                          every MoE layer goes through the library's MoE hook
                          and every Q8 matvec through its matvec hook

Only the two build outputs stay (git-ignored, they travel with the tree);
the patched source copies are deleted.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")
APP = os.path.join(OUT, "glm_cuda_app")
HARNESS = os.path.join(OUT, "libglmref_cuda.so")
CUDA_LIB_DIR = os.path.join(ROOT, "glm.c_b200")

CUDA_BLOCK = r'''
#if defined(GLM_ENABLE_CUDA)
#include "glm_cuda.h"
static int g_cuda_active = 0;

static int glm_cuda_backend_init(const Runtime *rt) {
    const RuntimeConfig *c = &rt->cfg;
    if (glm_cuda_init(0, c->dim, c->moe_ffn_dim, c->n_routed_experts, c->n_experts_used,
                      (int)c->group_size, c->n_layers) != 0) return -1;
    for (int l = 1; l < c->n_layers; l++) {
        const LayerMoeShared *w = &rt->moe_layers[l];
        const LayerMoeRouted *r = rt->has_moe_routed ? &rt->moe_routed_layers[l] : NULL;
        if (glm_cuda_upload_moe_layer(l, w->ffn_norm, w->gate_inp, w->exp_probs_b,
                                      w->gate_sh_q, w->gate_sh_s, w->up_sh_q, w->up_sh_s,
                                      w->down_sh_q, w->down_sh_s,
                                      r ? r->gate_q : NULL, r ? r->gate_s : NULL,
                                      r ? r->up_q : NULL, r ? r->up_s : NULL,
                                      r ? r->down_q : NULL, r ? r->down_s : NULL) != 0) return -1;
    }
    g_cuda_active = 1;
    return 0;
}

int glm_backend_try_cuda_moe(RunState *s, int layer_idx) {
    if (!g_cuda_active) return -1;
    if (glm_cuda_moe_layer(layer_idx, s->x, 1, s->moe_topk_idx, s->moe_topk_w) != 0) {
        fprintf(stderr, "[glm-cuda] moe layer %d failed: %s\n", layer_idx, glm_cuda_last_error());
        exit(1);
    }
    return 0;
}
#endif
'''

# (file, anchor, replacement): the anchor must occur exactly once.
EDITS = [
    ("model.h",
     "    BACKEND_METAL = 1,\n} BackendType;",
     "    BACKEND_METAL = 1,\n    BACKEND_CUDA = 2,\n} BackendType;"),
    ("backend.h",
     "int glm_backend_try_metal_matvec(const int8_t *qmat, const float *smat, const float *x, float *y, int rows, "
     "int dim, int gs);\n",
     "int glm_backend_try_metal_matvec(const int8_t *qmat, const float *smat, const float *x, float *y, int rows, "
     "int dim, int gs);\n#if defined(GLM_ENABLE_CUDA)\nint glm_backend_try_cuda_moe(RunState *s, int layer_idx);\n"
     "#endif\n"),
    ("backend.c",
     '#include "backend.h"\n',
     '#include "backend.h"\n' + CUDA_BLOCK),
    ("backend.c",
     "int glm_backend_try_metal_matvec(const int8_t *qmat, const float *smat, const float *x, float *y, int rows, "
     "int dim, int gs) {\n",
     "int glm_backend_try_metal_matvec(const int8_t *qmat, const float *smat, const float *x, float *y, int rows, "
     "int dim, int gs) {\n#if defined(GLM_ENABLE_CUDA)\n"
     "    if (g_cuda_active) return glm_cuda_matvec_q80(qmat, smat, x, y, rows, dim, gs) == 0 ? 0 : -1;\n#endif\n"),
    ("backend.c",
     "int glm_backend_init(BackendType backend, const Runtime *rt, RunState *st) {\n",
     "int glm_backend_init(BackendType backend, const Runtime *rt, RunState *st) {\n#if defined(GLM_ENABLE_CUDA)\n"
     "    if (backend == BACKEND_CUDA) {\n        if (glm_cuda_backend_init(rt) != 0) {\n"
     '            fprintf(stderr, "[glm-cuda] init failed: %s\\n", glm_cuda_last_error());\n            exit(1);\n'
     "        }\n        return 0;\n    }\n#endif\n"),
    ("backend.c",
     "void glm_backend_free(int use_metal) {\n",
     "void glm_backend_free(int use_metal) {\n#if defined(GLM_ENABLE_CUDA)\n"
     "    if (g_cuda_active) {\n        glm_cuda_free();\n        g_cuda_active = 0;\n    }\n#endif\n"),
    ("infer.c",
     "    if (layer_idx <= 0 || layer_idx >= rt->cfg.n_layers) return;\n    if (rt->cfg.moe_ffn_dim <= 0) return;\n"
     "    const LayerMoeShared *w = &rt->moe_layers[layer_idx];\n",
     "    if (layer_idx <= 0 || layer_idx >= rt->cfg.n_layers) return;\n    if (rt->cfg.moe_ffn_dim <= 0) return;\n"
     "#if defined(GLM_ENABLE_CUDA)\n    if (glm_backend_try_cuda_moe(s, layer_idx) == 0) return;\n#endif\n"
     "    const LayerMoeShared *w = &rt->moe_layers[layer_idx];\n"),
    ("infer.c",
     '            } else if (strcmp(v, "metal") == 0) {\n                backend = BACKEND_METAL;\n'
     "                backend_set = 1;\n            } else {\n",
     '            } else if (strcmp(v, "metal") == 0) {\n                backend = BACKEND_METAL;\n'
     "                backend_set = 1;\n#if defined(GLM_ENABLE_CUDA)\n"
     '            } else if (strcmp(v, "cuda") == 0) {\n                backend = BACKEND_CUDA;\n'
     "                backend_set = 1;\n#endif\n            } else {\n"),
    ("infer.c",
     '        if (env_backend && strcmp(env_backend, "metal") == 0) backend = BACKEND_METAL;\n',
     '        if (env_backend && strcmp(env_backend, "metal") == 0) backend = BACKEND_METAL;\n'
     "#if defined(GLM_ENABLE_CUDA)\n"
     '        if (env_backend && strcmp(env_backend, "cuda") == 0) backend = BACKEND_CUDA;\n#endif\n'),
]

# the reference Makefile's flags (Makefile:2,97-99; BLAS none) plus the cuda switch
CFLAGS = ["-O3", "-D_FILE_OFFSET_BITS=64", "-fopenmp", "-w", "-DGLM_ENABLE_CUDA=1"]


def patch_sources(ref_dir: str, dst: str) -> None:
    for name in ("main.c", "infer.c", "backend.c", "backend.h", "model.h"):
        shutil.copy(os.path.join(ref_dir, name), os.path.join(dst, name))
    for name, anchor, repl in EDITS:
        path = os.path.join(dst, name)
        src = open(path).read()
        n = src.count(anchor)
        if n != 1:
            raise RuntimeError(f"{name}: patch anchor found {n} times (glm.c changed?):\n{anchor}")
        open(path, "w").write(src.replace(anchor, repl))


def build(ref_dir: str) -> list[str]:
    """Build _ref/glm_cuda_app and _ref/libglmref_cuda.so; returns their paths."""
    lib = os.path.join(CUDA_LIB_DIR, "libglm_cuda.so")
    if not os.path.exists(lib):
        raise FileNotFoundError(f"{lib} missing: build the CUDA library first")
    cc = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
    link = ["-L" + CUDA_LIB_DIR, "-lglm_cuda", "-Wl,-rpath,$ORIGIN/../../glm.c_b200", "-lm"]
    os.makedirs(OUT, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="glm_cuda_patch_")
    try:
        patch_sources(ref_dir, tmp)
        inc = ["-I" + tmp, "-I" + os.path.join(ROOT, "include")]
        subprocess.run([cc, *CFLAGS, *inc, "-o", APP, os.path.join(tmp, "main.c"), os.path.join(tmp, "infer.c"),
                        os.path.join(tmp, "backend.c"), *link], check=True)
        subprocess.run([cc, *CFLAGS, "-fPIC", "-shared", *inc, "-o", HARNESS, os.path.join(HERE, "ref_harness.c"),
                        os.path.join(tmp, "backend.c"), *link], check=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return [APP, HARNESS]


if __name__ == "__main__":
    print("\n".join(build(sys.argv[1])))
