"""B200-native (sm_100a) backend for glm.c's mixture-of-experts FFN hot path.

  build      nvcc build of libglm_cuda.so (the product: include/glm_cuda.h)
  glm_cuda   ctypes binding of that C-ABI
  synth      seeded synthetic inputs with the benchmark configurations' shapes

The directory name contains a dot, so Python code loads it under the module
name `glm_c_b200` with `load_package()` below (also usable by path from any
script at the repository root).
"""
from __future__ import annotations

import importlib.util
import os
import sys

PACKAGE_NAME = "glm_c_b200"


def load_package(root: str | None = None):
    """Import this directory as the package `glm_c_b200` and return it."""
    if PACKAGE_NAME in sys.modules:
        return sys.modules[PACKAGE_NAME]
    pkg_dir = os.path.join(root, "glm.c_b200") if root else os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location(PACKAGE_NAME, os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[PACKAGE_NAME] = mod
    spec.loader.exec_module(mod)
    return mod
