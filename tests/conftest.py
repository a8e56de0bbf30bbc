"""Shared test setup: the `gpu` marker, the package loader and the oracle path.

CPU tests (-m "not gpu") check the oracle against the golden fixtures and the
compiled reference, the host-side logic, and that the C-ABI library loads and
exports what include/glm_cuda.h declares. GPU tests (-m gpu) are the parity
tests proper: they call the CUDA path through the C-ABI and compare with the
CPU oracle.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def pkg():
    from __graft_entry__ import load_package

    return load_package()


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    if not os.path.exists(oracle.ORC_SO):
        oracle.build()
    return oracle


@pytest.fixture(scope="session")
def golden():
    import make_golden

    return make_golden

