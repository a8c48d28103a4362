"""Shared pytest setup.

Marker ``gpu``: the test needs a CUDA device (run on a B200 with ``-m gpu``).
Everything unmarked runs on a CPU-only host.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "tests/golden", "llm-on-cpu_b200"):
    p = os.path.join(REPO, sub)
    if p not in sys.path:
        sys.path.insert(0, p)
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import orc

    return orc.Oracle()


@pytest.fixture(scope="session")
def reference():
    import orc

    if not orc.ref_available():
        pytest.skip("reference operators not built (oracle/_ref needs the reference tree at build time)")
    return orc.Reference()
