"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on a CPU-only host: the oracle against the golden vectors
and the reference build, the host logic, and the C-ABI library's exports and
argument validation (no kernel launches).  `-m gpu` runs the CUDA codec
through the C-ABI against the oracle and the golden vectors.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(REPO, "vlx-tee_b200"), os.path.join(REPO, "oracle"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import ztcp_oracle

    ztcp_oracle.build()
    return ztcp_oracle


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
