"""Shared test setup: import paths and the `gpu` marker.

CPU tests (`-m "not gpu"`) check the oracle against the reference's golden
vectors, the host logic and that the C-ABI library loads; GPU tests (`-m gpu`)
run the CUDA path through the C ABI and compare it with the oracle.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "hyperion-fa3-kernel-_b200")
for p in (REPO, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def hyperion():
    import hyperion_b200

    return hyperion_b200


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.lib()
    return O
