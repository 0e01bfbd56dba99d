"""Shared pytest setup: import paths and the `gpu` marker."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flashatte-hand_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def cuda_available() -> bool:
    import torch
    return torch.cuda.is_available()


@pytest.fixture(scope="session")
def lib():
    import flashdecode
    return flashdecode.load_library()
