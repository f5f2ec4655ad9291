import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "torch-rbln_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_sessionstart(session):
    """Build the in-tree native libraries when they are missing (a fresh
    checkout); nvcc cross-compiles for sm_100a without a GPU."""
    lib = os.path.join(ROOT, "torch-rbln_b200", "torch_rbln_b200", "_lib", "librbln_attn_torch.so")
    if not os.path.exists(lib):
        from torch_rbln_b200 import _build

        _build.build()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200) and the built CUDA extension")


@pytest.fixture(autouse=True)
def _seed():
    # the reference's test/conftest.py:14-18 seeds every test with 0
    import torch

    torch.manual_seed(0)
