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
        # loaded from its file: importing it through the package would run
        # the package's check that the libraries already exist
        import importlib.util

        path = os.path.join(ROOT, "torch-rbln_b200", "torch_rbln_b200", "_build.py")
        spec = importlib.util.spec_from_file_location("torch_rbln_b200_build", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200) and the built CUDA extension")


@pytest.fixture(autouse=True)
def _seed():
    # the reference's test/conftest.py:14-18 seeds every test with 0
    import torch

    torch.manual_seed(0)
