"""Shared pytest setup: markers and import paths.

``-m gpu`` tests need a B200 (sm_100) and the in-tree CUDA library; the rest
run on CPU.
"""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "cake-opt-vc_attention_b200"
for p in (str(REPO), str(PKG_ROOT), str(REPO / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def has_b200():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda_device():
    if not has_b200():
        if os.environ.get("VC_REQUIRE_CUDA") == "1":
            pytest.fail("VC_REQUIRE_CUDA=1 but no sm_100 GPU is visible")
        pytest.skip("needs an sm_100 GPU")
    import torch
    return torch.device("cuda:0")
