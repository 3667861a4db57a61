"""Shared pytest setup: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs the oracle / host / C-ABI loading checks on any CPU box;
``-m gpu`` runs the parity tests of the CUDA kernels through the C ABI.
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "qwen3asr.rs_b200", REPO / "oracle", REPO / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device; runs the kernels")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
