"""Test configuration: markers and import paths.

``-m "not gpu"`` runs here without a GPU (oracle vs golden vectors, C-ABI loading and argument
errors, host logic, gloo multi-process sharding). ``-m gpu`` holds the parity tests proper, which
call the CUDA kernels through the torch ops and the C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO_ROOT = Path(__file__).resolve().parents[1]
PACKAGE_DIR = REPO_ROOT / "inference-performance-lab_b200"

for path in (str(PACKAGE_DIR), str(REPO_ROOT)):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: requires an NVIDIA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "vllm: requires the vLLM serving environment")


def cuda_available() -> bool:
    import torch

    return torch.cuda.is_available()


requires_cuda = pytest.mark.skipif(not cuda_available(), reason="CUDA is unavailable")
