"""Shared pytest configuration.

Markers:
  gpu          needs a CUDA device (run with ``-m gpu`` on a GPU box)
  multigpu     needs at least two CUDA devices (also marked gpu)
  performance  timing-sensitive checks (run when BITSCOM_RUN_PERF=1)
"""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA device")
    config.addinivalue_line("markers", "multigpu: test needs at least two CUDA devices")
    config.addinivalue_line("markers", "performance: timing-sensitive test (BITSCOM_RUN_PERF=1)")


@pytest.fixture
def run_perf_enabled():
    return os.getenv("BITSCOM_RUN_PERF", "0") == "1"


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
