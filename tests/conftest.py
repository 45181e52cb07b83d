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


GPU_TEST_TIMEOUT_S = 600  # wall-clock limit of one GPU test (pytest-timeout)


def pytest_collection_modifyitems(config, items):
    """Give every GPU test a hard wall-clock limit when pytest-timeout is
    installed (the kernels' own waits are bounded; this also bounds host-side
    hangs such as a missing peer process)."""
    if not config.pluginmanager.hasplugin("timeout"):
        return
    for item in items:
        if item.get_closest_marker("gpu") is not None and item.get_closest_marker("timeout") is None:
            item.add_marker(pytest.mark.timeout(GPU_TEST_TIMEOUT_S))


@pytest.fixture
def run_perf_enabled():
    return os.getenv("BITSCOM_RUN_PERF", "0") == "1"


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
