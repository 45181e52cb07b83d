"""Loads the reference implementation's pure-torch CPU code as a test oracle.

The reference package ``bitscom`` is imported from ``BITSCOM_REF_PATH`` (default:
the reference build under ``baseline/_ref`` of this repository) with its two
native extension modules blocked, so every call runs the reference's own CPU
fallbacks (its quantization module imports the extensions inside try/except).
Tests that need the oracle skip when it is not installed.
"""

from __future__ import annotations

import importlib
import importlib.abc
import os
import sys
from pathlib import Path

import pytest

_BLOCKED = {"bitscom._lowbit_c", "bitscom._lowbit_cuda"}


class _BlockExtensions(importlib.abc.MetaPathFinder):
    def find_spec(self, fullname, path=None, target=None):
        if fullname in _BLOCKED:
            raise ImportError(f"{fullname} is blocked: the oracle runs the reference's CPU code")
        return None


def _candidates():
    env = os.environ.get("BITSCOM_REF_PATH")
    if env:
        yield Path(env)
    yield Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def load():
    """Return the reference ``bitscom.quantization`` module, or skip."""
    if "bitscom.quantization" in sys.modules:
        return sys.modules["bitscom.quantization"]
    for cand in _candidates():
        if (cand / "bitscom" / "quantization.py").exists():
            if not any(isinstance(f, _BlockExtensions) for f in sys.meta_path):
                sys.meta_path.insert(0, _BlockExtensions())
            sys.path.insert(0, str(cand))
            try:
                mod = importlib.import_module("bitscom.quantization")
            finally:
                sys.path.remove(str(cand))
            assert not mod._HAS_CUDA_KERNELS
            return mod
    pytest.skip("reference oracle not installed (set BITSCOM_REF_PATH)")
