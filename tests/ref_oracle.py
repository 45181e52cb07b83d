"""Loads the reference implementation's pure-torch CPU code as a test oracle.

The reference package ``bitscom`` is imported, with its two native extension
modules blocked so every call runs the reference's own CPU fallbacks (its
quantization module imports the extensions inside try/except), from the first
of:

1. ``BITSCOM_REF_PATH``;
2. the reference build under ``baseline/_ref`` of this repository
   (``baseline/install_reference.py``);
3. a copy of the reference's Python sources (``.py`` files only, never its
   shipped ``__pycache__`` or extension modules) taken from
   ``<reference_path>/python/bitscom``, ``reference_path`` being named by
   ``BASELINE.json``.

Tests that need the oracle skip when none of these exists.
"""

from __future__ import annotations

import importlib
import importlib.abc
import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import pytest

_BLOCKED = {"bitscom._lowbit_c", "bitscom._lowbit_cuda"}


class _BlockExtensions(importlib.abc.MetaPathFinder):
    def find_spec(self, fullname, path=None, target=None):
        if fullname in _BLOCKED:
            raise ImportError(f"{fullname} is blocked: the oracle runs the reference's CPU code")
        return None


_ROOT = Path(__file__).resolve().parents[1]
_SOURCE_COPY = None


def _source_copy():
    """Copy the reference's package sources (.py only) to a temp dir."""
    global _SOURCE_COPY
    if _SOURCE_COPY is not None:
        return _SOURCE_COPY
    try:
        ref = json.loads((_ROOT / "BASELINE.json").read_text()).get("reference_path")
    except (OSError, ValueError):
        return None
    src = Path(ref or "") / "python" / "bitscom"
    if not ref or not (src / "quantization.py").is_file():
        return None
    dst = Path(tempfile.mkdtemp(prefix="bitscom_ref_oracle_"))
    (dst / "bitscom").mkdir()
    for f in src.glob("*.py"):
        shutil.copyfile(f, dst / "bitscom" / f.name)
    _SOURCE_COPY = dst
    return dst


def _candidates():
    env = os.environ.get("BITSCOM_REF_PATH")
    if env:
        yield Path(env)
    yield _ROOT / "baseline" / "_ref"
    copy = _source_copy()
    if copy is not None:
        yield copy


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
