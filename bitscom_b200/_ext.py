"""Loader of the native extension ``bitscom_b200._C``.

The extension is built in-tree (``python setup.py build_ext --inplace``).  On a
machine with a CUDA device the CUDA code paths never fall back silently: if the
extension is missing, :func:`require` raises with the import error, so a GPU
test or benchmark that would otherwise run on a torch fallback fails loudly.
"""

from __future__ import annotations

import torch

try:  # torch.distributed must be imported first: the extension subclasses c10d.Backend
    import torch.distributed  # noqa: F401
    from . import _C  # type: ignore[attr-defined]

    HAS_EXT = True
    IMPORT_ERROR: BaseException | None = None
except Exception as exc:  # pragma: no cover - depends on the build
    _C = None
    HAS_EXT = False
    IMPORT_ERROR = exc


def available() -> bool:
    """True when the native extension imported."""
    return HAS_EXT


def require(what: str = "this operation"):
    """Return the extension module or raise a clear error."""
    if not HAS_EXT:
        raise RuntimeError(
            f"bitscom_b200 native extension is required for {what} but failed to import "
            f"({IMPORT_ERROR!r}); build it with `python setup.py build_ext --inplace`"
        ) from IMPORT_ERROR
    return _C


def use_cuda_kernels(t: torch.Tensor) -> bool:
    """CUDA tensors always take the native kernels; a missing extension raises."""
    if not t.is_cuda:
        return False
    require("CUDA tensors")
    return True
