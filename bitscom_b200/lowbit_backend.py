"""Registration of the ``lowbit`` torch.distributed backend.

Usage (same calls as reference python/bitscom/lowbit_backend.py:52-93)::

    import bitscom_b200 as bitscom
    bitscom.init(bitwidth=4, error_feedback=True)
    torch.distributed.init_process_group(backend="lowbit", ...)

The factory builds the native ``ProcessGroupLowBit`` (csrc/backend) around two
inner backends created on prefixed views of the same store: gloo for CPU
tensors and, when CUDA is available, NCCL for CUDA tensors.  CUDA low-bit
collectives run on the fused NVLink kernels; everything else is forwarded.
Options beyond the reference's two (bitwidth, error_feedback) are keyword
arguments of :func:`register_lowbit_backend`.
"""

from __future__ import annotations

import datetime
from typing import Any, Dict

import torch
import torch.distributed as dist

from . import _ext

_REGISTERED = False
_BACKEND_BITWIDTH = 4
_BACKEND_ERROR_FEEDBACK = False
_BACKEND_EXTRA: Dict[str, Any] = {}
_HAS_EXTENSION = _ext.HAS_EXT
_EXTENSION_IMPORT_ERROR = _ext.IMPORT_ERROR

_EXTRA_DEFAULTS = {
    "stochastic_rounding": False,
    "fp8": False,
    "force_lowbit": False,
    "algo": "auto",
    "workspace_mb": 256,
    "max_ctas": 0,
    "seed": 0x5EED,
    "blocking_wait": False,
    "oneshot_max_bytes": None,  # None: from the tuning table for this world size
}
_ALGOS = {"auto": 0, "twoshot": 1, "oneshot": 2}


def create_backend(store, rank: int, size: int, timeout, bitwidth: int = 4, error_feedback: bool = False, **extra):
    """Build a ProcessGroupLowBit (the counterpart of the reference's
    ``_lowbit_c.create_backend``, cpp/src/bindings.cc:17-26)."""
    C = _ext.require("the lowbit backend")
    if isinstance(timeout, (int, float)):
        timeout = datetime.timedelta(milliseconds=timeout)
    opts = C.LowBitOptions()
    opts.bitwidth = int(bitwidth)
    opts.error_feedback = bool(error_feedback)
    opts.timeout = timeout
    cfg = dict(_EXTRA_DEFAULTS)
    cfg.update(extra)
    opts.stochastic_rounding = bool(cfg["stochastic_rounding"])
    opts.fp8 = bool(cfg["fp8"])
    opts.force_lowbit = bool(cfg["force_lowbit"])
    opts.algo = _ALGOS[cfg["algo"]] if isinstance(cfg["algo"], str) else int(cfg["algo"])
    opts.workspace_bytes = int(cfg["workspace_mb"]) << 20
    opts.max_ctas = int(cfg["max_ctas"])
    opts.seed = int(cfg["seed"])
    opts.blocking_wait = bool(cfg["blocking_wait"])
    from .tuning import entries as _tuning_entries

    opts.tuning = [list(e) for e in _tuning_entries(size)]
    if cfg["oneshot_max_bytes"] is None:
        from .tuning import oneshot_max_bytes

        opts.oneshot_max_bytes = oneshot_max_bytes(size)
    else:
        opts.oneshot_max_bytes = int(cfg["oneshot_max_bytes"])

    cpu_inner = dist.ProcessGroupGloo(dist.PrefixStore("lowbit_gloo/", store), rank, size, timeout)
    cuda_inner = None
    if torch.cuda.is_available() and dist.is_nccl_available():
        nopts = dist.ProcessGroupNCCL.Options()
        nopts._timeout = timeout
        cuda_inner = dist.ProcessGroupNCCL(dist.PrefixStore("lowbit_nccl/", store), rank, size, nopts)
    return C.ProcessGroupLowBit(store, rank, size, cpu_inner, cuda_inner, opts)


def _create_lowbit_pg(store, rank, size, timeout):
    """Factory called by torch.distributed for ``backend="lowbit"``."""
    if not _HAS_EXTENSION:
        raise RuntimeError(
            "bitscom_b200 C++ extension is not available. Build it with "
            "`python setup.py build_ext --inplace` first."
        ) from _EXTENSION_IMPORT_ERROR
    return create_backend(
        store=store,
        rank=rank,
        size=size,
        timeout=timeout,
        bitwidth=_BACKEND_BITWIDTH,
        error_feedback=_BACKEND_ERROR_FEEDBACK,
        **_BACKEND_EXTRA,
    )


def register_lowbit_backend(bitwidth: int = 4, error_feedback: bool = False, **extra) -> None:
    """Register ``"lowbit"`` with torch.distributed (idempotent for equal options)."""
    global _REGISTERED, _BACKEND_BITWIDTH, _BACKEND_ERROR_FEEDBACK, _BACKEND_EXTRA
    if bitwidth not in (1, 2, 4, 8, 12, 16):
        raise ValueError(f"bitwidth must be one of (1, 2, 4, 8, 12, 16), got {bitwidth}")
    unknown = set(extra) - set(_EXTRA_DEFAULTS)
    if unknown:
        raise TypeError(f"unknown lowbit backend options: {sorted(unknown)}")
    if "algo" in extra and isinstance(extra["algo"], str) and extra["algo"] not in _ALGOS:
        raise ValueError(f"algo must be one of {sorted(_ALGOS)}")
    if _REGISTERED:
        if (
            bitwidth != _BACKEND_BITWIDTH
            or bool(error_feedback) != _BACKEND_ERROR_FEEDBACK
            or dict(extra) != _BACKEND_EXTRA
        ):
            raise RuntimeError(
                "lowbit backend is already registered with different options: "
                f"bitwidth={_BACKEND_BITWIDTH}, error_feedback={_BACKEND_ERROR_FEEDBACK}, extra={_BACKEND_EXTRA}"
            )
        return
    _BACKEND_BITWIDTH = bitwidth
    _BACKEND_ERROR_FEEDBACK = bool(error_feedback)
    _BACKEND_EXTRA = dict(extra)
    if not _HAS_EXTENSION:
        raise RuntimeError(
            "bitscom_b200 C++ extension is not available. Build it with "
            "`python setup.py build_ext --inplace` before registering the backend."
        ) from _EXTENSION_IMPORT_ERROR
    dist.Backend.register_backend(name="lowbit", func=_create_lowbit_pg, devices=["cpu", "cuda"])
    _REGISTERED = True


def is_extension_available() -> bool:
    return _HAS_EXTENSION


def backend_options() -> Dict[str, Any]:
    """The options the next ``init_process_group(backend="lowbit")`` will use."""
    out = {"bitwidth": _BACKEND_BITWIDTH, "error_feedback": _BACKEND_ERROR_FEEDBACK}
    cfg = dict(_EXTRA_DEFAULTS)
    cfg.update(_BACKEND_EXTRA)
    out.update(cfg)
    return out
