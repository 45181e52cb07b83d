"""bitscom_b200: Blackwell-native low-bit communication for PyTorch.

Usage (API of the reference package ``bitscom``)::

    import bitscom_b200 as bitscom
    bitscom.init(bitwidth=4, error_feedback=True)      # registers backend "lowbit"
    import torch.distributed as dist
    dist.init_process_group(backend="lowbit")
    group = bitscom.LowBitGroup(bitwidth=4)
    group.all_reduce(tensor)

DDP::

    ddp = torch.nn.parallel.DistributedDataParallel(model)
    bitscom.register_lowbit_hook(ddp, bitwidth=4, error_feedback=True)
"""

from .api import LowBitGroup
from .lowbit_backend import backend_options, is_extension_available, register_lowbit_backend
from .parallel.comm import Communicator
from .parallel.fsdp import LowBitShardedDP
from .parallel.graphs import GraphedStep
from .parallel.hooks import LowBitHookState, lowbit_allreduce_hook, register_lowbit_hook
from .quantization import (
    SUPPORTED_BITWIDTHS,
    CompressedTensor,
    compress_tensor,
    decompress_tensor,
    dequantize_tensor,
    ef_roundtrip,
    pack_lowbit,
    quantize_tensor,
    roundtrip_tensor,
    unpack_lowbit,
    validate_bitwidth,
)

__all__ = [
    "register_lowbit_backend",
    "is_extension_available",
    "backend_options",
    "LowBitGroup",
    "SUPPORTED_BITWIDTHS",
    "init",
    "stats",
    "Communicator",
    "LowBitHookState",
    "lowbit_allreduce_hook",
    "register_lowbit_hook",
    "LowBitShardedDP",
    "GraphedStep",
    "CompressedTensor",
    "compress_tensor",
    "decompress_tensor",
    "quantize_tensor",
    "dequantize_tensor",
    "pack_lowbit",
    "unpack_lowbit",
    "roundtrip_tensor",
    "ef_roundtrip",
    "validate_bitwidth",
]

__version__ = "0.1.0"


def init(bitwidth: int = 4, error_feedback: bool = False, **options) -> None:
    """Register the ``lowbit`` backend; call before ``init_process_group``."""
    register_lowbit_backend(bitwidth=bitwidth, error_feedback=error_feedback, **options)


def stats(group=None) -> dict:
    """Per-op counters of the fused paths (launches, wire bytes, algorithm
    choices) of every communicator created in this process, plus the
    ``lowbit`` backend counters of ``group`` when it uses that backend."""
    import torch
    import torch.distributed as dist

    from .parallel.comm import _CACHE

    out = {}
    for (gkey, dev), comm in list(_CACHE.items()):
        if comm is not None:
            out[f"{gkey}/cuda:{dev}"] = comm.stats()
    if dist.is_available() and dist.is_initialized():
        pg = group or dist.group.WORLD
        try:
            be = pg._get_backend(torch.device("cuda" if torch.cuda.is_available() else "cpu"))
            if hasattr(be, "stats"):
                out["lowbit_backend"] = dict(be.stats())
        except Exception:
            pass
    return out
