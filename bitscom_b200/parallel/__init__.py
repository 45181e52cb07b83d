"""Parallel runtime: fused communicator, DDP hook, sharded data parallel, pipeline-A."""

from .comm import Communicator
from .fsdp import LowBitShardedDP
from .hooks import LowBitHookState, lowbit_allreduce_hook, register_lowbit_hook
from .pipeline import DualStreamScheduler, hierarchical_allreduce, should_use_dual_stream

__all__ = [
    "Communicator", "LowBitShardedDP", "LowBitHookState", "lowbit_allreduce_hook", "register_lowbit_hook",
    "DualStreamScheduler", "hierarchical_allreduce", "should_use_dual_stream",
]
