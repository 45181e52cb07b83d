"""Parallel runtime: fused communicator, DDP hook, sharded data parallel,
pipeline-A, whole-step CUDA-graph capture."""

from .bucketing import GradBucketer
from .comm import Communicator
from .fsdp import LowBitShardedDP
from .graphs import DDP_EAGER_WARMUP, GraphedStep
from .hooks import LowBitHookState, lowbit_allreduce_hook, register_lowbit_hook
from .pipeline import DualStreamScheduler, hierarchical_allreduce, should_use_dual_stream

__all__ = [
    "Communicator", "GradBucketer", "LowBitShardedDP", "LowBitHookState", "lowbit_allreduce_hook", "register_lowbit_hook",
    "DualStreamScheduler", "hierarchical_allreduce", "should_use_dual_stream", "GraphedStep", "DDP_EAGER_WARMUP",
]
