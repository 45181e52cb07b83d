"""Whole-step CUDA-graph capture for data-parallel training with the low-bit
DDP hook.

A small-image training step (ResNet-18 on 32x32 inputs, batch 256) issues a
few hundred kernels of a few microseconds each; in eager mode the host, not
the GPU, sets the pace.  :class:`GraphedStep` captures forward, backward (with
the DDP comm hook and its fused all-reduce launches) and the optimizer step
into one CUDA graph and replays it, so a step costs one graph launch on the
host.

Why the low-bit collective can be replayed:

* the fused kernel takes its launch epoch (flag value and buffer parity) from
  a counter in device memory that the last CTA of each launch advances, so
  every replay gets a fresh epoch on every rank (ranks replay the same launch
  sequence, so their epochs agree);
* under capture the Philox offset of stochastic rounding is derived from that
  epoch, so replays draw fresh random numbers;
* the hook does no host synchronisation: it orders the comm stream after the
  current stream, launches, and returns a CUDA-aware future that completes in
  stream order.

Requirements on the step function (the usual whole-network capture rules):
static input tensors (copy each batch into them: :meth:`GraphedStep.__call__`
does), no host reads of device values inside the step, gradients kept
allocated between steps (``zero_grad(set_to_none=False)``), an optimizer
whose state exists before capture (the warm-up steps create it), and DDP
buffer broadcasting off (``broadcast_buffers=False``), since that is an NCCL
call on the default group inside the step.  DDP's reducer runs eagerly
during the warm-up iterations (at least 11, after which DDP stops sampling
its runtime statistics with host-synchronising events) and during capture;
replays skip the host side of DDP entirely.

No counterpart in the reference: its collectives synchronise with the host
(``.item()`` on scales, blocking waits; reference
python/bitscom/api.py:216-225, cpp/src/process_group_lowbit.cc:292-305), so a
step that uses them cannot be captured.
"""

from __future__ import annotations

from typing import Any, Callable, Optional, Sequence

import torch

# DDP records host-synchronising timing events for its first iterations; the
# PyTorch capture recipe asks for at least 11 eager DDP iterations first.
DDP_EAGER_WARMUP = 11


class GraphedStep:
    """Capture ``fn(*inputs)`` once and replay it.

    Args:
        fn: the training step; takes the static input tensors and returns a
            tensor (or a tuple of tensors), e.g. the loss.
        example_inputs: tensors with the shapes, dtypes, devices and memory
            formats of every later call's inputs (their values are used for
            the warm-up steps).
        warmup: eager iterations before capture (each one is a real training
            step on ``example_inputs``).
        pool: optional graph memory pool shared with other graphs.

    Calling the object copies the given inputs into the static buffers on the
    current stream and replays the graph; it returns the static outputs,
    which later calls overwrite.
    """

    def __init__(
        self,
        fn: Callable[..., Any],
        example_inputs: Sequence[torch.Tensor],
        *,
        warmup: int = DDP_EAGER_WARMUP,
        pool: Optional[Any] = None,
    ):
        if not example_inputs:
            raise ValueError("GraphedStep needs at least one input tensor")
        if not all(isinstance(t, torch.Tensor) and t.is_cuda for t in example_inputs):
            raise ValueError("GraphedStep inputs must be CUDA tensors")
        self.fn = fn
        self.static_inputs = [self._clone(t) for t in example_inputs]
        side = torch.cuda.Stream(device=self.static_inputs[0].device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(max(0, warmup)):
                fn(*self.static_inputs)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool):
            self.static_outputs = fn(*self.static_inputs)
        self.replays = 0

    @staticmethod
    def _clone(t: torch.Tensor) -> torch.Tensor:
        fmt = torch.channels_last if t.dim() == 4 and t.is_contiguous(memory_format=torch.channels_last) \
            and not t.is_contiguous() else torch.contiguous_format
        return t.detach().clone(memory_format=fmt)

    def __call__(self, *inputs: torch.Tensor):
        if len(inputs) != len(self.static_inputs):
            raise ValueError(f"expected {len(self.static_inputs)} inputs, got {len(inputs)}")
        for dst, src in zip(self.static_inputs, inputs):
            if src is not dst:
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        self.replays += 1
        return self.static_outputs

    def pool(self):
        """The graph's memory pool (pass it to another GraphedStep to share)."""
        return self.graph.pool()
