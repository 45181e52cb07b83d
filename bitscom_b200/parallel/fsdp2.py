"""Low-bit collectives for PyTorch FSDP2 (``fully_shard``).

Two ways to run FSDP2's parameter all-gathers and gradient reduce-scatters
on the fused low-bit kernels:

1. on a ``lowbit`` process group: FSDP2's default collectives call the
   backend's ``_allgather_base`` / ``_reduce_scatter_base``, which run the
   fused kernels (``bitscom.init(bitwidth=8, force_lowbit=True)``).  Error
   feedback there is keyed by buffer, which FSDP2 reallocates per module and
   step, so it is best left off on that path;
2. :func:`enable_lowbit_fsdp2` on modules already wrapped by
   ``fully_shard`` over ANY process group (NCCL included): it installs a
   :class:`LowBitAllGather` and a :class:`LowBitReduceScatter` per FSDP
   module (``FSDPModule.set_custom_all_gather`` /
   ``set_custom_reduce_scatter``), each calling the fused kernels through a
   :class:`~bitscom_b200.parallel.comm.Communicator` of that group, on the
   stream FSDP2 calls them on (its all-gather / reduce-scatter streams, so
   FSDP2's own prefetching and overlap are kept).  Each instance owns its
   module's error-feedback residual, so residuals never mix across modules.

The reference forwards reduce-scatter and all-gather to NCCL uncompressed
(cpp/src/process_group_lowbit.cc:351-369); this is its low-bit sharded-data-
parallel counterpart.  Inputs that are not fp32/bf16/fp16 (FSDP2 flattens
mixed-dtype modules to uint8) and groups without a peer-to-peer workspace
fall back to the group's own collective.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .comm import Communicator

_FUSED = (torch.float32, torch.bfloat16, torch.float16)

try:  # FSDP2 custom-collective interfaces (torch >= 2.8)
    from torch.distributed.fsdp._fully_shard._fsdp_api import AllGather as _AllGatherBase
    from torch.distributed.fsdp._fully_shard._fsdp_api import ReduceScatter as _ReduceScatterBase
except ImportError:  # pragma: no cover - older torch
    _AllGatherBase = object
    _ReduceScatterBase = object


class _LowBitComm:
    def __init__(self, bits: int, fmt: str, error_feedback: bool, residual_dtype: torch.dtype, seed: int):
        if fmt == "e4m3" and bits != 8:
            raise ValueError("the E4M3 format needs bits=8")
        self.bits = bits
        self.fmt = fmt
        self.error_feedback = error_feedback
        self.residual_dtype = residual_dtype
        self.seed = seed
        self.calls = 0
        self.fused_calls = 0
        self.residual: Optional[torch.Tensor] = None

    def allocate(self, size, *, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        return torch.empty(*size, dtype=dtype, device=device)

    def _comm(self, group, t: torch.Tensor) -> Optional[Communicator]:
        if not (t.is_cuda and t.dtype in _FUSED and t.is_contiguous()):
            return None
        return Communicator.for_group(group, t.device.index)

    def _residual_for(self, t: torch.Tensor) -> Optional[torch.Tensor]:
        if not self.error_feedback:
            return None
        if self.residual is None or self.residual.numel() != t.numel() or self.residual.device != t.device:
            self.residual = torch.zeros(t.numel(), dtype=self.residual_dtype, device=t.device)
        return self.residual

    def state_dict(self) -> dict:
        return {"calls": self.calls, "residual": None if self.residual is None else self.residual.detach().cpu()}

    def load_state_dict(self, state: dict) -> None:
        self.calls = int(state.get("calls", 0))
        r = state.get("residual")
        self.residual = None if r is None else r.clone()


class LowBitAllGather(_LowBitComm, _AllGatherBase):
    """FSDP2 parameter all-gather on the fused low-bit kernel."""

    def __call__(self, output_tensor, input_tensor, group, async_op: bool = False):
        comm = self._comm(group, input_tensor)
        if comm is None:
            return dist.all_gather_into_tensor(output_tensor, input_tensor, group=group, async_op=async_op)
        self.calls += 1
        self.fused_calls += 1
        res = self._residual_for(input_tensor)
        comm.all_gather(output_tensor.view(-1), input_tensor.view(-1), bits=self.bits, fmt=self.fmt, residual=res,
                        seed=self.seed, offset=self.calls)
        return None  # ordered on the calling stream; FSDP2 waits on its event


class LowBitReduceScatter(_LowBitComm, _ReduceScatterBase):
    """FSDP2 gradient reduce-scatter (SUM or AVG) on the fused low-bit kernel."""

    def __call__(self, output_tensor, input_tensor, group, op=None, async_op: bool = False):
        comm = self._comm(group, input_tensor)
        sum_like = op is None or op in (dist.ReduceOp.SUM, dist.ReduceOp.AVG)
        if comm is None or not sum_like:
            return dist.reduce_scatter_tensor(output_tensor, input_tensor, op=op, group=group, async_op=async_op)
        self.calls += 1
        self.fused_calls += 1
        world = dist.get_world_size(group)
        comm.reduce_scatter(output_tensor.view(-1), input_tensor.view(-1), bits=self.bits, fmt=self.fmt,
                            residual=self._residual_for(input_tensor), seed=self.seed, offset=self.calls,
                            post_scale=1.0 / world if op == dist.ReduceOp.AVG else 1.0)
        return None


def enable_lowbit_fsdp2(
    model: torch.nn.Module,
    *,
    bits: int = 8,
    fmt: str = "int",
    error_feedback: bool = True,
    gather_error_feedback: bool = False,
    residual_dtype: torch.dtype = torch.bfloat16,
    seed: int = 0x5EED,
    group: Optional[dist.ProcessGroup] = None,
) -> dict:
    """Install low-bit all-gather / reduce-scatter comms on every FSDP2 module
    of ``model`` (call after ``fully_shard``).  Gradient reduce-scatters carry
    an error-feedback residual per module when ``error_feedback``; parameter
    all-gathers quantise the current shard without one unless
    ``gather_error_feedback``.  ``group``: the FSDP mesh's process group, to
    set up its peer-to-peer workspace now (a collective over the group)
    rather than at the first all-gather.  Returns ``{module_name:
    (all_gather, reduce_scatter)}``."""
    from torch.distributed.fsdp import FSDPModule

    if group is not None and torch.cuda.is_available():
        Communicator.for_group(group, torch.cuda.current_device())

    installed = {}
    for name, mod in model.named_modules():
        if not isinstance(mod, FSDPModule):
            continue
        ag = LowBitAllGather(bits, fmt, gather_error_feedback, residual_dtype, seed)
        rs = LowBitReduceScatter(bits, fmt, error_feedback, residual_dtype, seed)
        mod.set_custom_all_gather(ag)
        mod.set_custom_reduce_scatter(rs)
        installed[name] = (ag, rs)
    if not installed:
        raise ValueError("no FSDP2 module found: call fully_shard first")
    return installed


__all__ = ["LowBitAllGather", "LowBitReduceScatter", "enable_lowbit_fsdp2"]
