"""Sharded data parallelism (ZeRO-3 style) over the fused low-bit
reduce-scatter and all-gather kernels.

The reference cannot do this: its ``reduce_scatter`` / ``all_gather`` are
forwarded to NCCL in full precision (reference
cpp/src/process_group_lowbit.cc:351-369) and ``LowBitGroup`` only simulates
quantisation for them (python/bitscom/api.py:466-498).

:class:`LowBitShardedDP` flattens every parameter of a module into one
padded fp32 vector.  Each rank owns one shard of it (its fp32 master copy
and the optimizer state); the module's parameters and gradients are views
into full-size working buffers.  One training step is:

1. forward / backward on the working parameters (under autocast as usual);
2. ``reduce_scatter`` of the flat gradient with the fused low-bit kernel
   (``rs_bits``, error feedback per rank, mean over ranks) into this rank's
   gradient shard;
3. the optimizer updates the fp32 master shard;
4. ``all_gather`` of the master shards with the fused low-bit kernel
   (``ag_bits``; error feedback on the quantised parameters, so the working
   copy tracks the master without drift) back into the working parameters.

Gathering the whole model at once fits B200 memory comfortably (GPT-2 medium:
1.4 GB of fp32 working parameters); the per-rank saving is the optimizer
state and master copy (1/W each).
"""

from __future__ import annotations

from typing import Callable, Iterable, List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .comm import Communicator

_ALIGN = 8192  # shard length granularity (one packed sub-chunk)


def _cpu_copy(obj):
    """Deep copy with every tensor cloned to host memory."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().to("cpu", copy=True)
    if isinstance(obj, dict):
        return {k: _cpu_copy(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_cpu_copy(v) for v in obj)
    return obj


class LowBitShardedDP(nn.Module):
    """Wraps ``module`` for sharded data-parallel training with low-bit
    reduce-scatter of gradients and low-bit all-gather of parameters.

    Args:
        module: the model (its parameters are re-pointed into flat buffers).
        optimizer_factory: ``params -> torch.optim.Optimizer``; called with the
            list ``[master_shard]`` (one fp32 tensor).
        process_group: group to shard over (default: the default group).
        rs_bits / ag_bits: wire bitwidths of the two collectives.
        fp8: use the block-scaled E4M3 format for 8-bit collectives.
        error_feedback: per-rank EF residuals for both collectives.
        stochastic_rounding: SR in the gradient reduce-scatter.
        use_fused: use the fused kernels (False: NCCL fp reduce-scatter /
            all-gather after a quantisation roundtrip, for comparison).
        max_ctas: CTAs per fused launch (0 = two per SM).
        residual_dtype: element type of the EF residuals (bf16, the default,
            or fp32; bf16 halves their HBM traffic at the same EF error).
    """

    def __init__(
        self,
        module: nn.Module,
        optimizer_factory: Callable[[List[torch.Tensor]], torch.optim.Optimizer],
        process_group: Optional[dist.ProcessGroup] = None,
        rs_bits: int = 8,
        ag_bits: int = 8,
        fp8: bool = False,
        error_feedback: bool = True,
        stochastic_rounding: bool = False,
        use_fused: bool = True,
        max_ctas: int = 0,
        residual_dtype: torch.dtype = torch.bfloat16,
    ):
        super().__init__()
        self.module = module
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.rs_bits, self.ag_bits = rs_bits, ag_bits
        self.fmt = "e4m3" if fp8 else "int"
        self.error_feedback = error_feedback
        self.stochastic_rounding = stochastic_rounding
        self.max_ctas = max_ctas
        params = [p for p in module.parameters() if p.requires_grad]
        if not params:
            raise ValueError("module has no trainable parameters")
        dev = params[0].device
        self.device = dev
        numel = sum(p.numel() for p in params)
        per = -(-numel // self.world)
        self.shard = -(-per // _ALIGN) * _ALIGN
        total = self.shard * self.world
        self.numel = numel
        # Working parameters and gradients (full size, fp32) + master shard.
        self.flat_param = torch.zeros(total, dtype=torch.float32, device=dev)
        self.flat_grad = torch.zeros(total, dtype=torch.float32, device=dev)
        off = 0
        self._views = []
        with torch.no_grad():
            for p in params:
                n = p.numel()
                self.flat_param[off : off + n].copy_(p.detach().reshape(-1).float())
                p.data = self.flat_param[off : off + n].view_as(p)
                p.grad = self.flat_grad[off : off + n].view_as(p)
                self._views.append((p, off, n))
                off += n
        # Every rank starts from rank 0's parameters.
        dist.broadcast(self.flat_param, src=dist.get_global_rank(process_group, 0) if process_group else 0,
                       group=process_group)
        lo = self.rank * self.shard
        self.master = self.flat_param[lo : lo + self.shard].clone().requires_grad_(True)
        self.master.grad = torch.zeros_like(self.master)
        self.optimizer = optimizer_factory([self.master])
        if residual_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("residual_dtype must be torch.float32 or torch.bfloat16")
        self.rs_residual = torch.zeros(total, dtype=residual_dtype, device=dev) if error_feedback else None
        self.ag_residual = torch.zeros(self.shard, dtype=residual_dtype, device=dev) if error_feedback else None
        self.comm = None
        if use_fused and dev.type == "cuda":
            self.comm = (Communicator.create_local(dev.index) if self.world == 1
                         else Communicator.for_group(process_group, dev.index))
        self._calls = 0

    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    def parameters_for_clipping(self) -> Iterable[torch.Tensor]:
        return [self.master]

    @torch.no_grad()
    def step(self) -> None:
        """Reduce-scatter gradients, update the master shard, all-gather parameters."""
        self._calls += 1
        g_shard = self.master.grad
        if self.comm is not None:
            self.comm.reduce_scatter(
                g_shard, self.flat_grad, bits=self.rs_bits, fmt=self.fmt, residual=self.rs_residual,
                stochastic_rounding=self.stochastic_rounding, offset=2 * self._calls,
                post_scale=1.0 / self.world, max_ctas=self.max_ctas,
            )
        else:
            from ..quantization import roundtrip_tensor

            x = roundtrip_tensor(self.flat_grad, self.rs_bits) if self.rs_bits < 16 else self.flat_grad
            dist.reduce_scatter_tensor(g_shard, x, op=dist.ReduceOp.AVG, group=self.pg)
        self.optimizer.step()
        if self.comm is not None:
            self.comm.all_gather(
                self.flat_param, self.master.detach(), bits=self.ag_bits, fmt=self.fmt, residual=self.ag_residual,
                offset=2 * self._calls + 1, max_ctas=self.max_ctas,
            )
        else:
            from ..quantization import roundtrip_tensor

            m = roundtrip_tensor(self.master.detach(), self.ag_bits) if self.ag_bits < 16 else self.master.detach()
            dist.all_gather_into_tensor(self.flat_param, m.contiguous(), group=self.pg)
        self.flat_grad.zero_()

    def zero_grad(self, set_to_none: bool = False) -> None:
        self.flat_grad.zero_()

    def state_dict_shard(self) -> dict:
        """This rank's master shard, its slice of the working parameters (the
        values every rank decoded from the last low-bit all-gather), optimizer
        state and EF residuals."""
        lo = self.rank * self.shard
        return {
            "master": self.master.detach().cpu(),
            "working": self.flat_param[lo : lo + self.shard].cpu(),
            # a copy: the optimizer's state_dict() refers to the live state
            # tensors, which later steps update in place
            "optimizer": _cpu_copy(self.optimizer.state_dict()),
            "rs_residual": None if self.rs_residual is None else self.rs_residual.cpu(),
            "ag_residual": None if self.ag_residual is None else self.ag_residual.cpu(),
            "calls": self._calls,
        }

    @torch.no_grad()
    def load_state_dict_shard(self, state: dict) -> None:
        """Restore what :meth:`state_dict_shard` saved on this rank, then
        all-gather the master shards into the working parameters (every rank
        calls this, since the gather is collective)."""
        master = state["master"]
        if master.numel() != self.master.numel():
            raise ValueError(f"checkpoint shard has {master.numel()} elements, this rank owns {self.master.numel()}")
        self.master.copy_(master.to(self.master.device))
        self.optimizer.load_state_dict(state["optimizer"])
        for name in ("rs_residual", "ag_residual"):
            mine, saved = getattr(self, name), state.get(name)
            if mine is not None:
                if saved is None:
                    mine.zero_()
                else:
                    mine.copy_(saved.to(mine.device, mine.dtype))
        self._calls = int(state.get("calls", 0))
        # Working parameters: the saved decoded slices (exact resume), or the
        # fp32 masters for a checkpoint without them.
        work = state.get("working")
        src = self.master.detach() if work is None else work.to(self.device, torch.float32)
        dist.all_gather_into_tensor(self.flat_param, src.contiguous(), group=self.pg)
        self.flat_grad.zero_()
