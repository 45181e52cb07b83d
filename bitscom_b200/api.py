"""High-level API: :class:`LowBitGroup`.

Same constructor, attributes and collective methods as reference
python/bitscom/api.py:29-525, with the same dispatch of ``all_reduce``:

1. ``local_group`` only (single node), <8 bits, SUM: fp all-reduce on the local
   group, or the low-bit all-reduce on it with ``local_quantize=True``
   (reference :95-112);
2. ``local_group`` + ``inter_group``: hierarchical pipeline-A with the
   dual-stream scheduler (:114-125, parallel/pipeline.py);
3. <8 bits, world > 1, SUM: the low-bit all-reduce (:127-131);
4. otherwise an fp all-reduce, after a quantise/dequantise roundtrip when
   ``simulate_quantization`` is set (:133-139).

The low-bit all-reduce of CUDA tensors runs the fused sm_100a NVLink kernel
(one launch: quantise + pack + peer stores + dequantise-reduce + requantise +
broadcast + unpack) whenever the group's ranks share a node with peer access;
otherwise (CPU tensors, multi-node groups) it runs the staged path with the
reference's exact arithmetic (one scale per rank, per-shard packing,
all-to-all, fp32 dequantise-sum, requantise, all-gather), with scales kept on
the device so the CUDA variant never syncs the host.

Additions: ``error_feedback`` (residual carried across calls), ``fp8``
(block-scaled E4M3 wire format for 8-bit), low-bit ``reduce_scatter_tensor`` /
``all_gather_into_tensor`` (the reference only simulated these), ``algo``.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _ext
from .ops.quant import pack_codes, quantize_codes, quantize_pack, unpack_dequant
from .parallel import pipeline as _pipeline
from .parallel.comm import Communicator
from .quantization import (
    SUPPORTED_BITWIDTHS,
    CompressedTensor,
    compress_tensor,
    decompress_tensor,
    packed_nbytes,
    roundtrip_tensor,
)

_FUSED_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


class _ImmediateWork:
    """Work-like handle of a collective that is already ordered on the caller's stream."""

    def __init__(self, result: Optional[torch.Tensor] = None):
        self._result = result

    def wait(self, timeout=None):
        return True

    def is_completed(self):
        return True

    def get_future(self):
        fut = torch.futures.Future()
        fut.set_result([self._result] if self._result is not None else [])
        return fut


class LowBitGroup:
    """Low-bit collectives over a torch.distributed process group.

    Args:
        bitwidth: 1, 2, 4, 8, 12 or 16.
        process_group: group to use (default: the default group).
        simulate_quantization: roundtrip through quantisation before the fp
            collective on paths that are not compressed.
        stochastic_rounding: stochastic rounding in the low-bit paths.
        error_feedback: carry the quantisation residual of each tensor across
            calls (keyed by ``ef_key`` or by storage pointer and size).
        fp8: 8-bit collectives use the block-scaled E4M3 wire format and are
            compressed (the reference leaves 8-bit uncompressed).
        algo: "auto", "oneshot" or "twoshot" for the fused all-reduce.
        use_fused: allow the fused NVLink kernels (default True).
    """

    def __init__(
        self,
        bitwidth: int = 4,
        process_group: Optional[dist.ProcessGroup] = None,
        simulate_quantization: bool = False,
        stochastic_rounding: bool = False,
        *,
        error_feedback: bool = False,
        fp8: bool = False,
        algo: str = "auto",
        use_fused: bool = True,
        seed: int = 0x5EED,
    ):
        if bitwidth not in SUPPORTED_BITWIDTHS:
            raise ValueError(f"bitwidth must be one of {SUPPORTED_BITWIDTHS}, got {bitwidth}")
        self.bitwidth = bitwidth
        self.pg = process_group or dist.distributed_c10d._get_default_group()
        self.simulate_quantization = simulate_quantization
        self.stochastic_rounding = stochastic_rounding
        self.error_feedback = error_feedback
        self.fp8 = fp8
        self.algo = algo
        self.use_fused = use_fused
        self.seed = int(seed)
        self._calls = 0
        # Error-feedback residuals by key: the caller's ``ef_key``, or
        # ("auto", i) for the i-th distinct tensor (storage, offset, size)
        # all-reduced without a key, so a resumed run that issues its calls in
        # the same order finds its residuals again.
        self._residuals: Dict[object, torch.Tensor] = {}
        self._auto_keys: Dict[tuple, int] = {}
        self._pending: Dict[object, torch.Tensor] = {}  # restored, not used yet

    # ------------------------------------------------------------------ info
    @property
    def rank(self) -> int:
        return dist.get_rank(self.pg)

    @property
    def world_size(self) -> int:
        return dist.get_world_size(self.pg)

    @property
    def _compress_8bit(self) -> bool:
        return self.fp8 and self.bitwidth == 8

    def _communicator(self, group, t: torch.Tensor) -> Optional[Communicator]:
        if not (self.use_fused and t.is_cuda and t.dtype in _FUSED_DTYPES and _ext.available()):
            return None
        return Communicator.for_group(group, t.device.index)

    def _residual(self, t: torch.Tensor, key=None) -> Optional[torch.Tensor]:
        if not self.error_feedback:
            return None
        k = key
        if k is None:
            ident = (t.untyped_storage().data_ptr(), t.storage_offset(), t.numel(), str(t.device))
            idx = self._auto_keys.setdefault(ident, len(self._auto_keys))
            k = ("auto", idx)
        r = self._residuals.get(k)
        if r is None and k in self._pending:
            r = self._pending.pop(k)
            if r.numel() == t.numel():
                r = self._residuals[k] = r.to(device=t.device, dtype=torch.float32).contiguous()
        if r is None or r.numel() != t.numel() or r.device != t.device:
            r = torch.zeros(t.numel(), dtype=torch.float32, device=t.device)
            self._residuals[k] = r
        return r

    def _next_offset(self) -> int:
        self._calls += 1
        return self._calls

    # ---------------------------------------------------------- all-reduce
    def all_reduce(
        self,
        tensor: torch.Tensor,
        op=dist.ReduceOp.SUM,
        async_op: bool = False,
        local_group: Optional[dist.ProcessGroup] = None,
        inter_group: Optional[dist.ProcessGroup] = None,
        chunk_size: Optional[int] = None,
        local_quantize: bool = False,
        *,
        ef_key=None,
    ):
        """Low-bit all-reduce; see the module docstring for the dispatch."""
        if local_group is not None and inter_group is None and self.bitwidth < 8 and op == dist.ReduceOp.SUM:
            if local_quantize:
                flat = tensor.contiguous().view(-1)
                reduced = self._lowbit_allreduce_via_alltoall_group(flat, local_group).view_as(tensor)
                tensor.copy_(reduced.to(dtype=tensor.dtype))
            else:
                dist.all_reduce(tensor, op=op, group=local_group)
            return _ImmediateWork(tensor) if async_op else None

        if self._should_use_pipeline_a(op, local_group, inter_group):
            self._hierarchical_lowbit_allreduce_pipeline_a(
                tensor,
                local_group=local_group,
                inter_group=inter_group,
                chunk_size=chunk_size,
                local_quantize=local_quantize,
            )
            return _ImmediateWork(tensor) if async_op else None

        if self._should_use_lowbit_path(op):
            self._lowbit_allreduce_via_alltoall(tensor, ef_key=ef_key)
            return _ImmediateWork(tensor) if async_op else None

        if self.simulate_quantization:
            tensor.copy_(roundtrip_tensor(tensor, self.bitwidth))
        work = dist.all_reduce(tensor, op=op, group=self.pg, async_op=True)
        if not async_op:
            work.wait()
            return None
        return work

    def _should_use_lowbit_path(self, op) -> bool:
        return (self.bitwidth < 8 or self._compress_8bit) and self.world_size > 1 and op == dist.ReduceOp.SUM

    def _should_use_pipeline_a(self, op, local_group, inter_group) -> bool:
        return local_group is not None and inter_group is not None and self.bitwidth < 8 and op == dist.ReduceOp.SUM

    def _should_use_dual_stream_pipeline(self, *, is_cuda: bool, local_size: int, global_size: int) -> bool:
        return _pipeline.should_use_dual_stream(is_cuda=is_cuda, local_size=local_size, global_size=global_size)

    def _split_flat_chunks(self, flat: torch.Tensor, chunk_size: int) -> List[torch.Tensor]:
        return _pipeline.split_chunks(flat, chunk_size)

    def _lowbit_allreduce_via_alltoall(self, tensor: torch.Tensor, *, ef_key=None) -> None:
        flat = tensor.contiguous().view(-1)
        comm = self._communicator(self.pg, flat)
        if comm is not None:
            comm.all_reduce(
                flat,
                bits=self.bitwidth,
                fmt="e4m3" if self._compress_8bit else "int",
                residual=self._residual(tensor, ef_key),
                stochastic_rounding=self.stochastic_rounding,
                stochastic_requant=self.stochastic_rounding,
                seed=self.seed,
                offset=self._next_offset(),
                algo=self.algo,
            )
            if flat.data_ptr() != tensor.data_ptr():
                tensor.copy_(flat.view_as(tensor))
            return
        restored = self._staged_allreduce(flat, self.pg, self._residual(tensor, ef_key)).view_as(tensor)
        tensor.copy_(restored.to(dtype=tensor.dtype))

    def _lowbit_allreduce_via_alltoall_group(self, flat: torch.Tensor, group) -> torch.Tensor:
        """Low-bit SUM all-reduce of a flat tensor over ``group``; returns the
        reduced values (fp32 on the staged path, the input dtype when fused)."""
        if flat.numel() == 0:
            return flat
        comm = self._communicator(group, flat)
        if comm is not None:
            out = torch.empty_like(flat)
            comm.all_reduce(
                flat.contiguous(),
                out=out,
                bits=self.bitwidth,
                fmt="e4m3" if self._compress_8bit else "int",
                stochastic_rounding=self.stochastic_rounding,
                stochastic_requant=self.stochastic_rounding,
                seed=self.seed,
                offset=self._next_offset(),
                algo=self.algo,
            )
            return out
        return self._staged_allreduce(flat, group, None)

    def _staged_allreduce(self, flat: torch.Tensor, group, residual: Optional[torch.Tensor]) -> torch.Tensor:
        """Reference C8 arithmetic (api.py:179-257) without host syncs."""
        bits = 8 if self.bitwidth > 8 else self.bitwidth
        world = dist.get_world_size(group)
        n = int(flat.numel())
        if n == 0:
            return flat
        x = flat.to(torch.float32)
        if residual is not None:
            x = x + residual
        pad = (world - n % world) % world
        if pad:
            x = torch.cat([x, x.new_zeros(pad)])
        shard = x.numel() // world
        sr = self.stochastic_rounding
        # Philox keys of the two roundings: the group's seed, this rank and
        # the phase, so stochastic rounding is reproducible (and resumable)
        # and independent across ranks.
        rank = dist.get_rank(group) if world > 1 else 0
        seed1 = (self.seed ^ (rank << 40) ^ (1 << 56)) & (2**63 - 1)
        seed2 = (self.seed ^ (rank << 40) ^ (2 << 56)) & (2**63 - 1)
        q, scale = quantize_codes(x, bits, stochastic=sr, seed=seed1, offset=self._next_offset())
        if residual is not None:
            residual.copy_((x - q.to(torch.float32) * scale)[:n])
        send = torch.cat([pack_codes(q[s * shard : (s + 1) * shard], bits) for s in range(world)])
        per = send.numel() // world
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
        scales_in = torch.empty(world, dtype=torch.float32, device=x.device)
        dist.all_to_all_single(scales_in, scale.expand(world).contiguous(), group=group)
        local = torch.zeros(shard, dtype=torch.float32, device=x.device)
        for s in range(world):
            local.add_(unpack_dequant(recv[s * per : (s + 1) * per], bits, shard, scales_in[s : s + 1]))
        packed_r, scale_r = quantize_pack(local, bits, stochastic=sr, seed=seed2, offset=self._next_offset())
        gathered = torch.empty(world * packed_r.numel(), dtype=torch.uint8, device=x.device)
        dist.all_gather_into_tensor(gathered, packed_r, group=group)
        scales_r = torch.empty(world, dtype=torch.float32, device=x.device)
        dist.all_gather_into_tensor(scales_r, scale_r.view(1), group=group)
        pr = packed_r.numel()
        out = torch.cat(
            [unpack_dequant(gathered[s * pr : (s + 1) * pr], bits, shard, scales_r[s : s + 1]) for s in range(world)]
        )
        return out[:n]

    def _hierarchical_lowbit_allreduce_pipeline_a(
        self, tensor, *, local_group, inter_group, chunk_size, local_quantize
    ) -> None:
        _pipeline.hierarchical_allreduce(
            self, tensor, local_group=local_group, inter_group=inter_group,
            chunk_size=chunk_size, local_quantize=local_quantize,
        )

    # ----------------------------------------------- gather / scatter family
    def all_gather(self, tensor_list: List[torch.Tensor], tensor: torch.Tensor, async_op: bool = False):
        """All-gather into a list; low-bit on the fused path when compressed widths
        are configured, else fp (with optional simulation, reference :466-479)."""
        comm = self._communicator(self.pg, tensor) if self._lowbit_gather() else None
        if comm is not None and all(t.numel() == tensor.numel() and t.dtype == tensor.dtype for t in tensor_list):
            out = torch.empty(tensor.numel() * self.world_size, dtype=tensor.dtype, device=tensor.device)
            self.all_gather_into_tensor(out, tensor)
            for r, t in enumerate(tensor_list):
                t.copy_(out[r * tensor.numel() : (r + 1) * tensor.numel()].view_as(t))
            return _ImmediateWork(out) if async_op else None
        if self.simulate_quantization:
            tensor.copy_(roundtrip_tensor(tensor, self.bitwidth))
        work = dist.all_gather(tensor_list, tensor, group=self.pg, async_op=True)
        if not async_op:
            work.wait()
            return None
        return work

    def reduce_scatter(self, output: torch.Tensor, input_list: List[torch.Tensor], op=dist.ReduceOp.SUM,
                       async_op: bool = False):
        """Reduce-scatter from a list (reference :481-498)."""
        comm = self._communicator(self.pg, output) if (self._lowbit_gather() and op == dist.ReduceOp.SUM) else None
        if comm is not None and all(t.numel() == output.numel() and t.dtype == output.dtype for t in input_list):
            self.reduce_scatter_tensor(output, torch.cat([t.reshape(-1) for t in input_list]))
            return _ImmediateWork(output) if async_op else None
        if self.simulate_quantization:
            for t in input_list:
                t.copy_(roundtrip_tensor(t, self.bitwidth))
        work = dist.reduce_scatter(output, input_list, op=op, group=self.pg, async_op=True)
        if not async_op:
            work.wait()
            return None
        return work

    def _lowbit_gather(self) -> bool:
        return self.bitwidth < 8 or self._compress_8bit

    def reduce_scatter_tensor(self, output: torch.Tensor, input: torch.Tensor, *, average: bool = False,
                              ef_key=None) -> torch.Tensor:
        """Low-bit SUM (or mean) reduce-scatter of ``input`` (world*n) into ``output`` (n).

        Fused kernel when available; otherwise a simulated roundtrip + fp
        reduce-scatter.  Compresses at every bitwidth (8-bit int codes unless
        ``fp8``)."""
        comm = self._communicator(self.pg, input)
        if comm is not None:
            comm.reduce_scatter(
                output.view(-1), input.contiguous().view(-1), bits=self.bitwidth,
                fmt="e4m3" if self._compress_8bit else "int",
                residual=self._residual(input, ef_key), stochastic_rounding=self.stochastic_rounding,
                seed=self.seed, offset=self._next_offset(),
                post_scale=1.0 / self.world_size if average else 1.0,
            )
            return output
        x = input
        if self.bitwidth < 16:
            x = roundtrip_tensor(input, self.bitwidth)
        dist.reduce_scatter_tensor(output, x, op=dist.ReduceOp.AVG if average else dist.ReduceOp.SUM, group=self.pg)
        return output

    def all_gather_into_tensor(self, output: torch.Tensor, input: torch.Tensor, *, ef_key=None) -> torch.Tensor:
        """Low-bit all-gather of ``input`` (n) into ``output`` (world*n)."""
        comm = self._communicator(self.pg, input)
        if comm is not None:
            comm.all_gather(
                output.view(-1), input.contiguous().view(-1), bits=self.bitwidth,
                fmt="e4m3" if self._compress_8bit else "int",
                residual=self._residual(input, ef_key), stochastic_rounding=self.stochastic_rounding,
                seed=self.seed, offset=self._next_offset(),
            )
            return output
        x = roundtrip_tensor(input, self.bitwidth) if self.bitwidth < 16 else input
        dist.all_gather_into_tensor(output, x.contiguous(), group=self.pg)
        return output

    def broadcast(self, tensor: torch.Tensor, src: int = 0, async_op: bool = False):
        """fp broadcast (never compressed, reference :500-511)."""
        work = dist.broadcast(tensor, src=src, group=self.pg, async_op=True)
        if not async_op:
            work.wait()
            return None
        return work

    # ------------------------------------------------------------ compress
    def compress(self, tensor: torch.Tensor) -> CompressedTensor:
        return compress_tensor(tensor, self.bitwidth)

    def decompress(self, compressed: CompressedTensor, *, dtype: Optional[torch.dtype] = None,
                   device: Optional[torch.device] = None) -> torch.Tensor:
        return decompress_tensor(compressed, dtype=dtype, device=device)

    # --------------------------------------------------------- EF state
    def state_dict(self) -> dict:
        """Error-feedback residuals and the stochastic-rounding call counter.

        Residuals are saved under their ``ef_key``, or under ("auto", i) for
        the i-th distinct tensor all-reduced without one."""
        res = dict(self._pending)
        res.update(self._residuals)
        return {"calls": self._calls, "residuals": {k: v.detach().cpu().clone() for k, v in res.items()}}

    def load_state_dict(self, state: dict) -> None:
        """Restore a :meth:`state_dict`: each residual is attached to its key's
        tensor on that tensor's first all-reduce (same ``ef_key``, or the same
        position in the order of first use), so resumed training continues
        bit-identically."""
        self._calls = int(state.get("calls", 0))
        self._residuals = {}
        self._auto_keys = {}
        self._pending = {k: v.detach().clone() for k, v in state.get("residuals", {}).items()}


__all__ = ["LowBitGroup", "packed_nbytes"]
