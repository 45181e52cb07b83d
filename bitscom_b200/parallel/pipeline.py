"""Hierarchical "pipeline-A" all-reduce and its dual-stream chunk scheduler.

Reference: python/bitscom/api.py:259-459.  A flat tensor is cut into chunks
and every chunk goes through three phases:

* **local**    intra-node stage: fp ``reduce`` to the local leader (default), or
               a quantised all-gather and a leader-side dequantise-sum
               (``local_quantize=True``);
* **inter**    the leader runs the low-bit all-reduce on ``inter_group``
               (the fused NVLink kernel when the inter group shares a node,
               the staged low-bit path otherwise);
* **finalize** fp ``broadcast`` from the leader, or a quantised broadcast.

:class:`DualStreamScheduler` overlaps the phases of consecutive chunks on two
CUDA streams (intra: local+finalize, inter: inter) with the schedule
warm-up -> steady -> cool-down (reference api.py:400-459):

    warm-up : local(0), local(1) | inter(0)
    steady  : for i>=2: finalize(i-2) + local(i) on intra  ||  inter(i-1) on inter
    cool-down: finalize(n-2) | inter(n-1) | finalize(n-1)

It runs only when there is an inter-node stage (local group smaller than the
global group) and the data is on CUDA; otherwise chunks run sequentially.
Unlike the reference, the quantised phases here keep scales on the device
(no ``.item()`` host syncs), so the two streams really overlap, and every
kernel launches on the stream the phase runs on.
"""

from __future__ import annotations

from typing import Callable, List, Optional

import torch
import torch.distributed as dist

from ..ops.quant import quantize_pack, unpack_dequant


def should_use_dual_stream(*, is_cuda: bool, local_size: int, global_size: int) -> bool:
    """Dual-stream overlap only pays when an inter-node stage exists."""
    return bool(is_cuda) and local_size < global_size


def split_chunks(flat: torch.Tensor, chunk_size: int) -> List[torch.Tensor]:
    if chunk_size <= 0:
        raise ValueError(f"chunk_size must be > 0, got {chunk_size}")
    return [flat[s : s + chunk_size] for s in range(0, flat.numel(), chunk_size)]


class DualStreamScheduler:
    """Runs ``local``, ``inter`` and ``finalize`` callbacks over n chunks with
    the warm-up / steady / cool-down overlap schedule."""

    def __init__(self, device: torch.device):
        self.intra = torch.cuda.Stream(device=device)
        self.inter = torch.cuda.Stream(device=device)
        self.trace: List[str] = []  # (phase, chunk, stream) order, for tests

    def _on(self, stream, fn: Callable[[int], None], idx: int, tag: str) -> None:
        with torch.cuda.stream(stream):
            fn(idx)
        self.trace.append(f"{tag}{idx}@{'intra' if stream is self.intra else 'inter'}")

    def run(self, n: int, local: Callable[[int], None], inter: Callable[[int], None],
            finalize: Callable[[int], None]) -> None:
        if n == 0:
            return
        cur = torch.cuda.current_stream()
        self.intra.wait_stream(cur)
        self.inter.wait_stream(cur)
        ev_intra = [torch.cuda.Event() for _ in range(n)]
        ev_inter = [torch.cuda.Event() for _ in range(n)]

        def local_i(i):
            self._on(self.intra, local, i, "L")
            ev_intra[i].record(self.intra)

        def inter_i(i):
            self.inter.wait_event(ev_intra[i])
            self._on(self.inter, inter, i, "I")
            ev_inter[i].record(self.inter)

        def final_i(i):
            self.intra.wait_event(ev_inter[i])
            self._on(self.intra, finalize, i, "F")

        local_i(0)
        if n == 1:
            inter_i(0)
            final_i(0)
        else:
            local_i(1)
            inter_i(0)
            for i in range(2, n):  # steady state
                final_i(i - 2)
                local_i(i)
                inter_i(i - 1)
            final_i(n - 2)  # cool-down
            inter_i(n - 1)
            final_i(n - 1)
        cur.wait_stream(self.intra)
        cur.wait_stream(self.inter)


def hierarchical_allreduce(
    owner,
    tensor: torch.Tensor,
    *,
    local_group,
    inter_group,
    chunk_size: Optional[int],
    local_quantize: bool,
) -> None:
    """Pipeline-A all-reduce (SUM) of ``tensor`` in place.

    ``owner`` is the LowBitGroup (bitwidth, stochastic flag and its
    ``_lowbit_allreduce_via_alltoall_group`` for the inter stage).
    """
    flat = tensor.contiguous().view(-1)
    if flat.numel() == 0:
        return
    bits = owner.bitwidth
    sr = owner.stochastic_rounding
    chunk_elems = int(chunk_size) if chunk_size is not None else max(1, flat.numel() // 4)
    chunks = split_chunks(flat, chunk_elems)
    n = len(chunks)

    local_rank = dist.get_rank(local_group)
    local_size = dist.get_world_size(local_group)
    global_size = dist.get_world_size(owner.pg)
    leader_global = dist.get_global_rank(local_group, 0) if local_size > 0 else 0
    is_leader = local_rank == 0

    inter_in: List[Optional[torch.Tensor]] = [None] * n
    results: List[Optional[torch.Tensor]] = [None] * n
    shapes: List[int] = [c.numel() for c in chunks]

    def local_phase(i: int) -> None:
        c = chunks[i]
        if not local_quantize:
            dist.reduce(c, dst=leader_global, group=local_group, op=dist.ReduceOp.SUM)
            if is_leader:
                inter_in[i] = c.to(torch.float32)
            return
        packed, scale = quantize_pack(c, bits, stochastic=sr)
        gathered = torch.empty(local_size * packed.numel(), dtype=torch.uint8, device=c.device)
        dist.all_gather_into_tensor(gathered, packed, group=local_group)
        scales = torch.empty(local_size, dtype=torch.float32, device=c.device)
        dist.all_gather_into_tensor(scales, scale.view(1), group=local_group)
        if is_leader:
            acc = torch.zeros(c.numel(), dtype=torch.float32, device=c.device)
            per = packed.numel()
            for r in range(local_size):
                acc.add_(unpack_dequant(gathered[r * per : (r + 1) * per], bits, c.numel(), scales[r : r + 1]))
            inter_in[i] = acc

    def inter_phase(i: int) -> None:
        if is_leader:
            x = inter_in[i]
            if x.is_cuda:
                x.record_stream(torch.cuda.current_stream(x.device))
            results[i] = owner._lowbit_allreduce_via_alltoall_group(x, inter_group)

    def finalize_phase(i: int) -> None:
        c = chunks[i]
        if is_leader and results[i] is not None and results[i].is_cuda:
            results[i].record_stream(torch.cuda.current_stream(results[i].device))
        if not local_quantize:
            buf = results[i].to(c.dtype) if is_leader else torch.empty_like(c)
            dist.broadcast(buf, src=leader_global, group=local_group)
            c.copy_(buf)
            return
        nbytes = _packed_len(shapes[i], bits)
        if is_leader:
            packed, scale = quantize_pack(results[i], bits, stochastic=sr)
        else:
            packed = torch.empty(nbytes, dtype=torch.uint8, device=c.device)
            scale = torch.empty(1, dtype=torch.float32, device=c.device)
        dist.broadcast(packed, src=leader_global, group=local_group)
        dist.broadcast(scale, src=leader_global, group=local_group)
        c.copy_(unpack_dequant(packed, bits, c.numel(), scale).to(c.dtype))

    if should_use_dual_stream(is_cuda=flat.is_cuda, local_size=local_size, global_size=global_size):
        DualStreamScheduler(flat.device).run(n, local_phase, inter_phase, finalize_phase)
    else:
        for i in range(n):
            local_phase(i)
            inter_phase(i)
            finalize_phase(i)
    if flat.data_ptr() != tensor.data_ptr():
        tensor.copy_(flat.view_as(tensor))


def _packed_len(numel: int, bits: int) -> int:
    from ..quantization import packed_nbytes

    return packed_nbytes(numel, bits)
