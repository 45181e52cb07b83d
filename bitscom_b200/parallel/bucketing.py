"""Persistent gradient buckets for data parallelism without DDP.

The reference's end-to-end benchmarks synchronise gradients by hand after
backward: every step they concatenate all gradients into new flat tensors,
all-reduce them, divide by the world size and copy the slices back
(reference benchmarks/multimodel_stochastic_e2e_curve.py:207-244).
:class:`GradBucketer` does the same job without the per-step allocations and
copies: it assigns parameters to buckets once (reverse registration order,
the order in which backward produces gradients, like DDP), allocates one
flat buffer per bucket and makes every ``param.grad`` a view into its
bucket, so backward accumulates straight into the buffers.  ``sync()`` then
runs one low-bit all-reduce per bucket (the fused kernel on CUDA tensors,
with a persistent error-feedback residual per bucket) and averages.
"""

from __future__ import annotations

from typing import TYPE_CHECKING, Iterable, List, Optional

import torch

if TYPE_CHECKING:  # the api module imports this package
    from ..api import LowBitGroup


class GradBucketer:
    """Flat gradient buckets with low-bit all-reduce.

    Args:
        params: the parameters whose gradients are synchronised (those with
            ``requires_grad``).
        group: the :class:`LowBitGroup` that reduces the buckets (default: a
            4-bit group with error feedback over the default process group).
        bucket_mb: bucket capacity in MiB of gradient bytes.
        average: divide the reduced gradients by the world size.

    Buckets hold one dtype each (a dtype change starts a new bucket).  The
    gradients stay views into the buckets as long as nobody replaces
    ``param.grad`` (use ``zero_grad(set_to_none=False)``, or
    :meth:`zero_grad` here).
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], group: Optional["LowBitGroup"] = None,
                 bucket_mb: float = 25.0, average: bool = True):
        if group is None:
            from ..api import LowBitGroup

            group = LowBitGroup(bitwidth=4, error_feedback=True)
        self.group = group
        self.average = average
        ps = [p for p in params if p.requires_grad]
        if not ps:
            raise ValueError("no parameters require gradients")
        cap = max(1, int(bucket_mb * 2**20))
        self.buckets: List[List[torch.nn.Parameter]] = []
        cur: List[torch.nn.Parameter] = []
        size = 0
        for p in reversed(ps):
            nbytes = p.numel() * p.element_size()
            if cur and (size + nbytes > cap or p.dtype != cur[0].dtype or p.device != cur[0].device):
                self.buckets.append(cur)
                cur, size = [], 0
            cur.append(p)
            size += nbytes
        if cur:
            self.buckets.append(cur)
        self.buffers: List[torch.Tensor] = []
        with torch.no_grad():
            for b in self.buckets:
                buf = torch.zeros(sum(p.numel() for p in b), dtype=b[0].dtype, device=b[0].device)
                off = 0
                for p in b:
                    n = p.numel()
                    view = buf[off : off + n].view_as(p)
                    if p.grad is not None:
                        view.copy_(p.grad)
                    p.grad = view
                    off += n
                self.buffers.append(buf)

    def _rebind(self) -> None:
        """Point any gradient that was replaced (e.g. set to None) back into its bucket."""
        for b, buf in zip(self.buckets, self.buffers):
            off = 0
            for p in b:
                n = p.numel()
                view = buf[off : off + n].view_as(p)
                if p.grad is None or p.grad.data_ptr() != view.data_ptr():
                    with torch.no_grad():
                        if p.grad is not None:
                            view.copy_(p.grad)
                        else:
                            view.zero_()
                    p.grad = view
                off += n

    @torch.no_grad()
    def sync(self) -> None:
        """All-reduce every bucket (low-bit, one call per bucket) and average."""
        self._rebind()
        world = self.group.world_size
        for i, buf in enumerate(self.buffers):
            self.group.all_reduce(buf, ef_key=("grad_bucket", i))
            if self.average and world > 1:
                buf.div_(world)

    @torch.no_grad()
    def zero_grad(self) -> None:
        for buf in self.buffers:
            buf.zero_()
        self._rebind()

    def num_buckets(self) -> int:
        return len(self.buffers)
