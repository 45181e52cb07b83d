"""Python front end of the fused low-bit collectives (``LowBitComm``).

:class:`Communicator` binds one native ``LowBitComm`` (a symmetric NVLink
workspace, see csrc/runtime/comm.h) to a torch.distributed process group of
ANY backend (nccl, gloo or lowbit): the 64-byte CUDA IPC handles are exchanged
with ``all_gather_object`` over that group, every rank maps every peer, and
the group agrees all-or-nothing whether the peer-to-peer path is usable.  When
it is not (ranks on different hosts, two ranks on one GPU, no peer access),
:meth:`Communicator.for_group` returns ``None`` and callers use their staged
fallback.

All collectives run on the caller's current CUDA stream and return without a
host sync.  Calls on one communicator must be issued in the same order on
every rank (like NCCL).
"""

from __future__ import annotations

import contextlib
import os
import socket
import threading
from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

from .. import _ext

ALGOS = {"auto": 0, "twoshot": 1, "oneshot": 2}
FMTS = {"int": 0, "e4m3": 1, "sign": 2}  # "sign": 1-bit sign codes with a mean-|x| block scale

def _trace_range(name: str):
    """A ``lowbit:<name>`` profiler range while torch.profiler records (the
    trace analyzer attributes these to communication), nothing otherwise."""
    if torch.autograd.profiler._is_profiler_enabled:
        return torch.autograd.profiler.record_function("lowbit:" + name)
    return contextlib.nullcontext()


_CACHE: Dict[Tuple[str, int], Optional["Communicator"]] = {}
_LOCK = threading.Lock()


def _group_key(group) -> str:
    if group is None or group == dist.group.WORLD:
        return "WORLD"
    name = getattr(group, "group_name", None)
    if name:
        return str(name)
    return "ranks:" + ",".join(str(r) for r in dist.get_process_group_ranks(group))


def default_workspace_bytes() -> int:
    return int(os.environ.get("BITSCOM_WORKSPACE_MB", "256")) << 20


class Communicator:
    """Fused low-bit all-reduce / reduce-scatter / all-gather on one device."""

    def __init__(self, native, group=None):
        self._c = native
        self.group = group
        from ..tuning import entries, oneshot_max_bytes, schedule_lag

        native.set_oneshot_max_bytes(oneshot_max_bytes(native.world))
        for bits, fmt, one, ws in entries(native.world):
            native.set_tuning(bits, fmt, one, ws)
        lag = schedule_lag(native.world)
        if lag is not None and "BITSCOM_SCHED_LAG" not in os.environ:
            native.set_schedule_lag(lag)

    # ------------------------------------------------------------------ setup
    @classmethod
    def create_local(cls, device: Optional[int] = None, workspace_bytes: Optional[int] = None) -> "Communicator":
        """A world-size-1 communicator (the collectives become local
        quantise/dequantise passes; used by tests and single-GPU runs)."""
        C = _ext.require("Communicator")
        dev = torch.cuda.current_device() if device is None else int(device)
        return cls(C.LowBitComm(0, 1, dev, workspace_bytes or default_workspace_bytes()), None)

    @classmethod
    def for_group(
        cls, group=None, device: Optional[int] = None, workspace_bytes: Optional[int] = None
    ) -> Optional["Communicator"]:
        """The cached communicator of ``group`` on ``device`` (collective on
        first use), or None when peer-to-peer mapping is not possible."""
        dev = torch.cuda.current_device() if device is None else int(device)
        key = (_group_key(group), dev)
        with _LOCK:
            if key in _CACHE:
                return _CACHE[key]
        comm = cls._rendezvous(group, dev, workspace_bytes or default_workspace_bytes())
        with _LOCK:
            _CACHE[key] = comm
        return comm

    @classmethod
    def _rendezvous(cls, group, dev: int, ws: int) -> Optional["Communicator"]:
        C = _ext.require("Communicator")
        rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        native, err = None, None
        try:
            native = C.LowBitComm(rank, world, dev, ws)
            handle = bytes(native.ipc_handle())
        except Exception as exc:  # pragma: no cover - allocation failures
            handle, err = b"", repr(exc)
        info = (socket.gethostname(), dev, handle)
        infos = [None] * world
        dist.all_gather_object(infos, info, group=group)
        ok = native is not None
        host = socket.gethostname()
        if ok:
            for r, (h, d, hd) in enumerate(infos):
                if h != host or len(hd) != 64 or (r != rank and d == dev):
                    ok = False
                    break
                if r != rank and not torch.cuda.can_device_access_peer(dev, d):
                    ok = False
                    break
        if ok and world > 1:
            try:
                native.open_peers([hd for (_, _, hd) in infos])
            except Exception as exc:
                ok, err = False, repr(exc)
        oks = [None] * world
        dist.all_gather_object(oks, ok, group=group)
        if not all(oks):
            if os.environ.get("BITSCOM_LOG_LEVEL"):
                print(f"[bitscom] rank {rank}: peer-to-peer workspace unavailable ({err}); using the staged path")
            return None
        return cls(native, group)

    @staticmethod
    def clear_cache() -> None:
        with _LOCK:
            _CACHE.clear()

    # ------------------------------------------------------------- properties
    @property
    def native(self):
        return self._c

    @property
    def rank(self) -> int:
        return self._c.rank

    @property
    def world_size(self) -> int:
        return self._c.world

    @property
    def device(self) -> int:
        return self._c.device

    @property
    def epoch(self) -> int:
        return self._c.epoch

    def set_timeout(self, seconds: float) -> None:
        """Bound of every device-side wait on a peer flag."""
        self._c.set_timeout_ms(seconds * 1e3)

    def set_schedule_lag(self, lag: int) -> None:
        """Chunk-group lag of the kernel's work order: -1 automatic, 0 phase-major."""
        self._c.set_schedule_lag(int(lag))

    def set_sub_per_item(self, spi: int) -> None:
        """Sub-chunks (8192 elements) per work item and completion flag: 0 automatic, 1..16 fixed."""
        self._c.set_sub_per_item(int(spi))

    def set_kernel_variant(self, variant: str) -> None:
        """Kernel organisation: "reg" (every warp loads and waits itself;
        default) or "ws" (warp-specialised: a producer warp waits on peers and
        stages data by bulk async copies).  Both produce identical bytes."""
        self._c.set_kernel_variant({"ws": 0, "reg": 1}[variant])

    @property
    def kernel_variant(self) -> str:
        return ("ws", "reg")[self._c.kernel_variant]

    def check_canaries(self) -> int:
        """Number of workspace guard regions that were overwritten (0 = none)."""
        return int(self._c.check_canaries())

    def status(self) -> int:
        return int(self._c.status())

    def check(self) -> None:
        """Raise if an earlier (completed) launch timed out waiting for a peer."""
        self._c.check()

    def stats(self) -> dict:
        s = self._c.stats()
        keys = ("calls", "launches", "elements", "wire_bytes", "oneshot", "twoshot", "timed_launches", "kernel_ms")
        return {k: getattr(s, k) for k in keys}

    def set_timing(self, on: bool = True) -> None:
        """Time every launch on the device (CUDA events); see ``stats()["kernel_ms"]``."""
        self._c.set_timing(bool(on))

    # ------------------------------------------------------------ collectives
    def all_reduce(
        self,
        tensor: torch.Tensor,
        *,
        out: Optional[torch.Tensor] = None,
        bits: int = 4,
        fmt: str = "int",
        residual: Optional[torch.Tensor] = None,
        stochastic_rounding: bool = False,
        stochastic_requant: bool = False,
        seed: int = 0,
        offset: int = 0,
        post_scale: float = 1.0,
        algo: str = "auto",
        max_ctas: int = 0,
    ) -> torch.Tensor:
        """Low-bit SUM all-reduce (times ``post_scale``) in place or into ``out``.

        ``residual`` (fp32 or bf16, ``tensor.numel()`` elements) enables error
        feedback: the kernel quantises ``tensor + residual`` and writes the new
        residual.
        """
        with _trace_range("all_reduce"):
            self._c.allreduce(
                tensor, out, residual, bits, FMTS[fmt], ALGOS[algo], stochastic_rounding, stochastic_requant,
                int(seed), int(offset), float(post_scale), int(max_ctas),
            )
        return tensor if out is None else out

    def reduce_scatter(
        self,
        output: torch.Tensor,
        input: torch.Tensor,
        *,
        bits: int = 8,
        fmt: str = "int",
        residual: Optional[torch.Tensor] = None,
        stochastic_rounding: bool = False,
        seed: int = 0,
        offset: int = 0,
        post_scale: float = 1.0,
        max_ctas: int = 0,
    ) -> torch.Tensor:
        """Low-bit SUM reduce-scatter: ``input`` holds world*n elements, ``output`` n."""
        with _trace_range("reduce_scatter"):
            self._c.reduce_scatter(
                input, output, residual, bits, FMTS[fmt], stochastic_rounding, int(seed), int(offset),
                float(post_scale), int(max_ctas),
            )
        return output

    def all_gather(
        self,
        output: torch.Tensor,
        input: torch.Tensor,
        *,
        bits: int = 8,
        fmt: str = "int",
        residual: Optional[torch.Tensor] = None,
        stochastic_rounding: bool = False,
        seed: int = 0,
        offset: int = 0,
        max_ctas: int = 0,
    ) -> torch.Tensor:
        """Low-bit all-gather: ``output`` holds world*n elements (rank-major)."""
        with _trace_range("all_gather"):
            self._c.all_gather(
                input, output, residual, bits, FMTS[fmt], stochastic_rounding, int(seed), int(offset), int(max_ctas)
            )
        return output
