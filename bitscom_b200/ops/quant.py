"""Sync-free building blocks used by the staged collective paths.

Unlike the reference-compatible functions in :mod:`bitscom_b200.quantization`
(which return the scale as a Python float, hence a host sync on CUDA), these
keep the scale as a one-element float32 tensor on the data's device, so a
chain quantise -> collective -> dequantise runs without host round trips.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _ext
from ..quantization import _pack_cpu, _quant_bounds, _unpack_cpu, _sr_uniforms, _draw_seed, packed_nbytes


def quantize_codes(
    x: torch.Tensor, bits: int, *, stochastic: bool = False, seed: Optional[int] = None, offset: int = 0
) -> Tuple[torch.Tensor, torch.Tensor]:
    """(int16 codes, float32[1] scale) with the per-tensor reference semantics."""
    if stochastic and seed is None:
        seed = _draw_seed()
    seed = 0 if seed is None else int(seed)
    if _ext.use_cuda_kernels(x):
        xx = x if x.dtype in (torch.float32, torch.bfloat16, torch.float16) else x.float()
        _, q, scale_d, _ = _ext._C.quantize(xx.contiguous().view(-1), bits, stochastic, seed, offset, False, True)
        return q, scale_d.to(torch.float32)
    qmin, qmax = _quant_bounds(bits)
    xf = x.detach().to(torch.float32).contiguous().view(-1)
    amax = xf.abs().max() if xf.numel() else torch.zeros((), dtype=torch.float32)
    scale_d = torch.where(amax == 0, torch.ones((), dtype=torch.float64), amax.double() / qmax)
    v = xf / scale_d.float()
    if stochastic:
        lo = torch.floor(v)
        q = lo + (_sr_uniforms(v.numel(), seed, offset) < (v - lo)).to(torch.float32)
    else:
        q = torch.round(v)
    return q.clamp_(qmin, qmax).to(torch.int16), scale_d.float().view(1)


def pack_codes(q: torch.Tensor, bits: int) -> torch.Tensor:
    if _ext.use_cuda_kernels(q):
        return _ext._C.pack(q.contiguous().view(-1), bits)
    qmin, _ = _quant_bounds(bits)
    return _pack_cpu((q.to(torch.int64).view(-1) - qmin) & ((1 << bits) - 1), bits)


def unpack_dequant(packed: torch.Tensor, bits: int, numel: int, scale: torch.Tensor) -> torch.Tensor:
    """float32 values from packed reference bytes and a device scale tensor."""
    if _ext.use_cuda_kernels(packed):
        _, out = _ext._C.unpack(packed.contiguous().view(-1), bits, numel, False, torch.float32, 1.0, scale.view(1))
        return out
    qmin, _ = _quant_bounds(bits)
    q = (_unpack_cpu(packed.contiguous(), bits, numel) + qmin).to(torch.float32)
    return q * scale.to(torch.float32).view(())


def quantize_pack(
    x: torch.Tensor, bits: int, *, stochastic: bool = False, seed: Optional[int] = None, offset: int = 0
) -> Tuple[torch.Tensor, torch.Tensor]:
    """(packed bytes, float32[1] scale) in one pass on CUDA."""
    if _ext.use_cuda_kernels(x):
        if stochastic and seed is None:
            seed = _draw_seed()
        xx = x if x.dtype in (torch.float32, torch.bfloat16, torch.float16) else x.float()
        packed, _, scale_d, _ = _ext._C.quantize(
            xx.contiguous().view(-1), bits, stochastic, 0 if seed is None else int(seed), offset, True, False
        )
        return packed, scale_d.to(torch.float32)
    q, s = quantize_codes(x, bits, stochastic=stochastic, seed=seed, offset=offset)
    return pack_codes(q, bits), s


__all__ = ["quantize_codes", "pack_codes", "unpack_dequant", "quantize_pack", "packed_nbytes"]
