"""Per-tensor symmetric quantisation and bit-packing, byte-compatible with the
reference's ``compress()`` output.

Public names and semantics follow reference ``python/bitscom/quantization.py``:

* bitwidths {1, 2, 4, 8, 12, 16}; 1-bit codes are the unsigned pair {0, 1},
  every other width is signed ``[-2^(b-1), 2^(b-1)-1]`` (reference :27-43);
* ``scale = max|x| / qmax`` (1.0 for an all-zero tensor), computed in double
  and applied as float32; ``q = clamp(round_half_even(x / scale))`` (:60-94);
* packed layout: the little-endian, LSB-first bit stream of ``q - qmin`` —
  whole bytes for 1/2/4/8 bits, 3-byte pairs for 12 bits, 2 bytes per code
  for 16 bits, zero padding (:118-196).

CUDA tensors run the sm_100a kernels of ``csrc/kernels/quant_kernels.cu`` for
every bitwidth (the reference had CUDA kernels for 1/2/4/8 only and a host
sync inside every quantisation).  CPU tensors use the torch code below.
Stochastic rounding draws from Philox-4x32-10 keyed by ``(seed, offset)`` on
both devices, so CPU and CUDA results agree bit-for-bit for the same seed; when
no seed is given one is drawn from torch's default generator, so
``torch.manual_seed`` makes runs reproducible.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

from . import _ext
from .ops.philox import uniforms_for_elements

SUPPORTED_BITWIDTHS = (1, 2, 4, 8, 12, 16)


def validate_bitwidth(bitwidth: int) -> None:
    """Raise ValueError unless ``bitwidth`` is one of SUPPORTED_BITWIDTHS."""
    if bitwidth not in SUPPORTED_BITWIDTHS:
        raise ValueError(f"bitwidth must be one of {SUPPORTED_BITWIDTHS}, got {bitwidth}")


def _quant_bounds(bitwidth: int) -> Tuple[int, int]:
    """(qmin, qmax) of a bitwidth."""
    if bitwidth == 1:
        return 0, 1
    half = 1 << (bitwidth - 1)
    return -half, half - 1


def _group(bitwidth: int) -> Tuple[int, int]:
    """(codes, bytes) of the smallest whole-byte group of the bit stream."""
    if bitwidth <= 8:
        return 8 // bitwidth, 1
    if bitwidth == 12:
        return 2, 3
    return 1, 2


def packed_nbytes(numel: int, bitwidth: int) -> int:
    """Bytes of the packed reference layout for ``numel`` codes."""
    g, nb = _group(bitwidth)
    return -(-numel // g) * nb


@dataclass(frozen=True)
class CompressedTensor:
    """Packed codes plus everything needed to restore the tensor."""

    packed: torch.Tensor
    scale: float
    numel: int
    shape: Tuple[int, ...]
    bitwidth: int
    dtype: torch.dtype

    @property
    def packed_bytes(self) -> int:
        return int(self.packed.numel())


def _draw_seed() -> int:
    return int(torch.randint(0, 2**62, (1,), dtype=torch.int64).item())


def _sr_uniforms(n: int, seed: int, offset: int) -> torch.Tensor:
    return torch.from_numpy(uniforms_for_elements(n, seed, offset))


def quantize_tensor(
    tensor: torch.Tensor,
    bitwidth: int,
    *,
    stochastic_rounding: bool = False,
    seed: Optional[int] = None,
    offset: int = 0,
) -> Tuple[torch.Tensor, float]:
    """Quantise to int16 codes with one symmetric scale; returns (q, scale)."""
    validate_bitwidth(bitwidth)
    if not tensor.is_floating_point():
        raise TypeError("quantize_tensor expects a floating-point tensor")
    if stochastic_rounding and seed is None:
        seed = _draw_seed()
    seed = 0 if seed is None else int(seed)
    if _ext.use_cuda_kernels(tensor):
        x = tensor.detach()
        if x.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            x = x.float()
        _, q, scale_t, _ = _ext._C.quantize(
            x.contiguous(), bitwidth, stochastic_rounding, seed, offset, False, True
        )
        return q.view(tensor.shape), float(scale_t.item())

    qmin, qmax = _quant_bounds(bitwidth)
    x = tensor.detach().to(torch.float32).contiguous()
    amax = float(x.abs().max().item()) if x.numel() else 0.0
    scale = 1.0 if amax == 0.0 else amax / float(qmax)
    v = x / scale
    if stochastic_rounding:
        lo = torch.floor(v)
        u = _sr_uniforms(v.numel(), seed, offset).view(v.shape)
        q = lo + (u < (v - lo)).to(torch.float32)
    else:
        q = torch.round(v)
    return q.clamp_(qmin, qmax).to(torch.int16), scale


def dequantize_tensor(
    q_tensor: torch.Tensor,
    scale: float,
    *,
    dtype: torch.dtype = torch.float32,
    device: torch.device | None = None,
    shape: Sequence[int] | None = None,
) -> torch.Tensor:
    """``q * scale`` in float32, then reshaped and cast."""
    if device is None:
        device = q_tensor.device
    if q_tensor.dtype == torch.int16 and _ext.use_cuda_kernels(q_tensor):
        out_dt = dtype if dtype in (torch.float32, torch.bfloat16, torch.float16) and torch.device(device) == q_tensor.device else torch.float32
        out = _ext._C.dequantize(q_tensor.contiguous(), float(scale), None, out_dt)
    else:
        out = q_tensor.to(torch.float32) * float(scale)
    if shape is not None:
        out = out.view(*shape)
    return out.to(device=device, dtype=dtype)


def _pack_cpu(values: torch.Tensor, bitwidth: int) -> torch.Tensor:
    """LSB-first bit stream of non-negative codes (int64), zero padded."""
    g, nb = _group(bitwidth)
    n = values.numel()
    pad = (-n) % g
    if pad:
        values = torch.cat([values, values.new_zeros(pad)])
    grp = values.view(-1, g)
    shifts = torch.arange(g, dtype=torch.int64) * bitwidth
    word = (grp << shifts).sum(dim=1)  # at most 24 significant bits
    byte_shifts = torch.arange(nb, dtype=torch.int64) * 8
    return ((word.unsqueeze(1) >> byte_shifts) & 0xFF).to(torch.uint8).reshape(-1)


def _unpack_cpu(packed: torch.Tensor, bitwidth: int, numel: int) -> torch.Tensor:
    g, nb = _group(bitwidth)
    groups = -(-numel // g)
    b = packed.reshape(-1)[: groups * nb].to(torch.int64).view(groups, nb)
    word = (b << (torch.arange(nb, dtype=torch.int64) * 8)).sum(dim=1)
    shifts = torch.arange(g, dtype=torch.int64) * bitwidth
    codes = (word.unsqueeze(1) >> shifts) & ((1 << bitwidth) - 1)
    return codes.reshape(-1)[:numel]


def pack_lowbit(q_tensor: torch.Tensor, bitwidth: int) -> Tuple[torch.Tensor, int]:
    """Pack int16 codes into the reference byte layout; returns (bytes, numel)."""
    validate_bitwidth(bitwidth)
    numel = int(q_tensor.numel())
    if _ext.use_cuda_kernels(q_tensor):
        return _ext._C.pack(q_tensor.to(torch.int16).contiguous().view(-1), bitwidth), numel
    qmin, _ = _quant_bounds(bitwidth)
    values = q_tensor.to(torch.int64).contiguous().view(-1) - qmin
    values = values & ((1 << bitwidth) - 1)
    return _pack_cpu(values, bitwidth), numel


def unpack_lowbit(packed: torch.Tensor, bitwidth: int, numel: int) -> torch.Tensor:
    """Inverse of :func:`pack_lowbit`: bytes back to int16 codes."""
    validate_bitwidth(bitwidth)
    if _ext.use_cuda_kernels(packed):
        q, _ = _ext._C.unpack(packed.contiguous().view(-1), bitwidth, numel, True, None, 1.0, None)
        return q
    qmin, _ = _quant_bounds(bitwidth)
    return (_unpack_cpu(packed.contiguous(), bitwidth, numel) + qmin).to(torch.int16)


def compress_tensor(
    tensor: torch.Tensor,
    bitwidth: int,
    *,
    stochastic_rounding: bool = False,
    seed: Optional[int] = None,
) -> CompressedTensor:
    """quantise + pack (one fused kernel pass on CUDA)."""
    validate_bitwidth(bitwidth)
    if not tensor.is_floating_point():
        raise TypeError("compress_tensor expects a floating-point tensor")
    if _ext.use_cuda_kernels(tensor):
        if stochastic_rounding and seed is None:
            seed = _draw_seed()
        x = tensor.detach()
        if x.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            x = x.float()
        packed, _, scale_t, _ = _ext._C.quantize(
            x.contiguous(), bitwidth, stochastic_rounding, 0 if seed is None else int(seed), 0, True, False
        )
        scale = float(scale_t.item())
    else:
        q, scale = quantize_tensor(tensor, bitwidth, stochastic_rounding=stochastic_rounding, seed=seed)
        packed, _ = pack_lowbit(q, bitwidth)
    return CompressedTensor(
        packed=packed,
        scale=scale,
        numel=int(tensor.numel()),
        shape=tuple(tensor.shape),
        bitwidth=bitwidth,
        dtype=tensor.dtype,
    )


def decompress_tensor(
    compressed: CompressedTensor,
    *,
    dtype: torch.dtype | None = None,
    device: torch.device | None = None,
) -> torch.Tensor:
    """unpack + dequantise (one fused kernel pass on CUDA)."""
    dtype = dtype or compressed.dtype
    p = compressed.packed
    if _ext.use_cuda_kernels(p):
        direct = dtype in (torch.float32, torch.bfloat16, torch.float16)
        _, out = _ext._C.unpack(
            p.contiguous().view(-1),
            compressed.bitwidth,
            compressed.numel,
            False,
            dtype if direct else torch.float32,
            float(compressed.scale),
            None,
        )
        out = out.view(*compressed.shape)
        return out.to(device=device or p.device, dtype=dtype)
    q = unpack_lowbit(p, compressed.bitwidth, compressed.numel)
    return dequantize_tensor(q, compressed.scale, dtype=dtype, device=device, shape=compressed.shape)


def roundtrip_tensor(tensor: torch.Tensor, bitwidth: int) -> torch.Tensor:
    """dequantise(quantise(tensor)) in the tensor's dtype and device."""
    validate_bitwidth(bitwidth)
    if _ext.use_cuda_kernels(tensor) and tensor.dtype in (torch.float32, torch.bfloat16, torch.float16):
        return _ext._C.ef_roundtrip(tensor.detach().contiguous(), None, bitwidth, False, 0, 0).view(tensor.shape)
    compressed = compress_tensor(tensor, bitwidth)
    return decompress_tensor(compressed, dtype=tensor.dtype, device=tensor.device)


def ef_roundtrip(
    tensor: torch.Tensor,
    residual: Optional[torch.Tensor],
    bitwidth: int,
    *,
    stochastic_rounding: bool = False,
    seed: Optional[int] = None,
    offset: int = 0,
) -> torch.Tensor:
    """Error-feedback roundtrip: ``c = x + residual``; returns ``dequant(quant(c))``
    and overwrites ``residual`` with ``c - dequant(quant(c))`` (fp32, in place).

    The EF arithmetic of reference benchmarks/error_feedback_comparison.py:20-37
    and cpp/src/process_group_lowbit.cc:191-252, as one fused pass on CUDA.
    """
    validate_bitwidth(bitwidth)
    if stochastic_rounding and seed is None:
        seed = _draw_seed()
    seed = 0 if seed is None else int(seed)
    if residual is not None and (residual.dtype != torch.float32 or residual.numel() != tensor.numel()):
        raise ValueError("residual must be a float32 tensor with tensor.numel() elements")
    if _ext.use_cuda_kernels(tensor) and tensor.dtype in (torch.float32, torch.bfloat16, torch.float16):
        r = residual.view(-1) if residual is not None else None
        return _ext._C.ef_roundtrip(
            tensor.detach().contiguous(), r, bitwidth, stochastic_rounding, seed, offset
        ).view(tensor.shape)
    c = tensor.detach().to(torch.float32)
    if residual is not None:
        c = c + residual.view(c.shape)
    q, scale = quantize_tensor(c, bitwidth, stochastic_rounding=stochastic_rounding, seed=seed, offset=offset)
    y = q.to(torch.float32) * float(scale)
    if residual is not None:
        residual.copy_((c - y).view(residual.shape))
    return y.to(tensor.dtype)
