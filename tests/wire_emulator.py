"""CPU model of the fused collectives' block-scaled arithmetic (deterministic rounding).

Each 1024-element block gets ``scale = amax / qmax`` (float32; 1.0 when the
block is all zero) and codes ``clamp(rint(x * (1/scale)))``; E4M3 blocks use
``amax / 448`` and saturating round-to-nearest fp8.  The owner of a shard sums
the W dequantised contributions in rank order in float32 and (two-shot)
requantises with fresh block scales.  Used to check the kernels bit-for-bit.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch

BLOCK = 1024
SUB = 8192


def _bounds(bits):
    if bits == 1:
        return 0, 1
    return -(1 << (bits - 1)), (1 << (bits - 1)) - 1


def _block_mean_abs(xb: torch.Tensor) -> torch.Tensor:
    """The kernel's mean |x| per block, in its exact fp32 order: lane l sums
    its 32 elements (k*32+l)*4+m in (k, m) order, then an xor butterfly over
    the lanes (offsets 16, 8, 4, 2, 1), then times 2^-10."""
    a = xb.abs().view(-1, 8, 32, 4).permute(0, 2, 1, 3).reshape(-1, 32, 32)  # [block, lane, j]
    s = torch.zeros(a.shape[0], 32, dtype=torch.float32)
    for j in range(32):
        s = s + a[:, :, j]
    lanes = torch.arange(32)
    for o in (16, 8, 4, 2, 1):
        s = s + s[:, lanes ^ o]
    return (s[:, :1] * (1.0 / BLOCK)).to(torch.float32)


def block_quant(x: torch.Tensor, bits: int, fmt: str = "int") -> torch.Tensor:
    """Dequantised values of x (float32, length a multiple of BLOCK)."""
    xb = x.view(-1, BLOCK)
    if fmt == "sign":
        scale = _block_mean_abs(xb)
        return torch.where(xb >= 0, scale, -scale).view(-1)
    amax = xb.abs().amax(dim=1, keepdim=True)
    one = torch.ones((), dtype=torch.float32)
    if fmt == "e4m3":
        scale = torch.where(amax > 0, amax / 448.0, one)
        inv = one / scale
        q = (xb * inv).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).to(torch.float32)
        return (q * scale).view(-1)
    qmin, qmax = _bounds(bits)
    scale = torch.where(amax > 0, amax / float(qmax), one)
    inv = one / scale
    q = torch.round(xb * inv).clamp(qmin, qmax)
    return (q * scale).view(-1)


def _pad(x: torch.Tensor, n: int) -> torch.Tensor:
    return torch.cat([x, x.new_zeros(n - x.numel())]) if n > x.numel() else x


def allreduce_two_shot(
    inputs: List[torch.Tensor],
    bits: int,
    residuals: Optional[List[torch.Tensor]] = None,
    post_scale: float = 1.0,
    fmt: str = "int",
) -> Tuple[torch.Tensor, Optional[List[torch.Tensor]]]:
    """Expected output (identical on all ranks) and new residuals."""
    W = len(inputs)
    n = inputs[0].numel()
    shard = -(-(-(-n // W)) // SUB) * SUB
    deq, new_res = [], []
    for r, x in enumerate(inputs):
        c = x.to(torch.float32).view(-1)
        if residuals is not None:
            c = c + residuals[r]
        cp = _pad(c, W * shard)
        d = block_quant(cp, bits, fmt)
        deq.append(d)
        if residuals is not None:
            new_res.append((cp - d)[:n])
    out = torch.empty(W * shard, dtype=torch.float32)
    for o in range(W):
        acc = torch.zeros(shard, dtype=torch.float32)
        for s in range(W):
            acc = acc + deq[s][o * shard : (o + 1) * shard]
        out[o * shard : (o + 1) * shard] = block_quant(acc, bits, fmt) * post_scale
    return out[:n], (new_res if residuals is not None else None)


def allreduce_one_shot(
    inputs: List[torch.Tensor],
    bits: int,
    residuals: Optional[List[torch.Tensor]] = None,
    post_scale: float = 1.0,
    fmt: str = "int",
):
    n = inputs[0].numel()
    padded = -(-n // SUB) * SUB
    acc = torch.zeros(padded, dtype=torch.float32)
    new_res = []
    for r, x in enumerate(inputs):
        c = x.to(torch.float32).view(-1)
        if residuals is not None:
            c = c + residuals[r]
        cp = _pad(c, padded)
        d = block_quant(cp, bits, fmt)
        if residuals is not None:
            new_res.append((cp - d)[:n])
        acc = acc + d
    return (acc * post_scale)[:n], (new_res if residuals is not None else None)


def reduce_scatter(inputs: List[torch.Tensor], bits: int, post_scale: float = 1.0, fmt: str = "int"):
    """Per-rank outputs of the fused reduce-scatter (input = W shards of n)."""
    W = len(inputs)
    n = inputs[0].numel() // W
    shard = -(-n // SUB) * SUB
    deq = []
    for x in inputs:
        parts = [block_quant(_pad(x[s * n : (s + 1) * n].float(), shard), bits, fmt) for s in range(W)]
        deq.append(parts)
    outs = []
    for o in range(W):
        acc = torch.zeros(shard, dtype=torch.float32)
        for s in range(W):
            acc = acc + deq[s][o]
        outs.append((acc * post_scale)[:n])
    return outs


def all_gather(inputs: List[torch.Tensor], bits: int, fmt: str = "int") -> torch.Tensor:
    n = inputs[0].numel()
    padded = -(-n // SUB) * SUB
    return torch.cat([block_quant(_pad(x.float().view(-1), padded), bits, fmt)[:n] for x in inputs])
