"""Philox-4x32-10 counter RNG on the host (numpy), bit-identical to the device
version in ``csrc/kernels/common.cuh``.

Written from Salmon, Moraes, Dror & Shaw, "Parallel random numbers: as easy as
1, 2, 3" (SC'11): 10 rounds of two 32x32->64-bit multiplications with the
multipliers 0xD2511F53 / 0xCD9E8D57 and a Weyl key schedule with increments
0x9E3779B9 / 0xBB67AE85.

Used for stochastic rounding on the CPU so that CPU and CUDA quantisation with
the same ``(seed, offset)`` draw the same numbers.
"""

from __future__ import annotations

import numpy as np

_M0 = np.uint64(0xD2511F53)
_M1 = np.uint64(0xCD9E8D57)
_W0 = np.uint32(0x9E3779B9)
_W1 = np.uint32(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)
_S32 = np.uint64(32)


def philox4x32_10(x, y, z, w, k0: int, k1: int):
    """Vectorised Philox over uint32 counter arrays; returns four uint32 arrays."""
    x = np.asarray(x, dtype=np.uint64) & _MASK
    y = np.asarray(y, dtype=np.uint64) & _MASK
    z = np.asarray(z, dtype=np.uint64) & _MASK
    w = np.asarray(w, dtype=np.uint64) & _MASK
    k0 = np.uint32(k0 & 0xFFFFFFFF)
    k1 = np.uint32(k1 & 0xFFFFFFFF)
    with np.errstate(over="ignore"):
        for _ in range(10):
            p0 = _M0 * x
            p1 = _M1 * z
            hi0, lo0 = p0 >> _S32, p0 & _MASK
            hi1, lo1 = p1 >> _S32, p1 & _MASK
            x, y, z, w = (hi1 ^ y ^ np.uint64(k0)), lo1, (hi0 ^ w ^ np.uint64(k1)), lo0
            k0 = np.uint32(k0 + _W0)
            k1 = np.uint32(k1 + _W1)
    return (x.astype(np.uint32), y.astype(np.uint32), z.astype(np.uint32), w.astype(np.uint32))


def uniforms_for_elements(n: int, seed: int, offset: int) -> np.ndarray:
    """Uniform [0,1) draws for elements 0..n-1 with the device's counter layout.

    Element e uses output lane ``e % 4`` of the call with counter
    ``(e // 4, 0, offset_lo, offset_hi)`` and key ``(seed_lo, seed_hi)``; the
    24 high bits become the float ``(r >> 8) * 2**-24``.
    """
    groups = (n + 3) // 4
    g = np.arange(groups, dtype=np.uint64)
    x, y, z, w = philox4x32_10(
        g & _MASK,
        g >> _S32,
        np.full(groups, offset & 0xFFFFFFFF, dtype=np.uint64),
        np.full(groups, (offset >> 32) & 0xFFFFFFFF, dtype=np.uint64),
        seed & 0xFFFFFFFF,
        (seed >> 32) & 0xFFFFFFFF,
    )
    r = np.stack([x, y, z, w], axis=1).reshape(-1)[:n]
    return (r >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
