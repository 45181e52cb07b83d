"""Quantisation / packing semantics and byte compatibility with the reference.

Mirrors reference tests/test_quantization.py (validation, full-range
pack/unpack, roundtrip bound, dtype override, SR unbiasedness) and adds
bit-for-bit comparisons against the reference's own CPU code.
"""

import numpy as np
import pytest
import torch

from bitscom_b200.quantization import (
    SUPPORTED_BITWIDTHS,
    _quant_bounds,
    compress_tensor,
    decompress_tensor,
    dequantize_tensor,
    ef_roundtrip,
    pack_lowbit,
    packed_nbytes,
    quantize_tensor,
    roundtrip_tensor,
    unpack_lowbit,
    validate_bitwidth,
)

from . import ref_oracle


def test_validate_bitwidth_accepts_supported_values():
    for b in SUPPORTED_BITWIDTHS:
        validate_bitwidth(b)


@pytest.mark.parametrize("bitwidth", [0, 3, 5, 7, 9, 15, 32])
def test_validate_bitwidth_rejects_unsupported_values(bitwidth):
    with pytest.raises(ValueError):
        validate_bitwidth(bitwidth)


@pytest.mark.parametrize("bitwidth", SUPPORTED_BITWIDTHS)
def test_pack_unpack_full_range(bitwidth):
    qmin, qmax = _quant_bounds(bitwidth)
    q = torch.arange(qmin, qmax + 1, dtype=torch.int16)
    packed, numel = pack_lowbit(q, bitwidth)
    assert packed.dtype == torch.uint8
    assert packed.numel() == packed_nbytes(numel, bitwidth)
    out = unpack_lowbit(packed, bitwidth, numel)
    assert out.dtype == torch.int16 and torch.equal(out, q)


@pytest.mark.parametrize("bitwidth", SUPPORTED_BITWIDTHS)
def test_roundtrip_error_bounded_by_quant_step(bitwidth):
    x = torch.linspace(-3.0, 3.0, steps=4096).reshape(64, 64)
    q, scale = quantize_tensor(x, bitwidth)
    y = roundtrip_tensor(x, bitwidth)
    assert y.shape == x.shape and y.dtype == x.dtype and q.dtype == torch.int16
    if bitwidth == 1:
        # 1-bit codes are unsigned {0, 1}: negatives collapse to 0 (reference semantics)
        pos = x >= 0
        assert torch.max(torch.abs(y[pos] - x[pos])).item() <= scale + 1e-6
    else:
        assert torch.max(torch.abs(y - x)).item() <= scale + 1e-6


def test_compress_decompress_dtype_override():
    x = torch.randn(128)
    c = compress_tensor(x, bitwidth=4)
    y = decompress_tensor(c, dtype=torch.float64)
    assert y.dtype == torch.float64 and y.shape == x.shape and c.packed.dtype == torch.uint8


def test_all_zero_tensor_uses_unit_scale():
    q, scale = quantize_tensor(torch.zeros(17), 4)
    assert scale == 1.0 and torch.equal(q, torch.zeros(17, dtype=torch.int16))


def test_stochastic_rounding_cpu_is_unbiased():
    x = torch.full((4096,), 0.3)
    x[0] = 1.0  # 2-bit qmax = 1 -> scale = 1
    means = []
    for _ in range(64):
        q, _ = quantize_tensor(x, bitwidth=2, stochastic_rounding=True)
        means.append(float(q[1:].float().mean()))
    assert abs(sum(means) / len(means) - 0.3) < 0.02


def test_stochastic_rounding_is_reproducible_with_seed():
    x = torch.randn(1000)
    a, _ = quantize_tensor(x, 4, stochastic_rounding=True, seed=123)
    b, _ = quantize_tensor(x, 4, stochastic_rounding=True, seed=123)
    c, _ = quantize_tensor(x, 4, stochastic_rounding=True, seed=124)
    assert torch.equal(a, b) and not torch.equal(a, c)
    torch.manual_seed(5)
    d, _ = quantize_tensor(x, 4, stochastic_rounding=True)
    torch.manual_seed(5)
    e, _ = quantize_tensor(x, 4, stochastic_rounding=True)
    assert torch.equal(d, e)


def test_ef_roundtrip_cpu_matches_definition():
    torch.manual_seed(0)
    x = torch.randn(3000)
    r = torch.randn(3000) * 0.01
    r0 = r.clone()
    y = ef_roundtrip(x, r, 4)
    c = x + r0
    q, s = quantize_tensor(c, 4)
    ref = q.float() * s
    assert torch.equal(y, ref)
    assert torch.equal(r, c - ref)


# ----------------------------------------------------------------------------
# byte compatibility with the reference's CPU code
# ----------------------------------------------------------------------------
CASES = [
    ("randn", 4099),
    ("randn", 1),
    ("randn", 7),
    ("linspace", 1031),
    ("zeros", 33),
    ("outliers", 2**14 + 3),
]


def _make(kind, n, seed=0):
    g = torch.Generator().manual_seed(seed)
    if kind == "randn":
        return torch.randn(n, generator=g)
    if kind == "linspace":
        return torch.linspace(-2.5, 3.0, n)
    if kind == "zeros":
        return torch.zeros(n)
    x = torch.randn(n, generator=g) * 1e-3
    idx = torch.randint(0, n, (max(1, n // 100),), generator=g)
    x[idx] = torch.randn(idx.numel(), generator=g) * 1e-1
    return x


@pytest.mark.parametrize("bitwidth", SUPPORTED_BITWIDTHS)
@pytest.mark.parametrize("kind,n", CASES)
def test_compress_bytes_match_reference(bitwidth, kind, n):
    ref = ref_oracle.load()
    x = _make(kind, n)
    ours = compress_tensor(x, bitwidth)
    theirs = ref.compress_tensor(x, bitwidth)
    assert ours.scale == theirs.scale
    assert ours.numel == theirs.numel and ours.shape == theirs.shape
    assert torch.equal(ours.packed, theirs.packed)
    # and each side decodes the other's bytes identically
    a = decompress_tensor(ours)
    b = ref.decompress_tensor(theirs)
    assert torch.equal(a, b)


@pytest.mark.parametrize("bitwidth", SUPPORTED_BITWIDTHS)
def test_quantize_and_pack_match_reference(bitwidth):
    ref = ref_oracle.load()
    x = _make("outliers", 50001, seed=3).reshape(3, -1)
    q, s = quantize_tensor(x, bitwidth)
    rq, rs = ref.quantize_tensor(x, bitwidth)
    assert s == rs and torch.equal(q, rq)
    p, n = pack_lowbit(q, bitwidth)
    rp, rn = ref.pack_lowbit(rq, bitwidth)
    assert n == rn and torch.equal(p, rp)
    assert torch.equal(unpack_lowbit(rp, bitwidth, rn), ref.unpack_lowbit(p, bitwidth, n))
    assert torch.equal(dequantize_tensor(q, s, shape=x.shape), ref.dequantize_tensor(rq, rs, shape=x.shape))


def test_seed0_2pow20_roundtrip_all_bitwidths_match_reference():
    """CPU roundtrip config: seed-0 N(0,1) tensor of 2^20 elements."""
    ref = ref_oracle.load()
    torch.manual_seed(0)
    x = torch.randn(2**20)
    for b in SUPPORTED_BITWIDTHS:
        assert torch.equal(roundtrip_tensor(x, b), ref.roundtrip_tensor(x, b)), b


def test_philox_known_answers():
    from bitscom_b200.ops.philox import philox4x32_10

    # Known-answer vectors of Philox-4x32-10 (Salmon et al., SC'11, Random123 KAT).
    out = philox4x32_10([0], [0], [0], [0], 0, 0)
    assert [int(v[0]) for v in out] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    m = 0xFFFFFFFF
    out = philox4x32_10([m], [m], [m], [m], m, m)
    assert [int(v[0]) for v in out] == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    out = philox4x32_10([0x243F6A88], [0x85A308D3], [0x13198A2E], [0x03707344], 0xA4093822, 0x299F31D0)
    assert [int(v[0]) for v in out] == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_philox_uniforms_are_uniform():
    from bitscom_b200.ops.philox import uniforms_for_elements

    u = uniforms_for_elements(1 << 16, seed=7, offset=3)
    assert u.dtype == np.float32 and u.min() >= 0.0 and u.max() < 1.0
    assert abs(float(u.mean()) - 0.5) < 0.01
