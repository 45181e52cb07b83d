"""sm_100a quantisation kernels vs the CPU implementation (which is itself
byte-compatible with the reference).  Needs a CUDA device."""

import pytest
import torch

import bitscom_b200
from bitscom_b200 import _ext
from bitscom_b200.quantization import (
    SUPPORTED_BITWIDTHS,
    compress_tensor,
    decompress_tensor,
    dequantize_tensor,
    ef_roundtrip,
    pack_lowbit,
    quantize_tensor,
    roundtrip_tensor,
    unpack_lowbit,
)

pytestmark = pytest.mark.gpu

SIZES = [1, 7, 1023, 1024, 4099, (1 << 20) + 5]


def _x(n, dtype=torch.float32, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, generator=g) * 0.5
    if n > 10:
        x[n // 3] = 4.0
    return x.to(dtype)


def test_native_extension_is_loaded_from_tree(cuda):
    assert _ext.available()
    assert "bitscom_b200" in _ext._C.__file__


@pytest.mark.parametrize("bits", SUPPORTED_BITWIDTHS)
@pytest.mark.parametrize("n", SIZES)
def test_quantize_matches_cpu(cuda, bits, n):
    x = _x(n)
    q_cpu, s_cpu = quantize_tensor(x, bits)
    q_gpu, s_gpu = quantize_tensor(x.to(cuda), bits)
    assert s_gpu == s_cpu
    assert torch.equal(q_gpu.cpu(), q_cpu)


@pytest.mark.parametrize("bits", SUPPORTED_BITWIDTHS)
@pytest.mark.parametrize("n", SIZES)
def test_compress_bytes_match_cpu(cuda, bits, n):
    x = _x(n, seed=n)
    c_cpu = compress_tensor(x, bits)
    c_gpu = compress_tensor(x.to(cuda), bits)
    assert c_gpu.packed.is_cuda and c_gpu.scale == c_cpu.scale
    assert torch.equal(c_gpu.packed.cpu(), c_cpu.packed)
    assert torch.equal(decompress_tensor(c_gpu).cpu(), decompress_tensor(c_cpu))
    # cross-device: bytes made on one side decode identically on the other
    assert torch.equal(decompress_tensor(c_cpu.__class__(**{**c_cpu.__dict__, "packed": c_cpu.packed.to(cuda)})).cpu(),
                       decompress_tensor(c_cpu))


@pytest.mark.parametrize("bits", SUPPORTED_BITWIDTHS)
def test_pack_unpack_dequant_match_cpu(cuda, bits):
    x = _x(5003, seed=bits)
    q, s = quantize_tensor(x, bits)
    p_cpu, n = pack_lowbit(q, bits)
    p_gpu, _ = pack_lowbit(q.to(cuda), bits)
    assert torch.equal(p_gpu.cpu(), p_cpu)
    assert torch.equal(unpack_lowbit(p_cpu.to(cuda), bits, n).cpu(), q)
    assert torch.equal(dequantize_tensor(q.to(cuda), s).cpu(), dequantize_tensor(q, s))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bits", [2, 4, 8, 12])
def test_low_precision_inputs(cuda, dtype, bits):
    x = _x(70001, dtype=dtype, seed=bits)
    c_cpu = compress_tensor(x.float(), bits)
    c_gpu = compress_tensor(x.to(cuda), bits)
    assert c_gpu.scale == c_cpu.scale and torch.equal(c_gpu.packed.cpu(), c_cpu.packed)
    y = decompress_tensor(c_gpu)
    assert y.dtype == dtype
    assert torch.equal(y.cpu(), decompress_tensor(c_cpu).to(dtype))


def test_misaligned_views(cuda):
    base = _x(10000).to(cuda)
    for off in (1, 2, 3, 5):
        x = base[off:]
        c = compress_tensor(x, 4)
        ref = compress_tensor(x.cpu(), 4)
        assert torch.equal(c.packed.cpu(), ref.packed)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_stochastic_rounding_matches_cpu_philox(cuda, bits):
    x = _x(40000, seed=9)
    q_cpu, _ = quantize_tensor(x, bits, stochastic_rounding=True, seed=1234, offset=7)
    q_gpu, _ = quantize_tensor(x.to(cuda), bits, stochastic_rounding=True, seed=1234, offset=7)
    assert torch.equal(q_gpu.cpu(), q_cpu)


def test_stochastic_rounding_cuda_is_unbiased(cuda):
    x = torch.full((8192,), 0.3, device=cuda)
    x[0] = 1.0
    means = [float(quantize_tensor(x, 2, stochastic_rounding=True)[0][1:].float().mean()) for _ in range(32)]
    assert abs(sum(means) / len(means) - 0.3) < 0.02


@pytest.mark.parametrize("bits", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("sr", [False, True])
def test_ef_roundtrip_matches_cpu(cuda, bits, sr):
    x = _x(30011, seed=bits)
    r = torch.randn(30011) * 0.01
    r_gpu = r.to(cuda)
    y_cpu = ef_roundtrip(x, r, bits, stochastic_rounding=sr, seed=99)
    y_gpu = ef_roundtrip(x.to(cuda), r_gpu, bits, stochastic_rounding=sr, seed=99)
    assert torch.equal(y_gpu.cpu(), y_cpu)
    assert torch.equal(r_gpu.cpu(), r)


def test_roundtrip_cuda_matches_cpu(cuda):
    x = _x(1 << 16)
    for b in SUPPORTED_BITWIDTHS:
        assert torch.equal(roundtrip_tensor(x.to(cuda), b).cpu(), roundtrip_tensor(x, b))


def test_kernels_run_on_current_stream(cuda):
    s = torch.cuda.Stream()
    x = _x(1 << 18).to(cuda)
    with torch.cuda.stream(s):
        c = compress_tensor(x, 4)
        y = decompress_tensor(c)
    s.synchronize()
    assert torch.equal(y.cpu(), decompress_tensor(compress_tensor(x.cpu(), 4)))


@pytest.mark.parametrize("bits", [2, 4, 8, 12, 16])
@pytest.mark.parametrize("amax", [7.0, 0.7, 3.0e-3, 12345.678])
def test_quantize_near_ties_matches_cpu(cuda, bits, amax):
    """Values whose quotient x / scale sits on, or one or two ulps around, a
    half-integer: the kernel must round the correctly rounded fp32 quotient
    half-to-even, exactly as the reference's CPU code does."""
    from bitscom_b200.quantization import _quant_bounds

    _, qmax = _quant_bounds(bits)
    scale = torch.tensor(amax / qmax, dtype=torch.float64).float()
    k = torch.arange(-qmax, qmax, dtype=torch.float32)
    mid = (k + 0.5) * scale
    vals = [mid]
    for d in (1, 2):
        up, dn = mid.clone(), mid.clone()
        for _ in range(d):
            up = torch.nextafter(up, torch.full_like(up, float("inf")))
            dn = torch.nextafter(dn, torch.full_like(dn, -float("inf")))
        vals += [up, dn]
    x = torch.cat(vals + [torch.tensor([amax, -amax])]).clamp(-amax, amax)
    q_cpu, s_cpu = quantize_tensor(x, bits)
    q_gpu, s_gpu = quantize_tensor(x.to(cuda), bits)
    assert s_gpu == s_cpu
    assert torch.equal(q_gpu.cpu(), q_cpu)
    c_cpu, c_gpu = compress_tensor(x, bits), compress_tensor(x.to(cuda), bits)
    assert torch.equal(c_gpu.packed.cpu(), c_cpu.packed)
