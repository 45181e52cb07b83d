"""The allocation-free C entry point ``bitscom_lowbit_allreduce_local_noalloc``.

It exists for callers that cannot call cudaMalloc (code that owns its device
memory through its own arena, or runs where the allocator must not grow); its
scratch is a static device array inside the library.  These tests call it
through its exported C symbol with ctypes, as such a caller would, and check
two consecutive calls bit-for-bit against the regular entry point (a one-rank
Communicator running the same kernel on a cudaMalloc'd workspace).  The file
is named to be collected last.
"""

import ctypes

import pytest
import torch

from bitscom_b200 import _ext
from bitscom_b200.parallel.comm import Communicator

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    so = ctypes.CDLL(_ext.require("the no-alloc entry point test").__file__)
    fn = so.bitscom_lowbit_allreduce_local_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                   ctypes.c_float, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    so.bitscom_noalloc_max_elems.restype = ctypes.c_longlong
    so.bitscom_noalloc_scratch_bytes.restype = ctypes.c_longlong
    so.bitscom_noalloc_strerror.restype = ctypes.c_char_p
    so.bitscom_noalloc_strerror.argtypes = [ctypes.c_int]
    so.bitscom_noalloc_status.restype = ctypes.c_int
    so.bitscom_noalloc_status.argtypes = [ctypes.c_int]
    return so


def _call(lib, x, out, residual, bits, post_scale):
    dt = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[x.dtype]
    rc = lib.bitscom_lowbit_allreduce_local_noalloc(
        x.data_ptr(), out.data_ptr(), residual.data_ptr() if residual is not None else None,
        x.numel(), dt, bits, post_scale, torch.cuda.current_stream().cuda_stream,
    )
    return rc


@pytest.mark.parametrize("dtype,bits,n", [
    (torch.float32, 4, 300001),
    (torch.bfloat16, 8, 300001),
    (torch.float32, 2, 300001),
    (torch.float16, 4, 300001),
    # at the scratch limit with the widest sub-chunks
    (torch.float32, 12, 1 << 20),
    (torch.float32, 16, 1 << 20),
])
def test_noalloc_matches_regular_entry_point_twice(lib, dtype, bits, n):
    torch.manual_seed(0)
    assert n <= lib.bitscom_noalloc_max_elems()
    ref_comm = Communicator.create_local(0, workspace_bytes=64 << 20)
    res_ref = torch.randn(n, device="cuda") * 1e-4
    res_na = res_ref.clone()
    for call in range(2):  # two calls in a row: scratch reuse + residual carried
        x = (torch.randn(n, device="cuda") * (1.0 + call)).to(dtype)
        exp = torch.empty_like(x)
        ref_comm.all_reduce(x, out=exp, bits=bits, residual=res_ref, post_scale=0.25, algo="twoshot")
        got = torch.empty_like(x)
        rc = _call(lib, x, got, res_na, bits, 0.25)
        assert rc == 0, lib.bitscom_noalloc_strerror(rc)
        torch.cuda.synchronize()
        assert lib.bitscom_noalloc_status(0) == 0
        assert torch.equal(got, exp), f"call {call}"
        assert torch.equal(res_na, res_ref), f"call {call}"


def test_noalloc_without_residual(lib):
    x = torch.randn(8192 * 3 + 17, device="cuda")
    exp = torch.empty_like(x)
    Communicator.create_local(0, workspace_bytes=64 << 20).all_reduce(x, out=exp, bits=4, algo="twoshot")
    got = torch.empty_like(x)
    assert _call(lib, x, got, None, 4, 1.0) == 0
    torch.cuda.synchronize()
    assert torch.equal(got, exp)


def test_noalloc_rejects_oversize_and_bad_arguments(lib):
    cap = lib.bitscom_noalloc_max_elems()
    assert cap == 1 << 20
    assert 0 < lib.bitscom_noalloc_scratch_bytes() < 16 << 20
    big = torch.empty(cap + 1, device="cuda")
    rc = _call(lib, big, big, None, 4, 1.0)
    assert rc == -2 and b"capacity" in lib.bitscom_noalloc_strerror(rc)
    x = torch.empty(16, device="cuda")
    assert _call(lib, x, x, None, 3, 1.0) == -1
