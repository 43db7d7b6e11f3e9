"""The allocation-free GEMM entry point, called through its exported C symbol.

`b200_gemm_bf16_noalloc` serves callers that cannot allocate device memory:
its split-K scratch is a fixed area compiled into the library instead of
memory taken from PyTorch's allocator.  This test loads the extension as a
plain shared library, calls the symbol twice in a row with fresh inputs and
checks each result against the ordinary op (torch.ops.b200.gemm_bf16_out)
with the same tolerance as the other GEMM tests, reads the kernel's status
word back through `b200_gemm_bf16_noalloc_status` (0 = no device-side
error), and checks that the second call changes neither PyTorch's allocator
counters nor the device's free memory.  It also checks that a shape needing
more scratch than the fixed maximum is refused with the documented code.
(This file is named so pytest collects it last.)
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOO_LARGE = -1


def _entry():
    from vllm_cmp170hx_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    f = lib.b200_gemm_bf16_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return f


def _status():
    from vllm_cmp170hx_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    g = lib.b200_gemm_bf16_noalloc_status
    g.restype = ctypes.c_int
    g.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_void_p]
    word = ctypes.c_uint32(0xFFFFFFFF)
    rc = g(ctypes.byref(word), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    return word.value


def _call(f, x, w, y, splits=0):
    M, K = x.shape
    N = w.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return f(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(), y.stride(0), M, N, K, splits, stream)


def _rel_err(y, r):
    return ((y.float() - r.float()).norm() / r.float().norm().clamp_min(1e-12)).item()


# (M, N, K, splits): the first two split K through fp32 partials in the fixed scratch (more than
# 8 splits, or more than 128 rows); the last lets the library choose, which for a small M reduces
# the splits on chip and leaves the scratch alone.
CASES = [(8, 1024, 4096, 16), (256, 1024, 4096, 2), (8, 1024, 4096, 0)]


@pytest.mark.parametrize("M,N,K,splits", CASES)
def test_noalloc_matches_existing_entry_point_twice(M, N, K, splits):
    from vllm_cmp170hx_b200 import ops

    f = _entry()
    torch.manual_seed(0)
    for call in range(2):
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
        expected = ops.gemm(x, w)
        y = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        torch.cuda.synchronize()
        allocs = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        free0 = torch.cuda.mem_get_info()[0]
        rc = _call(f, x, w, y, splits)
        torch.cuda.synchronize()
        assert rc == 0, (call, rc)
        assert _status() == 0, call
        if call == 1:  # the first call may load the kernel's module; the second allocates nothing
            assert torch.cuda.memory_stats().get("allocation.all.allocated", 0) == allocs
            assert torch.cuda.mem_get_info()[0] > free0 - (2 << 20)
        assert _rel_err(y, expected) < 1e-2, (call, _rel_err(y, expected))
        err = (y.float() - expected.float()).abs().max().item()
        assert err <= 2e-2 * expected.float().abs().max().item() + 1e-3, (call, err)


def test_noalloc_refuses_more_scratch_than_its_maximum():
    f = _entry()
    M, N, K = 64, 8192, 8192
    x = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    y = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    assert _call(f, x, w, y, splits=16) == TOO_LARGE
