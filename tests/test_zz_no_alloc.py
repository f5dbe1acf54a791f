"""The allocation-free C entry point ``es_gemm_bf16_noalloc``, called through its
exported symbol, against the regular GEMM entry point.

This file is named so that pytest collects it last.  The entry point serves
callers that cannot allocate device memory (their own memory pools, runtimes
that forbid cudaMalloc after start-up, non-Python hosts); it keeps its scratch
in a fixed-size static device array, so this test also checks that a second
call in a row, which reuses that scratch, gives the same result.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200 import _C  # noqa: E402
from torch_einshard_b200.ops import _native, gemm  # noqa: E402


def _entry():
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.es_gemm_bf16_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _call(fn, a, b, b_mn):
    """a: [M, K] row-major view (row pitch a.stride(0)); b: [N, K] (b_mn=0) or [K, N] (b_mn=1)."""
    m, k = a.shape
    n = b.shape[0] if b_mn == 0 else b.shape[1]
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    rc = fn(a.data_ptr(), a.stride(0), 0, b.data_ptr(), b.stride(0), b_mn, out.data_ptr(), out.stride(0), m, n, k,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return out


def _existing(a, b, b_mn):
    bb = b.t()[None] if b_mn == 0 else b[None]
    return gemm.native_bmm(a[None], bb)[0]


@pytest.mark.parametrize("m,n,k,b_mn", [(512, 768, 256, 0), (300, 500, 200, 1), (96, 40, 37, 0), (130, 45, 21, 1)])
def test_noalloc_matches_existing_entry_point_twice(m, n, k, b_mn):
    torch.manual_seed(7)
    fn = _entry()
    a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    b = (torch.randn(n, k, device="cuda", dtype=torch.bfloat16) if b_mn == 0
         else torch.randn(k, n, device="cuda", dtype=torch.bfloat16))
    want = _existing(a, b, b_mn).float()
    first = _call(fn, a, b, b_mn)
    second = _call(fn, a, b, b_mn)
    torch.cuda.synchronize()
    scale = want.abs().max().item() + 1.0
    for got in (first, second):
        assert (got.float() - want).abs().max().item() <= 2e-2 * scale
    _native.check_errors(a.device)


def test_noalloc_rejects_operands_beyond_scratch():
    fn = _entry()
    # K = 4097 gives an unaligned row pitch; 4096 rows of it need > 16 MiB of padded copy
    a = torch.randn(4096, 4097, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(64, 4097, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(4096, 64, device="cuda", dtype=torch.bfloat16)
    rc = fn(a.data_ptr(), a.stride(0), 0, b.data_ptr(), b.stride(0), 0, out.data_ptr(), out.stride(0), 4096, 64, 4097,
            torch.cuda.current_stream().cuda_stream)
    assert rc == -2
