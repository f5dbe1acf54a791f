"""The allocation-free C entry point ``es_gemm_bf16_noalloc``, called through its
exported symbol, against an fp32 PyTorch product of the same operands.

This file is named so that pytest collects it last.  The entry point serves
callers that cannot allocate device memory (their own memory pools, runtimes
that forbid cudaMalloc after start-up, non-Python hosts); it keeps its scratch
in a fixed-size static device array, so every case runs twice in a row, the
second call reusing the scratch the first one wrote.  Operands are given in
both storage orders (A as [M][K] or [K][M], B as [N][K] or [K][N]), with
aligned row pitches and with pitches the TMA engine cannot address (those go
through the padded copies in the scratch).  The status getter
``es_gemm_bf16_noalloc_status`` is checked after a bounded wait that runs out.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200 import _C  # noqa: E402
from torch_einshard_b200.ops import _native  # noqa: E402


def _lib():
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.es_gemm_bf16_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    status = lib.es_gemm_bf16_noalloc_status
    status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    status.restype = ctypes.c_int
    return fn, status


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _read_status(status):
    code = ctypes.c_int(-1)
    assert status(ctypes.byref(code), _stream()) == 0
    return code.value


def _stored(rows, cols, pitch):
    """A [rows, cols] bf16 view whose row pitch is ``pitch`` elements."""
    base = torch.randn(rows, pitch, device="cuda", dtype=torch.bfloat16)
    return base[:, :cols]


def _call(fn, a_store, a_mn, b_store, b_mn, m, n, k):
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    rc = fn(a_store.data_ptr(), a_store.stride(0), a_mn, b_store.data_ptr(), b_store.stride(0), b_mn,
            out.data_ptr(), out.stride(0), m, n, k, _stream())
    assert rc == 0
    return out


CASES = [
    # m, n, k, a_mn, b_mn, a pitch pad, b pitch pad (0 = dense rows)
    (512, 768, 256, 0, 0, 0, 0),
    (300, 500, 200, 0, 1, 0, 0),
    (96, 40, 37, 0, 0, 0, 0),       # K = 37: unaligned pitch for both operands
    (130, 45, 21, 0, 1, 0, 0),
    (256, 384, 128, 1, 0, 0, 0),    # A stored [K][M], aligned
    (256, 320, 192, 1, 1, 8, 0),    # A stored [K][M] with a padded (aligned) pitch
    (200, 136, 96, 1, 0, 3, 0),     # A stored [K][M], pitch M + 3: padded copy in the scratch
    (160, 72, 64, 1, 1, 5, 7),      # both operands with unaligned pitches
]


@pytest.mark.parametrize("m,n,k,a_mn,b_mn,a_pad,b_pad", CASES)
def test_noalloc_matches_fp32_matmul_twice(m, n, k, a_mn, b_mn, a_pad, b_pad):
    torch.manual_seed(7)
    fn, status = _lib()
    a_store = _stored(k, m, m + a_pad) if a_mn else _stored(m, k, k + a_pad)
    b_store = _stored(k, n, n + b_pad) if b_mn else _stored(n, k, k + b_pad)
    a = a_store.t() if a_mn else a_store           # [M, K]
    b = b_store if b_mn else b_store.t()           # [K, N]
    want = torch.matmul(a.float(), b.float())
    first = _call(fn, a_store, a_mn, b_store, b_mn, m, n, k)
    second = _call(fn, a_store, a_mn, b_store, b_mn, m, n, k)
    torch.cuda.synchronize()
    scale = want.abs().max().item() + 1.0
    for got in (first, second):
        assert (got.float() - want).abs().max().item() <= 2e-2 * scale
    assert _read_status(status) == 0


def test_noalloc_rejects_operands_beyond_scratch():
    fn, _ = _lib()
    # K = 4097 gives an unaligned row pitch; 4096 rows of it need > 16 MiB of padded copy
    a = torch.randn(4096, 4097, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(64, 4097, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(4096, 64, device="cuda", dtype=torch.bfloat16)
    rc = fn(a.data_ptr(), a.stride(0), 0, b.data_ptr(), b.stride(0), 0, out.data_ptr(), out.stride(0), 4096, 64, 4097,
            _stream())
    assert rc == -2


def test_noalloc_status_reports_a_wait_that_ran_out():
    fn, status = _lib()
    mod = _native.require()
    assert _read_status(status) == 0
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    result = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    # a bounded wait (50 ms) on a flag that nothing sets, recording into the status word
    mod.wait_probe_noalloc_status(flag, 1, 50_000_000, result)
    code = _read_status(status)
    assert int(result.item()) == 0
    assert code != 0
    assert _read_status(status) == 0  # the getter cleared it
    # the entry point still works afterwards
    a = torch.randn(128, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(96, 64, device="cuda", dtype=torch.bfloat16)
    got = _call(fn, a, 0, b, 0, 128, 96, 64)
    torch.cuda.synchronize()
    want = a.float() @ b.float().t()
    assert (got.float() - want).abs().max().item() <= 2e-2 * (want.abs().max().item() + 1.0)
    assert _read_status(status) == 0
