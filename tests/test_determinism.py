"""Run-to-run determinism of the native kernels (same inputs twice -> the same
bits).  A data race in a pipeline or flag protocol (a stage read before it is
filled, a tile stored twice) shows up as a bitwise difference between runs;
none of these kernels reduces in a run-dependent order, so equality is exact."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200.ops import _native, gemm  # noqa: E402
from torch_einshard_b200.ops.conv_impl import conv2d_native  # noqa: E402
from torch_einshard_b200.ops.fft_impl import fft_c2c  # noqa: E402

REPEATS = 4


def _repeat(fn):
    _native.reset_errors()
    outs = [fn().clone() for _ in range(REPEATS)]
    torch.cuda.synchronize()
    _native.check_errors("cuda")
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    return outs[0]


@pytest.mark.parametrize("mode", [0, 1, 2], ids=["1sm", "2sm", "2sm_wide"])
@pytest.mark.parametrize("shape", [(1, 1000, 1100, 520), (3, 257, 640, 192), (1, 2048, 2048, 4096)])
def test_gemm_bitwise_repeatable(mode, shape):
    mod = _native.require()
    mod.set_gemm_pair_mode(mode)
    try:
        b, m, n, k = shape
        x = torch.randn(b, m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(b, k, n, device="cuda", dtype=torch.bfloat16)
        _repeat(lambda: gemm.native_bmm(x, w))
    finally:
        mod.set_gemm_pair_mode(-1)


def test_conv_bitwise_repeatable():
    x = torch.randn(2, 37, 300, 128, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(192, 3, 3, 128, device="cuda", dtype=torch.bfloat16) * 0.05
    bias = torch.randn(192, device="cuda", dtype=torch.float32)
    _repeat(lambda: conv2d_native(x, w, bias, 1, 1))


@pytest.mark.parametrize("n,dim", [(1024, -1), (64, 1), (512, 0)])
def test_fft_bitwise_repeatable(n, dim):
    shape = [8, 8, 8]
    shape[dim] = n
    x = torch.randn(*shape, device="cuda", dtype=torch.complex64)
    mod = _native.require()
    _repeat(lambda: fft_c2c(mod, x, dim, False))
