"""GEMM + SiLU (einshard's activation="silu") against fp32 PyTorch.

The large shape runs on the wide kernel, whose epilogue writes the
pre-activation and its SiLU from one pass over the accumulator; the small one
takes the GEMM followed by the native elementwise pass.  Forward values, the
pre-activation kept for backward, and the gradients of both operands through
the public API are checked against fp32 autograd of the same bf16 values.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200 import einshard  # noqa: E402
from torch_einshard_b200.ops import _native  # noqa: E402


def _rel(got, want):
    return (got.float() - want).abs().max().item() / (want.abs().max().item() + 1e-6)


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 512), (130, 200, 64), (4096, 3584, 1024)])
def test_gemm_silu_forward_and_pre_activation(m, n, k):
    mod = _native.require()
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(1, m, k, device="cuda", dtype=torch.bfloat16, generator=g)
    b = torch.randn(1, n, k, device="cuda", dtype=torch.bfloat16, generator=g).transpose(1, 2)
    out, pre = mod.gemm_silu(a, b, _native.error_word("cuda"))
    torch.cuda.synchronize()
    _native.check_errors("cuda")
    want_pre = a.float() @ b.float()
    assert _rel(pre, want_pre) < 1e-2
    assert _rel(out, torch.nn.functional.silu(want_pre)) < 1e-2


@pytest.mark.parametrize("rows,cols", [(2, 4096), (3, 1001)])
def test_silu_elementwise_kernels(rows, cols):
    mod = _native.require()
    h = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16) * 4
    grad = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16)
    hr = h.float().requires_grad_(True)
    y = torch.nn.functional.silu(hr)
    y.backward(grad.float())
    assert _rel(mod.silu_forward(h), y.detach()) < 1e-2
    assert _rel(mod.silu_backward(grad, h), hr.grad) < 1e-2


@pytest.mark.parametrize("n,c,h", [(1024, 512, 4096), (64, 96, 160)])
def test_einshard_activation_matches_fp32_autograd(n, c, h):
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(2, n, c, device="cuda", dtype=torch.bfloat16, generator=g).requires_grad_(True)
    w = (torch.randn(h, c, device="cuda", dtype=torch.bfloat16, generator=g) * 0.05).requires_grad_(True)
    dy = torch.randn(2, n, h, device="cuda", dtype=torch.bfloat16, generator=g)
    y = einshard("b n c, h c -> b n h", x, w, activation="silu")
    y.backward(dy)
    torch.cuda.synchronize()
    _native.check_errors("cuda")
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    yr = torch.nn.functional.silu(torch.einsum("bnc,hc->bnh", xr, wr))
    yr.backward(dy.float())
    assert _rel(y, yr.detach()) < 2e-2
    assert _rel(x.grad, xr.grad) < 3e-2
    assert _rel(w.grad, wr.grad) < 3e-2


def test_activation_rejects_partial_outputs():
    x = torch.randn(4, 8, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="partial"):
        einshard("a b, b c -> a c // tp", x, x.t().contiguous(), activation="silu")
