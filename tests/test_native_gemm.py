"""tcgen05 GEMM numerics against a plain fp32 PyTorch matmul."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200.ops import _native, gemm  # noqa: E402


@pytest.fixture(params=[0, 1, 2], ids=["1sm", "2sm", "2sm_wide"], autouse=True)
def kernel_variant(request):
    """Run every case on the 1-SM, the 2-SM (CTA pair) and the wide 2-SM kernel."""
    mod = _native.require()
    mod.set_gemm_pair_mode(request.param)
    yield request.param
    mod.set_gemm_pair_mode(-1)


def _operand(shape_rows, shape_cols, batch, dtype, transposed):
    """[batch, rows, cols] view; transposed=True stores it column-major."""
    if transposed:
        return torch.randn(batch, shape_cols, shape_rows, device="cuda", dtype=dtype).transpose(1, 2)
    return torch.randn(batch, shape_rows, shape_cols, device="cuda", dtype=dtype)


def _check(a, b, out_dtype=None, tol=None):
    _native.reset_errors()
    c = gemm.native_bmm(a, b, out_dtype=out_dtype)
    torch.cuda.synchronize()
    _native.check_errors(a.device)
    ref = torch.matmul(a.float(), b.float())
    k = a.shape[-1]
    tol = tol or (2e-2 if c.dtype != torch.float32 else 1e-3)
    scale = ref.abs().max().item() + 1.0
    err = (c.float() - ref).abs().max().item()
    assert err <= tol * scale * max(1.0, (k / 256) ** 0.5), f"max err {err} (scale {scale})"


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_majorness(a_t, b_t):
    torch.manual_seed(0)
    a = _operand(256, 192, 1, torch.bfloat16, a_t)
    b = _operand(192, 512, 1, torch.bfloat16, b_t)
    _check(a, b)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (1, 8, 8), (300, 500, 200), (129, 257, 72), (1000, 24, 1032)])
def test_gemm_ragged_shapes(m, n, k):
    torch.manual_seed(1)
    a = _operand(m, k, 1, torch.bfloat16, False)
    b = _operand(k, n, 1, torch.bfloat16, True)
    _check(a, b)


def test_gemm_batched_fp16_and_fp32_out():
    torch.manual_seed(2)
    a = _operand(200, 136, 3, torch.float16, False)
    b = _operand(136, 264, 3, torch.float16, False)
    _check(a, b)
    _check(a, b, out_dtype=torch.float32)


def test_gemm_unaligned_row_pitch_is_padded():
    torch.manual_seed(3)
    a = torch.randn(1, 70, 37, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1, 37, 45, device="cuda", dtype=torch.bfloat16)
    _check(a, b)


def test_gemm_large_multi_wave():
    torch.manual_seed(4)
    a = _operand(4096, 2048, 1, torch.bfloat16, False)
    b = _operand(2048, 3072, 1, torch.bfloat16, True)
    _check(a, b)


def test_gemm_autograd_matches_torch():
    torch.manual_seed(5)
    a = torch.randn(2, 192, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    b = torch.randn(2, 128, 320, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    out = gemm.matmul(a, b)
    g = torch.randn_like(out)
    out.backward(g)
    ra, rb = a.detach().float().requires_grad_(), b.detach().float().requires_grad_()
    torch.matmul(ra, rb).backward(g.float())
    for got, ref in ((a.grad, ra.grad), (b.grad, rb.grad)):
        scale = ref.abs().max().item() + 1.0
        assert (got.float() - ref).abs().max().item() <= 3e-2 * scale
    _native.check_errors(a.device)


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("m,n,k", [(1000, 128, 320), (777, 100, 64), (4096, 8, 128)])
def test_gemm_narrow_n_runs_transposed(a_t, b_t, m, n, k):
    """N narrower than a tile with M larger: computed as C^T = B^T A^T, stored transposed."""
    torch.manual_seed(5)
    a = _operand(m, k, 1, torch.bfloat16, a_t)
    b = _operand(k, n, 1, torch.bfloat16, b_t)
    _check(a, b)
    _check(a, b, out_dtype=torch.float32)


def test_gemm_narrow_n_batched_silu():
    torch.manual_seed(6)
    a = _operand(640, 96, 3, torch.bfloat16, False)
    b = _operand(96, 64, 3, torch.bfloat16, True)
    _native.reset_errors()
    c = gemm.native_bmm(a, b, act="silu")
    ref = torch.nn.functional.silu(torch.matmul(a.float(), b.float()))
    assert (c.float() - ref).abs().max().item() <= 2e-2 * (ref.abs().max().item() + 1)
