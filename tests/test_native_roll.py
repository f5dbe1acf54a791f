"""Native multi-axis roll (csrc/copy.cu roll_copy) against torch.roll on CUDA:
every dtype size, rolled innermost and outer dims, negative and oversized
shifts, several axes in one pass, and the gradient (roll by the negated shifts)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200 import einroll  # noqa: E402
from torch_einshard_b200.ops import _native  # noqa: E402
from torch_einshard_b200.ops.native_ops import local_roll  # noqa: E402

CASES = [
    ((7, 33), {1: 5}),
    ((7, 33), {0: -3, 1: 40}),
    ((4, 6, 8, 16), {1: 2, 3: 3}),
    ((4, 6, 8, 16), {0: 1, 2: -9}),
    ((3, 5, 128), {0: 2, 1: 4}),            # tail of 128 elements: vector units
    ((2, 3, 4, 5, 6, 7, 2, 3, 2), {0: 1, 4: 2, 8: 1}),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.complex64, torch.int8])
@pytest.mark.parametrize("shape,shifts", CASES)
def test_local_roll_matches_torch_roll(dtype, shape, shifts):
    if dtype == torch.int8:
        x = torch.randint(-100, 100, shape, device="cuda", dtype=dtype)
    else:
        x = torch.randn(shape, device="cuda", dtype=dtype)
    dims = list(shifts)
    want = torch.roll(x, shifts=[shifts[d] for d in dims], dims=dims)
    got = local_roll(x, shifts)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_local_roll_gradient_and_einroll():
    x = torch.randn(6, 10, 12, device="cuda", requires_grad=True)
    g = torch.randn(6, 10, 12, device="cuda")
    y = einroll("a b c", x, {"a": 2, "c": -5})
    y.backward(g)
    assert torch.equal(y, torch.roll(x.detach(), shifts=(2, -5), dims=(0, 2)))
    assert torch.equal(x.grad, torch.roll(g, shifts=(-2, 5), dims=(0, 2)))
    mod = _native.require()
    assert mod.launch_count() > 0


def test_local_roll_of_lazy_conjugate_views():
    """Lazy conjugate / negative views (autograd passes conj(grad) that way) are
    rolled by value, forward and backward."""
    from torch_einshard_b200.ops.native_ops import local_roll
    z = torch.randn(3, 6, 5, dtype=torch.complex64, device="cuda")
    for view in (z.conj(), torch.neg(z.conj()).conj()):
        torch.testing.assert_close(local_roll(view, {1: 2, 2: -1}), torch.roll(view, (2, -1), (1, 2)))
    zr = z.clone().requires_grad_(True)
    zt = z.clone().requires_grad_(True)
    local_roll(zr, {1: 1}).conj().abs().sum().backward()
    torch.roll(zt, 1, 1).conj().abs().sum().backward()
    torch.testing.assert_close(zr.grad, zt.grad)
