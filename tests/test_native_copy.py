"""Native strided gather copy against torch's .contiguous()."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200.ops import _native, native_ops  # noqa: E402


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.uint8, torch.complex64, torch.float64])
def test_permutes(dtype):
    torch.manual_seed(0)
    base = torch.randn(3, 5, 64, 7, device="cuda").to(dtype) if dtype != torch.uint8 else \
        torch.randint(0, 255, (3, 5, 64, 7), device="cuda", dtype=torch.uint8)
    for perm in [(0, 1, 2, 3), (3, 2, 1, 0), (1, 0, 2, 3), (0, 2, 1, 3), (2, 0, 3, 1)]:
        view = base.permute(perm)
        out = native_ops.strided_copy(view)
        assert out is not None and torch.equal(out, view.contiguous()), perm
    sl = base[:, 1:4, ::2, 2:]
    assert torch.equal(native_ops.strided_copy(sl), sl.contiguous())
    _native.check_errors()


@pytest.mark.parametrize("shape,k", [((2, 10, 12, 128), 3), ((1, 7, 9, 64), 5), ((3, 4, 300, 8), 3)])
def test_window_views(shape, k):
    x = torch.randn(*shape, device="cuda", dtype=torch.bfloat16)
    u = x.unfold(1, k, 1).unfold(2, k, 1)            # b h w c kh kw
    view = u.permute(0, 1, 2, 4, 5, 3)                 # b h w kh kw c
    out = native_ops.strided_copy(view)
    assert torch.equal(out, view.contiguous())
    _native.check_errors()


def test_einwindow_uses_native(monkeypatch):
    import torch_einshard_b200 as es
    calls = []
    real = native_ops.strided_copy
    monkeypatch.setattr(native_ops, "strided_copy", lambda v: calls.append(1) or real(v))
    x = torch.randn(2, 16, 24, 128, device="cuda", dtype=torch.bfloat16)
    y = es.einwindow("b h w c -> b h w kh kw c", x, {"h": "kh", "w": "kw"}, {"h": 1, "w": 1})
    ref = torch.nn.functional.pad(x, (0, 0, 1, 1, 1, 1)).unfold(1, 3, 1).unfold(2, 3, 1).permute(0, 1, 2, 4, 5, 3)
    assert torch.equal(y, ref)
    assert calls
