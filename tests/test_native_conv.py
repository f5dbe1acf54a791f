"""Implicit-GEMM conv2d (tcgen05, NHWC) against an fp32 PyTorch reference:
both forward kernels (the CTA-pair kernel with resident weights and the
weights-streaming kernel), per-side zero padding, backward."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200.ops import _native  # noqa: E402
from torch_einshard_b200.ops.conv_impl import conv2d_native  # noqa: E402


def _ref(x, w, bias, pad=0):
    out = F.conv2d(x.float().permute(0, 3, 1, 2), w.float().permute(0, 3, 1, 2),
                   None if bias is None else bias.float(), padding=pad)
    return out.permute(0, 2, 3, 1)


def _close(got, want, tol=2e-2):
    scale = want.abs().max().item() + 1e-6
    err = (got.float() - want).abs().max().item()
    assert err <= tol * scale, (err, scale)


@pytest.mark.parametrize("B,H,W,C,O,K", [(1, 8, 8, 64, 128, 3), (2, 17, 300, 64, 96, 3), (1, 5, 513, 128, 128, 1),
                                         (3, 9, 40, 192, 256, 5), (1, 4, 4, 64, 8, 3),
                                         (2, 40, 1000, 128, 128, 3), (1, 10, 70, 64, 256, 7)])
@pytest.mark.parametrize("kernel", [0, 1])
def test_conv_forward(B, H, W, C, O, K, kernel, monkeypatch):
    from torch_einshard_b200.ops import conv_impl
    monkeypatch.setattr(conv_impl, "_KERNEL", kernel)
    torch.manual_seed(0)
    x = torch.randn(B, H, W, C, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(O, K, K, C, device="cuda") * 0.05).to(torch.bfloat16)
    bias = torch.randn(O, device="cuda")
    got = conv2d_native(x, w, bias)
    _close(got, _ref(x, w, bias))
    again = conv2d_native(x, w, bias)
    assert torch.equal(got, again)
    _native.check_errors()


def test_conv_backward():
    torch.manual_seed(1)
    x = torch.randn(2, 12, 33, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(128, 3, 3, 64, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    bias = torch.randn(128, device="cuda", requires_grad=True)
    y = conv2d_native(x, w, bias)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    br = bias.detach().clone().requires_grad_(True)
    _ref(xr, wr, br).backward(g.float())
    _close(x.grad, xr.grad)
    _close(w.grad, wr.grad)
    _close(bias.grad, br.grad, tol=1e-3)
    _native.check_errors()


def test_einconv_local_uses_native(monkeypatch):
    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import conv_impl
    calls = []
    real = conv_impl._run
    monkeypatch.setattr(conv_impl, "_run", lambda *a, **k: calls.append(1) or real(*a, **k))
    torch.manual_seed(2)
    x = torch.randn(2, 16, 40, 64, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(3, 3, 64, 128, device="cuda") * 0.05).to(torch.bfloat16)
    y = es.einconv("b h w c, kh kw c o -> b h w o", x, w, {"h": "kh", "w": "kw"})
    want = _ref(x, w.permute(3, 0, 1, 2), None, pad=1)
    _close(y, want)
    assert calls


@pytest.mark.parametrize("pad", [1, 2])
def test_conv_kernel_padding_forward_backward(pad):
    torch.manual_seed(3)
    K = 2 * pad + 1
    x = torch.randn(2, 9, 37, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(64, K, K, 64, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    y = conv2d_native(x, w, None, pad, pad)
    assert y.shape == (2, 9, 37, 64)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    yr = _ref(xr, wr, None, pad=pad)
    yr.backward(g.float())
    _close(y, yr)
    _close(x.grad, xr.grad)
    _close(w.grad, wr.grad)
    _native.check_errors()


def test_einconv_pads_in_kernel_without_copy(monkeypatch):
    """Local zero-boundary axes are padded by the kernel: no halo_tensor copy is made."""
    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import conv as conv_mod
    calls = []
    real = conv_mod.halo_tensor

    def spy(spec, x, halos, **kw):
        if halos:
            calls.append(dict(halos))
        return real(spec, x, halos, **kw)
    monkeypatch.setattr(conv_mod, "halo_tensor", spy)
    x = torch.randn(2, 16, 40, 64, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(3, 3, 64, 128, device="cuda") * 0.05).to(torch.bfloat16)
    y = es.einconv("b h w c, kh kw c o -> b h w o", x, w, {"h": "kh", "w": "kw"}, checkpoint=None)
    _close(y, _ref(x, w.permute(3, 0, 1, 2), None, pad=1))
    assert calls == []


@pytest.mark.parametrize("B,H,W,C,O,KH,KW,ph,pw", [
    (2, 12, 33, 64, 128, 3, 3, 0, 0),     # one partial column block per row
    (1, 9, 130, 128, 64, 3, 3, 1, 1),     # O < one M tile, three column blocks, padding
    (3, 5, 64, 64, 192, 1, 3, 0, 1),      # two M tiles, 1 x 3 kernel, exact column blocks
    (2, 7, 20, 192, 64, 5, 5, 2, 2),      # N = 25 * 192 spans many N tiles
    (4, 64, 256, 128, 128, 3, 3, 1, 1),   # split-K over 59 slices, the last one past the end
])
def test_conv_weight_gradient_native(B, H, W, C, O, KH, KW, ph, pw):
    torch.manual_seed(2)
    mod = _native.require()
    x = torch.randn(B, H, W, C, device="cuda", dtype=torch.bfloat16)
    Ho, Wo = H + 2 * ph - KH + 1, W + 2 * pw - KW + 1
    dy = torch.randn(B, Ho, Wo, O, device="cuda", dtype=torch.bfloat16)
    dw = torch.empty(O, KH, KW, C, device="cuda", dtype=torch.float32)
    mod.conv2d_wgrad(x, dy, dw, ph, pw, -1, -1, _native.error_word(x.device))
    torch.cuda.synchronize()
    _native.check_errors()
    ref = torch.nn.grad.conv2d_weight(x.float().permute(0, 3, 1, 2), (O, C, KH, KW), dy.float().permute(0, 3, 1, 2),
                                      padding=(ph, pw)).permute(0, 2, 3, 1)
    scale = ref.abs().max().item()
    assert (dw - ref).abs().max().item() <= 1e-4 * scale + 1e-3, (dw - ref).abs().max().item()


@pytest.mark.parametrize("kernel", [0, 1])
@pytest.mark.parametrize("ph,pw", [((1, 0), (0, 1)), ((0, 2), (2, 0)), ((1, 1), (0, 0))])
def test_conv_per_side_padding_forward_backward(ph, pw, kernel, monkeypatch):
    """Zero padding that differs per side (the global edge of a sharded axis)."""
    from torch_einshard_b200.ops import conv_impl
    monkeypatch.setattr(conv_impl, "_KERNEL", kernel)
    torch.manual_seed(4)
    x = torch.randn(2, 11, 300, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(128, 3, 3, 64, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    bias = torch.randn(128, device="cuda", requires_grad=True)
    y = conv2d_native(x, w, bias, ph, pw)
    assert y.shape == (2, 11 + sum(ph) - 2, 300 + sum(pw) - 2, 128)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    br = bias.detach().clone().requires_grad_(True)
    xp = F.pad(xr.permute(0, 3, 1, 2), (pw[0], pw[1], ph[0], ph[1]))
    yr = F.conv2d(xp, wr.permute(0, 3, 1, 2), br).permute(0, 2, 3, 1)
    yr.backward(g.float())
    _close(y, yr)
    _close(x.grad, xr.grad)
    _close(w.grad, wr.grad)
    _close(bias.grad, br.grad, tol=1e-3)
    _native.check_errors()


@pytest.mark.parametrize("gtop,gbot,ph", [(1, 1, (0, 0)), (1, 0, (0, 1)), (0, 2, (2, 0)), (2, 2, (0, 0))])
def test_conv_ghost_rows_forward_backward(gtop, gbot, ph):
    """Rows read from a separate ghost tensor above and below x (the halo of a
    sharded axis) give the conv of the assembled input, forward and backward."""
    from torch_einshard_b200.ops.conv_impl import conv2d_ghost_rows
    torch.manual_seed(5)
    B, H, W, C, O, K = 2, 9, 300, 64, 128, 5 if max(gtop, gbot) > 1 else 3
    x = torch.randn(B, H, W, C, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    g = torch.randn(B, gtop + gbot, W, C, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(O, K, K, C, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    bias = torch.randn(O, device="cuda", requires_grad=True)
    pw = (K // 2, K // 2)
    # ghosts are constants here: the adjoint keeps the shard's rows
    y = conv2d_ghost_rows(x, g, gtop, gbot, lambda dv: dv[:, gtop:gtop + H], w, bias, ph, pw)
    full = torch.cat([g[:, :gtop].float(), x.detach().float(), g[:, gtop:].float()], 1).requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    br = bias.detach().clone().requires_grad_(True)
    xp = F.pad(full.permute(0, 3, 1, 2), (pw[0], pw[1], ph[0], ph[1]))
    yr = F.conv2d(xp, wr.permute(0, 3, 1, 2), br).permute(0, 2, 3, 1)
    assert y.shape == yr.shape
    _close(y, yr)
    gy = torch.randn_like(y)
    y.backward(gy)
    yr.backward(gy.float())
    _close(x.grad, full.grad[:, gtop:gtop + H])
    _close(w.grad, wr.grad)
    _close(bias.grad, br.grad, tol=1e-3)
    _native.check_errors()


@pytest.mark.parametrize("gl,gr,gtop,gbot,ph,pw", [(1, 1, 1, 1, (0, 0), (0, 0)), (1, 0, 0, 1, (1, 0), (0, 1)),
                                                   (0, 1, 0, 0, (1, 1), (1, 0))])
def test_conv_ghost_2d_native(gl, gr, gtop, gbot, ph, pw):
    """The two-axis ghost conv on the native kernels (wider ghost rows, output
    column ranges, transposed strips) against a conv of the assembled input."""
    from torch_einshard_b200.ops.conv_impl import conv2d_ghost_2d
    torch.manual_seed(6)
    B, H, W, C, O = 2, 20, 300, 64, 128
    full = torch.randn(B, gtop + H + gbot, gl + W + gr, C, device="cuda", dtype=torch.bfloat16)
    x = full[:, gtop:gtop + H, gl:gl + W].contiguous()
    cols = torch.cat([full[:, gtop:gtop + H, :gl], full[:, gtop:gtop + H, gl + W:]], 2).contiguous()
    ghosts = torch.cat([full[:, :gtop], full[:, gtop + H:]], 1).contiguous() if gtop + gbot else None
    w = (torch.randn(O, 3, 3, C, device="cuda") * 0.05).to(torch.bfloat16)
    bias = torch.randn(O, device="cuda")
    got = conv2d_ghost_2d(x, ghosts, gtop, gbot, cols, gl, gr, w, bias, ph, pw)
    xp = F.pad(full.float().permute(0, 3, 1, 2), (pw[0], pw[1], ph[0], ph[1]))
    want = F.conv2d(xp, w.float().permute(0, 3, 1, 2), bias).permute(0, 2, 3, 1)
    assert got.shape == want.shape
    _close(got, want)
    _native.check_errors()


def test_einconv_1d_runs_native_as_height_one(monkeypatch):
    """A 1-D einconv runs on the native kernels as a 2-D conv of height 1
    (forward and backward) and matches F.conv1d."""
    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import conv_impl
    calls = []
    real = conv_impl._run
    monkeypatch.setattr(conv_impl, "_run", lambda *a, **k: calls.append(1) or real(*a, **k))
    torch.manual_seed(7)
    x = torch.randn(3, 500, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(5, 64, 128, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    y = es.einconv("b l c, k c o -> b l o", x, w, {"l": "k"}, checkpoint=None)
    assert calls
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    yr = F.conv1d(xr.permute(0, 2, 1), wr.permute(2, 1, 0), padding=2).permute(0, 2, 1)
    _close(y, yr)
    g = torch.randn_like(y)
    y.backward(g)
    yr.backward(g.float())
    _close(x.grad, xr.grad)
    _close(w.grad, wr.grad)
    _native.check_errors()
