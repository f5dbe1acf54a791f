"""Native complex64 FFT kernels against torch.fft (fp32 reference), and the
einfft slab path (transpose fused into the FFT loads) on 2+ GPUs."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200.ops import _native  # noqa: E402
from torch_einshard_b200.ops.fft_impl import fft_c2c  # noqa: E402


def _close(got, want, tol=2e-5):
    scale = want.abs().max().item() + 1e-30
    err = (got - want).abs().max().item()
    assert err <= tol * scale, (err, scale)


@pytest.mark.parametrize("n", [2, 4, 8, 16, 32, 64, 128, 256, 512, 1024])
@pytest.mark.parametrize("inverse", [False, True])
def test_fft_lengths_last_dim(n, inverse):
    mod = _native.require()
    x = torch.randn(7, n, dtype=torch.complex64, device="cuda")
    got = fft_c2c(mod, x, 1, inverse)
    want = torch.fft.ifft(x.cdouble(), dim=1, norm="forward") if inverse else torch.fft.fft(x.cdouble(), dim=1)
    _close(got.cdouble(), want, tol=1e-5 * (1 + n.bit_length()))
    _native.check_errors()


@pytest.mark.parametrize("shape,dim", [((3, 64, 10), 1), ((5, 1024, 24), 1), ((1024, 6), 0), ((2, 3, 256, 1), 2),
                                       ((32, 128), 0), ((4, 8, 16), 0)])
def test_fft_strided_axes(shape, dim):
    mod = _native.require()
    x = torch.randn(*shape, dtype=torch.complex64, device="cuda")
    got = fft_c2c(mod, x, dim, False)
    want = torch.fft.fft(x.cdouble(), dim=dim)
    _close(got.cdouble(), want, tol=1e-4)
    # twice in a row on the same input gives identical results (no shared-state races)
    again = fft_c2c(mod, x, dim, False)
    assert torch.equal(got, again)


def test_fft_unsupported_falls_back():
    mod = _native.require()
    x = torch.randn(4, 12, dtype=torch.complex64, device="cuda")
    assert fft_c2c(mod, x, 1, False) is None
    assert fft_c2c(mod, x.to(torch.complex128), 0, False) is None


def test_fft_autograd_matches_torch():
    mod = _native.require()
    x = torch.randn(6, 256, dtype=torch.complex64, device="cuda", requires_grad=True)
    g = torch.randn(6, 256, dtype=torch.complex64, device="cuda")
    y = fft_c2c(mod, x, 1, False, scale=0.5)
    y.backward(g)
    x2 = x.detach().clone().requires_grad_(True)
    (torch.fft.fft(x2, dim=1) * 0.5).backward(g)
    _close(x.grad, x2.grad, tol=1e-4)


def test_einfft_local_uses_native(monkeypatch):
    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import fft_impl
    calls = []
    real = fft_impl._run
    monkeypatch.setattr(fft_impl, "_run", lambda *a, **k: calls.append(1) or real(*a, **k))
    x = torch.randn(2, 64, 32, dtype=torch.complex64, device="cuda")
    y = es.einfft("b x y -> b kx ky", x, {"x": "kx", "y": "ky"})
    torch.testing.assert_close(y, torch.fft.fftn(x, dim=(1, 2)), rtol=1e-4, atol=1e-3)
    assert len(calls) == 2


def _slab(rank, world):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native, fft_impl

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("sp",))
    assert es.setup_native_comm(mesh)
    calls = []
    real = fft_impl._slab_run
    fft_impl._slab_run = lambda *a, **k: calls.append(1) or real(*a, **k)
    for (b, X, Y, Z) in [(1, 64, 32, 16), (2, 128, 64, 8)]:
        torch.manual_seed(5)
        full = torch.randn(b, X, Y, Z, dtype=torch.complex64, device="cuda")
        xl, yl = X // world, Y // world
        local = full[:, rank * xl:(rank + 1) * xl].contiguous().requires_grad_(True)
        for _ in range(2):  # repeated calls reuse the symmetric region (epochs)
            out = es.einfft("b x/sp y z -> b kx ky/sp kz", local, {"x": "kx", "y": "ky", "z": "kz"}, mesh=mesh)
            want = torch.fft.fftn(full.cdouble(), dim=(1, 2, 3))[:, :, rank * yl:(rank + 1) * yl]
            scale = want.abs().max().item()
            assert (out.cdouble() - want).abs().max().item() < 1e-5 * scale * 8
        g = torch.randn_like(out)
        out.backward(g)
        # gradient oracle: full-tensor autograd through torch.fft.fftn
        full_g = torch.zeros(b, X, Y, Z, dtype=torch.complex64, device="cuda")
        gs = [torch.empty_like(g) for _ in range(world)]
        dist.all_gather(gs, g)
        full_g = torch.cat(gs, dim=2)
        ref = full.detach().clone().requires_grad_(True)
        torch.fft.fftn(ref, dim=(1, 2, 3)).backward(full_g)
        want_g = ref.grad[:, rank * xl:(rank + 1) * xl]
        assert (local.grad - want_g).abs().max().item() < 1e-4 * want_g.abs().max().item()
        # inverse with ortho norm round-trips
        back = es.einfft("b kx ky/sp kz -> b x/sp y z", out.detach(), {"kx": "x", "ky": "y", "kz": "z"},
                         inverse=True, mesh=mesh)
        assert (back - local.detach()).abs().max().item() < 1e-4 * local.abs().max().item()
    assert calls, "the native slab path did not run"
    torch.cuda.synchronize()
    _native.check_errors()


@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_einfft_slab_two_gpus():
    from gpu_harness import run_gpus
    run_gpus(_slab, 2)


@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_einfft_slab_four_gpus():
    from gpu_harness import run_gpus
    run_gpus(_slab, 4)


@pytest.mark.parametrize("shape,dim", [((16, 1024), 1), ((3, 1024, 16), 1), ((1024, 40), 0), ((2, 1024, 8, 2), 1),
                                       ((300, 1024), 1)])
@pytest.mark.parametrize("inverse", [False, True])
def test_fft_1024_pipelined_kernel(shape, dim, inverse):
    """1024-point lines in whole tiles take the persistent cp.async-pipelined kernel."""
    mod = _native.require()
    x = torch.randn(*shape, dtype=torch.complex64, device="cuda")
    got = fft_c2c(mod, x, dim, inverse, scale=0.25)
    want = (torch.fft.ifft(x.cdouble(), dim=dim, norm="forward") if inverse else torch.fft.fft(x.cdouble(), dim=dim)) * 0.25
    _close(got.cdouble(), want, tol=2e-4)
    assert torch.equal(fft_c2c(mod, x, dim, inverse, scale=0.25), got)


@pytest.mark.parametrize("n", [4, 64, 512, 2048])
def test_real_fft_native_matches_torch(n):
    from torch_einshard_b200.ops.fft_impl import irfft_native, rfft_native
    x = torch.randn(3, n, 5, device="cuda", dtype=torch.float32)
    got = rfft_native(x, 1)
    want = torch.fft.rfft(x.double(), dim=1)
    _close(got.cdouble(), want, tol=2e-5 * n.bit_length())
    back = irfft_native(got, n, 1)
    want_back = torch.fft.irfft(want, n=n, dim=1, norm="forward")
    _close(back.double(), want_back, tol=2e-5 * n.bit_length())
    # gradients flow through the native pieces
    xr = x.clone().requires_grad_(True)
    rfft_native(xr, 1).abs().sum().backward()
    xt = x.clone().requires_grad_(True)
    torch.fft.rfft(xt, dim=1).abs().sum().backward()
    _close(xr.grad, xt.grad, tol=1e-3)


def test_einfft_real_local_uses_native(monkeypatch):
    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import fft_impl
    calls = []
    real = fft_impl._run
    monkeypatch.setattr(fft_impl, "_run", lambda *a, **k: calls.append(1) or real(*a, **k))
    x = torch.randn(4, 64, 32, device="cuda")
    y = es.einfft("b x y -> b kx ky", x, {"x": "kx", "y": "ky"}, real=True)
    torch.testing.assert_close(y, torch.fft.rfftn(x, dim=(1, 2)), rtol=1e-4, atol=1e-3)
    back = es.einfft("b kx ky -> b x y", y, {"kx": "x", "ky": "y"}, real=True, inverse=True, signal_sizes={"y": 32})
    torch.testing.assert_close(back, x, rtol=1e-4, atol=1e-4)
    assert calls
