"""Native complex64 FFTs (``_C.fft_c2c`` / ``_C.fft_slab``) with autograd.

``fft_c2c(mod, x, dim, inverse)`` is the unnormalised DFT along one dim
(inverse = conjugate twiddles, no 1/n), the contract of ``_local_fft`` in
``ops/fft.py``.  ``slab_fft`` runs the slab pipeline of ``einfft``: FFTs over
the local transform dims, then the all-to-all slab transpose fused with the
FFT along the axis that becomes local (its loads read peer GPUs' symmetric
memory), then any remaining FFTs.  The adjoint of either is the same routine
with the direction flipped (and, for the slab, the exchanged roles swapped),
which is what the backward passes run.

Twiddle tables exp(-+2 pi i j / n) are computed on the host in float64, rounded
to complex64 and cached per (device, n, direction).

Replaces the reference's ``torch.fft`` calls (``src/torch_einshard/fft.py:202-205,549-553,861-870``).
"""

import math

import torch

from . import _native
from .native_ops import local_roll

__all__ = ["supported_length", "fft_c2c", "try_fft", "slab_fft", "rfft_native", "irfft_native"]

_MAX_LOG = 10
_TWIDDLES = {}


def supported_length(n):
    return 2 <= n <= (1 << _MAX_LOG) and (n & (n - 1)) == 0


def twiddles(n, inverse, device):
    key = (device, n, bool(inverse))
    tw = _TWIDDLES.get(key)
    if tw is None:
        sign = 1.0 if inverse else -1.0
        j = torch.arange(n, dtype=torch.float64)
        angle = sign * 2.0 * math.pi * j / n
        tw = torch.complex(torch.cos(angle), torch.sin(angle)).to(torch.complex64).to(device)
        _TWIDDLES[key] = tw
    return tw


def _eligible(x, dim):
    return (x.is_cuda and x.dtype == torch.complex64 and x.dim() > 0 and supported_length(x.shape[dim]))


def _run(mod, x, dim, inverse, scale=1.0, out=None):
    x = x.resolve_conj().resolve_neg().contiguous()  # the kernel reads raw memory
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    mod.fft_c2c(x, out, dim, bool(inverse), twiddles(x.shape[dim], inverse, x.device), float(scale))
    return out


class _FFT(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, inverse, scale):
        ctx.dim, ctx.inverse, ctx.scale = dim, inverse, scale
        return _run(_native.require(), x, dim, inverse, scale)

    @staticmethod
    def backward(ctx, grad):
        # y = s F x  =>  dL/dx = s F^H g, and F^H is the unnormalised opposite direction
        return _run(_native.require(), grad, ctx.dim, not ctx.inverse, ctx.scale), None, None, None


def fft_c2c(mod, x, dim, inverse, scale=1.0):
    """Unnormalised DFT of ``x`` along ``dim`` on the native kernel, or ``None``
    when the kernel does not cover the call (the caller then uses torch.fft)."""
    dim = dim % x.dim() if x.dim() else 0
    if mod is None or not _eligible(x, dim):
        return None
    if x.shape[dim] == 1:
        return x.clone()
    if torch.is_grad_enabled() and x.requires_grad:
        return _FFT.apply(x, dim, bool(inverse), float(scale))
    return _run(mod, x, dim, inverse, scale)


# ------------------------------------------------------------------ slab pipeline

def _slab_geometry(shape, gather_dim, split_dim, P):
    """Canonical [A, S, B, D, C] (mode 0) or [A, D, B, S, C] (mode 1) sizes of the
    pre-exchange tensor, where S = gather_dim (local slab Sl) and D = split_dim."""
    def prod(dims):
        out = 1
        for d in dims:
            out *= shape[d]
        return out
    nd = len(shape)
    if gather_dim < split_dim:
        mode = 0
        A = prod(range(0, gather_dim))
        B = prod(range(gather_dim + 1, split_dim))
        C = prod(range(split_dim + 1, nd))
    else:
        mode = 1
        A = prod(range(0, split_dim))
        B = prod(range(split_dim + 1, gather_dim))
        C = prod(range(gather_dim + 1, nd))
    return mode, A, B, C


def slab_eligible(x, comm, gather_dim, split_dim, P, pre_dims, post_dims):
    if comm is None or not x.is_cuda or x.dtype != torch.complex64:
        return False
    mod = _native.module()
    if mod is None or not hasattr(mod, "fft_slab"):
        return False
    n = x.shape[gather_dim] * P
    D = x.shape[split_dim]
    if not supported_length(n) or D % P:
        return False
    for d in list(pre_dims) + list(post_dims):
        if not supported_length(x.shape[d]) and x.shape[d] != 1:
            return False
    return x.numel() * 8 <= comm.data_bytes


def _slab_run(x, spec):
    mod = _native.require()
    comm, P, rank = spec["comm"], spec["P"], spec["rank"]
    g, s = spec["gather"], spec["split"]
    inverse = spec["inverse"]
    x = x.contiguous()
    # 1) FFTs over the local dims; the last writes this rank's symmetric region
    comm.acquire()
    region = comm.region(x.numel() * 8).view(torch.complex64).view(x.shape)
    pre = [d for d in spec["pre"] if x.shape[d] > 1]
    if not pre:
        region.copy_(x)
    for k, d in enumerate(pre):
        src = x if k == 0 else cur
        dst = region if k == len(pre) - 1 else None
        cur = _run(mod, src, d, inverse, 1.0, out=dst)
    # 2) exchange fused with the FFT along the gathered dim
    n = x.shape[g] * P
    D = x.shape[s]
    Dl = D // P
    mode, A, B, C = _slab_geometry(x.shape, g, s, P)
    out_shape = list(x.shape)
    out_shape[g] = n
    out_shape[s] = Dl
    out = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    mod.fft_slab(comm.id, out, n, A, B, C, D, Dl, rank * Dl, mode, twiddles(n, inverse, x.device),
                 float(spec["scale"]), bool(inverse), _native.error_word(x.device))
    # 3) remaining local FFTs
    for d in spec["post"]:
        if out.shape[d] > 1:
            out = _run(mod, out, d, inverse, 1.0)
    return out


class _SlabFFT(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, spec):
        ctx.spec = spec
        return _slab_run(x, spec)

    @staticmethod
    def backward(ctx, grad):
        s = ctx.spec
        adjoint = dict(s, pre=[s["gather"]], gather=s["split"], split=s["gather"],
                       post=[d for d in s["pre"] if d != s["split"]], inverse=not s["inverse"])
        return _slab_run(grad, adjoint), None


def slab_fft(x, comm, P, rank, *, pre_dims, gather_dim, split_dim, post_dims=(), inverse=False, scale=1.0):
    """Unnormalised (times ``scale``) FFT over ``pre_dims`` + ``gather_dim`` +
    ``post_dims`` with the slab exchange: ``gather_dim`` is sharded (P equal
    blocks) on the input and local on the output, ``split_dim`` the reverse."""
    spec = dict(comm=comm, P=P, rank=rank, pre=list(pre_dims), gather=gather_dim, split=split_dim,
                post=list(post_dims), inverse=bool(inverse), scale=float(scale))
    if torch.is_grad_enabled() and x.requires_grad:
        return _SlabFFT.apply(x, spec)
    return _slab_run(x, spec)


# ------------------------------------------------------------------ real transforms

_HALF_TW = {}


def _half_twiddles(n, device):
    """exp(-2 pi i k / n) for k < n/2 (float64 on the host, complex64 on device)."""
    key = (device, n)
    tw = _HALF_TW.get(key)
    if tw is None:
        k = torch.arange(n // 2, dtype=torch.float64)
        angle = -2.0 * math.pi * k / n
        tw = torch.complex(torch.cos(angle), torch.sin(angle)).to(torch.complex64).to(device)
        _HALF_TW[key] = tw
    return tw


def _real_ok(n):
    return n % 2 == 0 and supported_length(n // 2)


def rfft_native(x, dim):
    """Unnormalised real-to-half-spectrum DFT along ``dim`` (``torch.fft.rfft``
    contract) as a complex DFT of half length: z[m] = x[2m] + i x[2m+1],
    Z = DFT(z), then X[k] = (Z[k] + conj Z[-k]) / 2 - i w^k (Z[k] - conj Z[-k]) / 2
    with w = exp(-2 pi i / n).  ``None`` when the native kernels do not apply."""
    mod = _native.module()
    dim = dim % x.dim()
    n = x.shape[dim]
    if mod is None or not x.is_cuda or x.dtype != torch.float32 or not _real_ok(n):
        return None
    xm = x.movedim(dim, -1).contiguous()
    z = torch.view_as_complex(xm.reshape(*xm.shape[:-1], n // 2, 2))
    Z = fft_c2c(mod, z, z.dim() - 1, False)
    Zc = torch.conj(local_roll(torch.flip(Z, dims=(-1,)), {Z.dim() - 1: 1}))  # conj Z[-k mod n/2]
    even = (Z + Zc) * 0.5
    odd = (Z - Zc) * (-0.5j)
    w = _half_twiddles(n, x.device)
    head = even + w * odd
    nyquist = (even[..., :1] - odd[..., :1])
    return torch.cat([head, nyquist], dim=-1).movedim(-1, dim)


def irfft_native(X, n, dim):
    """Unnormalised half-spectrum-to-real inverse DFT (``torch.fft.irfft(...,
    norm="forward")`` contract) of output length ``n`` along ``dim``."""
    mod = _native.module()
    dim = dim % X.dim()
    if (mod is None or not X.is_cuda or X.dtype != torch.complex64 or not _real_ok(n)
            or X.shape[dim] != n // 2 + 1):
        return None
    Xm = X.movedim(dim, -1)
    h = n // 2
    lo = Xm[..., :h]
    hi = torch.conj(torch.flip(Xm[..., 1:h + 1], dims=(-1,)))  # conj X[h - k]
    even = (lo + hi) * 0.5
    odd = (lo - hi) * 0.5 * torch.conj(_half_twiddles(n, X.device))
    Z = (even + 1j * odd).contiguous()
    z = fft_c2c(mod, Z, Z.dim() - 1, True, scale=2.0)
    return torch.view_as_real(z).reshape(*z.shape[:-1], n).movedim(-1, dim)


def try_fft(x, dim, inverse, scale=1.0):
    """Native FFT along one axis of a CUDA complex tensor, or None when the
    kernels do not cover the call (not CUDA complex64, length not a supported
    power of two); the caller then uses ``torch.fft``.  Replaces the
    reference's ``torch.fft`` calls (``src/torch_einshard/fft.py:202-205``)."""
    if not x.is_cuda:
        return None
    mod = _native.module()
    if mod is None or not hasattr(mod, "fft_c2c"):
        return None
    return fft_c2c(mod, x, dim, inverse, scale)
