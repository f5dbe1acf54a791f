"""Native batched GEMM with autograd: ``matmul(A[B,M,K], B[B,K,N]) -> [B,M,N]``.

Forward and both backward products run on the tcgen05 kernel
(``csrc/gemm_tc.cuh``).  Transposed operands are passed as strided views: the
kernel reads either operand K-major or MN-major, so ``dA = dC @ B^T`` and
``dB = A^T @ dC`` need no transpose copies.  Operands whose strides the TMA
engine cannot address (row stride not a multiple of 16 bytes, unaligned base)
are first copied into a padded buffer.

Replaces the reference's ``torch.einsum`` (``src/torch_einshard/einsum.py:132``).
"""

import torch

from . import _native

__all__ = ["eligible", "matmul", "native_bmm", "silu"]

_NATIVE_DTYPES = (torch.bfloat16, torch.float16)
_ACTS = {None: 0, "silu": 1}
_OUT_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def eligible(x, y) -> bool:
    """True when the contraction of ``x`` and ``y`` should run natively."""
    if not (x.is_cuda and y.is_cuda) or x.dtype != y.dtype or x.dtype not in _NATIVE_DTYPES:
        return False
    if _native.available():
        return True
    if _native.allow_fallback():
        return False
    _native.require()  # raises: native extension missing on a CUDA machine
    return False


def _tma_ready(t: torch.Tensor, contiguous_dim: int) -> bool:
    other = 2 if contiguous_dim == 1 else 1
    if t.stride(contiguous_dim) != 1 and t.size(contiguous_dim) > 1:
        return False
    if t.data_ptr() % 16:
        return False
    row = t.stride(other) if t.size(other) > 1 else t.size(contiguous_dim)
    if (row * t.element_size()) % 16:
        return False
    if t.size(0) > 1 and (t.stride(0) * t.element_size()) % 16:
        return False
    return True


def _padded_copy(t: torch.Tensor) -> torch.Tensor:
    """Contiguous copy whose last-dim row pitch is padded to 16 bytes."""
    b, r, c = t.shape
    align = 16 // t.element_size()
    pitch = -(-c // align) * align
    buf = t.new_zeros((b, r, pitch))
    buf[:, :, :c].copy_(t)
    return buf[:, :, :c]


def _prepare(t: torch.Tensor) -> torch.Tensor:
    # either the last dim (row-major) or the middle dim (column-major) must be contiguous
    if _tma_ready(t, 2) or _tma_ready(t, 1):
        return t
    t = t.contiguous()
    return t if _tma_ready(t, 2) else _padded_copy(t)


def native_bmm(a: torch.Tensor, b: torch.Tensor, out_dtype=None, act=None) -> torch.Tensor:
    mod = _native.require()
    a, b = _prepare(a), _prepare(b)
    out_dtype = a.dtype if out_dtype is None else out_dtype
    return mod.gemm(a, b, _OUT_CODE[out_dtype], _ACTS[act], _native.error_word(a.device))


class _NativeMatmul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return native_bmm(a, b)

    @staticmethod
    def backward(ctx, grad):
        a, b = ctx.saved_tensors
        # a transposed-view b (e.g. an [out, in] weight) gets its gradient directly in
        # that memory order, (dC^T A)^T, so no copy is needed later
        return _grads(ctx, a, b, grad)


def _grads(ctx, a, b, grad):
    grad_a = native_bmm(grad, b.transpose(1, 2)) if ctx.needs_input_grad[0] else None
    grad_b = None
    if ctx.needs_input_grad[1]:
        if b.stride(1) == 1 and b.size(1) > 1:
            grad_b = native_bmm(grad.transpose(1, 2), a).transpose(1, 2)
        else:
            grad_b = native_bmm(a.transpose(1, 2), grad)
    return grad_a, grad_b


class _NativeMatmulSilu(torch.autograd.Function):
    """silu(a @ b): the wide kernel writes the pre-activation H and silu(H) from
    one pass over its accumulator; backward forms dH = dY * silu'(H) in one
    elementwise pass and reuses the GEMM pair of the plain product."""

    @staticmethod
    def forward(ctx, a, b):
        mod = _native.require()
        a2, b2 = _prepare(a), _prepare(b)
        out, pre = mod.gemm_silu(a2, b2, _native.error_word(a.device))
        ctx.save_for_backward(a, b, pre)
        return out

    @staticmethod
    def backward(ctx, grad):
        a, b, pre = ctx.saved_tensors
        dpre = _native.require().silu_backward(grad.contiguous(), pre)
        return _grads(ctx, a, b, dpre)


class _NativeSilu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h):
        h = h.contiguous()
        ctx.save_for_backward(h)
        return _native.require().silu_forward(h)

    @staticmethod
    def backward(ctx, grad):
        (h,) = ctx.saved_tensors
        return _native.require().silu_backward(grad.contiguous(), h)


def silu(t: torch.Tensor) -> torch.Tensor:
    """SiLU on the native elementwise kernel for 16-bit CUDA tensors, else torch."""
    if t.is_cuda and t.dtype in _NATIVE_DTYPES and _native.available():
        return _NativeSilu.apply(t)
    return torch.nn.functional.silu(t)


def matmul(a: torch.Tensor, b: torch.Tensor, activation=None) -> torch.Tensor:
    if activation == "silu":
        if a.requires_grad or b.requires_grad:
            return _NativeMatmulSilu.apply(a, b)
        return _native.require().gemm_silu(_prepare(a), _prepare(b), _native.error_word(a.device))[0]
    if activation is not None:
        raise ValueError(f"unsupported activation {activation!r} (supported: 'silu')")
    if a.requires_grad or b.requires_grad:
        return _NativeMatmul.apply(a, b)
    return native_bmm(a, b)
