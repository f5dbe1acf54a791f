"""Native local data movement.

* ``strided_copy``: materialise a strided view with one gather kernel
  (``csrc/copy.cu``); ``None`` when the native path does not apply (CPU
  tensors, rank above 8, an empty view, no extension).  Used for einwindow's
  window tensors (the reference builds them with
  ``src/torch_einshard/halo.py:414-417``, ``unfold`` plus ``permute().contiguous()``).
* ``local_roll``: cyclic shifts along several dims in one kernel
  (``csrc/copy.cu:roll_copy``), differentiable; replaces the reference's
  ``torch.roll`` (``src/torch_einshard/roll.py:23``).
"""

import torch

from . import _native

__all__ = ["strided_copy", "local_roll"]

_MAX_RANK = 8


def strided_copy(view: torch.Tensor):
    """Materialise an arbitrary strided view contiguously with one kernel."""
    if not view.is_cuda or view.dim() > _MAX_RANK or view.numel() == 0 or view.is_conj() or view.is_neg():
        return None
    mod = _native.module()
    if mod is None or not hasattr(mod, "strided_copy"):
        return None
    out = torch.empty(view.shape, dtype=view.dtype, device=view.device)
    mod.strided_copy(view, out)
    return out


class _LocalRoll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, shifts):
        ctx.shifts = shifts
        return _roll_native(x, shifts)

    @staticmethod
    def backward(ctx, grad):
        return _roll_native(grad, [-s for s in ctx.shifts]), None


def _roll_native(x, shifts):
    # the kernel moves raw memory: resolve lazy conjugate / negative views first
    # (autograd hands conj(grad) of torch.conj to backward as such a view)
    x = x.resolve_conj().resolve_neg().contiguous()
    out = torch.empty_like(x)
    _native.require().roll_copy(x, out, [int(s) for s in shifts])
    return out


def local_roll(x, shifts_by_dim):
    """``torch.roll`` along several dims at once: one native kernel for CUDA
    tensors (rank 1 to 9), ``torch.roll`` otherwise."""
    if not shifts_by_dim:
        return x
    if x.is_cuda and 1 <= x.dim() <= 9 and x.numel() > 0 and _native.available():
        shifts = [0] * x.dim()
        for dim, shift in shifts_by_dim.items():
            shifts[dim] += shift
        return _LocalRoll.apply(x, shifts)
    dims = list(shifts_by_dim)
    return torch.roll(x, shifts=[shifts_by_dim[d] for d in dims], dims=dims)
