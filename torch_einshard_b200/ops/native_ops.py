"""Native local data-movement kernels (strided gather copies, roll).

Each function returns ``None`` when the native path does not apply, and the
caller then uses the torch implementation.

Replaces the reference's window build (``src/torch_einshard/halo.py:36-55``)
and ``torch.roll`` (``src/torch_einshard/roll.py:23``).
"""

import torch

from . import _native

__all__ = ["strided_copy"]

_MAX_RANK = 8


def strided_copy(view: torch.Tensor):
    """Materialise an arbitrary strided view contiguously with one kernel."""
    if not view.is_cuda or view.dim() > _MAX_RANK or view.numel() == 0:
        return None
    mod = _native.module()
    if mod is None or not hasattr(mod, "strided_copy"):
        return None
    out = torch.empty(view.shape, dtype=view.dtype, device=view.device)
    mod.strided_copy(view, out)
    return out
