"""One-call setup of the native NVLink communicators for a mesh.

No reference counterpart (the reference only uses ``torch.distributed``).
"""

__all__ = ["setup_native_comm"]


def setup_native_comm(mesh=None, *, enable=True):
    """Create peer-mapped communicators for every group of ``mesh`` (CUDA + NCCL only).

    Returns True when the native path is active.  Safe to call on CPU/gloo,
    where it does nothing and returns False.
    """
    import torch
    import torch.distributed as dist
    if not enable or not torch.cuda.is_available() or not dist.is_initialized():
        return False
    try:
        from . import symmetric
    except ImportError:
        return False
    return symmetric.activate(mesh)
