"""Native NVLink communicators (peer-mapped symmetric buffers + sm_100a kernels).

A communicator exists for a process group only when every member is a CUDA
device of this node with peer access and the native extension is loaded; the
collective helpers ask :func:`communicator_for` and fall back to
``torch.distributed`` when it returns ``None``.  The implementation is filled in
by :mod:`torch_einshard_b200.parallel.symmetric`.
"""

__all__ = ["communicator_for", "world_communicator", "enable", "disable", "enabled"]

_state = {"enabled": False, "factory": None}


def enable(factory):
    """Register the factory mapping a process group to a communicator (or None)."""
    _state["factory"] = factory
    _state["enabled"] = True


def disable():
    _state["enabled"] = False


def enabled() -> bool:
    return _state["enabled"] and _state["factory"] is not None


def communicator_for(group):
    if not enabled():
        return None
    return _state["factory"](group)


def world_communicator():
    if not enabled():
        return None
    import torch.distributed as dist
    return _state["factory"](dist.group.WORLD)
