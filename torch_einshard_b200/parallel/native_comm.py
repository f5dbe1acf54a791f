"""Native NVLink communicators (peer-mapped symmetric buffers + sm_100a kernels).

A communicator exists for a process group only when every member is a CUDA
device of this node with peer access and the native extension is loaded; the
collective helpers ask :func:`communicator_for` and fall back to
``torch.distributed`` when it returns ``None``.  The implementation is filled in
by :mod:`torch_einshard_b200.parallel.symmetric`.

Native backend of the reference's collective helpers
(``src/torch_einshard/helpers.py:27-309``).
"""

__all__ = ["communicator_for", "workspace_for", "world_communicator", "enable", "disable", "enabled"]

_state = {"enabled": False, "factory": None, "workspace": None}


def enable(factory, workspace=None):
    """Register the factory mapping a process group to a communicator (or None),
    and optionally the one returning a communicator with at least n bytes."""
    _state["factory"] = factory
    _state["workspace"] = workspace
    _state["enabled"] = True


def disable():
    _state["enabled"] = False


def enabled() -> bool:
    return _state["enabled"] and _state["factory"] is not None


def communicator_for(group):
    if not enabled():
        return None
    return _state["factory"](group)


def workspace_for(group, nbytes):
    """A communicator of ``group`` whose symmetric region holds ``nbytes``
    (collective: every member must ask with the same size), or None."""
    if not enabled():
        return None
    if _state["workspace"] is None:
        comm = _state["factory"](group)
        return comm if comm is not None and comm.data_bytes >= nbytes else None
    return _state["workspace"](group, nbytes)


def world_communicator():
    if not enabled():
        return None
    import torch.distributed as dist
    return _state["factory"](dist.group.WORLD)
