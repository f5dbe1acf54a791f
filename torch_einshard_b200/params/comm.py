"""Parameter communication: initial-value sync and gradient reduction.

* ``init_param_`` / ``init_params_`` attach init-time metadata and broadcast
  the parameter from group rank 0 over every ``init_sync`` group.
* ``reduce_grad_`` / ``reduce_module_grads_`` all-reduce gradients over the
  parameter's native reduction groups; ``register_native_grad_reduction_hooks_``
  does it from autograd hooks.
* ``register_grad_reduction_hook_`` installs a DDP communication hook: the
  bucket is all-reduced over the data-parallel group and averaged, then
  parameters with extra reduction groups are reduced over those groups
  (coalesced per group).  When every parameter of a bucket needs the same
  extra groups, one all-reduce over the compound group replaces both.  On
  CUDA buckets with a native communicator the all-reduce, the 1/dp scale and
  the copy back into the bucket run as one kernel over NVLink.

Contract of ``src/torch_einshard/params.py:706-896,1672-1839``.
"""

from collections.abc import Mapping

import torch
import torch.distributed as dist

from ..parallel import collectives
from .registry import (
    attached_state,
    check_metadata_keys,
    get_parameter_state,
    init_state,
    prepare_updates,
    register_parameter_state,
    set_parameter_state,
)
from .state import (
    NativeGradReductionHandle,
    as_name_tuple,
    check_group_components,
    check_groups_disjoint,
    check_state_metadata,
    mesh_dim_names_from,
    parts,
    parts_of,
)

__all__ = [
    "init_param_",
    "init_params_",
    "sync_param_",
    "sync_module_params_",
    "reduce_grad_",
    "reduce_module_grads_",
    "register_native_grad_reduction_hooks_",
    "register_grad_reduction_hook_",
]


def mesh_group(mesh, name):
    try:
        return mesh[name].get_group()
    except (KeyError, RuntimeError) as error:
        if "-" in name and not hasattr(mesh, "device_mesh"):
            raise ValueError(f"Compound mesh group {name!r} requires es.wrap_mesh(mesh)") from error
        raise ValueError(f"Mesh does not contain parameter metadata group {name!r}") from error


def groups_exist(mesh, names):
    for name in names:
        mesh_group(mesh, name)


def _pending_error(state):
    return ValueError("Parameter gradient communication is still pending inference")


def native_reduce_groups(state):
    if state is None:
        return ()
    gc = state.grad_comm
    if gc.pending_inference:
        if gc.backend in ("native", "ddp"):
            raise _pending_error(state)
        return ()
    if gc.mode == "none" or gc.backend != "native":
        return ()
    return gc.mesh_dims


def ddp_reduce_groups(state):
    if state is None:
        return ()
    gc = state.grad_comm
    if gc.pending_inference:
        if gc.backend in ("native", "ddp"):
            raise _pending_error(state)
        return ()
    if gc.mode == "none" or gc.backend not in ("native", "ddp"):
        return ()
    return gc.mesh_dims


def validation_grad_groups(state, *, allow_pending):
    gc = state.grad_comm
    if gc.pending_inference:
        if gc.backend in ("native", "ddp") and not allow_pending:
            raise _pending_error(state)
        return ()
    if gc.mode == "none" or gc.backend == "external":
        return ()
    return gc.mesh_dims if gc.backend in ("native", "ddp") else ()


def _require_state_object(state):
    from .state import ParameterState
    if isinstance(state, ParameterState):
        return state
    raise TypeError("Parameter metadata must be a ParameterState")


# ------------------------------------------------------------------ init sync

def init_param_(param, mesh, *, sync=None, sharded=(), mesh_dim_names=(), source="init"):
    if not isinstance(param, torch.nn.Parameter):
        raise TypeError("Parameter initialization requires a torch.nn.Parameter")
    mesh_dim_names = mesh_dim_names_from(mesh, mesh_dim_names)
    state = init_state(sync=sync, sharded=sharded, mesh_dim_names=mesh_dim_names, source=source)
    if state.shared:
        if mesh is None:
            raise ValueError("Parameter initialization sync requires mesh")
        groups_exist(mesh, state.shared)
    register_parameter_state(param, state)
    return sync_param_(param, get_parameter_state(param), mesh)


def init_params_(module, mesh, *, sync=None, sharded=None, mesh_dim_names=(), source="init"):
    if isinstance(module, torch.nn.Parameter):
        return init_param_(module, mesh, sync=sync, sharded=() if sharded is None else sharded,
                           mesh_dim_names=mesh_dim_names, source=source)
    if not isinstance(module, torch.nn.Module):
        raise TypeError("Parameter initialization requires a torch.nn.Module or torch.nn.Parameter")
    named = tuple(module.named_parameters())
    names = tuple(name for name, _ in named)
    check_metadata_keys(sync, names, "sync")
    check_metadata_keys(sharded, names, "sharded")
    mesh_dim_names = mesh_dim_names_from(mesh, mesh_dim_names)
    updates = []
    for name, param in named:
        value = sharded.get(name) if isinstance(sharded, Mapping) else sharded
        updates.append((param, init_state(
            sync=sync.get(name) if isinstance(sync, Mapping) else sync,
            sharded=() if value is None else value,
            mesh_dim_names=mesh_dim_names,
            source=source,
        )))
    prepared = prepare_updates(updates)
    for _, state in prepared:
        check_state_metadata(state)
    if mesh is None and any(state.shared for _, state in prepared):
        raise ValueError("Parameter initialization sync requires mesh")
    if mesh is not None:
        for _, state in prepared:
            groups_exist(mesh, state.shared)
    for param, state in prepared:
        set_parameter_state(param, state)
    for param, state in prepared:
        sync_param_(param, state, mesh)
    return module


def sync_param_(param, state, mesh):
    """Broadcast ``param`` from group rank 0 over each ``init_sync`` group
    (reference ``src/torch_einshard/params.py:880-887``).  CUDA parameters on a
    group with a native communicator take the NVLS broadcast (rank 0 writes the
    tensor once through the switch into every rank's heap); otherwise
    ``torch.distributed.broadcast``."""
    from ..parallel import symmetric
    state = _require_state_object(state)
    for name in state.shared:
        group = mesh_group(mesh, name)
        if dist.get_world_size(group) == 1:
            continue
        comm = symmetric.communicator_for(group) if param.is_cuda else None
        if comm is not None and param.data.is_contiguous() and comm.broadcast_(param.data, 0):
            continue
        dist.broadcast(param.data, src=dist.get_global_rank(group, 0), group=group)
    return param


def sync_module_params_(module, mesh):
    for param in module.parameters():
        state = get_parameter_state(param)
        if state is not None:
            sync_param_(param, state, mesh)
    return module


# ------------------------------------------------------------------ gradient reduction

def reduce_grad_(param, state, mesh):
    if param.grad is None:
        return param
    state = _require_state_object(state)
    for name in native_reduce_groups(state):
        param.grad = collectives.all_reduce(param.grad, mesh_group(mesh, name))
    return param


def reduce_module_grads_(module, mesh):
    for param in module.parameters():
        state = get_parameter_state(param)
        if state is not None:
            reduce_grad_(param, state, mesh)
    return module


def register_native_grad_reduction_hooks_(module, mesh):
    """Reduce each registered parameter's gradient from an autograd hook.

    Every registered parameter must take part in backward in the same order on
    every rank; models with rank-dependent control flow or unused parameters
    should use the DDP communication hook or an external backend.
    """
    handle = NativeGradReductionHandle()
    specs = []
    for param in module.parameters():
        state = attached_state(param)
        if state is None or state.grad_comm.backend != "native":
            continue
        groups = tuple((name, mesh_group(mesh, name)) for name in native_reduce_groups(state))
        if not groups:
            continue
        if not param.requires_grad:
            raise ValueError("Cannot register gradient reduction hook for a parameter that does not require gradients")
        specs.append((param, groups))
    try:
        for param, groups in specs:
            def hook(grad, *, groups=groups):
                for _, group in groups:
                    if dist.get_world_size(group) > 1:
                        grad = collectives.all_reduce(grad, group)
                return grad

            handle._add_hook(param.register_hook(hook))
    except Exception:
        handle.remove()
        raise
    return handle


def _check_no_ddp_overlap(ddp_group, reduce_groups):
    if ddp_group is None or not reduce_groups:
        return
    check_group_components((ddp_group,), "ddp_group")
    check_group_components(reduce_groups, "grad")
    for name in reduce_groups:
        overlap = parts(ddp_group) & parts(name)
        if overlap:
            raise ValueError(f"Parameter gradient reduction groups overlap with ddp_group: {', '.join(sorted(overlap))}")


def _check_combined(ddp_group, combined_group, combined_reduce):
    if combined_group is None:
        return
    if ddp_group is None:
        raise ValueError("combined_reduce_group requires a named ddp_group")
    check_group_components((ddp_group, combined_group, *combined_reduce), "combined_reduce")
    check_groups_disjoint((ddp_group, *combined_reduce), "combined_reduce")
    if parts(combined_group) != parts_of((ddp_group, *combined_reduce)):
        raise ValueError("combined_reduce_group must cover ddp_group and combined_reduce")


def _allreduce_mean(buffer, group, divisor):
    """All-reduce ``buffer`` in place over ``group`` and divide it by ``divisor``.

    Returns a future.  CUDA buckets on a group with a native communicator run
    one fused reduce+divide kernel over NVLink; otherwise NCCL/gloo followed
    by an in-place divide.
    """
    from ..parallel import symmetric
    comm = symmetric.communicator_for(group) if buffer.is_cuda else None
    if comm is not None and comm.all_reduce_div_(buffer, divisor):
        future = torch.futures.Future()
        future.set_result(buffer)
        return future
    future = dist.all_reduce(buffer, group=group, async_op=True).get_future()
    if divisor == 1:
        return future.then(lambda _: buffer)

    def finish(_):
        buffer.div_(divisor)
        return buffer

    return future.then(finish)


def register_grad_reduction_hook_(ddp_model, mesh, ddp_group="dp", combined_reduce_group=None, combined_reduce=None):
    combined_reduce = as_name_tuple(combined_reduce)
    if combined_reduce_group is not None and not combined_reduce:
        raise ValueError("combined_reduce must be provided with combined_reduce_group")
    if combined_reduce and combined_reduce_group is None:
        raise ValueError("combined_reduce_group must be provided with combined_reduce")
    _check_combined(ddp_group, combined_reduce_group, combined_reduce)
    if ddp_group is not None:
        groups_exist(mesh, (ddp_group,))
    if combined_reduce_group is not None:
        groups_exist(mesh, (combined_reduce_group,))
        groups_exist(mesh, combined_reduce)
    for param in ddp_model.parameters():
        state = attached_state(param)
        if state is not None:
            groups = ddp_reduce_groups(state)
            _check_no_ddp_overlap(ddp_group, groups)
            groups_exist(mesh, groups)

    def bucket_views(bucket):
        buffer = bucket.buffer()
        views, offset = [], 0
        for param in bucket.parameters():
            views.append((param, buffer.narrow(0, offset, param.numel()).view_as(param), get_parameter_state(param)))
            offset += param.numel()
        return views

    def combined_applies(views):
        if combined_reduce_group is None or not views:
            return False
        wanted = set(combined_reduce)
        return all(state is not None and set(ddp_reduce_groups(state)) == wanted for _, _, state in views)

    def reduce_extra_groups(buffer, views):
        names = sorted({name for _, _, state in views for name in ddp_reduce_groups(state)})
        for name in names:
            members = [view for _, view, state in views if name in ddp_reduce_groups(state)]
            if not members:
                continue
            flat = torch.cat([view.reshape(-1) for view in members])
            dist.all_reduce(flat, group=mesh_group(mesh, name))
            offset = 0
            for view in members:
                view.copy_(flat.narrow(0, offset, view.numel()).view_as(view))
                offset += view.numel()
        return buffer

    def hook(_state, bucket):
        buffer = bucket.buffer()
        group = mesh_group(mesh, ddp_group) if ddp_group is not None else None
        dp = dist.get_world_size(group)
        views = bucket_views(bucket)
        if combined_applies(views):
            cgroup = mesh_group(mesh, combined_reduce_group)
            csize = dist.get_world_size(cgroup)
            if csize == 1 and dp == 1:
                future = torch.futures.Future()
                future.set_result(buffer)
                return future
            if csize > 1:
                return _allreduce_mean(buffer, cgroup, dp)
        if dp == 1:
            future = torch.futures.Future()
            future.set_result(buffer)
        else:
            future = _allreduce_mean(buffer, group, dp)
        return future.then(lambda _: reduce_extra_groups(buffer, views))

    ddp_model.register_comm_hook(None, hook)
    return ddp_model
