"""Per-rank shard metadata of parameters (checkpoint-facing).

``param_local_slices`` maps a parameter's global shape to the slice this rank
owns, from the mesh coordinate of this rank (or its rank in a compound group)
and the balanced split rule; ``factors`` keeps shard boundaries on multiples of
a factor (e.g. head size).  ``param_shard_metadata`` packs global shape, local
slices, local shape and shard dims into :class:`ParamShardMetadata`.
Contract of ``src/torch_einshard/params.py:1569-1669``.
"""

import torch.distributed as dist

from ..notation.spec import AxisGroup, EllipsisAxis
from ..parallel.collectives import compute_split_shapes_for_factors
from .registry import get_parameter_state
from .state import ParameterState, ParamShardMetadata

__all__ = ["param_shard_dims", "param_local_slices", "param_local_shape", "param_shard_metadata"]


def require_state(param_or_state):
    if isinstance(param_or_state, ParameterState):
        return param_or_state
    state = get_parameter_state(param_or_state)
    if state is None:
        raise ValueError("Parameter does not have an attached ParameterState")
    return state


def param_shard_dims(param_or_state):
    return require_state(param_or_state).layout_shard_dims


def _rank_and_size(mesh, shard_dim):
    if not dist.is_initialized():
        raise RuntimeError("Parameter shard metadata requires an initialized process group")
    device_mesh = getattr(mesh, "device_mesh", mesh)
    if not hasattr(device_mesh, "mesh_dim_names") or not hasattr(device_mesh, "mesh"):
        raise TypeError("mesh must be a PyTorch DeviceMesh or torch_einshard.wrap_mesh(mesh)")
    if shard_dim in device_mesh.mesh_dim_names:
        index = device_mesh.mesh_dim_names.index(shard_dim)
        coord = (device_mesh.mesh == dist.get_rank()).nonzero()[0].tolist()
        return coord[index], device_mesh.mesh.shape[index]
    if "-" not in shard_dim:
        raise ValueError(f"Mesh does not contain sharded parameter dimension {shard_dim!r}")
    if not hasattr(mesh, "device_mesh"):
        raise ValueError(f"Compound sharded parameter dimension {shard_dim!r} requires es.wrap_mesh(mesh)")
    group = mesh[shard_dim].get_group()
    return dist.get_rank(group), dist.get_world_size(group)


def _axis_shard_dim(axis):
    if isinstance(axis, EllipsisAxis):
        raise ValueError("Parameter shard metadata does not support ellipsis axes")
    if isinstance(axis, AxisGroup):
        if axis.axes.all_shard_dims():
            raise NotImplementedError("Parameter shard metadata does not support sharded factored-axis groups")
        return ""
    return axis.shard_dim


def _factor(axis, factors):
    if not factors:
        return 1
    if isinstance(axis, EllipsisAxis):
        raise ValueError("Parameter shard metadata does not support ellipsis axes")
    if isinstance(axis, AxisGroup):
        raise NotImplementedError("Parameter shard metadata does not support factored-axis groups")
    return int(factors.get(axis.name, 1))


def param_local_slices(param_or_state, global_shape, mesh, factors=None):
    state = require_state(param_or_state)
    axes = state.axes
    global_shape = tuple(int(n) for n in global_shape)
    if len(global_shape) != len(axes):
        raise ValueError(
            f"Global shape rank {len(global_shape)} does not match parameter metadata rank {len(axes)}"
        )
    slices = []
    for axis, size in zip(axes, global_shape):
        shard_dim = _axis_shard_dim(axis)
        if not shard_dim:
            slices.append(slice(None))
            continue
        rank, chunks = _rank_and_size(mesh, shard_dim)
        sections = compute_split_shapes_for_factors(size, chunks, _factor(axis, factors))
        start = sum(sections[:rank])
        slices.append(slice(start, start + sections[rank]))
    return tuple(slices)


def shape_from_slices(global_shape, slices):
    shape = []
    for size, piece in zip(global_shape, slices):
        start = 0 if piece.start is None else piece.start
        stop = size if piece.stop is None else piece.stop
        shape.append(stop - start)
    return tuple(shape)


def param_local_shape(param_or_state, global_shape, mesh, factors=None):
    return shape_from_slices(global_shape, param_local_slices(param_or_state, global_shape, mesh, factors=factors))


def param_shard_metadata(param_or_state, global_shape, mesh, factors=None):
    state = require_state(param_or_state)
    global_shape = tuple(int(n) for n in global_shape)
    slices = param_local_slices(state, global_shape, mesh, factors=factors)
    return ParamShardMetadata(global_shape=global_shape, local_slices=slices,
                              local_shape=shape_from_slices(global_shape, slices), shard_dims=param_shard_dims(state))
