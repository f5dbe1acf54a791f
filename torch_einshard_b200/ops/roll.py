"""``einroll``: cyclic shifts along named axes of a possibly sharded tensor.

The call is planned once: every axis of the spec with a nonzero shift becomes
a move, either local (the axis is not sharded) or sharded (on a mesh dim).
Shifts along different axes commute, so all local moves run first as one
native gather kernel (``csrc/copy.cu:roll_copy``, every local axis in a single
pass over the tensor; its adjoint is the roll by the negated shifts), and then
each sharded move exchanges exactly the intervals that cross shard boundaries
(``parallel/mappings.py:roll_sharded_forward_backward``; one peer copy per
interval on the native path).  A sharded axis without split metadata is
gathered, rolled and split again, with the reference's ``RuntimeWarning``.

Contract (arguments, errors, warning text) of the reference's
``src/torch_einshard/roll.py:10-45``.
"""

import warnings
from dataclasses import dataclass

from ..notation.families import cached_expand_axis_families, expand_family_mapping
from ..notation.parser import parse_sharding
from ..parallel.collectives import resolve_split_shapes
from ..parallel.mappings import (
    allgather_forward_split_backward,
    roll_sharded_forward_backward,
    split_forward_allgather_backward,
)
from .native_ops import local_roll

__all__ = ["einroll"]


@dataclass(frozen=True)
class _Move:
    dim: int
    name: str
    mesh_dim: object  # None for a local axis
    shift: int


def _plan(shard, shifts, families):
    shard, _ = cached_expand_axis_families(shard, families=families)
    shifts = expand_family_mapping(shifts, families, label="Shift")
    spec = parse_sharding(f"{shard} -> {shard}")[0]
    moves = []
    for dim, axis in enumerate(spec.axes):
        shift = shifts.get(axis.name, 0)
        if shift:
            moves.append(_Move(dim, axis.name, None if axis.local() else axis.shard_dim, shift))
    return moves


def _sharded(z, move, mesh, shapes):
    if mesh is None:
        raise ValueError("Distributed einroll operations require mesh")
    group = mesh[move.mesh_dim].get_group()
    split = resolve_split_shapes(shapes, move.mesh_dim, move.name, group)
    if split is not None:
        return roll_sharded_forward_backward(z, group, move.dim, move.shift, split)
    warnings.warn(
        f"Using gather/roll/split fallback for sharded roll axis {move.name!r}; "
        "provide shapes to enable direct slice exchange.",
        RuntimeWarning,
        stacklevel=3,
    )
    full = allgather_forward_split_backward(z, group, move.dim, split)
    full = local_roll(full, {move.dim: move.shift})
    return split_forward_allgather_backward(full, group, move.dim, split)


def einroll(shard, x, shifts, *, mesh=None, shapes=None, families=None):
    moves = _plan(shard, shifts, families)
    z = local_roll(x, {m.dim: m.shift for m in moves if m.mesh_dim is None})
    for move in moves:
        if move.mesh_dim is not None:
            z = _sharded(z, move, mesh, shapes)
    return z
