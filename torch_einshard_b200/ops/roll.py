"""``einroll``: per-axis cyclic shifts of (possibly sharded) tensors.

Local axes use ``torch.roll``; a sharded axis with split metadata exchanges
exactly the intervals that cross shard boundaries (one peer copy per interval
on the native path, P2P otherwise); without metadata the axis is gathered,
rolled and split again with a ``RuntimeWarning``.  Contract of
``src/torch_einshard/roll.py:10-45``.
"""

import warnings

import torch

from ..notation.families import cached_expand_axis_families, expand_family_mapping
from ..notation.parser import parse_sharding
from ..parallel.collectives import resolve_split_shapes
from ..parallel.mappings import (
    allgather_forward_split_backward,
    roll_sharded_forward_backward,
    split_forward_allgather_backward,
)

__all__ = ["einroll"]


def einroll(shard, x, shifts, *, mesh=None, shapes=None, families=None):
    shard, _ = cached_expand_axis_families(shard, families=families)
    shifts = expand_family_mapping(shifts, families, label="Shift")
    spec = parse_sharding(f"{shard} -> {shard}")[0]
    z = x
    for dim, axis in enumerate(spec.axes):
        shift = shifts.get(axis.name, 0)
        if shift == 0:
            continue
        if axis.local():
            z = torch.roll(z, shifts=shift, dims=dim)
            continue
        if mesh is None:
            raise ValueError("Distributed einroll operations require mesh")
        group = mesh[axis.shard_dim].get_group()
        split_shapes = resolve_split_shapes(shapes, axis.shard_dim, axis.name, group)
        if split_shapes is not None:
            z = roll_sharded_forward_backward(z, group, dim, shift, split_shapes)
            continue
        warnings.warn(
            f"Using gather/roll/split fallback for sharded roll axis {axis.name!r}; "
            "provide shapes to enable direct slice exchange.",
            RuntimeWarning,
            stacklevel=2,
        )
        z = allgather_forward_split_backward(z, group, dim, split_shapes)
        z = torch.roll(z, shifts=shift, dims=dim)
        z = split_forward_allgather_backward(z, group, dim, split_shapes)
    return z
