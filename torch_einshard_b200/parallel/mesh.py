"""Device meshes with compound mesh groups.

:class:`CompoundDeviceMesh` wraps a ``torch.distributed.device_mesh.DeviceMesh``
and adds groups that span several named mesh dimensions: ``mesh["dp-sp"]`` is
the process group of all ranks that share every *other* mesh coordinate.  The
groups are created lazily (collectively, on every rank, in a deterministic
order) and cached; ``dp-sp`` and ``sp-dp`` name the same group.  Same contract
as ``src/torch_einshard/mesh.py:15-103``.

On NVSwitch systems every rank subset has uniform bandwidth, so a compound
group is only a rank list; the native communicator for it is created on first
use by :mod:`.symmetric`.
"""

from itertools import product

import torch
import torch.distributed as dist

__all__ = ["CompoundDeviceMesh", "wrap_mesh", "validate_mesh_dim_names"]


class _GroupHandle:
    """``mesh[name]`` result for compound names: exposes ``get_group()``."""

    def __init__(self, group, ranks=None):
        self.group = group
        self.ranks = ranks

    def get_group(self):
        return self.group


def validate_mesh_dim_names(names) -> tuple:
    """Normalise ``mesh_dim_names`` to a tuple of valid, non-overlapping names."""
    if names is None:
        return ()
    if isinstance(names, str):
        result = (names,)
    elif isinstance(names, torch.Tensor) or (hasattr(names, "shape") and hasattr(names, "dtype")):
        raise TypeError("mesh_dim_names must be an iterable of strings")
    else:
        try:
            result = tuple(names)
        except TypeError as error:
            raise TypeError("mesh_dim_names must be an iterable of strings") from error
    if not all(isinstance(name, str) for name in result):
        raise TypeError("mesh_dim_names entries must be strings")
    if not all(result):
        raise ValueError("mesh_dim_names entries must be non-empty strings")
    seen = set()
    for name in result:
        parts = name.split("-")
        if not all(parts):
            raise ValueError("mesh_dim_names entries cannot contain empty compound components")
        if len(set(parts)) != len(parts):
            raise ValueError("mesh_dim_names entries cannot repeat compound components")
    for name in result:
        parts = set(name.split("-"))
        if parts & seen:
            raise ValueError("mesh_dim_names entries cannot overlap compound components")
        seen |= parts
    if len(set(result)) != len(result):
        raise ValueError("mesh_dim_names entries must be unique")
    return result


class CompoundDeviceMesh:
    def __init__(self, device_mesh):
        self.device_mesh = device_mesh
        self.mesh = device_mesh.mesh
        self.mesh_dim_names = validate_mesh_dim_names(device_mesh.mesh_dim_names)
        if len(self.mesh_dim_names) != self.mesh.dim():
            raise ValueError("mesh_dim_names length must match mesh rank")
        self._dim_index = {name: index for index, name in enumerate(self.mesh_dim_names)}
        self._groups = {}

    def __getitem__(self, name):
        if name in self._dim_index or "-" not in name:
            return self.device_mesh[name]
        parts = tuple(name.split("-"))
        if not all(parts):
            raise ValueError("Compound mesh groups cannot contain empty mesh dimensions")
        if len(set(parts)) != len(parts):
            raise ValueError("Compound mesh groups cannot repeat mesh dimensions")
        if not all(part in self._dim_index for part in parts):
            return self.device_mesh[name]
        return _GroupHandle(self._compound_group(parts))

    def _compound_group(self, parts):
        key = tuple(sorted(parts, key=self._dim_index.__getitem__))
        if key in self._groups:
            return self._groups[key]
        if not dist.is_initialized():
            raise RuntimeError("Compound mesh groups require an initialized process group")
        spanned = {self._dim_index[name] for name in key}
        fixed = [d for d in range(self.mesh.dim()) if d not in spanned]
        grid = self.mesh.detach().cpu()
        me = dist.get_rank()
        mine = None
        # every rank creates every group, in the same order (new_group is collective)
        for fixed_coord in product(*(range(grid.shape[d]) for d in fixed)):
            members = [
                int(grid[coord])
                for coord in product(*(range(n) for n in grid.shape))
                if all(coord[d] == fixed_coord[i] for i, d in enumerate(fixed))
            ]
            group = dist.new_group(ranks=members)
            if me in members:
                mine = group
        self._groups[key] = mine
        return mine

    def coordinate(self, rank=None):
        """Mesh coordinate of ``rank`` (default: this process)."""
        rank = dist.get_rank() if rank is None else rank
        return (self.mesh == rank).nonzero()[0].tolist()


def wrap_mesh(device_mesh):
    if isinstance(device_mesh, CompoundDeviceMesh):
        return device_mesh
    return CompoundDeviceMesh(device_mesh)
