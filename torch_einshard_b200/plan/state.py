"""Symbolic tensor placement state (``TensorState``) and plan step records.

A ``TensorState`` is the planner's frozen view of one tensor spec: the ordered
axis names, where each axis is sharded, which mesh dims hold partial sums and
which mesh dims the tensor is replicated over (compound names such as
``dp-sp`` count as using both components).  Mirrors
``src/torch_einshard/symbolic.py:53-101``.
"""

from dataclasses import dataclass

from ..notation.spec import Axes, Axis, EllipsisAxis, TensorSpec

__all__ = [
    "StateAxis",
    "TensorState",
    "PlanStep",
    "axes_of",
    "flat_axes_of",
    "partials_of",
    "mesh_dim_components",
    "mesh_dims_components",
    "require_expanded_axes",
    "tensor_spec",
    "local_axis",
    "sharded_axis",
]


def axes_of(spec):
    return spec.axes if hasattr(spec, "axes") else spec


def flat_axes_of(spec):
    axes = axes_of(spec)
    return axes.flat() if hasattr(axes, "flat") else axes


def partials_of(spec) -> tuple:
    return tuple(getattr(spec, "partials", ()))


def mesh_dim_components(name: str) -> set:
    """A mesh group name together with its ``-``-separated components."""
    return {name, *name.split("-")}


def mesh_dims_components(names) -> set:
    out = set()
    for name in names:
        out |= mesh_dim_components(name)
    return out


def require_expanded_axes(spec) -> Axes:
    axes = flat_axes_of(spec)
    if any(isinstance(axis, EllipsisAxis) for axis in axes):
        raise ValueError("Symbolic TensorState requires ellipsis expansion")
    return Axes(axes)


@dataclass(frozen=True)
class StateAxis:
    name: str
    shard_dim: str = ""

    def local(self) -> bool:
        return not self.shard_dim


@dataclass(frozen=True)
class TensorState:
    axes: tuple
    placements: tuple
    partials: tuple
    replicated_dims: tuple = ()

    @classmethod
    def from_spec(cls, spec, mesh_dim_names=()):
        axes = tuple(StateAxis(axis.name, axis.shard_dim) for axis in require_expanded_axes(spec))
        names = [axis.name for axis in axes]
        if len(names) != len(set(names)):
            raise ValueError("Symbolic TensorState requires unique axis names")
        partials = partials_of(spec)
        used = mesh_dims_components([axis.shard_dim for axis in axes if axis.shard_dim] + list(partials))
        replicated = tuple(dim for dim in mesh_dim_names if not (mesh_dim_components(dim) & used))
        return cls(
            axes=axes,
            placements=tuple((axis.name, axis.shard_dim or None) for axis in axes),
            partials=partials,
            replicated_dims=replicated,
        )

    def placement(self, name):
        for axis_name, shard_dim in self.placements:
            if axis_name == name:
                return shard_dim
        raise KeyError(name)

    def placement_dict(self) -> dict:
        return dict(self.placements)

    def axis(self, name) -> StateAxis:
        for axis in self.axes:
            if axis.name == name:
                return axis
        raise KeyError(name)

    def names(self) -> tuple:
        return tuple(axis.name for axis in self.axes)


@dataclass(frozen=True)
class PlanStep:
    """One primitive of a transition plan: a mapping name plus its arguments."""

    name: str
    args: tuple = ()


def tensor_spec(axes, partials=()):
    return TensorSpec(Axes(axes), partials)


def local_axis(name):
    return Axis(name)


def sharded_axis(name, shard_dim):
    return Axis(name, shard_dim)
