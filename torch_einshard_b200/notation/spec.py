"""Axis and tensor-spec data model of the einshard notation.

A parsed expression is a triple ``(input0, input1_or_None, output)`` of
:class:`TensorSpec`.  Each spec holds an :class:`Axes` list whose entries are
plain/sharded :class:`Axis` objects, at most one :class:`EllipsisAxis` and
factored :class:`AxisGroup` entries.  Input specs may carry a
:class:`TensorAnnotation` (``[param, grad=..., init_sync=...]``).

The ``repr`` strings, equality/hash rules and annotation value grammar are part
of the public interface (user code and tests compare them), so they follow the
reference notation exactly: ``src/torch_einshard/sharding.py:4-232``.
"""

from dataclasses import dataclass

__all__ = [
    "Axis",
    "EllipsisAxis",
    "AxisGroup",
    "Axes",
    "GradAnnotation",
    "InitSyncAnnotation",
    "TensorAnnotation",
    "TensorSpec",
]


class Axis:
    """A named tensor axis, optionally sharded over mesh dimension ``shard_dim``.

    Two axes are equal when both the name and the mesh dimension agree, so
    ``a/dp`` and ``a`` are different axes that share a name.
    """

    __slots__ = ("name", "shard_dim")

    def __init__(self, name: str, shard_dim: str = "") -> None:
        self.name = name
        self.shard_dim = shard_dim

    def local(self) -> bool:
        return self.shard_dim == "" or self.shard_dim is None

    def __repr__(self) -> str:
        return self.name if self.local() else f"{self.name} / {self.shard_dim}"

    def __hash__(self) -> int:
        return hash(self.name) ^ hash(self.shard_dim)

    def __eq__(self, other):
        if not isinstance(other, Axis):
            return NotImplemented
        return (self.name, self.shard_dim) == (other.name, other.shard_dim)


class EllipsisAxis:
    """The ``...`` placeholder; it stands for any number of local axes."""

    name = "..."
    shard_dim = ""

    def local(self) -> bool:
        return True

    def __repr__(self) -> str:
        return "..."

    def __hash__(self) -> int:
        return hash(EllipsisAxis)

    def __eq__(self, other) -> bool:
        return isinstance(other, EllipsisAxis)


class AxisGroup:
    """A factored axis ``(h p)``: one tensor dimension made of several axes."""

    def __init__(self, axes) -> None:
        self.axes = Axes(axes)

    def local(self) -> bool:
        return self.axes.local()

    def __iter__(self):
        return iter(self.axes)

    def __len__(self) -> int:
        return len(self.axes)

    def __repr__(self) -> str:
        return "(" + " ".join(str(axis) for axis in self.axes) + ")"


class Axes(list):
    """Ordered axes of one tensor spec."""

    def __repr__(self) -> str:
        return " × ".join(str(axis) for axis in self)

    def local(self) -> bool:
        return all(axis.local() for axis in self)

    def flat(self) -> "Axes":
        """Axes with every factored group expanded in place."""
        out = Axes()
        for axis in self:
            if isinstance(axis, AxisGroup):
                out.extend(axis.axes)
            else:
                out.append(axis)
        return out

    def all_shard_dims(self) -> list:
        """Mesh dimensions of every sharded axis, groups included, in order."""
        return [axis.shard_dim for axis in self.flat() if axis.shard_dim]


_RESERVED_GRAD_WORDS = frozenset({"async", "ddp", "external", "none"})


@dataclass(frozen=True)
class GradAnnotation:
    """Gradient-communication request of a ``[param, grad=...]`` operand.

    ``mode`` is ``inferred`` (mesh groups derived from the formula), ``explicit``
    (groups named in the value) or ``none``.  ``backend`` is ``native`` (einshard
    hooks), ``ddp`` (DDP comm hook), ``external`` or ``none``.  ``schedule`` is
    ``backend_default`` or ``async``.
    """

    mode: str = "inferred"
    mesh_dims: tuple = ()
    backend: str = "native"
    schedule: str = "backend_default"

    @classmethod
    def from_value(cls, value: str) -> "GradAnnotation":
        if ":" in value:
            group, _, suffix = value.rpartition(":")
            if not group or not suffix:
                raise ValueError("Invalid grad annotation")
            if group in _RESERVED_GRAD_WORDS:
                raise ValueError("Grad annotation suffix requires an explicit mesh group")
            per_suffix = {
                "async": dict(backend="native", schedule="async"),
                "ddp": dict(backend="ddp"),
                "external": dict(backend="external"),
            }
            if suffix not in per_suffix:
                raise ValueError(f"Unknown grad annotation suffix {suffix!r}")
            return cls(mode="explicit", mesh_dims=(group,), **per_suffix[suffix])
        keyword = {
            "async": dict(schedule="async"),
            "ddp": dict(backend="ddp"),
            "external": dict(backend="external"),
            "none": dict(mode="none", backend="none"),
        }
        if value in keyword:
            return cls(**keyword[value])
        return cls(mode="explicit", mesh_dims=(value,))

    def __repr__(self) -> str:
        if self.mode == "none":
            return "none"
        if self.mode == "inferred":
            if self.backend == "native" and self.schedule == "async":
                return "async"
            if self.backend in ("ddp", "external"):
                return self.backend
        if self.mode == "explicit" and self.mesh_dims:
            group = self.mesh_dims[0]
            if self.backend == "native" and self.schedule == "async":
                return f"{group}:async"
            if self.backend in ("ddp", "external"):
                return f"{group}:{self.backend}"
            return group
        return "inferred"


@dataclass(frozen=True)
class InitSyncAnnotation:
    """Initial-value synchronisation request ``init_sync=<group>|none|external``."""

    mode: str = "inferred"
    mesh_dims: tuple = ()

    @classmethod
    def from_value(cls, value: str) -> "InitSyncAnnotation":
        if ":" in value:
            raise ValueError("init_sync annotations do not accept suffixes")
        if value in ("none", "external"):
            return cls(mode=value)
        return cls(mode="explicit", mesh_dims=(value,))

    def __repr__(self) -> str:
        if self.mode in ("none", "external"):
            return self.mode
        if self.mode == "explicit" and self.mesh_dims:
            return self.mesh_dims[0]
        return "inferred"


@dataclass(frozen=True)
class TensorAnnotation:
    """Bracketed operand annotation ``[param, grad=..., init_sync=...]``."""

    is_param: bool = False
    grad: GradAnnotation = None
    init_sync: InitSyncAnnotation = None

    @classmethod
    def from_items(cls, items) -> "TensorAnnotation":
        fields = {}
        for key, value in items:
            if key in fields:
                raise ValueError(f"Duplicate tensor annotation {key!r}")
            if key == "param":
                fields[key] = True
            elif key == "grad":
                fields[key] = GradAnnotation.from_value(value)
            elif key == "init_sync":
                fields[key] = InitSyncAnnotation.from_value(value)
            else:
                raise ValueError(f"Unknown tensor annotation {key!r}")
        return cls(
            is_param=fields.get("param", False),
            grad=fields.get("grad"),
            init_sync=fields.get("init_sync"),
        )

    def __bool__(self) -> bool:
        return bool(self.is_param) or self.grad is not None or self.init_sync is not None

    def __repr__(self) -> str:
        parts = []
        if self.is_param:
            parts.append("param")
        if self.grad is not None:
            parts.append(f"grad={self.grad!r}")
        if self.init_sync is not None:
            parts.append(f"init_sync={self.init_sync!r}")
        return "[" + ", ".join(parts) + "]"


class TensorSpec:
    """One tensor of an expression: axes, partial mesh dims, annotation."""

    def __init__(self, axes, partials=None, annotation=None) -> None:
        if sum(1 for axis in axes if isinstance(axis, EllipsisAxis)) > 1:
            raise ValueError("Tensor specs may contain at most one ellipsis")
        self.axes = axes
        self.partials = tuple(partials) if partials else ()
        self.annotation = annotation if annotation is not None else TensorAnnotation()

    def local(self) -> bool:
        return self.axes.local() and not self.partials

    def __iter__(self):
        return iter(self.axes)

    def __len__(self) -> int:
        return len(self.axes)

    def __getitem__(self, index):
        return self.axes[index]

    def __repr__(self) -> str:
        text = repr(self.axes)
        if self.partials:
            if len(self.partials) == 1:
                text += f" // {self.partials[0]}"
            else:
                text += " // (" + ",".join(self.partials) + ")"
        if self.annotation:
            text += f" {self.annotation!r}"
        return text
