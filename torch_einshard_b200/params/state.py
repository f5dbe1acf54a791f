"""Parameter metadata objects and their validation rules.

``ParameterState`` is attached to ``nn.Parameter`` objects as the attribute
``einshard_state``.  It records the parameter's layout spec, which mesh
dimensions it is sharded over, which mesh groups must agree on its initial
value (``init_sync``) and over which groups its gradient must be reduced
(``grad_comm``).  ``ParamShardMetadata`` is the checkpoint-facing record of
one rank's shard.  Field names, modes and error texts are part of the public
format and follow ``src/torch_einshard/params.py:13-737``.
"""

from dataclasses import dataclass, field

import torch

from ..notation.parser import parse_sharding
from ..notation.spec import AxisGroup, EllipsisAxis, TensorAnnotation, TensorSpec
from ..plan.state import TensorState

PARAM_STATE_ATTR = "einshard_state"

__all__ = [
    "PARAM_STATE_ATTR",
    "ParameterInitSync",
    "ParameterGradComm",
    "ParameterState",
    "ParamShardMetadata",
    "NativeGradReductionHandle",
]


# ------------------------------------------------------------------ name helpers

def as_name_tuple(value):
    if value is None:
        return ()
    if isinstance(value, str):
        return (value,)
    out = tuple(value)
    if not all(isinstance(item, str) for item in out):
        raise TypeError("Parameter metadata entries must be strings")
    return out


def duplicates(values):
    seen, out = set(), []
    for value in values:
        if value in seen and value not in out:
            out.append(value)
        seen.add(value)
    return out


def components(name):
    """A group name and its ``-``-separated components."""
    return {name, *name.split("-")}


def components_of(names):
    out = set()
    for name in names:
        out |= components(name)
    return out


def parts(name):
    """Only the ``-``-separated components of a group name."""
    return set(name.split("-"))


def parts_of(names):
    out = set()
    for name in names:
        out |= parts(name)
    return out


def check_group_components(names, label):
    for name in names:
        pieces = name.split("-")
        if not all(pieces):
            raise ValueError(f"Parameter {label} contains empty mesh dimensions: {name}")
        if len(set(pieces)) != len(pieces):
            raise ValueError(f"Parameter {label} contains repeated mesh dimensions: {name}")


def check_groups_disjoint(names, label):
    seen = set()
    for name in names:
        overlap = seen & parts(name)
        if overlap:
            raise ValueError(f"Parameter {label} groups overlap on mesh dimensions: {', '.join(sorted(overlap))}")
        seen |= parts(name)


def check_layout(layout_shard_dims, init_sync=None):
    check_group_components(layout_shard_dims, "layout")
    seen = set()
    for dim in layout_shard_dims:
        overlap = seen & components(dim)
        if overlap:
            raise ValueError(
                "Parameter specs cannot shard multiple axes over the same mesh dimension: "
                + ", ".join(sorted(overlap))
            )
        seen |= components(dim)
    if init_sync is None or init_sync.mode in ("none", "external") or not init_sync.mesh_dims:
        return
    sharded = components_of(layout_shard_dims)
    check_group_components(init_sync.mesh_dims, "init_sync")
    check_groups_disjoint(init_sync.mesh_dims, "init_sync")
    for name in init_sync.mesh_dims:
        overlap = sharded & components(name)
        if overlap:
            raise ValueError(
                "Parameter init_sync annotation overlaps with sharded axis dimensions: " + ", ".join(sorted(overlap))
            )


def check_grad_comm(layout_shard_dims, grad_comm):
    if grad_comm.mode == "none" or not grad_comm.mesh_dims:
        return
    check_group_components(grad_comm.mesh_dims, "grad")
    if grad_comm.backend == "external":
        return
    check_groups_disjoint(grad_comm.mesh_dims, "grad")
    sharded = components_of(layout_shard_dims)
    for name in grad_comm.mesh_dims:
        overlap = sharded & components(name)
        if overlap:
            raise ValueError(
                "Parameter grad annotation overlaps with sharded axis dimensions: " + ", ".join(sorted(overlap))
            )


# ------------------------------------------------------------------ mesh dim names

def normalize_mesh_dim_names(names):
    if names is None:
        return ()
    if isinstance(names, str):
        names = (names,)
    elif isinstance(names, torch.Tensor) or (hasattr(names, "shape") and hasattr(names, "dtype")):
        raise TypeError("mesh_dim_names must be an iterable of strings")
    else:
        try:
            names = tuple(names)
        except TypeError as error:
            raise TypeError("mesh_dim_names must be an iterable of strings") from error
    if not all(isinstance(name, str) for name in names):
        raise TypeError("mesh_dim_names entries must be strings")
    if not all(names):
        raise ValueError("mesh_dim_names entries must be non-empty strings")
    check_group_components(names, "mesh_dim_names")
    check_groups_disjoint(names, "mesh_dim_names")
    repeated = duplicates(names)
    if repeated:
        raise ValueError(f"mesh_dim_names entries must be unique: {', '.join(repeated)}")
    return names


def check_name_count(mesh, names):
    grid = getattr(mesh, "mesh", None)
    if grid is None or not hasattr(grid, "dim"):
        return
    if len(names) != grid.dim():
        raise ValueError("mesh_dim_names length must match mesh rank")


def check_names_match_mesh(mesh, names):
    mesh_names = getattr(mesh, "mesh_dim_names", None)
    if mesh_names is None:
        return
    if names != normalize_mesh_dim_names(mesh_names):
        raise ValueError("mesh_dim_names must match mesh.mesh_dim_names")


def mesh_dim_names_from(mesh=None, mesh_dim_names=()):
    """Resolve mesh dim names from an explicit argument or from ``mesh``."""
    if mesh_dim_names is not None and not (isinstance(mesh_dim_names, tuple) and not mesh_dim_names):
        names = normalize_mesh_dim_names(mesh_dim_names)
        check_name_count(mesh, names)
        check_names_match_mesh(mesh, names)
        return names
    if mesh is None:
        return ()
    names = normalize_mesh_dim_names(getattr(mesh, "mesh_dim_names", None))
    check_name_count(mesh, names)
    return names


def group_known(name, mesh_dim_names):
    if name in mesh_dim_names:
        return True
    pieces = name.split("-")
    if len(set(pieces)) != len(pieces):
        return False
    return len(pieces) > 1 and all(piece in mesh_dim_names for piece in pieces)


def check_known_groups(mesh_dim_names, groups, label):
    if not mesh_dim_names or not groups:
        return
    missing = [name for name in groups if not group_known(name, mesh_dim_names)]
    if missing:
        raise ValueError(f"Parameter {label} references unknown mesh dimensions: {', '.join(missing)}")


def check_parameter_groups(mesh_dim_names, layout_shard_dims, init_sync, grad_comm):
    check_known_groups(mesh_dim_names, layout_shard_dims, "layout")
    if init_sync.mesh_dims:
        check_known_groups(mesh_dim_names, init_sync.mesh_dims, "init_sync")
    if grad_comm.mode != "none" and grad_comm.backend != "external":
        check_known_groups(mesh_dim_names, grad_comm.mesh_dims, "grad")


# ------------------------------------------------------------------ layouts

def parse_layout_axes(layout):
    spec_in, other, spec_out = parse_sharding(f"{layout} -> {layout}")
    if other is not None or spec_in.partials or spec_out.partials:
        raise ValueError("Parameter specs must contain only axis layout notation")
    return spec_in.axes


def check_layout_value(layout):
    if not isinstance(layout, str):
        raise TypeError("Parameter layout must be a string")


def check_annotation_value(name, value):
    if not isinstance(value, str):
        raise TypeError(f"{name} must be a string annotation value")
    pieces = value.split(":")
    if len(pieces) > 2 or not all(pieces):
        raise ValueError(f"Invalid {name} annotation value {value!r}")
    if not all(token and token.isalnum() for token in pieces[0].split("-")):
        raise ValueError(f"Invalid {name} annotation value {value!r}")
    if len(pieces) == 2 and not pieces[1].isalnum():
        raise ValueError(f"Invalid {name} annotation value {value!r}")


def spec_from_layout(layout, *, grad=None, init_sync=None):
    check_layout_value(layout)
    items = []
    if grad is not None:
        check_annotation_value("grad", grad)
        items.append(("grad", grad))
    if init_sync is not None:
        check_annotation_value("init_sync", init_sync)
        items.append(("init_sync", init_sync))
    annotation = TensorAnnotation.from_items(items) if items else None
    axes = parse_layout_axes(layout)
    if any(isinstance(axis, AxisGroup) for axis in axes):
        raise ValueError("Explicit parameter layouts cannot contain factored axes")
    return TensorSpec(axes, annotation=annotation)


def axis_signature(axis):
    if isinstance(axis, EllipsisAxis):
        return ("ellipsis",)
    if isinstance(axis, AxisGroup):
        return ("group", tuple(axis_signature(inner) for inner in axis.axes))
    return ("axis", axis.name, axis.shard_dim)


def layout_signature(spec):
    return tuple(axis_signature(axis) for axis in spec.axes)


def tensor_state_or_none(spec, mesh_dim_names):
    try:
        return TensorState.from_spec(spec, mesh_dim_names=mesh_dim_names)
    except ValueError:
        return None


# ------------------------------------------------------------------ state objects

@dataclass(frozen=True)
class ParameterInitSync:
    mode: str = "none"
    mesh_dims: tuple = ()

    @classmethod
    def from_annotation(cls, annotation, layout_shard_dims, mesh_dim_names):
        if annotation is not None:
            if annotation.mode in ("none", "external"):
                return cls(mode=annotation.mode)
            if annotation.mode == "explicit":
                return cls(mode="explicit", mesh_dims=annotation.mesh_dims)
        if not mesh_dim_names:
            return cls(mode="none")
        sharded = components_of(layout_shard_dims)
        return cls(mode="inferred",
                   mesh_dims=tuple(dim for dim in mesh_dim_names if not (components(dim) & sharded)))


@dataclass(frozen=True)
class ParameterGradComm:
    mode: str = "none"
    mesh_dims: tuple = ()
    backend: str = "none"
    schedule: str = "backend_default"

    @classmethod
    def from_annotation(cls, annotation, *, is_param=False):
        if annotation is None:
            return cls(mode="inferred", backend="native") if is_param else cls()
        return cls(mode=annotation.mode, mesh_dims=annotation.mesh_dims, backend=annotation.backend,
                   schedule=annotation.schedule)

    @property
    def pending_inference(self):
        return self.mode == "inferred" and not self.mesh_dims


@dataclass(frozen=True)
class ParameterState:
    spec: TensorSpec
    tensor_state: TensorState = None
    layout_shard_dims: tuple = ()
    mesh_dim_names: tuple = ()
    init_sync: ParameterInitSync = field(default_factory=ParameterInitSync)
    grad_comm: ParameterGradComm = field(default_factory=ParameterGradComm)
    source: str = "inferred"
    explicit_init_sync_none: bool = False
    explicit_grad_comm_none: bool = False

    @classmethod
    def from_spec(cls, spec, *, mesh_dim_names=(), source="inferred"):
        mesh_dim_names = mesh_dim_names_from(mesh_dim_names=mesh_dim_names)
        if getattr(spec, "partials", ()):
            raise ValueError("Parameter states must contain only axis layout notation")
        layout_shard_dims = tuple(spec.axes.all_shard_dims())
        annotation = getattr(spec, "annotation", None)
        is_param = bool(getattr(annotation, "is_param", False))
        init_annotation = getattr(annotation, "init_sync", None)
        grad_annotation = getattr(annotation, "grad", None)
        init_sync = ParameterInitSync.from_annotation(init_annotation, layout_shard_dims, mesh_dim_names)
        check_layout(layout_shard_dims, init_sync)
        grad_comm = ParameterGradComm.from_annotation(grad_annotation, is_param=is_param)
        check_grad_comm(layout_shard_dims, grad_comm)
        check_parameter_groups(mesh_dim_names, layout_shard_dims, init_sync, grad_comm)
        return cls(
            spec=spec,
            tensor_state=tensor_state_or_none(spec, mesh_dim_names),
            layout_shard_dims=layout_shard_dims,
            mesh_dim_names=mesh_dim_names,
            init_sync=init_sync,
            grad_comm=grad_comm,
            source=source,
            explicit_init_sync_none=init_annotation is not None and init_annotation.mode == "none",
            explicit_grad_comm_none=grad_annotation is not None and grad_annotation.mode == "none",
        )

    @classmethod
    def from_layout(cls, layout, *, mesh=None, mesh_dim_names=(), grad=None, init_sync=None, source="layout"):
        spec = spec_from_layout(layout, grad=grad, init_sync=init_sync)
        state = cls.from_spec(spec, mesh_dim_names=mesh_dim_names_from(mesh, mesh_dim_names), source=source)
        if state.tensor_state is None:
            raise ValueError("Explicit parameter layouts must be representable as TensorState")
        return state

    @property
    def axes(self):
        if self.spec is None:
            raise ValueError("ParameterState does not have an inferred parameter layout yet")
        return self.spec.axes

    @property
    def shared(self):
        if self.init_sync.mode in ("none", "external"):
            return ()
        return self.init_sync.mesh_dims

    @property
    def reduce(self):
        if self.grad_comm.mode == "none" or self.grad_comm.backend == "external":
            return ()
        return self.grad_comm.mesh_dims


@dataclass(frozen=True)
class ParamShardMetadata:
    """Checkpoint record of one rank's shard of a parameter."""

    global_shape: tuple
    local_slices: tuple
    local_shape: tuple
    shard_dims: tuple


class NativeGradReductionHandle:
    """Handle returned by :func:`register_native_grad_reduction_hooks_`.

    ``wait()`` completes outstanding asynchronous reductions (failed works are
    kept so that a retry can wait again); ``remove()`` waits and removes hooks.
    """

    def __init__(self):
        self._hooks = []
        self._works = []

    @property
    def pending(self):
        return len(self._works)

    def _add_hook(self, hook):
        self._hooks.append(hook)

    def _add_work(self, work):
        self._works.append(work)

    def wait(self):
        works, self._works = self._works, []
        for index, work in enumerate(works):
            try:
                work.wait()
            except Exception:
                self._works = works[index:] + self._works
                raise
        return self

    def remove(self):
        self.wait()
        for hook in self._hooks:
            hook.remove()
        self._hooks = []
        return self


# ------------------------------------------------------------------ object validation

def check_name_tuple(value, label):
    if not isinstance(value, tuple):
        raise TypeError(f"{label} must be a tuple of strings")
    if not all(isinstance(item, str) for item in value):
        raise TypeError(f"{label} entries must be strings")


def check_init_sync_object(init_sync):
    if not isinstance(init_sync, ParameterInitSync):
        raise TypeError("ParameterState init_sync must be a ParameterInitSync")
    check_name_tuple(init_sync.mesh_dims, "ParameterInitSync mesh_dims")
    if init_sync.mode not in ("none", "external", "explicit", "inferred"):
        raise ValueError(f"Unknown ParameterInitSync mode {init_sync.mode!r}")
    if init_sync.mode in ("none", "external") and init_sync.mesh_dims:
        raise ValueError("ParameterInitSync none/external modes cannot carry mesh_dims")
    if init_sync.mode == "explicit" and not init_sync.mesh_dims:
        raise ValueError("ParameterInitSync explicit mode requires mesh_dims")


def check_grad_comm_object(grad_comm):
    if not isinstance(grad_comm, ParameterGradComm):
        raise TypeError("ParameterState grad_comm must be a ParameterGradComm")
    check_name_tuple(grad_comm.mesh_dims, "ParameterGradComm mesh_dims")
    if grad_comm.mode not in ("none", "inferred", "explicit"):
        raise ValueError(f"Unknown ParameterGradComm mode {grad_comm.mode!r}")
    if grad_comm.backend not in ("none", "native", "ddp", "external"):
        raise ValueError(f"Unknown ParameterGradComm backend {grad_comm.backend!r}")
    if grad_comm.schedule not in ("backend_default", "synchronous", "async"):
        raise ValueError(f"Unknown ParameterGradComm schedule {grad_comm.schedule!r}")
    if grad_comm.mode == "none":
        if grad_comm.backend != "none" or grad_comm.mesh_dims:
            raise ValueError("ParameterGradComm none mode cannot carry backend or mesh_dims")
    elif grad_comm.backend == "none":
        raise ValueError("ParameterGradComm non-none modes require a backend")
    if grad_comm.mode == "explicit" and not grad_comm.mesh_dims:
        raise ValueError("ParameterGradComm explicit mode requires mesh_dims")
    if grad_comm.backend != "native" and grad_comm.schedule != "backend_default":
        raise ValueError("ParameterGradComm schedules other than backend_default require native backend")


def _check_inferred_init_sync(state, layout_shard_dims, mesh_dim_names, derived):
    if state.init_sync.mode != "inferred":
        return
    expected = ParameterInitSync.from_annotation(None, layout_shard_dims, mesh_dim_names).mesh_dims
    if state.init_sync.mesh_dims != expected:
        actual = ", ".join(state.init_sync.mesh_dims) or "<none>"
        wanted = ", ".join(expected) or "<none>"
        raise ValueError(
            f"ParameterState inferred init_sync mesh_dims {actual} do not match {derived}-derived mesh dims {wanted}"
        )


def check_state_object(state):
    if not isinstance(state, ParameterState):
        raise TypeError("Attached parameter metadata must be a ParameterState")
    check_init_sync_object(state.init_sync)
    check_grad_comm_object(state.grad_comm)
    if state.spec is None:
        check_name_tuple(state.layout_shard_dims, "ParameterState layout_shard_dims")
        names = normalize_mesh_dim_names(state.mesh_dim_names)
        if tuple(state.mesh_dim_names) != names:
            raise ValueError("ParameterState mesh_dim_names are malformed")
        if state.tensor_state is not None:
            raise ValueError("ParameterState without a layout cannot carry tensor_state")
        if state.grad_comm.mode != "none":
            raise ValueError("ParameterState without a layout cannot carry grad_comm")
        _check_inferred_init_sync(state, state.layout_shard_dims, names, "sharding")
        return
    if getattr(state.spec, "partials", ()):
        raise ValueError("Parameter states must contain only axis layout notation")
    layout_shard_dims = tuple(state.spec.axes.all_shard_dims())
    if tuple(state.layout_shard_dims) != layout_shard_dims:
        raise ValueError("ParameterState layout_shard_dims do not match spec axes")
    names = normalize_mesh_dim_names(state.mesh_dim_names)
    if tuple(state.mesh_dim_names) != names:
        raise ValueError("ParameterState mesh_dim_names are malformed")
    _check_inferred_init_sync(state, layout_shard_dims, names, "layout")


def check_state_metadata(state):
    check_state_object(state)
    check_layout(state.layout_shard_dims, state.init_sync)
    check_grad_comm(state.layout_shard_dims, state.grad_comm)
    check_parameter_groups(state.mesh_dim_names, state.layout_shard_dims, state.init_sync, state.grad_comm)


def check_state_rank(param, state):
    if state.spec is None or not hasattr(param, "ndim"):
        return
    axes = tuple(state.axes)
    if any(isinstance(axis, EllipsisAxis) for axis in axes):
        valid = param.ndim >= sum(not isinstance(axis, EllipsisAxis) for axis in axes)
    else:
        valid = param.ndim == len(axes)
    if not valid:
        raise ValueError(f"Parameter rank {param.ndim} does not match parameter layout rank {len(state.axes)}")
