"""Registration and merging of parameter metadata.

A parameter may be described several times (by a formula operand annotated
``[param]``, by layout helpers, by ``init_param_``); each description is
merged into the attached :class:`ParameterState`.  Merging keeps explicit
``none`` opt-outs sticky, resolves pending gradient inference against concrete
groups, and rejects layouts or groups that disagree.  Multi-parameter helpers
validate every update before attaching any (all-or-nothing).  Rules and error
texts: ``src/torch_einshard/params.py:740-1566``.
"""

from collections.abc import Mapping
from dataclasses import replace

import torch

from ..notation.spec import EllipsisAxis, TensorAnnotation
from .state import (
    PARAM_STATE_ATTR,
    ParameterGradComm,
    ParameterInitSync,
    ParameterState,
    as_name_tuple,
    axis_signature,
    check_annotation_value,
    check_grad_comm,
    check_known_groups,
    check_layout,
    check_layout_value,
    check_parameter_groups,
    check_state_metadata,
    check_state_rank,
    components_of,
    layout_signature,
    mesh_dim_names_from,
    parse_layout_axes,
)

_INCOMPATIBLE = "Parameter is already registered with incompatible metadata"


# ------------------------------------------------------------------ attach / lookup

def attached_state(param):
    return getattr(param, PARAM_STATE_ATTR, None)


def set_parameter_state(param, state):
    setattr(param, PARAM_STATE_ATTR, state)
    return param


def get_parameter_state(param):
    return attached_state(param)


def iter_parameter_states(module):
    for name, param in module.named_parameters():
        state = get_parameter_state(param)
        if state is not None:
            yield name, param, state


# ------------------------------------------------------------------ merge rules

def _explicit_init_none(state):
    if getattr(state, "explicit_init_sync_none", False):
        return True
    init_sync = getattr(getattr(state.spec, "annotation", None), "init_sync", None)
    return init_sync is not None and init_sync.mode == "none"


def _explicit_grad_none(state):
    if getattr(state, "explicit_grad_comm_none", False):
        return True
    grad = getattr(getattr(state.spec, "annotation", None), "grad", None)
    return grad is not None and grad.mode == "none"


def _merge_init_sync(old_state, new_state):
    old, new = old_state.init_sync, new_state.init_sync
    if _explicit_init_none(new_state):
        if old.mode != "none":
            raise ValueError(_INCOMPATIBLE)
        return old
    if new.mode == "none":
        return old
    if new.mode == "inferred" and old.mode != "none":
        return old
    if old.mode == "none":
        if _explicit_init_none(old_state):
            raise ValueError(_INCOMPATIBLE)
        return new
    compatible = old == new or (
        old.mode not in ("none", "external") and new.mode not in ("none", "external")
        and old.mesh_dims == new.mesh_dims
    )
    if not compatible:
        raise ValueError(_INCOMPATIBLE)
    return old


def _merge_schedule(old, new):
    if old.schedule == new.schedule or new.schedule == "backend_default":
        return old.schedule
    if old.schedule == "backend_default":
        return new.schedule
    raise ValueError(_INCOMPATIBLE)


def _merge_grad_comm(old_state, new_state):
    old, new = old_state.grad_comm, new_state.grad_comm
    if _explicit_grad_none(new_state):
        if old.mode != "none":
            raise ValueError(_INCOMPATIBLE)
        return old
    if new.mode == "none":
        return old
    if old.mode == "none":
        if _explicit_grad_none(old_state):
            raise ValueError(_INCOMPATIBLE)
        return new
    if old.backend != new.backend:
        raise ValueError(_INCOMPATIBLE)
    schedule = _merge_schedule(old, new)
    if old.pending_inference and new.pending_inference:
        return replace(old, schedule=schedule)
    if old.pending_inference or new.pending_inference:
        concrete, pending = (new, old) if old.pending_inference else (old, new)
        return replace(concrete if concrete.mode == "explicit" else pending, schedule=schedule)
    if old.mesh_dims != new.mesh_dims:
        raise ValueError(_INCOMPATIBLE)
    return replace(old, schedule=schedule)


def _merge_tensor_state(old, new):
    if new.tensor_state is None:
        return old.tensor_state
    if old.tensor_state is None:
        return new.tensor_state
    if len(new.tensor_state.replicated_dims) > len(old.tensor_state.replicated_dims):
        return new.tensor_state
    return old.tensor_state


def _merge_mesh_names(old, new):
    if not old.mesh_dim_names:
        return new.mesh_dim_names
    if not new.mesh_dim_names:
        return old.mesh_dim_names
    if old.mesh_dim_names != new.mesh_dim_names:
        raise ValueError("Parameter is already registered with incompatible mesh_dim_names")
    return old.mesh_dim_names


def _check_footprint(old, new):
    if old.spec is not None and new.spec is not None:
        if layout_signature(old.spec) != layout_signature(new.spec):
            raise ValueError("Parameter is already registered with a different layout")
        return
    if old.spec is None and new.spec is not None:
        compare = bool(old.layout_shard_dims)
    elif old.spec is not None and new.spec is None:
        compare = bool(new.layout_shard_dims)
    else:
        compare = bool(old.layout_shard_dims) and bool(new.layout_shard_dims)
    if compare and components_of(old.layout_shard_dims) != components_of(new.layout_shard_dims):
        raise ValueError("Parameter is already registered with a different sharded mesh footprint")


def merge_parameter_state(old, new):
    """Merge ``new`` metadata into ``old`` (either may be None)."""
    if old is None:
        return new
    _check_footprint(old, new)
    init_sync = _merge_init_sync(old, new)
    grad_comm = _merge_grad_comm(old, new)
    tensor_state = _merge_tensor_state(old, new)
    mesh_names = _merge_mesh_names(old, new)
    layout_dims = new.layout_shard_dims if (new.spec is not None or not old.layout_shard_dims) else old.layout_shard_dims
    spec = new.spec if new.spec is not None else old.spec
    check_layout(layout_dims, init_sync)
    check_grad_comm(layout_dims, grad_comm)
    check_parameter_groups(mesh_names, layout_dims, init_sync, grad_comm)
    init_none = _explicit_init_none(old) or _explicit_init_none(new)
    grad_none = _explicit_grad_none(old) or _explicit_grad_none(new)
    unchanged = (
        spec == old.spec and tuple(layout_dims) == tuple(old.layout_shard_dims) and init_sync == old.init_sync
        and grad_comm == old.grad_comm and tensor_state == old.tensor_state and mesh_names == old.mesh_dim_names
        and init_none == old.explicit_init_sync_none and grad_none == old.explicit_grad_comm_none
    )
    if unchanged:
        return old
    return replace(old, spec=spec, tensor_state=tensor_state, layout_shard_dims=layout_dims,
                   mesh_dim_names=mesh_names, init_sync=init_sync, grad_comm=grad_comm, source=old.source,
                   explicit_init_sync_none=init_none, explicit_grad_comm_none=grad_none)


def register_parameter_state(param, state):
    check_state_metadata(state)
    existing = attached_state(param)
    if existing is not None:
        check_state_metadata(existing)
    merged = merge_parameter_state(existing, state)
    check_state_metadata(merged)
    return set_parameter_state(param, merged)


def prepare_updates(updates):
    """Merge a batch of ``(param, state)`` updates without attaching anything."""
    merged, params = {}, {}
    for param, state in updates:
        check_state_rank(param, state)
        key = id(param)
        base = merged[key] if key in merged else attached_state(param)
        merged[key] = merge_parameter_state(base, state)
        params[key] = param
    return [(params[key], state) for key, state in merged.items()]


def _commit(prepared):
    for param, state in prepared:
        set_parameter_state(param, state)


# ------------------------------------------------------------------ module helpers

def _param_attr(module, name):
    param = getattr(module, name, None)
    if param is None:
        return None
    if not isinstance(param, torch.nn.Parameter):
        raise TypeError(f"module.{name} must be a torch.nn.Parameter")
    return param


def module_parameter(module, name):
    if not isinstance(name, str):
        raise TypeError("Parameter names must be strings")
    if not name:
        raise ValueError("Parameter names must be non-empty")
    try:
        return module.get_parameter(name)
    except AttributeError as error:
        raise ValueError(f"module does not define parameter {name!r}") from error


def _per_param(value, name):
    return value.get(name) if isinstance(value, Mapping) else value


def check_metadata_keys(value, names, label):
    if not isinstance(value, Mapping):
        return
    unknown = sorted(set(value) - set(names), key=repr)
    if unknown:
        raise ValueError(f"{label} metadata contains unknown parameter names: {', '.join(repr(n) for n in unknown)}")


def _axis_layout(axis):
    from ..notation.spec import AxisGroup
    if isinstance(axis, EllipsisAxis):
        raise ValueError("Parameter layout helpers do not support ellipsis axes")
    if isinstance(axis, AxisGroup):
        raise NotImplementedError("Parameter layout helpers do not support factored-axis groups")
    return f"{axis.name}/{axis.shard_dim}" if axis.shard_dim else axis.name


def _bias_layout(weight_layout):
    check_layout_value(weight_layout)
    axes = parse_layout_axes(weight_layout)
    if not axes:
        raise ValueError("Linear weight layout must contain at least one axis")
    return _axis_layout(axes[0])


def _check_bias_matches_first_axis(weight_layout, bias_layout, label):
    check_layout_value(weight_layout)
    check_layout_value(bias_layout)
    w_axes, b_axes = parse_layout_axes(weight_layout), parse_layout_axes(bias_layout)
    if not w_axes:
        raise ValueError(f"{label} weight layout must contain at least one axis")
    if len(b_axes) != 1 or axis_signature(b_axes[0]) != axis_signature(w_axes[0]):
        raise ValueError(f"{label} bias layout must match the first weight layout axis")


def _check_same_layout(layout, other, label):
    check_layout_value(layout)
    check_layout_value(other)
    a, b = parse_layout_axes(layout), parse_layout_axes(other)
    if tuple(axis_signature(x) for x in a) != tuple(axis_signature(x) for x in b):
        raise ValueError(f"{label} layout must match weight layout")


def register_parameter_layout(param, layout, *, mesh=None, mesh_dim_names=(), grad=None, init_sync=None,
                              source="layout"):
    if not isinstance(param, torch.nn.Parameter):
        raise TypeError("Parameter layout registration requires a torch.nn.Parameter")
    state = ParameterState.from_layout(layout, mesh=mesh, mesh_dim_names=mesh_dim_names, grad=grad,
                                       init_sync=init_sync, source=source)
    check_state_rank(param, state)
    return register_parameter_state(param, state)


def register_module_parameter_layouts_(module, layouts, *, mesh=None, mesh_dim_names=(), grad=None, init_sync=None,
                                       source="module"):
    if not isinstance(layouts, Mapping):
        raise TypeError("Parameter layouts must be a mapping from parameter name to layout")
    if not layouts:
        raise ValueError("Parameter layouts mapping must not be empty")
    names = tuple(layouts)
    check_metadata_keys(grad, names, "grad")
    check_metadata_keys(init_sync, names, "init_sync")
    mesh_dim_names = mesh_dim_names_from(mesh, mesh_dim_names)
    updates = [
        (module_parameter(module, name),
         ParameterState.from_layout(layout, mesh_dim_names=mesh_dim_names, grad=_per_param(grad, name),
                                    init_sync=_per_param(init_sync, name), source=source))
        for name, layout in layouts.items()
    ]
    _commit(prepare_updates(updates))
    return module


def register_linear_parameters_(module, *, weight_layout="out in", bias_layout=None, mesh=None, mesh_dim_names=(),
                                weight_grad=None, bias_grad=None, init_sync=None, weight_init_sync=None,
                                bias_init_sync=None, source="linear"):
    mesh_dim_names = mesh_dim_names_from(mesh, mesh_dim_names)
    weight = _param_attr(module, "weight")
    if weight is None:
        raise ValueError("module must define a weight parameter")
    explicit_bias = bias_layout is not None or bias_grad is not None or bias_init_sync is not None
    weight_init_sync = init_sync if weight_init_sync is None else weight_init_sync
    bias_init_sync = init_sync if bias_init_sync is None else bias_init_sync
    updates = [(weight, ParameterState.from_layout(weight_layout, mesh_dim_names=mesh_dim_names, grad=weight_grad,
                                                   init_sync=weight_init_sync, source=source))]
    bias = _param_attr(module, "bias")
    if bias is None and explicit_bias:
        raise ValueError("module does not define a bias parameter")
    if weight.ndim != 2:
        raise ValueError("Linear weight must be rank 2")
    if bias is not None and bias.ndim != 1:
        raise ValueError("Linear bias must be rank 1")
    if bias is not None and weight.shape[0] != bias.shape[0]:
        raise ValueError("Linear bias shape must match weight output dimension")
    if bias is not None:
        if bias_layout is None:
            bias_layout = _bias_layout(weight_layout)
        else:
            _check_bias_matches_first_axis(weight_layout, bias_layout, "Linear")
        updates.append((bias, ParameterState.from_layout(bias_layout, mesh_dim_names=mesh_dim_names, grad=bias_grad,
                                                         init_sync=bias_init_sync, source=source)))
    _commit(prepare_updates(updates))
    return module


def _default_conv_layout(rank):
    layouts = {3: "out in k", 4: "out in kh kw", 5: "out in kd kh kw"}
    if rank not in layouts:
        raise ValueError("Conv weight must be rank 3, 4, or 5")
    return layouts[rank]


def register_conv_parameters_(module, *, weight_layout=None, bias_layout=None, mesh=None, mesh_dim_names=(),
                              grad=None, weight_grad=None, bias_grad=None, init_sync=None, weight_init_sync=None,
                              bias_init_sync=None, source="conv"):
    mesh_dim_names = mesh_dim_names_from(mesh, mesh_dim_names)
    explicit_bias = bias_layout is not None or bias_grad is not None or bias_init_sync is not None
    weight_grad = grad if weight_grad is None else weight_grad
    bias_grad = grad if bias_grad is None else bias_grad
    weight_init_sync = init_sync if weight_init_sync is None else weight_init_sync
    bias_init_sync = init_sync if bias_init_sync is None else bias_init_sync
    weight = _param_attr(module, "weight")
    if weight is None:
        raise ValueError("module must define a weight parameter")
    bias = _param_attr(module, "bias")
    if bias is None and explicit_bias:
        raise ValueError("module does not define a bias parameter")
    if isinstance(module, torch.nn.modules.conv._ConvTransposeNd):
        raise NotImplementedError("ConvTranspose parameter registration is not supported")
    if getattr(module, "groups", 1) != 1:
        raise NotImplementedError("Conv parameter registration currently supports only groups=1")
    if weight.ndim not in (3, 4, 5):
        raise ValueError("Conv weight must be rank 3, 4, or 5")
    if bias is not None and bias.ndim != 1:
        raise ValueError("Conv bias must be rank 1")
    if bias is not None and weight.shape[0] != bias.shape[0]:
        raise ValueError("Conv bias shape must match weight output dimension")
    if weight_layout is None:
        weight_layout = _default_conv_layout(weight.ndim)
    updates = [(weight, ParameterState.from_layout(weight_layout, mesh_dim_names=mesh_dim_names, grad=weight_grad,
                                                   init_sync=weight_init_sync, source=source))]
    if bias is not None:
        if bias_layout is None:
            bias_layout = _bias_layout(weight_layout)
        else:
            _check_bias_matches_first_axis(weight_layout, bias_layout, "Conv")
        updates.append((bias, ParameterState.from_layout(bias_layout, mesh_dim_names=mesh_dim_names, grad=bias_grad,
                                                         init_sync=bias_init_sync, source=source)))
    _commit(prepare_updates(updates))
    return module


class _DefaultNormLayout:
    def __repr__(self):
        return '"c"'


_DEFAULT_NORM_LAYOUT = _DefaultNormLayout()


def register_norm_parameters_(module, *, layout=_DEFAULT_NORM_LAYOUT, weight_layout=None, bias_layout=None,
                              mesh=None, mesh_dim_names=(), grad=None, weight_grad=None, bias_grad=None,
                              init_sync=None, weight_init_sync=None, bias_init_sync=None, source="norm"):
    mesh_dim_names = mesh_dim_names_from(mesh, mesh_dim_names)
    explicit_bias = bias_layout is not None or bias_grad is not None or bias_init_sync is not None
    omitted = layout is _DEFAULT_NORM_LAYOUT
    layout = "c" if omitted else layout
    if weight_layout is None:
        weight_layout = layout
    elif not omitted:
        _check_same_layout(layout, weight_layout, "Norm weight")
    weight_grad = grad if weight_grad is None else weight_grad
    bias_grad = grad if bias_grad is None else bias_grad
    weight_init_sync = init_sync if weight_init_sync is None else weight_init_sync
    bias_init_sync = init_sync if bias_init_sync is None else bias_init_sync
    weight = _param_attr(module, "weight")
    if weight is None:
        raise ValueError("module must define a weight parameter")
    updates = [(weight, ParameterState.from_layout(weight_layout, mesh_dim_names=mesh_dim_names, grad=weight_grad,
                                                   init_sync=weight_init_sync, source=source))]
    bias = _param_attr(module, "bias")
    if bias is None and explicit_bias:
        raise ValueError("module does not define a bias parameter")
    if bias is not None and weight.shape != bias.shape:
        raise ValueError("Norm bias shape must match weight shape")
    if bias is not None:
        if bias_layout is None:
            bias_layout = weight_layout
        else:
            _check_same_layout(weight_layout, bias_layout, "Norm bias")
        updates.append((bias, ParameterState.from_layout(bias_layout, mesh_dim_names=mesh_dim_names, grad=bias_grad,
                                                         init_sync=bias_init_sync, source=source)))
    _commit(prepare_updates(updates))
    return module


# ------------------------------------------------------------------ formula operands

def _flat(spec):
    axes = spec.axes if hasattr(spec, "axes") else spec
    return axes.flat() if hasattr(axes, "flat") else axes


def infer_grad_mesh_dims(input_specs, output_spec, operand_index, *, include_axes=True):
    """Mesh dims a parameter operand's gradient must be reduced over.

    Every mesh dim that shards an axis of another operand or of the output
    which the parameter does not carry, plus every output partial.
    """
    param_names = {a.name for a in _flat(input_specs[operand_index]) if not isinstance(a, EllipsisAxis)}
    dims = []
    if include_axes:
        others = (*input_specs[:operand_index], *input_specs[operand_index + 1:], output_spec)
        for spec in others:
            for axis in _flat(spec):
                if isinstance(axis, EllipsisAxis) or axis.name in param_names:
                    continue
                if axis.shard_dim and axis.shard_dim not in dims:
                    dims.append(axis.shard_dim)
    for partial in getattr(output_spec, "partials", ()):
        if partial and partial not in dims:
            dims.append(partial)
    return tuple(dims)


def _with_inferred_grad(state, input_specs, output_spec, operand_index, *, include_axes=True, mesh_dim_names=()):
    grad_comm = state.grad_comm
    if not grad_comm.pending_inference:
        return state
    dims = infer_grad_mesh_dims(input_specs, output_spec, operand_index, include_axes=include_axes)
    grad_comm = ParameterGradComm() if not dims else replace(grad_comm, mesh_dims=dims)
    check_grad_comm(state.layout_shard_dims, grad_comm)
    check_parameter_groups(mesh_dim_names, state.layout_shard_dims, state.init_sync, grad_comm)
    return replace(state, grad_comm=grad_comm)


def parameter_operand_state(param, input_specs, output_spec, operand_index, *, mesh_dim_names=(), source="formula",
                            infer_grad=True):
    if not isinstance(param, torch.nn.Parameter):
        raise TypeError("Annotated parameter operands must be torch.nn.Parameter instances")
    mesh_dim_names = mesh_dim_names_from(mesh_dim_names=mesh_dim_names)
    state = ParameterState.from_spec(input_specs[operand_index], mesh_dim_names=mesh_dim_names, source=source)
    if not infer_grad:
        return state
    return _with_inferred_grad(state, input_specs, output_spec, operand_index,
                               include_axes=infer_grad != "partials", mesh_dim_names=mesh_dim_names)


def register_parameter_operand(param, input_specs, output_spec, operand_index, *, mesh_dim_names=(),
                               source="formula", infer_grad=True):
    state = parameter_operand_state(param, input_specs, output_spec, operand_index, mesh_dim_names=mesh_dim_names,
                                    source=source, infer_grad=infer_grad)
    check_state_rank(param, state)
    return register_parameter_state(param, state)


# ------------------------------------------------------------------ finalisation

def _finalized_grad(value):
    check_annotation_value("grad", value)
    annotation = TensorAnnotation.from_items((("grad", value),)).grad
    grad_comm = ParameterGradComm.from_annotation(annotation)
    if grad_comm.pending_inference or grad_comm.mode == "none":
        raise ValueError("Finalized grad communication must use an explicit mesh group")
    return grad_comm


def _finalized_state(state, grad, mesh_dim_names):
    if not state.grad_comm.pending_inference:
        raise ValueError("Parameter gradient communication is not pending inference")
    grad_comm = _finalized_grad(grad)
    mesh_dim_names = mesh_dim_names or state.mesh_dim_names
    check_grad_comm(state.layout_shard_dims, grad_comm)
    check_parameter_groups(mesh_dim_names, state.layout_shard_dims, state.init_sync, grad_comm)
    return replace(state, mesh_dim_names=mesh_dim_names, grad_comm=grad_comm, explicit_grad_comm_none=False)


def _check_finalized_groups(mesh, state):
    from .comm import groups_exist
    if mesh is None or state.grad_comm.backend not in ("native", "ddp"):
        return
    groups_exist(mesh, state.grad_comm.mesh_dims)


def finalize_parameter_grad_comm_(param, grad, *, mesh=None, mesh_dim_names=()):
    if not isinstance(param, torch.nn.Parameter):
        raise TypeError("Parameter grad finalization requires a torch.nn.Parameter")
    state = attached_state(param)
    if state is None:
        raise ValueError("Parameter does not have an attached ParameterState")
    finalized = _finalized_state(state, grad, mesh_dim_names_from(mesh, mesh_dim_names))
    _check_finalized_groups(mesh, finalized)
    return register_parameter_state(param, finalized)


def finalize_module_parameter_grad_comm_(module, grad, *, mesh=None, mesh_dim_names=()):
    if not isinstance(grad, Mapping):
        raise TypeError("grad finalization must be a mapping from parameter names to grad policies")
    if not grad:
        raise ValueError("grad finalization mapping must not be empty")
    mesh_dim_names = mesh_dim_names_from(mesh, mesh_dim_names)
    updates = []
    for name, value in grad.items():
        param = module_parameter(module, name)
        state = attached_state(param)
        if state is None:
            raise ValueError(f"module parameter {name!r} does not have attached ParameterState")
        finalized = _finalized_state(state, value, mesh_dim_names)
        _check_finalized_groups(mesh, finalized)
        updates.append((param, finalized))
    _commit(prepare_updates(updates))
    return module


# ------------------------------------------------------------------ init-time metadata

def _init_sync_value(sync, layout_shard_dims, mesh_dim_names):
    if sync is None:
        return ParameterInitSync.from_annotation(None, layout_shard_dims, mesh_dim_names)
    if not isinstance(sync, str):
        dims = as_name_tuple(sync)
        for name in dims:
            check_annotation_value("sync", name)
        return ParameterInitSync(mode="explicit", mesh_dims=dims)
    if sync in ("none", "external"):
        return ParameterInitSync(mode=sync)
    check_annotation_value("sync", sync)
    return ParameterInitSync(mode="explicit", mesh_dims=(sync,))


def init_state(*, sync, sharded, mesh_dim_names, source):
    layout_dims = as_name_tuple(sharded)
    check_known_groups(mesh_dim_names, layout_dims, "layout")
    init_sync = _init_sync_value(sync, layout_dims, mesh_dim_names)
    check_layout(layout_dims, init_sync)
    check_parameter_groups(mesh_dim_names, layout_dims, init_sync, ParameterGradComm())
    return ParameterState(spec=None, layout_shard_dims=layout_dims, mesh_dim_names=mesh_dim_names,
                          init_sync=init_sync, source=source, explicit_init_sync_none=sync == "none")


def validate_module_parameter_states_(module, mesh=None, *, allow_pending=False):
    from .comm import groups_exist, validation_grad_groups
    from .state import check_layout as _cl, check_names_match_mesh, check_state_object
    for name, param in module.named_parameters():
        state = attached_state(param)
        if state is None:
            continue
        try:
            check_state_object(state)
            check_state_rank(param, state)
            _cl(state.layout_shard_dims, state.init_sync)
            check_grad_comm(state.layout_shard_dims, state.grad_comm)
            check_parameter_groups(state.mesh_dim_names, state.layout_shard_dims, state.init_sync, state.grad_comm)
            grad_groups = validation_grad_groups(state, allow_pending=allow_pending)
            if mesh is not None:
                if state.mesh_dim_names:
                    check_names_match_mesh(mesh, state.mesh_dim_names)
                groups_exist(mesh, (*state.layout_shard_dims, *state.shared, *grad_groups))
        except (AttributeError, TypeError, ValueError) as error:
            raise ValueError(f"Invalid parameter metadata for {name!r}: {error}") from error
    return module
