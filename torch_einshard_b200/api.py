"""``einshard`` / ``einshard_like`` entry points.

``einshard(expr, *tensors, mesh=, shapes=, sizes=, families=, optimize=, policy=)``
expands axis families, parses the expression, registers metadata for operands
annotated ``[param]``, and runs either the local contraction (when no axis
changes placement and no partials are involved) or the distributed executor.
``einshard_like`` performs the same parsing, validation and parameter
registration without running anything.  Contract of
``src/torch_einshard/__init__.py:82-372``.
"""

from . import params as _params
from .notation.families import cached_expand_axis_families
from .notation.parser import parse_sharding
from .notation.spec import Axes, AxisGroup, EllipsisAxis, TensorSpec
from .ops import gemm as _gemm
from .ops.einsum import einsum
from .parallel.executor import distributed_1d
from .plan.policy import resolve_plan_policy
from .plan.state import TensorState
from .plan.trace import ExecutionPlan, set_last_plan
from .plan.transitions import build_binary_transition_plan, build_unary_transition_plan

try:
    from torch.compiler import disable as _no_compile
except (AttributeError, ImportError):  # pragma: no cover - older torch
    from torch._dynamo import disable as _no_compile

__all__ = ["einshard", "einshard_like", "local_operation"]


def _axes(spec):
    return spec.axes if hasattr(spec, "axes") else spec


def _partials(spec):
    return getattr(spec, "partials", ())


def _flat(spec):
    axes = _axes(spec)
    return axes.flat() if hasattr(axes, "flat") else axes


def _has_groups(spec):
    return any(isinstance(axis, AxisGroup) for axis in _axes(spec))


def _no_ellipsis(axes):
    return Axes(axis for axis in axes if not isinstance(axis, EllipsisAxis))


def local_operation(shard):
    """True when every rank can compute its output shard with no communication."""
    if any(_partials(spec) for spec in shard if spec is not None):
        return False
    if shard[1] is None:
        return Axes(set(_flat(shard[0])) ^ set(_flat(shard[2]))).local()
    axes0, axes1, out = _flat(shard[0]), _flat(shard[1]), _flat(shard[2])
    inputs = list(axes0) + list(axes1)
    for axis in out:
        if axis not in inputs and any(other.name == axis.name for other in inputs):
            return False
    by0 = {a.name: a for a in axes0}
    by1 = {a.name: a for a in axes1}
    for name in set(by0) & set(by1):
        a, b = by0[name], by1[name]
        if not a.local() or not b.local() or a != b:
            return False
    return True


def _input_specs(shard):
    return (shard[0],) if shard[1] is None else (shard[0], shard[1])


def _operand_registrations(shard, xs, mesh):
    infer = local_operation(shard)
    names = None
    found = []
    specs = _input_specs(shard)
    for index, spec in enumerate(specs):
        if not getattr(getattr(spec, "annotation", None), "is_param", False):
            continue
        if names is None:
            names = _params._mesh_dim_names_from(mesh)
        if index >= len(xs):
            raise ValueError("Annotated parameter operand is missing a tensor argument")
        found.append((xs[index], _params.parameter_operand_state(
            xs[index], specs, shard[2], index, mesh_dim_names=names, infer_grad=infer,
        )))
    return found


def _prepare(registrations):
    merged, params = {}, {}
    for param, state in registrations:
        key = id(param)
        base = merged[key] if key in merged else _params._parameter_state_from_attached_metadata(param)
        merged[key] = _params._merge_parameter_state(base, state)
        _params._validate_parameter_state_rank(param, merged[key])
        params[key] = param
    return [(params[key], state) for key, state in merged.items()]


def _commit(registrations):
    for param, state in registrations:
        _params.set_parameter_state(param, state)


def _run(shard, xs, mesh, shapes, sizes, policy, activation=None):
    if local_operation(shard):
        out = einsum(shard, *xs, sizes=sizes, activation=activation)
        plan = ExecutionPlan()
        plan.add("rank_local_einsum")
        set_last_plan(plan)
        return out
    if any(_has_groups(spec) for spec in shard if spec is not None):
        raise NotImplementedError("Factored axes are currently supported only for local reshape operations")
    if mesh is None:
        raise ValueError("Distributed einshard operations require mesh")
    out = distributed_1d(shard, *xs, mesh=mesh, shapes=shapes, policy=policy)
    if activation is not None:
        if getattr(shard[2], "partials", ()):
            raise ValueError("activation needs a complete output (no // partial sums)")
        out = _gemm.silu(out) if activation == "silu" else None
        if out is None:
            raise ValueError(f"unsupported activation {activation!r} (supported: 'silu')")
    return out


def einshard(shard, *xs, mesh=None, shapes=None, sizes=None, families=None, optimize=None, policy=None,
             activation=None):
    """Run an einshard expression on ``xs`` (see module docstring).

    ``activation`` ("silu" or None) is an extension of this framework: the
    elementwise activation of the result.  For a rank-local contraction it runs
    in the GEMM's epilogue (the wide kernel writes the pre-activation, kept for
    backward, and the activation from one pass over its accumulator); for a
    distributed one it follows the plan's last step.  An output with ``//``
    partial sums cannot take one."""
    policy = resolve_plan_policy(optimize=optimize, policy=policy)
    shard, sizes = cached_expand_axis_families(shard, sizes, families)
    shard = parse_sharding(shard)
    if activation is not None and getattr(shard[2], "partials", ()):
        raise ValueError("activation needs a complete output (no // partial sums)")
    registrations = _prepare(_operand_registrations(shard, xs, mesh))
    out = _run(shard, xs, mesh, shapes, sizes, policy, activation)
    _commit(registrations)
    return out


# ------------------------------------------------------------------ einshard_like validation

def _check_output_axes_once(shard, *, exact):
    key = (lambda a: a) if exact else (lambda a: a.name)
    inputs = {key(a) for a in _flat(shard[0]) if not isinstance(a, EllipsisAxis)}
    if shard[1] is not None:
        inputs |= {key(a) for a in _flat(shard[1]) if not isinstance(a, EllipsisAxis)}
    seen = set()
    for axis in _flat(shard[2]):
        if isinstance(axis, EllipsisAxis):
            continue
        k = key(axis)
        if k in seen:
            raise ValueError(f"Output dimension {axis} appears more than once")
        seen.add(k)
        if k not in inputs:
            raise ValueError(f"Output dimension {axis} must be present in input")


def _check_like_unary(shard):
    a_in, a_out = tuple(_flat(shard[0])), tuple(_flat(shard[2]))
    e_in = any(isinstance(a, EllipsisAxis) for a in a_in)
    e_out = any(isinstance(a, EllipsisAxis) for a in a_out)
    if e_in or e_out:
        if e_in != e_out:
            raise NotImplementedError("Distributed unary ellipsis requires ellipsis in both input and output")
        if len([a for a in a_in if not isinstance(a, EllipsisAxis)]) != \
                len([a for a in a_out if not isinstance(a, EllipsisAxis)]):
            raise ValueError("Input tensor rank is incompatible with ellipsis notation")
        return
    if len(a_in) != len(a_out):
        raise ValueError("Input and output dimensions must match in the equation")
    if {a.name for a in a_in} != {a.name for a in a_out}:
        raise ValueError("Input and output axes must match")


def _check_sharded_contracting_axes_kept(shard):
    in0 = [a for a in _flat(shard[0]) if not isinstance(a, EllipsisAxis)]
    in1 = [a for a in _flat(shard[1]) if not isinstance(a, EllipsisAxis)]
    n0, n1 = {a.name for a in in0}, {a.name for a in in1}
    out_names = {a.name for a in _flat(shard[2]) if not isinstance(a, EllipsisAxis)}
    partials = set(_partials(shard[2]))
    for axes, other in ((in0, n1), (in1, n0)):
        for axis in axes:
            if axis.name in other or axis.name in out_names:
                continue
            if axis.shard_dim and axis.shard_dim not in partials:
                raise ValueError(
                    f"Omitted sharded input-only dimension {axis} must be preserved as an output partial"
                )


def _check_mesh_dims(shard, mesh):
    names = _params._mesh_dim_names_from(mesh)
    groups = []
    for spec in shard:
        if spec is None:
            continue
        groups += [a.shard_dim for a in _flat(spec) if not isinstance(a, EllipsisAxis) and a.shard_dim]
        groups += list(_partials(spec))
    _params._validate_known_mesh_groups(names, groups, "operation")


def _check_states(shard, mesh):
    names = _params._mesh_dim_names_from(mesh)
    for spec in shard:
        if spec is None or any(isinstance(a, EllipsisAxis) for a in _flat(spec)):
            continue
        TensorState.from_spec(spec, mesh_dim_names=names)


def _check_plan(shard):
    if shard[1] is None:
        if any(isinstance(a, EllipsisAxis) for spec in shard if spec is not None for a in _flat(spec)):
            return
        build_unary_transition_plan(shard[0], shard[2])
        return
    build_binary_transition_plan(*(
        TensorSpec(_no_ellipsis(_axes(spec)), _partials(spec)) for spec in shard
    ))


def _validate_like(shard, mesh):
    if mesh is not None:
        _check_mesh_dims(shard, mesh)
    if shard[1] is not None:
        _check_sharded_contracting_axes_kept(shard)
    if local_operation(shard):
        if _partials(shard[0]) or (shard[1] is not None and _partials(shard[1])):
            raise ValueError("Local einsum does not support partial inputs")
        _check_output_axes_once(shard, exact=True)
        return
    _check_output_axes_once(shard, exact=False)
    if any(_has_groups(spec) for spec in shard if spec is not None):
        raise NotImplementedError("Factored axes are currently supported only for local reshape operations")
    if mesh is None:
        raise ValueError("Distributed einshard operations require mesh")
    _check_states(shard, mesh)
    if shard[1] is None:
        _check_like_unary(shard)
    elif _partials(shard[0]) or _partials(shard[1]):
        raise ValueError("Binary distributed einshard_like does not support partial inputs")
    _check_plan(shard)


@_no_compile
def einshard_like(shard, *xs, mesh=None, sizes=None, families=None):
    """Register annotated parameter metadata from an einshard formula without executing it.

    Parses and validates the same notation as :func:`einshard` and attaches
    metadata to operands annotated ``[param]``.  Other operands only line up
    formula operands with arguments; nothing is computed and ``None`` is
    returned.
    """
    shard, _ = cached_expand_axis_families(shard, sizes, families)
    shard = parse_sharding(shard)
    registrations = _prepare(_operand_registrations(shard, xs, mesh))
    _validate_like(shard, mesh)
    _commit(registrations)
    return None
