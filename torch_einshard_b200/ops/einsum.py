"""Local (per-rank) contraction of an einshard expression.

The notation is lowered to an einsum equation over single letters.  Axes are
keyed by the full axis object (``h/tp`` and ``h`` are different letters) unless
``name_only`` is set.  Factored groups ``(h p)`` are expanded by reshape before
the contraction (one unknown factor may be inferred from ``sizes``) and packed
again afterwards.  Contract and error texts follow
``src/torch_einshard/einsum.py:20-135``.

The contraction itself goes through :func:`.contraction.contract`, which
canonicalises two-operand contractions to a batched GEMM and runs the tcgen05
kernel for bf16/fp16 CUDA tensors.
"""

import string

from ..notation.spec import AxisGroup, EllipsisAxis
from .contraction import contract

__all__ = ["einsum", "expand_groups", "pack_groups"]


def _axes(spec):
    return spec.axes if hasattr(spec, "axes") else spec


def _flat(spec):
    axes = _axes(spec)
    return axes.flat() if hasattr(axes, "flat") else axes


def _has_groups(spec):
    return any(isinstance(axis, AxisGroup) for axis in _axes(spec))


def _factor_sizes(extent, group, sizes):
    known = [None if sizes is None else sizes.get(axis.name) for axis in group]
    missing = [axis for axis, size in zip(group, known) if size is None]
    product = 1
    for size in known:
        if size is not None:
            product *= size
    if len(missing) > 1:
        raise ValueError(f"Cannot infer multiple factor sizes for {', '.join(a.name for a in missing)}")
    if missing:
        if extent % product != 0:
            raise ValueError(f"Cannot infer factor size for {missing[0].name!r} from dimension {extent}")
        known[known.index(None)] = extent // product
    elif product != extent:
        raise ValueError(f"Factor sizes multiply to {product}, but tensor dimension is {extent}")
    return known


def expand_groups(tensor, spec, sizes):
    """Reshape so that every factored group becomes its member dimensions."""
    if not _has_groups(spec):
        return tensor
    axes = _axes(spec)
    n_ellipsis = tensor.dim() - sum(1 for axis in axes if not isinstance(axis, EllipsisAxis))
    shape, dim = [], 0
    for axis in axes:
        if isinstance(axis, EllipsisAxis):
            shape.extend(tensor.shape[dim:dim + n_ellipsis])
            dim += n_ellipsis
        elif isinstance(axis, AxisGroup):
            shape.extend(_factor_sizes(tensor.shape[dim], axis, sizes))
            dim += 1
        else:
            shape.append(tensor.shape[dim])
            dim += 1
    return tensor.reshape(shape)


def pack_groups(tensor, spec):
    """Merge member dimensions back into each factored group of ``spec``."""
    if not _has_groups(spec):
        return tensor
    axes = _axes(spec)
    fixed = sum(len(axis) if isinstance(axis, AxisGroup) else 1 for axis in axes if not isinstance(axis, EllipsisAxis))
    n_ellipsis = tensor.dim() - fixed
    shape, dim = [], 0
    for axis in axes:
        if isinstance(axis, EllipsisAxis):
            shape.extend(tensor.shape[dim:dim + n_ellipsis])
            dim += n_ellipsis
        elif isinstance(axis, AxisGroup):
            extent = 1
            for _ in axis:
                extent *= tensor.shape[dim]
                dim += 1
            shape.append(extent)
        else:
            shape.append(tensor.shape[dim])
            dim += 1
    return tensor.reshape(shape)


def _letters(spec, table, name_only, allow_missing=True):
    out = ""
    for axis in _flat(spec):
        if isinstance(axis, EllipsisAxis):
            out += "..."
            continue
        key = axis.name if name_only else axis
        if key not in table:
            if not allow_missing:
                raise AssertionError(f"Output dimension {axis} must be present in input")
            table[key] = string.ascii_letters[len(table)]
        out += table[key]
    return out


def equation_for(shard, name_only=False):
    """The einsum equation (letters) the local contraction of ``shard`` uses."""
    table = {}
    lhs = _letters(shard[0], table, name_only)
    if shard[1] is not None:
        lhs += "," + _letters(shard[1], table, name_only)
    return f"{lhs}->{_letters(shard[2], table, name_only, allow_missing=False)}"


def einsum(shard, *xs, name_only=False, sizes=None, activation=None):
    """Run the local contraction described by ``shard`` on ``xs``, optionally
    followed by an elementwise ``activation`` (fused into the GEMM epilogue)."""
    binary = shard[1] is not None
    if not name_only:
        assert not getattr(shard[0], "partials", ()), "Local einsum does not support partial inputs"
        if binary:
            assert not getattr(shard[1], "partials", ()), "Local einsum does not support partial inputs"
        xs = [expand_groups(xs[0], shard[0], sizes)] + list(xs[1:])
        if binary:
            xs[1] = expand_groups(xs[1], shard[1], sizes)
    table = {}
    lhs = _letters(shard[0], table, name_only)
    if binary:
        lhs += "," + _letters(shard[1], table, name_only)
    rhs = _letters(shard[2], table, name_only, allow_missing=False)
    output = contract(f"{lhs}->{rhs}", *xs, activation=activation)
    return output if name_only else pack_groups(output, shard[2])
