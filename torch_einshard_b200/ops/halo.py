"""``einhalo`` (ghost cells) and ``einwindow`` (sharding-aware im2col).

A halo of ``(left, right)`` cells is added to named axes.  Local axes are
padded with a ``constant`` fill, ``periodic`` wrap or ``replicate`` edge.  A
sharded axis fetches exactly the global intervals its halo covers from their
owner ranks (uneven shards, halos wider than a shard and periodic wrap are all
handled by the interval table); the backward pass scatter-adds halo gradients
to the owners.  ``einwindow`` adds the halo and then unfolds window axes.
Contract of ``src/torch_einshard/halo.py:14-418``.
"""

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..notation.families import cached_expand_axis_families, expand_family_mapping
from ..notation.parser import parse_sharding
from ..notation.spec import EllipsisAxis
from ..parallel.collectives import resolve_split_shapes, split_offsets

__all__ = ["einhalo", "einwindow", "halo_intervals", "halo_tensor", "normalize_halo"]


def _axes(spec):
    return spec.axes if hasattr(spec, "axes") else spec


def normalize_halo(value):
    if isinstance(value, int):
        if value < 0:
            raise ValueError("Halo widths must be non-negative")
        return value, value
    left, right = value
    if left < 0 or right < 0:
        raise ValueError("Halo widths must be non-negative")
    return left, right


def pad_dim(x, dim, left, right, *, boundary, fill):
    """Pad one local dimension with the requested boundary rule."""
    if left == 0 and right == 0:
        return x
    n = x.shape[dim]
    if boundary == "periodic":
        if n == 0:
            raise ValueError("Cannot periodic-pad an empty axis")
        index = torch.arange(-left, n + right, device=x.device).remainder(n)
        return torch.index_select(x, dim, index).contiguous()
    if boundary == "replicate":
        if n == 0:
            raise ValueError("Cannot replicate-pad an empty axis")
        index = torch.arange(-left, n + right, device=x.device).clamp(0, n - 1)
        return torch.index_select(x, dim, index).contiguous()
    if boundary == "constant":
        padding = [0, 0] * x.dim()
        padding[2 * (x.dim() - dim - 1)] = left
        padding[2 * (x.dim() - dim - 1) + 1] = right
        return F.pad(x, padding, mode="constant", value=fill)
    raise ValueError(f"Unsupported halo boundary {boundary!r}")


def _owner(ends, g):
    for rank, end in enumerate(ends):
        if g < end:
            return rank
    return len(ends) - 1


def _pieces(shapes, start, length, *, periodic):
    """Split global range [start, start+length) into (out_off, src_rank, src_off, len) pieces.

    Non-periodic requests outside [0, total) are skipped (their output cells
    are left for the boundary padding).
    """
    if length == 0:
        return []
    total = sum(shapes)
    if periodic and total == 0:
        raise ValueError("Cannot periodic-pad an empty axis")
    offsets = split_offsets(shapes)
    ends = [o + s for o, s in zip(offsets, shapes)]
    pieces, out_off, cursor, remaining = [], 0, start, length
    while remaining > 0:
        if periodic:
            g = cursor % total
        else:
            if cursor < 0:
                skip = min(remaining, -cursor)
                cursor, out_off, remaining = cursor + skip, out_off + skip, remaining - skip
                continue
            if cursor >= total:
                break
            g = cursor
        src = _owner(ends, g)
        take = min(remaining, ends[src] - g)
        if take == 0:
            cursor += 1
            continue
        pieces.append((out_off, src, g - offsets[src], take))
        cursor, out_off, remaining = cursor + take, out_off + take, remaining - take
    return pieces


def halo_intervals(shapes, left, right, *, periodic):
    """Per destination rank: the pieces that make up its haloed shard."""
    total = sum(shapes)
    table, start = [], 0
    for local in shapes:
        if periodic:
            lo, length = start - left, local + left + right
        else:
            lo = max(0, start - left)
            length = min(total, start + local + right) - lo
        table.append(_pieces(shapes, lo, length, periodic=periodic))
        start += local
    return table


def _resized(x, dim, length):
    shape = list(x.shape)
    shape[dim] = length
    return x.new_empty(shape)


def _halo_forward(x, group, dim, shapes, left, right, periodic):
    """The haloed shard of x along ``dim`` (native staged exchange, else NCCL P2P)."""
    size, rank = dist.get_world_size(group), dist.get_rank(group)
    if len(shapes) != size:
        raise ValueError(f"Error: passed shapes of size {len(shapes)} not equal to {size}")
    if x.shape[dim] != shapes[rank]:
        raise ValueError(f"Local tensor size {x.shape[dim]} does not match split shape {shapes[rank]}")
    table = halo_intervals(shapes, left, right, periodic=periodic)
    length = shapes[rank] + left + right if periodic else sum(p[3] for p in table[rank])
    from ..parallel import symmetric
    comm = symmetric.communicator_for(group) if x.is_cuda else None
    if comm is not None:
        out = comm.halo_gather(x.contiguous(), dim, table, length, shapes)
        if out is not None:
            return out
    out = _resized(x, dim, length)
    ops, landing, keep = [], [], []
    for out_off, src, src_off, n in table[rank]:
        target = out.narrow(dim, out_off, n)
        if src == rank:
            target.copy_(x.narrow(dim, src_off, n))
            continue
        incoming = torch.empty_like(target)
        landing.append((incoming, target))
        ops.append(dist.P2POp(dist.irecv, incoming, dist.get_global_rank(group, src), group))
    for dst, pieces in enumerate(table):
        if dst == rank:
            continue
        for _, src, src_off, n in pieces:
            if src == rank:
                outgoing = x.narrow(dim, src_off, n).contiguous()
                keep.append(outgoing)
                ops.append(dist.P2POp(dist.isend, outgoing, dist.get_global_rank(group, dst), group))
    if ops:
        for request in dist.batch_isend_irecv(ops):
            request.wait()
    for incoming, target in landing:
        target.copy_(incoming)
    return out.contiguous()


def _halo_adjoint(grad, group, dim, shapes, left, right, periodic, in_shape):
    """Adjoint of _halo_forward: every haloed row's gradient back to its owner, summed."""
    rank = dist.get_rank(group)
    table = halo_intervals(shapes, left, right, periodic=periodic)
    from ..parallel import symmetric
    comm = symmetric.communicator_for(group) if grad.is_cuda else None
    if comm is not None:
        out = comm.halo_scatter_add(grad.contiguous(), dim, table, in_shape)
        if out is not None:
            return out
    grad_in = grad.new_zeros(in_shape)
    ops, landing, keep = [], [], []
    for out_off, src, src_off, n in table[rank]:
        piece = grad.narrow(dim, out_off, n)
        if src == rank:
            grad_in.narrow(dim, src_off, n).add_(piece)
            continue
        outgoing = piece.contiguous()
        keep.append(outgoing)
        ops.append(dist.P2POp(dist.isend, outgoing, dist.get_global_rank(group, src), group))
    for dst, pieces in enumerate(table):
        if dst == rank:
            continue
        for _, src, src_off, n in pieces:
            if src != rank:
                continue
            target = grad_in.narrow(dim, src_off, n)
            incoming = torch.empty_like(target)
            landing.append((incoming, target))
            ops.append(dist.P2POp(dist.irecv, incoming, dist.get_global_rank(group, dst), group))
    if ops:
        for request in dist.batch_isend_irecv(ops):
            request.wait()
    for incoming, target in landing:
        target.add_(incoming)
    return grad_in


class _HaloExchange(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim, shapes, left, right, periodic):
        ctx.saved = (group, dim, shapes, left, right, periodic, tuple(x.shape))
        return _halo_forward(x, group, dim, shapes, left, right, periodic)

    @staticmethod
    def backward(ctx, grad):
        return _halo_adjoint(grad, *ctx.saved), None, None, None, None, None, None


def _sharded_halo(x, axis, dim, left, right, *, mesh, shapes, boundary, fill):
    z, lo, hi = _sharded_halo_unpadded(x, axis, dim, left, right, mesh=mesh, shapes=shapes, boundary=boundary)
    return pad_dim(z, dim, lo, hi, boundary=boundary, fill=fill) if lo or hi else z


def _sharded_halo_unpadded(x, axis, dim, left, right, *, mesh, shapes, boundary):
    """The exchanged part of a sharded halo: this rank's rows plus the ghost
    rows its neighbours hold, and how many rows of boundary fill are missing
    before and after them (the global edges)."""
    if mesh is None:
        raise ValueError("Sharded einhalo axes require mesh")
    group = mesh[axis.shard_dim].get_group()
    size, rank = dist.get_world_size(group), dist.get_rank(group)
    split = resolve_split_shapes(shapes, axis.shard_dim, axis.name, group)
    if split is None:
        split = [x.shape[dim]] * size
    if x.shape[dim] != split[rank]:
        raise ValueError(
            f"Local tensor size {x.shape[dim]} does not match split shape {split[rank]} for axis {axis.name!r}"
        )
    total = sum(split)
    if boundary == "periodic":
        if total == 0:
            raise ValueError("Cannot periodic-pad an empty axis")
        return _HaloExchange.apply(x, group, dim, split, left, right, True), 0, 0
    if boundary not in ("constant", "replicate"):
        raise ValueError(f"Unsupported halo boundary {boundary!r}")
    start, local = sum(split[:rank]), split[rank]
    lo, hi = max(0, start - left), min(total, start + local + right)
    z = _HaloExchange.apply(x, group, dim, split, left, right, False)
    return z, lo - (start - left), (start + local + right) - hi


def halo_ghost_rows(x, axis, dim, left, right, *, mesh, shapes, slab=None, shape=None):
    """Zero-boundary halo of a sharded axis for a consumer that reads the
    shard and its neighbours' rows in place (the pair conv's ghost rows):
    returns (G, gtop, gbot, missing_lo, missing_hi, adjoint).  G holds the
    gtop rows above the shard and the gbot rows below it along ``dim`` (only
    the rows peers own; the shard is not copied), missing_lo / missing_hi the
    zero rows beyond the global edges, and adjoint(dv) maps the gradient of
    the haloed shard (gtop + shard + gbot rows) back to the shard's gradient.
    ``slab(off, n)`` / ``shape``: exchange the rows of a tensor of that shape
    that is never assembled (only the sent rows are built)."""
    shape = list(x.shape) if shape is None else list(shape)
    if mesh is None:
        raise ValueError("Sharded einhalo axes require mesh")
    group = mesh[axis.shard_dim].get_group()
    size, rank = dist.get_world_size(group), dist.get_rank(group)
    split = resolve_split_shapes(shapes, axis.shard_dim, axis.name, group)
    if split is None:
        split = [x.shape[dim]] * size
    if shape[dim] != split[rank]:
        raise ValueError(
            f"Local tensor size {shape[dim]} does not match split shape {split[rank]} for axis {axis.name!r}"
        )
    total, start, local = sum(split), sum(split[:rank]), split[rank]
    lo, hi = max(0, start - left), min(total, start + local + right)
    table = halo_intervals(split, left, right, periodic=False)
    length = sum(p[3] for p in table[rank])
    from ..parallel import symmetric
    comm = symmetric.communicator_for(group) if x.is_cuda else None
    got = comm.halo_ghosts(x, dim, table, length, slab=slab, shape=shape) if comm is not None else None
    if got is None:
        whole = x if slab is None else slab(0, shape[dim])
        full = _halo_forward(whole, group, dim, split, left, right, False)
        gtop, gbot = start - lo, hi - (start + local)
        g = torch.cat([full.narrow(dim, 0, gtop), full.narrow(dim, gtop + local, gbot)], dim)
    else:
        g, gtop, gbot = got
    in_shape = tuple(shape)

    def adjoint(dv):
        return _halo_adjoint(dv, group, dim, split, left, right, False, in_shape)

    return g, gtop, gbot, lo - (start - left), (start + local + right) - hi, adjoint


def _check_axes(axes):
    seen = set()
    for axis in axes:
        if isinstance(axis, EllipsisAxis):
            raise NotImplementedError("einhalo does not support ellipsis axes")
        if not hasattr(axis, "name"):
            raise NotImplementedError("einhalo does not support factored axes")
        if axis.name in seen:
            raise ValueError(f"Axis {axis.name!r} appears more than once")
        seen.add(axis.name)


def halo_tensor(spec, x, halos, *, mesh=None, shapes=None, boundary="constant", fill=0):
    axes = _axes(spec)
    _check_axes(axes)
    unknown = set(halos) - {axis.name for axis in axes}
    if unknown:
        raise ValueError(f"Halo axis {sorted(unknown)[0]!r} is not present in the tensor spec")
    z = x
    for dim, axis in enumerate(axes):
        if axis.name not in halos:
            continue
        left, right = normalize_halo(halos[axis.name])
        if left == 0 and right == 0:
            continue
        if axis.local():
            z = pad_dim(z, dim, left, right, boundary=boundary, fill=fill)
        else:
            z = _sharded_halo(z, axis, dim, left, right, mesh=mesh, shapes=shapes, boundary=boundary, fill=fill)
    return z


def halo_tensor_unpadded(spec, x, halos, *, mesh=None, shapes=None):
    """Zero-boundary halo for a consumer that zero-pads by itself (the native
    conv's TMA fill): sharded axes get their neighbours' ghost rows, and the
    fill that ``halo_tensor`` would add (local axes, global edges of sharded
    axes) is returned as {axis name: (before, after)} instead of copied in."""
    axes = _axes(spec)
    _check_axes(axes)
    pads = {}
    z = x
    for dim, axis in enumerate(axes):
        if axis.name not in halos:
            continue
        left, right = normalize_halo(halos[axis.name])
        if left == 0 and right == 0:
            continue
        if axis.local():
            pads[axis.name] = (left, right)
            continue
        z, lo, hi = _sharded_halo_unpadded(z, axis, dim, left, right, mesh=mesh, shapes=shapes, boundary="constant")
        if lo or hi:
            pads[axis.name] = (lo, hi)
    return z, pads


def einhalo(shard, x, halos, *, boundary="constant", fill=0, mesh=None, shapes=None, families=None):
    shard, _ = cached_expand_axis_families(shard, families=families)
    halos = expand_family_mapping(halos, families, label="Halo")
    spec = parse_sharding(f"{shard} -> {shard}")[0]
    return halo_tensor(spec, x, halos, mesh=mesh, shapes=shapes, boundary=boundary, fill=fill)


def einwindow(shard, x, windows, radius, *, boundary="constant", fill=0, mesh=None, shapes=None, families=None):
    """Materialise sliding windows: ``b h w c -> b h w kh kw c`` with halo exchange."""
    shard, _ = cached_expand_axis_families(shard, families=families)
    windows = expand_family_mapping(windows, families, label="Window")
    radius = expand_family_mapping(radius, families, label="Radius")
    in_spec, other, out_spec = parse_sharding(shard)
    if other is not None:
        raise ValueError("einwindow expects a unary sharding expression")
    if in_spec.partials or out_spec.partials:
        raise ValueError("einwindow does not support partial tensor specs")
    in_axes, out_axes = _axes(in_spec), _axes(out_spec)
    _check_axes(in_axes)
    _check_axes(out_axes)
    in_names = [a.name for a in in_axes]
    out_names = [a.name for a in out_axes]
    missing = [name for name in windows if name not in in_names]
    if missing:
        raise ValueError(f"Window source axis {missing[0]!r} is not present in the input")
    missing = [name for name in windows if name not in radius]
    if missing:
        raise ValueError(f"Missing radius for window source axis {missing[0]!r}")
    extra = set(radius) - set(windows)
    if extra:
        raise ValueError(f"Radius axis {sorted(extra)[0]!r} has no matching window")
    expected = in_names + list(windows.values())
    if len(set(expected)) != len(expected):
        raise ValueError("Window axes must be distinct from input axes and each other")
    if sorted(expected) != sorted(out_names):
        raise ValueError("einwindow output axes must be exactly the input axes plus the requested window axes")
    out_by = {a.name: a for a in out_axes}
    for axis in in_axes:
        if out_by[axis.name] != axis:
            raise ValueError("einwindow output must preserve input axis sharding")
    for window_axis in windows.values():
        if not out_by[window_axis].local():
            raise ValueError("einwindow window axes must be local")

    halos = {name: radius[name] for name in windows}
    z = halo_tensor(in_spec, x, halos, mesh=mesh, shapes=shapes, boundary=boundary, fill=fill)
    names = list(in_names)
    for axis in in_axes:
        if axis.name not in windows:
            continue
        left, right = normalize_halo(radius[axis.name])
        window_axis = windows[axis.name]
        if window_axis in names:
            raise ValueError(f"Window axis {window_axis!r} conflicts with an existing axis")
        z = z.unfold(names.index(axis.name), left + right + 1, 1)
        names.append(window_axis)
    return _materialize_windows(z, [names.index(name) for name in out_names])


def _materialize_windows(unfolded, permutation):
    """Permute the unfolded view to the output order and materialise it.

    CUDA tensors use the native window-gather kernel when available (one read
    of the haloed input per window element, coalesced writes); otherwise
    ``permute().contiguous()``.
    """
    view = unfolded.permute(permutation)
    if view.is_cuda:
        from . import native_ops
        out = native_ops.strided_copy(view)
        if out is not None:
            return out
    return view.contiguous()
