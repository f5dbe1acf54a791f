"""``einfft``: named-axis FFTs over (possibly sharded) tensors.

Paths, chosen per call (``explain=True`` reports the choice instead of running):

* ``distributed-fftn``  - complex transform; every sharded transform axis
  stays sharded on the same mesh dimension with equal shards divisible by the
  group size.  Each such axis runs the four-step FFT (all-to-all, size-P FFT,
  twiddle, all-to-all, size-L FFT, all-to-all); local axes run local FFTs.
* ``distributed-rfft-local-half`` / ``distributed-rfft-sharded-half`` - real
  forward/inverse transforms whose half-spectrum axis is local, or forward
  transforms whose sharded half axis is re-chunked with a prefix all-to-all.
* ``distributed-fftn-slab`` (this framework only) - a slab transpose: one
  transform axis is sharded on the input and local on the output while
  another is local on the input and sharded on the output over the same mesh
  dim (``b x/sp y z -> b kx ky/sp kz``).  Local FFTs, one all-to-all
  repartition, then the remaining FFT.  The reference rejects this layout.
* ``fallback`` - gather sharded transform axes, FFT, split (``RuntimeWarning``).

Semantics, error texts and ``explain`` payloads follow
``src/torch_einshard/fft.py:16-895``.  The four-step decomposition is the
standard Cooley-Tukey split ``k = k2 + P*k1``, ``n = q*L + m``.
Local FFTs of CUDA complex64 tensors run on the native Stockham kernels when
the extension provides them (``ops/fft_impl.py``), else ``torch.fft``.
"""

import math
import warnings
from collections.abc import Mapping

import torch
import torch.distributed as dist

from ..notation.families import cached_expand_axis_families, expand_family_mapping
from ..notation.parser import parse_sharding
from ..notation.spec import Axes, Axis, AxisGroup, EllipsisAxis, TensorSpec
from ..parallel.collectives import resolve_split_shapes, split_offsets
from ..parallel.executor import distributed_1d
from ..parallel.mappings import allgather_forward_split_backward, alltoall_repartition, split_forward_allgather_backward

__all__ = ["einfft"]

_SHARED_DIM_REASON = "einfft transform axes cannot share a mesh dimension with another input or output axis"


def _axes(spec):
    return spec.axes if hasattr(spec, "axes") else spec


def _dim(axes, name):
    for dim, axis in enumerate(axes):
        if axis.name == name:
            return dim
    raise ValueError(f"Axis {name!r} is not present")


def _spec_names(spec, *, label):
    if spec.partials:
        raise ValueError("einfft does not support partial tensor specs")
    names = []
    for axis in _axes(spec):
        if isinstance(axis, EllipsisAxis):
            raise NotImplementedError(f"einfft does not support ellipsis axes in {label}")
        if isinstance(axis, AxisGroup):
            raise NotImplementedError(f"einfft does not support factored axes in {label}")
        if axis.name in names:
            raise ValueError(f"Axis {axis.name!r} appears more than once in {label}")
        names.append(axis.name)
    return names


def _transform_map(axes):
    if isinstance(axes, dict):
        return dict(axes)
    if isinstance(axes, (str, bytes)):
        raise TypeError("axes must be a mapping or iterable of axis names, not a string")
    try:
        return {name: name for name in axes}
    except TypeError as error:
        raise TypeError("axes must be a mapping or iterable of axis names") from error


def _expand_axes_arg(axes, families):
    if isinstance(axes, dict):
        return expand_family_mapping(axes, families, label="FFT axis")
    if isinstance(axes, (str, bytes)) or not families:
        return axes
    out = []
    for name in axes:
        out.extend(families.get(name, (name,)))
    return out


def _group(mesh, dim):
    return mesh[dim].get_group()


# ----------------------------------------------------------------- local transforms

def _local_fft(x, dim, inverse, scale=1.0):
    """``scale`` times the unnormalised DFT along ``dim`` (inverse without the 1/n).
    The native kernel folds the scale into its stores."""
    from . import fft_impl
    out = fft_impl.try_fft(x, dim, inverse, scale)
    if out is not None:
        return out
    out = torch.fft.ifft(x, dim=dim, norm="forward") if inverse else torch.fft.fft(x, dim=dim)
    return out if scale == 1.0 else out * scale


def _rfft(x, dim):
    """Unnormalised real-to-half-spectrum DFT: native kernels when they apply."""
    from . import fft_impl
    out = fft_impl.rfft_native(x, dim) if x.is_cuda else None
    return out if out is not None else torch.fft.rfft(x, dim=dim)


def _irfft(x, n, dim):
    """Unnormalised half-spectrum-to-real inverse DFT of length ``n``."""
    from . import fft_impl
    out = fft_impl.irfft_native(x, n, dim) if x.is_cuda else None
    return out if out is not None else torch.fft.irfft(x, n=n, dim=dim, norm="forward")


def _norm_scale(*, n, inverse, norm):
    if norm == "ortho":
        return 1.0 / math.sqrt(n)
    if norm in (None, "backward"):
        return 1.0 / n if inverse else 1.0
    if norm == "forward":
        return 1.0 if inverse else 1.0 / n
    raise ValueError(f"Invalid FFT norm {norm!r}")


def _normalize(x, *, n, inverse, norm):
    if norm == "ortho":
        return x / math.sqrt(n)
    if norm in (None, "backward"):
        return x / n if inverse else x
    if norm == "forward":
        return x if inverse else x / n
    raise ValueError(f"Invalid FFT norm {norm!r}")


# ------------------------------------------------------------------ exchanges

def _exchange_blocks(z, group, send_block, out_shape, recv_view):
    """All-to-all of equal blocks: ``send_block(p)`` goes to peer p; block from
    peer p lands in ``recv_view(out, p)``."""
    size, rank = dist.get_world_size(group), dist.get_rank(group)
    out = z.new_empty(out_shape)
    from ..parallel import symmetric
    comm = symmetric.communicator_for(group) if z.is_cuda else None
    if comm is not None and comm.block_exchange(z, send_block, out, recv_view):
        return out
    ops, landing = [], []
    for peer in range(size):
        outgoing = send_block(peer).contiguous()
        target = recv_view(out, peer)
        if peer == rank:
            target.copy_(outgoing)
            continue
        peer_global = dist.get_global_rank(group, peer)
        incoming = torch.empty_like(target)
        ops.append(dist.P2POp(dist.isend, outgoing, peer_global, group))
        ops.append(dist.P2POp(dist.irecv, incoming, peer_global, group))
        landing.append((incoming, target))
    if ops:
        for request in dist.batch_isend_irecv(ops):
            request.wait()
    for incoming, target in landing:
        target.copy_(incoming)
    return out


def _distributed_fft_1d_no_autograd(x, group, dim, *, inverse, norm):
    """Distributed 1-D FFT along a sharded axis with equal shards, local size % P == 0."""
    P, r = dist.get_world_size(group), dist.get_rank(group)
    L = x.shape[dim]
    c = L // P
    N = L * P
    z = x.movedim(dim, -1).contiguous()
    lead = z.shape[:-1]
    z = z.reshape(-1, L)
    B = z.shape[0]
    # 1) each rank collects columns m in [r*c, (r+1)*c) from every q-block
    z = _exchange_blocks(z, group, lambda p: z[:, p * c:(p + 1) * c], (B, P, c), lambda o, p: o[:, p, :])
    # 2) size-P transforms over q, then twiddle w_N^(m*k2)
    z = _local_fft(z, 1, inverse)
    m = torch.arange(r * c, (r + 1) * c, device=z.device, dtype=torch.float64)
    k2 = torch.arange(P, device=z.device, dtype=torch.float64)
    angle = (1.0 if inverse else -1.0) * 2.0 * math.pi * torch.outer(k2, m) / N
    z = z * torch.polar(torch.ones_like(angle), angle).to(z.dtype)
    # 3) rank r collects k2 = r for every m
    z = _exchange_blocks(z, group, lambda p: z[:, p, :], (B, P, c), lambda o, p: o[:, p, :]).reshape(B, L)
    # 4) size-L transforms over m -> k1
    z = _local_fft(z, 1, inverse)
    # 5) back to contiguous blocks: rank r' owns k in [r'L, (r'+1)L), local index j*P + k2
    z = _exchange_blocks(z, group, lambda p: z[:, p * c:(p + 1) * c], (B, P, c), lambda o, p: o[:, p, :])
    z = z.permute(0, 2, 1).reshape(B, L)
    z = _normalize(z, n=N, inverse=inverse, norm=norm)
    return z.reshape(*lead, L).movedim(-1, dim).contiguous()


def _adjoint_norm(inverse, norm):
    if norm == "ortho":
        return "ortho"
    if inverse:
        return "forward" if norm in (None, "backward") else None
    return None if norm == "forward" else "forward"


class _DistributedFFT1D(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim, shapes, inverse, norm):
        ctx.args = (group, dim, inverse, norm)
        return _distributed_fft_1d_no_autograd(x, group, dim, inverse=inverse, norm=norm)

    @staticmethod
    def backward(ctx, grad):
        group, dim, inverse, norm = ctx.args
        out = _distributed_fft_1d_no_autograd(grad, group, dim, inverse=not inverse, norm=_adjoint_norm(inverse, norm))
        return out, None, None, None, None, None


def _dist_fft(x, group, dim, shapes, *, inverse, norm):
    return _DistributedFFT1D.apply(x, group, dim, shapes, inverse, norm)


def _prefix_exchange(x, group, dim, src_shapes, dst_shapes):
    """Re-chunk a prefix of a sharded axis: ``src_shapes`` -> ``dst_shapes`` (sum may shrink)."""
    r, P = dist.get_rank(group), dist.get_world_size(group)
    src_off, dst_off = split_offsets(src_shapes), split_offsets(dst_shapes)
    src_total = sum(src_shapes)
    z = x.movedim(dim, -1).contiguous()
    lead = z.shape[:-1]
    z = z.reshape(-1, src_shapes[r])
    B = z.shape[0]
    my_lo, my_hi = src_off[r], src_off[r] + src_shapes[r]
    send, send_sizes = [], []
    for p in range(P):
        lo = max(my_lo, dst_off[p])
        hi = min(my_hi, dst_off[p] + dst_shapes[p], src_total)
        n = max(0, hi - lo)
        send.append(z[:, lo - my_lo:lo - my_lo + n].reshape(-1))
        send_sizes.append(B * n)
    recv_sizes, recv_cols = [], []
    d_lo, d_hi = dst_off[r], dst_off[r] + dst_shapes[r]
    for p in range(P):
        lo = max(d_lo, src_off[p])
        hi = min(d_hi, src_off[p] + src_shapes[p], src_total)
        n = max(0, hi - lo)
        recv_sizes.append(B * n)
        recv_cols.append((lo - d_lo, n))
    flat = torch.cat(send) if send else z.new_empty(0)
    recv = z.new_empty(sum(recv_sizes))
    dist.all_to_all_single(recv, flat, recv_sizes, send_sizes, group=group)
    out = z.new_zeros(B, dst_shapes[r])
    cursor = 0
    for (col, n), count in zip(recv_cols, recv_sizes):
        if count:
            out[:, col:col + n].copy_(recv[cursor:cursor + count].reshape(B, n))
        cursor += count
    return out.reshape(*lead, dst_shapes[r]).movedim(-1, dim).contiguous()


class _PrefixRepartition(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim, src_shapes, dst_shapes):
        ctx.args = (group, dim, dst_shapes, src_shapes)
        return _prefix_exchange(x, group, dim, src_shapes, dst_shapes)

    @staticmethod
    def backward(ctx, grad):
        return _prefix_exchange(grad, *ctx.args), None, None, None, None


# ------------------------------------------------------------------ planning

def _axis_plan(x, source, in_axis, out_axis, in_axes, shapes, mesh):
    if in_axis.local() or out_axis.local() or in_axis.shard_dim != out_axis.shard_dim:
        return None
    group = _group(mesh, in_axis.shard_dim)
    split = resolve_split_shapes(shapes, in_axis.shard_dim, in_axis.name, group)
    out_split = resolve_split_shapes(shapes, out_axis.shard_dim, out_axis.name, group)
    P, r = dist.get_world_size(group), dist.get_rank(group)
    dim = _dim(in_axes, source)
    if split is None:
        split = [x.shape[dim]] * P
    if out_split is None:
        out_split = split
    if split != out_split or len(set(split)) != 1:
        return None
    local = split[r]
    if x.shape[dim] != local or local != split[0] or local % P != 0:
        return None
    return group, dim, split, sum(split)


def _complex_plan(x, tmap, in_by, out_by, in_axes, shapes, mesh, *, require_complex=True):
    if require_complex and not torch.is_complex(x):
        return None
    plan, used = [], set()
    for source, target in tmap.items():
        dim = _dim(in_axes, source)
        in_axis, out_axis = in_by[source], out_by[target]
        if not out_axis.local():
            if out_axis.shard_dim in used:
                return None
            used.add(out_axis.shard_dim)
        if in_axis.local():
            plan.append(("local", source, target, dim, x.shape[dim]))
            continue
        if mesh is None or out_axis.local() or in_axis.shard_dim != out_axis.shard_dim:
            return None
        found = _axis_plan(x, source, in_axis, out_axis, in_axes, shapes, mesh)
        if found is None:
            return None
        group, dim, split, n = found
        plan.append(("distributed", source, target, dim, n, group, split))
    return plan


def _run_items(z, current, out_by, plan, *, inverse, per_axis_norm, last_scale=None):
    """Runs the plan; ``last_scale`` (when given) is folded into a final local FFT.
    Returns (z, scale_applied)."""
    applied = False
    for index, item in enumerate(plan):
        if item[0] == "local":
            _, source, target, dim, _ = item
            fold = last_scale is not None and index == len(plan) - 1
            z = _local_fft(z, dim, inverse, last_scale if fold else 1.0)
            applied = applied or fold
            current[dim] = Axis(target)
        else:
            _, source, target, dim, _, group, split = item
            z = _dist_fft(z, group, dim, split, inverse=inverse, norm=per_axis_norm)
            current[dim] = Axis(target, out_by[target].shard_dim)
    return z, applied


def _run_complex_plan(z, current, out_by, plan, *, inverse, norm):
    total = math.prod(item[4] for item in plan)
    scale = _norm_scale(n=total, inverse=inverse, norm=norm)
    z, applied = _run_items(z, current, out_by, plan, inverse=inverse, per_axis_norm="forward" if inverse else None,
                            last_scale=scale)
    return z if applied or scale == 1.0 else z * scale


def _real_input_ok(x):
    return x.dtype in (torch.float32, torch.float64)


def _complex_dtype(dtype):
    return torch.complex128 if dtype in (torch.float64, torch.complex128) else torch.complex64


def _real_plan(x, tmap, in_by, out_by, in_axes, shapes, mesh, *, inverse, signal_sizes):
    half_src = next(reversed(tmap))
    half_dst = tmap[half_src]
    h_in, h_out = in_by[half_src], out_by[half_dst]
    if not inverse and not h_in.local() and not h_out.local() and h_in.shard_dim == h_out.shard_dim:
        if not _real_input_ok(x) or mesh is None:
            return None
        group = _group(mesh, h_in.shard_dim)
        full = resolve_split_shapes(shapes, h_in.shard_dim, h_in.name, group)
        P, r = dist.get_world_size(group), dist.get_rank(group)
        dim = _dim(in_axes, half_src)
        if full is None:
            full = [x.shape[dim]] * P
        if len(set(full)) != 1:
            return None
        local = full[r]
        if x.shape[dim] != local or local % P != 0:
            return None
        n = sum(full)
        half = resolve_split_shapes(shapes, h_out.shard_dim, h_out.name, group)
        if half is None or sum(half) != n // 2 + 1:
            return None
        rest = {s: t for s, t in tmap.items() if s != half_src}
        if any(out_by[t].shard_dim == h_out.shard_dim for t in rest.values()):
            return None
        rest_plan = []
        if rest:
            rest_plan = _complex_plan(x, rest, in_by, out_by, in_axes, shapes, mesh, require_complex=False)
            if rest_plan is None:
                return None
        return ("sharded_half_forward", half_src, half_dst, dim, n, group, full, half, rest_plan)
    if not h_in.local() or not h_out.local():
        return None
    if not inverse and not _real_input_ok(x):
        return None
    rest = {s: t for s, t in tmap.items() if s != half_src}
    if not rest:
        return None
    plan = _complex_plan(x, rest, in_by, out_by, in_axes, shapes, mesh, require_complex=False)
    if plan is None:
        return None
    if inverse and signal_sizes is not None:
        if not isinstance(signal_sizes, Mapping):
            return plan
        sizes = {item[1]: item[4] for item in plan}
        for s, t in rest.items():
            want = signal_sizes.get(t, signal_sizes.get(s))
            if want is None:
                continue
            if want != sizes.get(s, x.shape[_dim(in_axes, s)]):
                return None
    return plan


def _signal_sizes(tmap, current, x, signal_sizes):
    if signal_sizes is None:
        signal_sizes = {}
    elif not isinstance(signal_sizes, Mapping):
        raise TypeError("signal_sizes must be a mapping from axis names to sizes")
    out = [signal_sizes.get(t, signal_sizes.get(s)) for s, t in tmap.items()]
    names = list(tmap)
    if out[-1] is None:
        out[-1] = 2 * (x.shape[_dim(current, names[-1])] - 1)
    for i, size in enumerate(out):
        if size is None:
            out[i] = x.shape[_dim(current, names[i])]
    return tuple(out)


def _run_real_plan(z, current, out_by, tmap, plan, *, inverse, norm, signal_sizes):
    half_src = next(reversed(tmap))
    half_dst = tmap[half_src]
    if isinstance(plan, tuple) and plan[0] == "sharded_half_forward":
        _, _, _, hdim, n, group, full, half, rest_plan = plan
        total = n * math.prod(item[4] for item in rest_plan)
        z = z.to(_complex_dtype(z.dtype))
        z = _dist_fft(z, group, hdim, full, inverse=False, norm=None)
        z = _PrefixRepartition.apply(z, group, hdim, full, half)
        current[hdim] = Axis(half_dst, out_by[half_dst].shard_dim)
        z, _ = _run_items(z, current, out_by, rest_plan, inverse=False, per_axis_norm=None)
        return _normalize(z, n=total, inverse=False, norm=norm)
    sizes = _signal_sizes(tmap, current, z, signal_sizes) if inverse else None
    planned = {item[1]: item[4] for item in plan}
    total = math.prod(
        planned.get(s, sizes[i] if inverse else z.shape[_dim(current, s)]) for i, s in enumerate(tmap)
    )
    per_axis = "forward" if inverse else None
    if inverse:
        z, _ = _run_items(z, current, out_by, plan, inverse=True, per_axis_norm=per_axis)
        hdim = _dim(current, half_src)
        z = _irfft(z, sizes[-1], hdim)
        current[hdim] = Axis(half_dst)
    else:
        hdim = _dim(current, half_src)
        z = _rfft(z, hdim)
        current[hdim] = Axis(half_dst)
        z, _ = _run_items(z, current, out_by, plan, inverse=False, per_axis_norm=per_axis)
    return _normalize(z, n=total, inverse=inverse, norm=norm)


# ------------------------------------------------------------------ slab transpose path

def _slab_pairs(tmap, in_by, out_by):
    """(src, dst, mesh_dim) when the layout is a slab transpose between transform axes."""
    gathered = [(s, in_by[s].shard_dim) for s, t in tmap.items() if not in_by[s].local() and out_by[t].local()]
    scattered = [(s, out_by[t].shard_dim) for s, t in tmap.items() if in_by[s].local() and not out_by[t].local()]
    if len(gathered) != 1 or len(scattered) != 1 or gathered[0][1] != scattered[0][1]:
        return None
    dim = gathered[0][1]
    for name, axis in in_by.items():
        if name not in (gathered[0][0],) and not axis.local() and axis.shard_dim == dim:
            return None
    for name, axis in out_by.items():
        if name != tmap[scattered[0][0]] and not axis.local() and axis.shard_dim == dim:
            return None
    for s, t in tmap.items():
        if s in (gathered[0][0], scattered[0][0]):
            continue
        if not (in_by[s].local() and out_by[t].local()):
            return None
    return gathered[0][0], scattered[0][0], dim


def _slab_plan(x, tmap, in_by, out_by, in_axes, shapes, mesh):
    if mesh is None or not torch.is_complex(x):
        return None
    pair = _slab_pairs(tmap, in_by, out_by)
    if pair is None:
        return None
    src, dst, mdim = pair
    group = _group(mesh, mdim)
    P, r = dist.get_world_size(group), dist.get_rank(group)
    src_dim, dst_dim = _dim(in_axes, src), _dim(in_axes, dst)
    try:
        src_shapes = resolve_split_shapes(shapes, mdim, src, group)
        dst_shapes = resolve_split_shapes(shapes, mdim, tmap[dst], group) if isinstance(shapes, dict) else None
    except ValueError:
        return None
    if src_shapes is None:
        src_shapes = [x.shape[src_dim]] * P
    if x.shape[src_dim] != src_shapes[r]:
        return None
    if dst_shapes is None:
        from ..parallel.collectives import compute_split_shapes
        dst_shapes = compute_split_shapes(x.shape[dst_dim], P)
    if sum(dst_shapes) != x.shape[dst_dim]:
        return None
    return dict(src=src, dst=dst, group=group, src_dim=src_dim, dst_dim=dst_dim,
                src_shapes=src_shapes, dst_shapes=dst_shapes, n_src=sum(src_shapes))


def _run_slab(z, current, out_by, tmap, plan, *, inverse, norm):
    total = 1
    for s, t in tmap.items():
        if s == plan["src"]:
            total *= plan["n_src"]
        else:
            total *= z.shape[_dim(current, s)]
    fused = _run_slab_native(z, current, tmap, plan, inverse=inverse, scale=_norm_scale(n=total, inverse=inverse,
                                                                                        norm=norm))
    if fused is not None:
        for s, t in tmap.items():
            dim = _dim(current, s)
            current[dim] = Axis(t)
        dst_t = tmap[plan["dst"]]
        current[plan["dst_dim"]] = Axis(dst_t, out_by[dst_t].shard_dim)
        return fused
    # 1) transforms over every axis that is local on the input
    for s, t in tmap.items():
        if s == plan["src"]:
            continue
        dim = _dim(current, s)
        z = _local_fft(z, dim, inverse)
        current[dim] = Axis(t)
    # 2) slab transpose: gather src, scatter dst on the same mesh dim
    z = alltoall_repartition(z, plan["group"], plan["src_dim"], plan["dst_dim"], plan["src_shapes"], plan["dst_shapes"])
    dst_t = tmap[plan["dst"]]
    current[plan["dst_dim"]] = Axis(dst_t, out_by[dst_t].shard_dim)
    # 3) the remaining transform over the now-local src axis, normalisation folded in
    z = _local_fft(z, plan["src_dim"], inverse, _norm_scale(n=total, inverse=inverse, norm=norm))
    current[plan["src_dim"]] = Axis(tmap[plan["src"]])
    return z


def _run_slab_native(z, current, tmap, plan, *, inverse, scale):
    """The slab pipeline on the native kernels: local FFTs, then the all-to-all
    fused into the loads of the FFT along the gathered axis (peer memory over
    NVLink).  ``None`` when the native path does not cover the call."""
    if not z.is_cuda or z.dtype != torch.complex64:
        return None
    P = len(plan["src_shapes"])
    if len(set(plan["src_shapes"])) != 1 or len(set(plan["dst_shapes"])) != 1:
        return None
    from ..parallel import symmetric
    from . import fft_impl
    comm = symmetric.workspace_for(plan["group"], z.numel() * z.element_size())
    pre = [_dim(current, s) for s in tmap if s != plan["src"]]
    if not fft_impl.slab_eligible(z, comm, plan["src_dim"], plan["dst_dim"], P, pre, ()):
        return None
    return fft_impl.slab_fft(z, comm, P, dist.get_rank(plan["group"]), pre_dims=pre, gather_dim=plan["src_dim"],
                             split_dim=plan["dst_dim"], inverse=inverse, scale=scale)


# ------------------------------------------------------------------ diagnostics

def _path_name(fast, *, real):
    if fast is None:
        return "fallback"
    if isinstance(fast, dict):
        return "distributed-fftn-slab"
    if real and isinstance(fast, tuple) and fast[0] == "sharded_half_forward":
        return "distributed-rfft-sharded-half"
    return "distributed-rfft-local-half" if real else "distributed-fftn"


def _fallback_reason(x, tmap, in_by, out_by, in_axes, shapes, mesh, *, real, inverse, signal_sizes):
    if real:
        half_src = next(reversed(tmap))
        h_in, h_out = in_by[half_src], out_by[tmap[half_src]]
        if not inverse and not _real_input_ok(x):
            return "forward real FFT fast path requires float32 or float64 input"
        if inverse and (not h_in.local() or not h_out.local()):
            return "inverse real FFT with a sharded half-spectrum axis is not optimized yet"
        if h_in.local() != h_out.local():
            return "real FFT half-spectrum axis must be local on both sides or sharded on the same mesh dimension"
        if not h_in.local() and h_in.shard_dim != h_out.shard_dim:
            return "real FFT half-spectrum axis must stay on the same mesh dimension"
        if inverse and signal_sizes is not None and isinstance(signal_sizes, Mapping):
            for s, t in list(tmap.items())[:-1]:
                want = signal_sizes.get(t, signal_sizes.get(s))
                if want is None:
                    continue
                dim = _dim(in_axes, s)
                have = None
                if in_by[s].local():
                    have = x.shape[dim]
                elif mesh is not None:
                    axis = in_by[s]
                    group = _group(mesh, axis.shard_dim)
                    split = resolve_split_shapes(shapes, axis.shard_dim, axis.name, group)
                    have = sum(split) if split is not None else x.shape[dim] * dist.get_world_size(group)
                if have is not None and want != have:
                    return "inverse real FFT non-half-axis signal_sizes request padding or cropping"
    if mesh is None and any(not in_by[s].local() or not out_by[t].local() for s, t in tmap.items()):
        return "distributed FFT layouts require mesh"
    if not real and not torch.is_complex(x):
        return "complex FFT fast path requires complex input"
    for s, t in tmap.items():
        a, b = in_by[s], out_by[t]
        if not a.local() and b.local():
            return "sharded transform axes must stay sharded for the fast path"
        if a.local() and not b.local():
            return "local transform axes cannot become sharded in the fast path"
        if not a.local() and a.shard_dim != b.shard_dim:
            return "sharded transform axes must stay on the same mesh dimension"
        if not a.local() and mesh is not None:
            group = _group(mesh, a.shard_dim)
            split = resolve_split_shapes(shapes, a.shard_dim, a.name, group)
            if split is not None:
                if len(set(split)) != 1:
                    return "fast path requires equal shard sizes"
                if split[dist.get_rank(group)] % dist.get_world_size(group) != 0:
                    return "fast path requires local shard size divisible by mesh size"
    return "layout is not supported by an optimized FFT path"


def _shared_dim_reason(tmap, in_by, out_by):
    for s, t in tmap.items():
        axis = in_by[s] if not in_by[s].local() else out_by[t]
        if not axis.local():
            for name, other in in_by.items():
                if name != s and not other.local() and other.shard_dim == axis.shard_dim:
                    return _SHARED_DIM_REASON
        out_axis = out_by[t]
        if out_axis.local():
            continue
        for name, other in out_by.items():
            if name != t and not other.local() and other.shard_dim == out_axis.shard_dim:
                return _SHARED_DIM_REASON
    return None


def _warn_fallback():
    warnings.warn(
        "einfft is using the gather/FFT/split fallback for a sharded transform axis; "
        "this is correct but materializes the full transform axis on every rank.",
        RuntimeWarning,
        stacklevel=3,
    )


# ------------------------------------------------------------------ entry point

def einfft(shard, x, axes, *, inverse=False, norm=None, mesh=None, shapes=None, families=None, real=False,
           signal_sizes=None, explain=False):
    """Named-axis FFT with sharding-aware fast paths and a gather/split fallback."""
    shard, _ = cached_expand_axis_families(shard, families=families)
    tmap = _transform_map(_expand_axes_arg(axes, families))
    in_spec, other, out_spec = parse_sharding(shard)
    if other is not None:
        raise ValueError("einfft expects a unary sharding expression")
    in_names = _spec_names(in_spec, label="input")
    out_names = _spec_names(out_spec, label="output")
    if len(in_names) != x.dim():
        raise ValueError("Input tensor rank does not match the input spec")
    if len(in_names) != len(out_names):
        raise ValueError("Input and output specs must have the same rank")

    if not tmap:
        if sorted(in_names) != sorted(out_names):
            raise ValueError("Output axes must match input axes when no FFT axes are requested")
        if explain:
            noop = [a.name for a in _axes(in_spec)] == out_names and _axes(in_spec) == _axes(out_spec)
            return {
                "fast_path": False,
                "path": "no-op-layout" if noop else "layout-only",
                "reason": "no transform axes requested" if noop else
                "no transform axes requested; only layout changes would run",
                "axes": {},
            }
        return distributed_1d((in_spec, None, out_spec), x, mesh=mesh, shapes=shapes)

    for s, t in tmap.items():
        if s not in in_names:
            raise ValueError(f"FFT source axis {s!r} is not present in the input")
        if t not in out_names:
            raise ValueError(f"FFT output axis {t!r} is not present in the output")
    if len(set(tmap)) != len(tmap):
        raise ValueError("FFT source axes must be distinct")
    if len(set(tmap.values())) != len(tmap):
        raise ValueError("FFT output axes must be distinct")
    if sorted(tmap.get(n, n) for n in in_names) != sorted(out_names):
        raise ValueError("Output axes must match input axes with FFT axes renamed")
    in_by = {a.name: a for a in _axes(in_spec)}
    out_by = {a.name: a for a in _axes(out_spec)}
    for name in in_names:
        if name not in tmap and in_by[name] != out_by[name]:
            raise ValueError("einfft output must preserve non-FFT axis sharding")

    current = Axes(Axis(a.name, a.shard_dim) for a in _axes(in_spec))
    z = x
    slab = None if real else _slab_plan(z, tmap, in_by, out_by, current, shapes, mesh)
    if slab is None:
        reason = _shared_dim_reason(tmap, in_by, out_by)
        if reason is not None:
            if explain:
                return {"fast_path": False, "path": "unsupported-layout", "reason": reason, "axes": dict(tmap)}
            raise NotImplementedError(reason)

    if slab is not None:
        fast = slab
    elif real:
        fast = _real_plan(z, tmap, in_by, out_by, current, shapes, mesh, inverse=inverse, signal_sizes=signal_sizes)
    else:
        fast = _complex_plan(z, tmap, in_by, out_by, current, shapes, mesh)

    if fast is not None:
        if explain:
            return {"fast_path": True, "path": _path_name(fast, real=real), "reason": None, "axes": dict(tmap)}
        if isinstance(fast, dict):
            z = _run_slab(z, current, out_by, tmap, fast, inverse=inverse, norm=norm)
        elif real:
            z = _run_real_plan(z, current, out_by, tmap, fast, inverse=inverse, norm=norm, signal_sizes=signal_sizes)
        else:
            z = _run_complex_plan(z, current, out_by, fast, inverse=inverse, norm=norm)
        if [a.name for a in current] == out_names and current == _axes(out_spec):
            return z
        return distributed_1d((TensorSpec(current), None, out_spec), z, mesh=mesh, shapes=shapes)

    if explain:
        return {
            "fast_path": False,
            "path": "fallback",
            "reason": _fallback_reason(z, tmap, in_by, out_by, current, shapes, mesh, real=real, inverse=inverse,
                                       signal_sizes=signal_sizes),
            "axes": dict(tmap),
        }
    if any(not in_by[s].local() or (real and not out_by[t].local()) for s, t in tmap.items()):
        _warn_fallback()
    dims = []
    for s in tmap:
        dim = _dim(current, s)
        dims.append(dim)
        axis = current[dim]
        if axis.local():
            continue
        if mesh is None:
            raise ValueError("Distributed einfft operations require mesh")
        group = _group(mesh, axis.shard_dim)
        z = allgather_forward_split_backward(z, group, dim,
                                             resolve_split_shapes(shapes, axis.shard_dim, axis.name, group))
        current[dim] = Axis(axis.name)
    if real:
        if inverse:
            z = torch.fft.irfftn(z, s=_signal_sizes(tmap, current, z, signal_sizes), dim=tuple(dims), norm=norm)
        else:
            z = torch.fft.rfftn(z, dim=tuple(dims), norm=norm)
    else:
        total = math.prod(z.shape[d] for d in dims)
        scale = _norm_scale(n=total, inverse=inverse, norm=norm)
        for k, d in enumerate(dims):
            z = _local_fft(z, d, inverse, scale if k == len(dims) - 1 else 1.0)
    for s, t in tmap.items():
        dim = _dim(current, s)
        out_axis = out_by[t]
        current[dim] = Axis(t)
        if out_axis.local():
            continue
        if mesh is None:
            raise ValueError("Distributed einfft operations require mesh")
        group = _group(mesh, out_axis.shard_dim)
        z = split_forward_allgather_backward(z, group, dim,
                                             resolve_split_shapes(shapes, out_axis.shard_dim, out_axis.name, group))
        current[dim] = Axis(t, out_axis.shard_dim)
    if [a.name for a in current] == out_names and current == _axes(out_spec):
        return z
    return distributed_1d((TensorSpec(current), None, out_spec), z, mesh=mesh, shapes=shapes)
