"""Collective helpers behind every autograd mapping (the "comm backend").

Public functions keep the reference helper contract
(``src/torch_einshard/helpers.py:5-361``): ``all_reduce`` returns a new tensor,
``all_gather``/``reduce_scatter``/``split`` accept uneven per-rank ``shapes``,
``all_to_all_repartition`` and ``roll_sharded`` return ``None`` when the split
metadata does not match the tensor, and ``owner_swap`` exchanges whole blocks
between mesh coordinates.

Backend choice, per call: CUDA tensors on a group that has a native
communicator (peer-mapped symmetric buffers over NVLink, see
:mod:`.symmetric`) run the sm_100a copy/reduce kernels; everything else
(CPU/gloo, groups without peer access, oversize messages) runs through
``torch.distributed``.  Both paths compute the same values.
"""

import os

import torch
import torch.distributed as dist

__all__ = [
    "init_process_group",
    "all_reduce",
    "broadcast",
    "split",
    "all_gather",
    "reduce_scatter",
    "all_to_all_repartition",
    "owner_swap",
    "roll_shards",
    "roll_sharded",
    "resolve_split_shapes",
    "compute_split_shapes",
    "compute_split_shapes_for_factors",
    "split_offsets",
]


def init_process_group(backend, use_cuda):
    """Initialise ``torch.distributed`` from SLURM or torchrun variables.

    Returns ``(local_rank, world_rank, world_size)``.
    """
    if "SLURM_NTASKS" in os.environ:
        world_size = int(os.getenv("SLURM_NTASKS", 1))
        world_rank = int(os.getenv("SLURM_PROCID", 0))
    else:
        world_size = int(os.getenv("WORLD_SIZE", 1))
        world_rank = int(os.getenv("RANK", 0))
    dist.init_process_group(backend=backend, rank=world_rank, world_size=world_size)
    if not use_cuda:
        local_rank = 0
    elif "LOCAL_RANK" in os.environ:
        local_rank = int(os.getenv("LOCAL_RANK"))
    else:
        local_rank = world_rank % torch.cuda.device_count()
    return local_rank, world_rank, world_size


def _native(group, tensor):
    if not tensor.is_cuda:
        return None
    from . import symmetric
    return symmetric.communicator_for(group)


def split_offsets(shapes):
    offsets, total = [], 0
    for size in shapes:
        offsets.append(total)
        total += size
    return offsets


def all_reduce(input, group, *, async_op=False):
    output = input.contiguous().clone()
    comm = None if async_op else _native(group, output)
    if comm is not None and comm.all_reduce_(output):
        return output
    work = dist.all_reduce(output, group=group, async_op=async_op)
    if async_op:
        return output, work
    return output


def broadcast(input, group, src=0):
    output = input.contiguous().clone()
    comm = _native(group, output)
    if comm is not None and comm.broadcast_(output, src):
        return output
    dist.broadcast(output, dist.get_global_rank(group, src), group=group)
    return output


def split(input, group, dim, shapes):
    """This rank's slice of ``input`` along ``dim`` (no communication)."""
    size = dist.get_world_size(group)
    if size == 1:
        return input
    if shapes is None:
        shapes = compute_split_shapes(input.shape[dim], size)
    rank = dist.get_rank(group)
    return input.narrow(dim, sum(shapes[:rank]), shapes[rank]).contiguous()


def all_gather(input, group, dim, shapes):
    """Concatenate every rank's shard along ``dim`` (uneven ``shapes`` allowed)."""
    size = dist.get_world_size(group)
    if shapes is not None and len(shapes) != size:
        raise ValueError(f"Error: passed shapes of size {len(shapes)} not equal to {size}")
    if dim >= input.dim():
        raise ValueError(f"Error: Gathering along {dim} for a tensor of size {input.dim()}")
    if size == 1:
        return input
    input = input.contiguous()
    rank = dist.get_rank(group)
    if shapes is not None and input.shape[dim] != shapes[rank]:
        raise ValueError(
            f"Error: local tensor size {input.shape[dim]} does not match shapes[{rank}] = {shapes[rank]}"
        )
    if shapes is None:
        shapes = [input.shape[dim]] * size
    comm = _native(group, input)
    if comm is not None:
        out = comm.all_gather(input, dim, shapes)
        if out is not None:
            return out
    if len(set(shapes)) != 1:
        # pad every shard to the largest one, gather, then drop the padding
        padded_shape = list(input.shape)
        padded_shape[dim] = max(shapes)
        padded = input.new_zeros(padded_shape)
        padded.narrow(dim, 0, input.shape[dim]).copy_(input)
        pieces = [torch.empty_like(padded) for _ in range(size)]
        dist.all_gather(pieces, padded, group=group)
        return torch.cat([piece.narrow(dim, 0, shapes[src]) for src, piece in enumerate(pieces)], dim=dim).contiguous()
    pieces = [torch.empty_like(input) for _ in range(size)]
    dist.all_gather(pieces, input, group=group)
    return torch.cat(pieces, dim=dim).contiguous()


def reduce_scatter(input, group, dim, shapes):
    """Sum over ranks, then keep this rank's slice along ``dim``."""
    size = dist.get_world_size(group)
    if size == 1:
        return input
    if shapes is None:
        shapes = compute_split_shapes(input.shape[dim], size)
    if len(shapes) != size:
        raise ValueError(f"Error: passed shapes of size {len(shapes)} not equal to {size}")
    comm = _native(group, input)
    if comm is not None and input.shape[dim] == sum(shapes):
        out = comm.reduce_scatter(input.contiguous(), dim, shapes)
        if out is not None:
            return out
    if len(set(shapes)) != 1:
        return split(all_reduce(input, group), group, dim, shapes)
    chunk = shapes[0]
    if input.shape[dim] != chunk * size:
        raise ValueError(
            f"Error: tensor size {input.shape[dim]} along dim {dim} does not match reduce_scatter shapes {shapes}"
        )
    moved = input.movedim(dim, 0).contiguous()
    output = moved.new_empty((chunk, *moved.shape[1:]))
    dist.reduce_scatter_tensor(output, moved, group=group)
    return output.movedim(0, dim).contiguous()


def all_to_all_repartition(input, group, source_dim, dest_dim, source_shapes, dest_shapes):
    """Gather ``source_dim`` while scattering ``dest_dim`` in one exchange.

    Returns ``None`` when split metadata is missing or inconsistent.
    """
    size = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if size == 1:
        return input
    if source_shapes is None or dest_shapes is None:
        return None
    if input.shape[source_dim] != source_shapes[rank] or input.shape[dest_dim] != sum(dest_shapes):
        return None
    comm = _native(group, input)
    if comm is not None:
        out = comm.all_to_all(input, source_dim, dest_dim, source_shapes, dest_shapes)
        if out is not None:
            return out
    src_off = split_offsets(source_shapes)
    dst_off = split_offsets(dest_shapes)
    out_shape = list(input.shape)
    out_shape[source_dim] = sum(source_shapes)
    out_shape[dest_dim] = dest_shapes[rank]
    output = input.new_empty(out_shape)
    ops, landing = [], []
    for peer in range(size):
        outgoing = input.narrow(dest_dim, dst_off[peer], dest_shapes[peer]).contiguous()
        target = output.narrow(source_dim, src_off[peer], source_shapes[peer])
        if peer == rank:
            target.copy_(outgoing)
            continue
        peer_global = dist.get_global_rank(group, peer)
        incoming = torch.empty_like(target)
        ops.append(dist.P2POp(dist.isend, outgoing, peer_global, group))
        ops.append(dist.P2POp(dist.irecv, incoming, peer_global, group))
        landing.append((incoming, target))
    for request in dist.batch_isend_irecv(ops):
        request.wait()
    for incoming, target in landing:
        target.copy_(incoming)
    return output.contiguous()


def _swap_partners(mesh, source_shard_dims, dest_shard_dims):
    device_mesh = getattr(mesh, "device_mesh", mesh)
    grid = device_mesh.mesh
    index = {name: i for i, name in enumerate(device_mesh.mesh_dim_names)}
    me = dist.get_rank()
    coord = (grid == me).nonzero()[0].tolist()
    send, recv = list(coord), list(coord)
    pairs = [(index[s], index[d]) for s, d in zip(source_shard_dims, dest_shard_dims)]
    if set(source_shard_dims) == set(dest_shard_dims):
        # a permutation of mesh dims: block at coord moves to the permuted coordinate
        for s, d in pairs:
            send[d] = coord[s]
            recv[s] = coord[d]
    else:
        for s, d in pairs:
            send[s], send[d] = coord[d], coord[s]
            recv[s], recv[d] = coord[d], coord[s]
    return me, int(grid[tuple(send)].item()), int(grid[tuple(recv)].item())


def owner_swap(input, mesh, source_shard_dims, dest_shard_dims, output_shape):
    """Move this rank's block to the rank that owns it after the mesh-dim swap."""
    me, send_rank, recv_rank = _swap_partners(mesh, source_shard_dims, dest_shard_dims)
    if send_rank == me and recv_rank == me:
        return input.contiguous()
    output = input.new_empty(output_shape)
    from . import symmetric
    comm = symmetric.world_communicator() if input.is_cuda else None
    if comm is not None and comm.send_recv(input.contiguous(), send_rank, output, recv_rank):
        return output
    ops = [
        dist.P2POp(dist.isend, input.contiguous(), send_rank),
        dist.P2POp(dist.irecv, output, recv_rank),
    ]
    for request in dist.batch_isend_irecv(ops):
        request.wait()
    return output.contiguous()


def roll_shards(input, group, shard_shift):
    """Shift whole shards by ``shard_shift`` ranks (cyclic)."""
    size = dist.get_world_size(group)
    if size == 1 or shard_shift % size == 0:
        return input
    rank = dist.get_rank(group)
    to_peer = dist.get_global_rank(group, (rank + shard_shift) % size)
    from_peer = dist.get_global_rank(group, (rank - shard_shift) % size)
    output = torch.empty_like(input)
    ops = [
        dist.P2POp(dist.isend, input.contiguous(), to_peer, group),
        dist.P2POp(dist.irecv, output, from_peer, group),
    ]
    for request in dist.batch_isend_irecv(ops):
        request.wait()
    return output


def roll_intervals(shapes, shift):
    """For every source rank, the ``(src_start, length, dst_rank, dst_start)`` pieces.

    Rolling a sharded axis by ``shift`` moves each element ``g`` to
    ``(g + shift) % total``; a source shard maps onto at most a few contiguous
    destination intervals.
    """
    total = sum(shapes)
    offsets = split_offsets(shapes)
    ends = [o + s for o, s in zip(offsets, shapes)]

    def owner(g):
        for r, end in enumerate(ends):
            if g < end:
                return r
        return len(shapes) - 1

    table = []
    for src, size in enumerate(shapes):
        pieces, start = [], 0
        while start < size:
            dst_global = (offsets[src] + start + shift) % total
            dst = owner(dst_global)
            length = min(size - start, ends[dst] - dst_global)
            if length == 0:
                break
            pieces.append((start, length, dst, dst_global - offsets[dst]))
            start += length
        table.append(pieces)
    return table


def roll_sharded(input, group, dim, shift, shapes):
    """Roll a sharded axis by exchanging exactly the crossing intervals."""
    size = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if shapes is None or len(shapes) != size:
        return None
    total = sum(shapes)
    shift = shift % total
    if size == 1:
        from ..ops.native_ops import local_roll
        return local_roll(input, {dim % input.dim(): shift})
    if shift == 0:
        return input
    if input.shape[dim] != shapes[rank]:
        return None
    table = roll_intervals(shapes, shift)
    comm = _native(group, input)
    if comm is not None:
        out = comm.interval_exchange(input, dim, table, shapes)
        if out is not None:
            return out
    output = torch.empty_like(input)
    ops, landing = [], []
    for start, length, dst, _ in table[rank]:
        if dst != rank:
            ops.append(dist.P2POp(dist.isend, input.narrow(dim, start, length).contiguous(),
                                  dist.get_global_rank(group, dst), group))
    for src in range(size):
        for start, length, dst, dst_start in table[src]:
            if dst != rank:
                continue
            target = output.narrow(dim, dst_start, length)
            if src == rank:
                target.copy_(input.narrow(dim, start, length))
                continue
            incoming = torch.empty_like(target)
            ops.append(dist.P2POp(dist.irecv, incoming, dist.get_global_rank(group, src), group))
            landing.append((incoming, target))
    for request in dist.batch_isend_irecv(ops):
        request.wait()
    for incoming, target in landing:
        target.copy_(incoming)
    return output.contiguous()


def resolve_split_shapes(shapes, shard_dim, axis_name, group=None):
    """Pick per-rank sizes from a list, ``{mesh_dim: list}`` or ``{mesh_dim: {axis: list}}``."""
    if shapes is None:
        return None
    if isinstance(shapes, dict):
        if shard_dim not in shapes:
            raise ValueError(f"Missing split shapes for mesh dimension {shard_dim!r}")
        shapes = shapes[shard_dim]
        if isinstance(shapes, dict):
            if axis_name not in shapes:
                raise ValueError(f"Missing split shapes for axis {axis_name!r} on mesh dimension {shard_dim!r}")
            shapes = shapes[axis_name]
    if group is not None:
        size = dist.get_world_size(group)
        if len(shapes) != size:
            raise ValueError(f"Error: passed shapes of size {len(shapes)} not equal to {size}")
    return shapes


def compute_split_shapes(size, num_chunks):
    """Balanced split: ceil-sized chunks, falling back to floor if the last would be empty."""
    if num_chunks == 1:
        return [size]
    chunk = -(-size // num_chunks)
    last = max(0, size - chunk * (num_chunks - 1))
    if last == 0:
        chunk = size // num_chunks
        last = size - chunk * (num_chunks - 1)
    return [chunk] * (num_chunks - 1) + [last]


def compute_split_shapes_for_factors(size, num_chunks, factor):
    """Split in whole multiples of ``factor``; the remainder goes to the last rank."""
    sections = compute_split_shapes(size // factor, num_chunks)
    if factor == 1:
        return sections
    sections = [s * factor for s in sections]
    sections[-1] += size % factor
    return sections
