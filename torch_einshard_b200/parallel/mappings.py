"""Autograd-paired collectives: the planner's primitive vocabulary.

Each primitive is a forward collective whose backward is its adjoint
(all-reduce <-> identity, all-gather <-> split or reduce-scatter, repartition
<-> inverse repartition, ...).  Names and pairings are the reference's
(``src/torch_einshard/mappings.py:1-200``); plan steps refer to them by the
wrapper function names below.
"""

import torch
import torch.distributed as dist

from . import collectives as C

__all__ = [
    "allreduce_forward_identity_backward",
    "identity_forward_allreduce_backward",
    "broadcast_forward_allreduce_backward",
    "allgather_forward_split_backward",
    "split_forward_allgather_backward",
    "reducescatter_forward_allgather_backward",
    "allgather_forward_reducescatter_backward",
    "alltoall_repartition",
    "owner_swap_forward_backward",
    "roll_shards_forward_backward",
    "roll_sharded_forward_backward",
]


class _AllReduceFwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        return C.all_reduce(x, group)

    @staticmethod
    def backward(ctx, g):
        return g, None


class _AllReduceBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        return C.all_reduce(g, ctx.group), None


class _Broadcast(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, src):
        ctx.group, ctx.src = group, src
        return C.broadcast(x, group, src)

    @staticmethod
    def backward(ctx, g):
        grad = C.all_reduce(g, ctx.group)
        if dist.get_rank(ctx.group) != ctx.src:
            grad = torch.zeros_like(grad)
        return grad, None, None


class _GatherSplit(torch.autograd.Function):
    """all-gather forward, split backward."""

    @staticmethod
    def forward(ctx, x, group, dim, shapes):
        ctx.args = (group, dim, shapes)
        return C.all_gather(x, group, dim, shapes)

    @staticmethod
    def backward(ctx, g):
        return C.split(g, *ctx.args), None, None, None


class _SplitGather(torch.autograd.Function):
    """split forward, all-gather backward."""

    @staticmethod
    def forward(ctx, x, group, dim, shapes):
        ctx.args = (group, dim, shapes)
        return C.split(x, group, dim, shapes)

    @staticmethod
    def backward(ctx, g):
        return C.all_gather(g, *ctx.args), None, None, None


class _ScatterGather(torch.autograd.Function):
    """reduce-scatter forward, all-gather backward."""

    @staticmethod
    def forward(ctx, x, group, dim, shapes):
        ctx.args = (group, dim, shapes)
        return C.reduce_scatter(x, group, dim, shapes)

    @staticmethod
    def backward(ctx, g):
        return C.all_gather(g, *ctx.args), None, None, None


class _GatherScatter(torch.autograd.Function):
    """all-gather forward, reduce-scatter backward."""

    @staticmethod
    def forward(ctx, x, group, dim, shapes):
        ctx.args = (group, dim, shapes)
        return C.all_gather(x, group, dim, shapes)

    @staticmethod
    def backward(ctx, g):
        return C.reduce_scatter(g, *ctx.args), None, None, None


class _Repartition(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, source_dim, dest_dim, source_shapes, dest_shapes):
        ctx.args = (group, dest_dim, source_dim, dest_shapes, source_shapes)
        return C.all_to_all_repartition(x, group, source_dim, dest_dim, source_shapes, dest_shapes)

    @staticmethod
    def backward(ctx, g):
        return (C.all_to_all_repartition(g, *ctx.args),) + (None,) * 5


class _OwnerSwap(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mesh, source_shard_dims, dest_shard_dims, output_shape):
        ctx.args = (mesh, dest_shard_dims, source_shard_dims, tuple(x.shape))
        return C.owner_swap(x, mesh, source_shard_dims, dest_shard_dims, output_shape)

    @staticmethod
    def backward(ctx, g):
        return (C.owner_swap(g, *ctx.args),) + (None,) * 5


class _RollShards(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, shard_shift):
        ctx.group, ctx.shift = group, shard_shift
        return C.roll_shards(x, group, shard_shift)

    @staticmethod
    def backward(ctx, g):
        return C.roll_shards(g, ctx.group, -ctx.shift), None, None


class _RollSharded(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim, shift, shapes):
        ctx.args = (group, dim, shift, shapes)
        return C.roll_sharded(x, group, dim, shift, shapes)

    @staticmethod
    def backward(ctx, g):
        group, dim, shift, shapes = ctx.args
        return C.roll_sharded(g, group, dim, -shift, shapes), None, None, None, None


def allreduce_forward_identity_backward(input, comm):
    return _AllReduceFwd.apply(input, comm)


def identity_forward_allreduce_backward(input, comm):
    return _AllReduceBwd.apply(input, comm)


def broadcast_forward_allreduce_backward(input, comm, src=0):
    return _Broadcast.apply(input, comm, src)


def allgather_forward_split_backward(input, comm, dim, shapes):
    return _GatherSplit.apply(input, comm, dim, shapes)


def split_forward_allgather_backward(input, comm, dim, shapes):
    return _SplitGather.apply(input, comm, dim, shapes)


def reducescatter_forward_allgather_backward(input, comm, dim, shapes):
    return _ScatterGather.apply(input, comm, dim, shapes)


def allgather_forward_reducescatter_backward(input, comm, dim, shapes):
    return _GatherScatter.apply(input, comm, dim, shapes)


def alltoall_repartition(input, comm, source_dim, dest_dim, source_shapes, dest_shapes):
    return _Repartition.apply(input, comm, source_dim, dest_dim, source_shapes, dest_shapes)


def owner_swap_forward_backward(input, mesh, source_shard_dims, dest_shard_dims, output_shape):
    return _OwnerSwap.apply(input, mesh, source_shard_dims, dest_shard_dims, output_shape)


def roll_shards_forward_backward(input, comm, shard_shift):
    return _RollShards.apply(input, comm, shard_shift)


def roll_sharded_forward_backward(input, comm, dim, shift, shapes):
    return _RollSharded.apply(input, comm, dim, shift, shapes)
