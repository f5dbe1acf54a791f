"""Native fused contraction + all-reduce paths (installed by ``setup_native_comm``).

Provides the fusion descriptors consumed by :mod:`.fused`:

* ``gemm_allreduce``  - forward ``AR(A @ B)`` runs as one kernel: the tcgen05
  GEMM tiles are reduced over NVLink as they finish (``csrc/gemm_ar.cu``).
  Backward needs no communication (the all-reduce's adjoint is the identity):
  ``dA = dC @ B^T`` and ``dB = A^T @ dC`` on the plain native GEMM.
* ``dgrad_allreduce`` - forward is the plain GEMM; in backward the gradient of
  the replicated operand, which must be all-reduced over the group, is
  computed by the fused kernel.

Both apply to two-operand contractions that canonicalise to a single
(batch-free) GEMM of CUDA bf16 tensors whose output fits the symmetric buffer.
"""

import torch
import torch.distributed as dist

from . import _native, fused
from .contraction import canonical_gemm
from .einsum import equation_for
from .gemm import _prepare, native_bmm

__all__ = ["install", "gemm_allreduce"]


def _comm(group):
    from ..parallel import native_comm
    return native_comm.communicator_for(group)


def gemm_allreduce(comm, a, b):
    """``sum over ranks of a @ b`` for a: [1, M, K], b: [1, K, N] (bf16)."""
    mod = _native.require()
    a, b = _prepare(a), _prepare(b)
    out = torch.empty((1, a.shape[1], b.shape[2]), dtype=torch.bfloat16, device=a.device)
    mod.gemm_allreduce(comm.cid, a, b, out, _native.error_word(a.device))
    return out


def _fits(comm, m, n):
    tiles = -(-m // 128) * -(-n // 256)
    return tiles * 128 * 256 * 2 <= comm.capacity and tiles <= 120000


def _ar_or_fallback(comm, a, b):
    if _fits(comm, a.shape[1], b.shape[2]):
        return gemm_allreduce(comm, a, b)
    out = native_bmm(a, b)
    if not comm.all_reduce_(out):
        dist.all_reduce(out, group=comm.group)
    return out


def _grad_b(a, b, grad):
    if b.stride(1) == 1 and b.size(1) > 1:
        return native_bmm(grad.transpose(1, 2), a).transpose(1, 2)
    return native_bmm(a.transpose(1, 2), grad)


class _GemmAllReduce(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, comm):
        ctx.save_for_backward(a, b)
        return _ar_or_fallback(comm, a, b)

    @staticmethod
    def backward(ctx, grad):
        a, b = ctx.saved_tensors
        ga = native_bmm(grad, b.transpose(1, 2)) if ctx.needs_input_grad[0] else None
        gb = _grad_b(a, b, grad) if ctx.needs_input_grad[1] else None
        return ga, gb, None


class _GemmDgradAllReduce(torch.autograd.Function):
    """Plain GEMM forward; the replicated operand's gradient is all-reduced in backward."""

    @staticmethod
    def forward(ctx, a, b, comm, operand):
        ctx.save_for_backward(a, b)
        ctx.comm, ctx.operand = comm, operand
        return native_bmm(a, b)

    @staticmethod
    def backward(ctx, grad):
        a, b = ctx.saved_tensors
        comm, operand = ctx.comm, ctx.operand
        ga = gb = None
        if ctx.needs_input_grad[0]:
            ga = _ar_or_fallback(comm, grad, b.transpose(1, 2)) if operand == 0 else native_bmm(grad, b.transpose(1, 2))
        if ctx.needs_input_grad[1]:
            if operand == 1:
                gb = _ar_or_fallback(comm, a.transpose(1, 2), grad)
            else:
                gb = _grad_b(a, b, grad)
        return ga, gb, None, None


class _Fusion:
    def __init__(self, kind, operand=None):
        self.kind = kind
        self.operand = operand

    @staticmethod
    def _gemm_views(shard, x, y):
        equation = equation_for(shard)
        plan = canonical_gemm(equation, tuple(x.shape), tuple(y.shape))
        if plan is None or plan["batch"] or plan["x_only"] or plan["y_only"]:
            return None
        size = plan["size"]
        ex, ey, ez = plan["ex"], plan["ey"], plan["ez"]
        rows, cols, red = plan["rows"], plan["cols"], plan["red"]
        m = 1
        for c in rows:
            m *= size[c]
        n = 1
        for c in cols:
            n *= size[c]
        k = 1
        for c in red:
            k *= size[c]
        if min(m, n, k) == 0:
            return None
        a = x.permute([ex.index(c) for c in rows + red]).reshape(1, m, k)
        b = y.permute([ey.index(c) for c in red + cols]).reshape(1, k, n)
        order = rows + cols
        shape = [size[c] for c in order]
        perm = [order.index(c) for c in ez]
        return a, b, shape, perm

    def run_gemm_allreduce(self, shard, x, y, group):
        views = self._gemm_views(shard, x, y)
        comm = _comm(group)
        if views is None or comm is None:
            from .einsum import einsum
            from ..parallel.mappings import allreduce_forward_identity_backward
            return allreduce_forward_identity_backward(einsum(shard, x, y), group)
        a, b, shape, perm = views
        out = _GemmAllReduce.apply(a, b, comm)
        return out.reshape(shape).permute(perm)

    def run_dgrad_allreduce(self, shard, x, y, group):
        views = self._gemm_views(shard, x, y)
        comm = _comm(group)
        if views is None or comm is None:
            from .einsum import einsum
            from ..parallel.mappings import identity_forward_allreduce_backward
            if self.operand == 0:
                x = identity_forward_allreduce_backward(x, group)
            else:
                y = identity_forward_allreduce_backward(y, group)
            return einsum(shard, x, y)
        a, b, shape, perm = views
        out = _GemmDgradAllReduce.apply(a, b, comm, self.operand)
        return out.reshape(shape).permute(perm)


def _eligible_tensors(executor):
    x, y = executor.x0, executor.y0
    return x.is_cuda and y.is_cuda and x.dtype == torch.bfloat16 and y.dtype == torch.bfloat16


def provider(executor):
    """Fusion descriptor for a binary executor, or None."""
    if executor.post is not None or not _eligible_tensors(executor):
        return None
    tp = executor.tp
    out_steps = [s for s in tp.output_steps if s.name != "rank_local_einsum"]
    if (len(out_steps) == 1 and out_steps[0].name == "allreduce_forward_identity_backward"
            and not tp.input0_steps and not tp.input1_steps):
        if _comm(executor.group(out_steps[0].args[0])) is not None:
            return _Fusion("gemm_allreduce")
        return None
    if out_steps:
        return None
    in0, in1 = tp.input0_steps, tp.input1_steps
    for operand, (mine, other) in enumerate(((in0, in1), (in1, in0))):
        if len(mine) == 1 and not other and mine[0].name == "identity_forward_allreduce_backward":
            if _comm(executor.group(mine[0].args[0])) is not None:
                return _Fusion("dgrad_allreduce", operand)
    return None


def install():
    fused.register_fusion_provider(provider)
