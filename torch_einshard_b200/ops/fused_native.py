"""Fused contraction + collective paths of the binary executor.

``provider(executor)`` inspects a binary plan while the native communicators
are active (``setup_native_comm``) and returns a fusion descriptor when one of
the patterns below applies (CUDA bf16 operands, a native communicator for the
group); otherwise ``None`` and the executor runs the unfused steps.  Fuses the
planner steps ``rank_local_einsum`` + ``allreduce_forward_identity_backward`` /
``reducescatter_forward_allgather_backward`` and
``allgather_forward_reducescatter_backward`` + ``rank_local_einsum``
(``src/torch_einshard/mappings.py:169-187``,
``src/torch_einshard/distributed.py:84-620``):

* ``gemm_allreduce``  - forward ``AR(A @ B)`` runs as one launch: the wide
  tcgen05 GEMM writes its output units into the symmetric heap and reducer
  clusters of the same launch sum each unit in the NVSwitch as soon as every
  rank produced it (``csrc/gemm_nvls.cu``; on heaps without multicast, the
  older epilogue kernels ``csrc/gemm_ar.cu`` / ``gemm_push.cu`` on request).
  Backward needs no communication (the all-reduce's adjoint is the identity):
  ``dA = dC @ B^T`` and ``dB = A^T @ dC`` on the plain native GEMM.
* ``dgrad_allreduce`` - forward is the plain GEMM; in backward the gradient of
  the replicated operand, which must be all-reduced over the group, is
  computed by the same fused kernel.
* ``gemm_reducescatter`` / ``allgather_gemm`` - the row reduce-scatter epilogue
  and the all-gather fused into the GEMM's operand loads (``csrc/gemm_ag.cu``).

All apply to two-operand contractions that canonicalise to a single
(batch-free) GEMM of CUDA bf16 tensors.

Fuses the reference's ``mappings.py:169-187`` collectives with the contraction
of ``einsum.py:132``.
"""

import torch
import torch.distributed as dist

from . import _native
from .contraction import canonical_gemm
from .einsum import equation_for
from .gemm import _prepare, native_bmm

__all__ = ["install", "gemm_allreduce", "gemm_reducescatter", "gemm_allgather"]


def _comm(group):
    from ..parallel import symmetric
    return symmetric.communicator_for(group)


def gemm_allreduce(comm, a, b):
    """``sum over ranks of a @ b`` for a: [1, M, K], b: [1, K, N] (bf16)."""
    mod = _native.require()
    a, b = _prepare(a), _prepare(b)
    out = torch.empty((1, a.shape[1], b.shape[2]), dtype=torch.bfloat16, device=a.device)
    comm.enter("copy")
    mod.gemm_allreduce(comm.cid, a, b, out, _native.error_word(a.device))
    return out


def gemm_allreduce_push(comm, a, b):
    """``sum over ranks of a @ b`` with the push-model fused kernel (wide GEMM;
    partials and reduced tiles cross NVLink as stores)."""
    mod = _native.require()
    a, b = _prepare(a), _prepare(b)
    out = torch.empty((1, a.shape[1], b.shape[2]), dtype=torch.bfloat16, device=a.device)
    comm.enter("copy")
    mod.gemm_allreduce_push(comm.cid, a, b, out, _native.error_word(a.device))
    return out


def _push_fits(comm, m, n):
    mod = _native.module()
    return (mod is not None and hasattr(mod, "gemm_allreduce_push")
            and mod.gemm_push_region_bytes(m, n, comm.size) <= comm.capacity
            and -(-m // 128) * -(-n // 256) <= 120000)


def gemm_reducescatter(comm, a, b, seg, shard):
    """This rank's rows of the reduce-scatter of ``a @ b`` over the ranks: rows are
    segments of ``seg`` rows, rank p keeps rows [p*shard, (p+1)*shard) of each."""
    mod = _native.require()
    a, b = _prepare(a), _prepare(b)
    out = torch.empty((1, a.shape[1] // comm.size, b.shape[2]), dtype=torch.bfloat16, device=a.device)
    comm.enter("copy")
    mod.gemm_reducescatter(comm.cid, a, b, out, seg, shard, _native.error_word(a.device))
    return out


def gemm_allgather(comm, a_local, b, seg, shard):
    """``(gather_rows(a_local) @ b, gathered a)`` in one kernel: copy warps of the
    GEMM pull peers' row shards over NVLink while the tensor cores run."""
    mod = _native.require()
    a_local = a_local.contiguous()
    b = _prepare(b)
    rows = a_local.shape[1] * comm.size
    xfull = torch.empty((1, rows, a_local.shape[2]), dtype=torch.bfloat16, device=a_local.device)
    out = torch.empty((1, rows, b.shape[2]), dtype=torch.bfloat16, device=a_local.device)
    comm.enter("copy")
    mod.gemm_allgather(comm.cid, a_local, b, out, xfull, seg, shard, _native.error_word(a_local.device))
    return out, xfull


def _ag_fits(comm, a_local, seg, shard):
    rows = a_local.shape[1] * comm.size
    return (a_local.dtype == torch.bfloat16 and shard % 256 == 0 and (a_local.shape[2] * 2) % 16 == 0
            and a_local.numel() * 2 <= comm.capacity and rows // 128 <= 21000 and a_local.shape[1] % shard == 0)


def _gather_rows(comm, x, seg, shard):
    """Inverse layout of the row reduce-scatter: [1, M/P, N] -> [1, M, N]."""
    m_local, n = x.shape[1], x.shape[2]
    segments = m_local // shard
    view = x.reshape(segments, shard, n)
    full = comm.all_gather(view, 1, [shard] * comm.size)
    if full is None:
        parts = [torch.empty_like(view) for _ in range(comm.size)]
        dist.all_gather(parts, view.contiguous(), group=comm.group)
        full = torch.cat(parts, dim=1)
    return full.reshape(1, segments * seg, n)


def _scatter_rows(comm, full, seg, shard):
    """Row reduce-scatter of an unfused [1, M, N] tensor (fallback)."""
    m, n = full.shape[1], full.shape[2]
    view = full.reshape(m // seg, seg, n)
    out = comm.reduce_scatter(view, 1, [shard] * comm.size)
    if out is None:
        dist.all_reduce(view, group=comm.group)
        out = view[:, comm.rank * shard:(comm.rank + 1) * shard].contiguous()
    return out.reshape(1, (m // seg) * shard, n)


def _rs_fits(comm, m, n, seg, shard):
    return _fits(comm, m, n) and seg % 128 == 0 and shard % 128 == 0 and shard * comm.size == seg and m % seg == 0


class _GemmReduceScatter(torch.autograd.Function):
    """Forward: rows of RS(a @ b) in one kernel.  Backward: gather dC, then the
    plain GEMMs (the reduce-scatter's adjoint is the all-gather)."""

    @staticmethod
    def forward(ctx, a, b, comm, seg, shard):
        ctx.save_for_backward(a, b)
        ctx.args = (comm, seg, shard)
        return _reducescatter(comm, a, b, seg, shard)

    @staticmethod
    def backward(ctx, grad):
        a, b = ctx.saved_tensors
        comm, seg, shard = ctx.args
        full = _gather_rows(comm, grad.contiguous(), seg, shard)
        ga = native_bmm(full, b.transpose(1, 2)) if ctx.needs_input_grad[0] else None
        gb = _grad_b(a, b, full) if ctx.needs_input_grad[1] else None
        return ga, gb, None, None, None


class _AllGatherGemm(torch.autograd.Function):
    """Forward: gather the row-sharded operand a, then the GEMM.  Backward: the
    gradient of the local rows is the row reduce-scatter of dC @ b^T, computed
    by the fused GEMM + reduce-scatter kernel; db uses the gathered a."""

    @staticmethod
    def forward(ctx, a_local, b, comm, seg, shard):
        from ..parallel import symmetric
        ws = symmetric.workspace_for(comm.group, a_local.numel() * a_local.element_size())
        if ws is not None and _ag_fits(ws, a_local, seg, shard):
            comm = ws
            out, a_full = gemm_allgather(comm, a_local, b, seg, shard)
        else:
            a_full = _gather_rows(comm, a_local.contiguous(), seg, shard)
            out = native_bmm(a_full, b)
        ctx.save_for_backward(a_full, b)
        ctx.args = (comm, seg, shard)
        return out

    @staticmethod
    def backward(ctx, grad):
        a_full, b = ctx.saved_tensors
        comm, seg, shard = ctx.args
        ga = gb = None
        if ctx.needs_input_grad[0]:
            ga = _reducescatter(comm, grad, b.transpose(1, 2), seg, shard)
        if ctx.needs_input_grad[1]:
            gb = _grad_b(a_full, b, grad)
        return ga, gb, None, None, None


def _fits(comm, m, n):
    tiles = -(-m // 128) * -(-n // 256)
    return tiles * 128 * 256 * 2 <= comm.capacity and tiles <= 120000


def gemm_allreduce_nvls(comm, a, b):
    """``sum over ranks of a @ b`` on every rank, one launch: the wide GEMM
    writes its output units into the symmetric heap and reducer clusters of the
    same launch sum each unit through the NVSwitch as soon as every rank has
    produced it (``csrc/gemm_nvls.cu``).  None when the group has no NVLS heap."""
    from ..parallel import symmetric
    m, n = a.shape[1], b.shape[2]
    ws = symmetric.workspace_for(comm.group, m * n * 2)
    if ws is None or not ws.nvls or ws.broken:
        return None
    mod = _native.require()
    a, b = _prepare(a), _prepare(b)
    out = torch.empty((1, m, n), dtype=torch.bfloat16, device=a.device)
    ws.enter("tile")
    mod.gemm_allreduce_nvls(ws.cid, a, b, out, _NVLS_REDUCER_CLUSTERS, _NVLS_LAG,
                            _native.error_word(a.device))
    return out


def gemm_reducescatter_nvls(comm, a, b, seg, shard):
    """This rank's row segments of ``sum over ranks of a @ b`` in one launch:
    the wide GEMM writes its output units into the symmetric heap and each
    unit's owner (the rank whose rows it holds) sums it in the NVSwitch and
    stores it into its output.  None when the group has no NVLS heap."""
    from ..parallel import symmetric
    m, n = a.shape[1], b.shape[2]
    ws = symmetric.workspace_for(comm.group, m * n * 2)
    if ws is None or not ws.nvls or ws.broken:
        return None
    mod = _native.require()
    a, b = _prepare(a), _prepare(b)
    out = torch.empty((1, m // comm.size, n), dtype=torch.bfloat16, device=a.device)
    ws.enter("tile")
    mod.gemm_reducescatter_nvls(ws.cid, a, b, out, seg, shard, _NVLS_REDUCER_CLUSTERS, _NVLS_LAG,
                                _native.error_word(a.device))
    return out


def _nvls_rs_fits(comm, a, b, seg, shard):
    return (_nvls_fits(comm, a, b) and seg > 0 and shard % 32 == 0 and shard * comm.size == seg
            and a.shape[1] % seg == 0)


def _reducescatter(comm, a, b, seg, shard):
    """Row reduce-scatter of a @ b: the fused NVLS kernel, else the older fused
    epilogue, else the GEMM followed by the collective."""
    if _nvls_rs_fits(comm, a, b, seg, shard):
        out = gemm_reducescatter_nvls(comm, a, b, seg, shard)
        if out is not None:
            return out
    if _fusable(comm, _MAX_FUSED_EPILOGUE_RANKS) and _rs_fits(comm, a.shape[1], b.shape[2], seg, shard):
        return gemm_reducescatter(comm, a, b, seg, shard)
    return _scatter_rows(comm, native_bmm(a, b), seg, shard)


def _nvls_fits(comm, a, b):
    m, n = a.shape[1], b.shape[2]
    tiles = -(-m // 256) * -(-n // 512)
    return (comm.nvls and _FUSED_NVLS and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and a.shape[0] == 1
            and n % 8 == 0 and tiles * 16 <= 120000)


def _ar_or_fallback(comm, a, b):
    if _nvls_fits(comm, a, b):
        out = gemm_allreduce_nvls(comm, a, b)
        if out is not None:
            return out
    if _fusable(comm, _MAX_FUSED_EPILOGUE_RANKS):
        if _push_fits(comm, a.shape[1], b.shape[2]):
            return gemm_allreduce_push(comm, a, b)
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


def gemm_allreduce_overlapped(a, b, group, chunks, gemm_into):
    """out = all_reduce(a @ b) with the rows in ``chunks`` pieces: piece i's
    all-reduce (``torch.distributed``, asynchronous) runs while piece i + 1's
    GEMM runs, so the collective overlaps the contraction without a fused
    kernel.  ``gemm_into(a_rows, b, out_rows)`` computes one piece in place.
    Pieces are whole multiples of 256 rows (one wide-kernel tile row)."""
    m, n = a.shape[1], b.shape[2]
    out = torch.empty(a.shape[0], m, n, dtype=a.dtype, device=a.device)
    step = -(-m // max(1, chunks))
    step = -(-step // 256) * 256
    works = []
    for lo in range(0, m, step):
        hi = min(m, lo + step)
        piece = out[:, lo:hi]
        gemm_into(a[:, lo:hi], b, piece)
        works.append(dist.all_reduce(piece, group=group, async_op=True))
    for work in works:
        work.wait()
    return out


def _native_gemm_into(a, b, out):
    _native.require().gemm_out(_prepare(a), _prepare(b), out, 0, _native.error_word(a.device))


class _GemmAllReduceOverlap(torch.autograd.Function):
    """Row-parallel contraction whose all-reduce overlaps the GEMM in row
    pieces (forward); backward is the plain GEMM pair (the all-reduce's
    adjoint is the identity)."""

    @staticmethod
    def forward(ctx, a, b, group, chunks):
        ctx.save_for_backward(a, b)
        return gemm_allreduce_overlapped(a, b, group, chunks, _native_gemm_into)

    @staticmethod
    def backward(ctx, grad):
        a, b = ctx.saved_tensors
        ga = native_bmm(grad, b.transpose(1, 2)) if ctx.needs_input_grad[0] else None
        gb = _grad_b(a, b, grad) if ctx.needs_input_grad[1] else None
        return ga, gb, None, None


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
    def __init__(self, kind, operand=None, axis=None, overlap_chunks=0):
        self.kind = kind
        self.operand = operand
        self.axis = axis  # gathered / scattered axis name
        self.overlap_chunks = overlap_chunks  # gemm_allreduce: > 1 row pieces on torch.distributed, no fused kernel

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

    @staticmethod
    def _row_segment(shard, x, y, name, P):
        """(views, seg, shard_rows) when ``name`` is a GEMM row axis whose blocks
        per rank are whole row ranges of the flattened rows; else None."""
        views = _Fusion._gemm_views(shard, x, y)
        if views is None:
            return None
        equation = equation_for(shard)
        plan = canonical_gemm(equation, tuple(x.shape), tuple(y.shape))
        ez = plan["ez"]
        out_axes = [a for a in shard[2].axes]
        letter = ez[[a.name for a in out_axes].index(name)]
        rows, size = plan["rows"], plan["size"]
        if letter not in rows or size[letter] % P:
            return None
        seg = 1
        for c in rows[rows.index(letter):]:
            seg *= size[c]
        return views, seg, seg // P, letter, plan

    def run_gemm_reducescatter(self, shard, x, y, group, name):
        comm = _comm(group)
        found = self._row_segment(shard, x, y, name, comm.size) if comm is not None else None
        if found is None:
            return None
        (a, b, shape, perm), seg, rows_per_rank, letter, plan = found
        out = _GemmReduceScatter.apply(a, b, comm, seg, rows_per_rank)
        order = plan["rows"] + plan["cols"]
        shape = list(shape)
        shape[order.index(letter)] //= comm.size
        return out.reshape(shape).permute(perm)

    def run_allgather_gemm(self, shard, x_local, y, group, name, dim):
        """Operand ``self.operand`` is sharded along ``name`` (tensor dim ``dim``)."""
        comm = _comm(group)
        if comm is None:
            return None
        P = comm.size
        # plan against the gathered shapes
        full_shape = list((x_local if self.operand == 0 else y).shape)
        full_shape[dim] *= P
        xs = torch.empty(full_shape, device="meta", dtype=x_local.dtype) if self.operand == 0 else x_local
        ys = y if self.operand == 0 else torch.empty(full_shape, device="meta", dtype=y.dtype)
        found = self._row_segment_input(shard, xs, ys, name, P)
        if found is None:
            return None
        a_perm, b_perm, m, n, k, seg, rows_per_rank, shape, perm = found
        if self.operand == 0:
            a_local = x_local.permute(a_perm).reshape(1, m // P, k)
            b = y.permute(b_perm).reshape(1, k, n)
        else:
            return None
        out = _AllGatherGemm.apply(a_local, b, comm, seg, rows_per_rank)
        return out.reshape(shape).permute(perm)

    @staticmethod
    def _row_segment_input(shard, x, y, name, P):
        equation = equation_for(shard)
        plan = canonical_gemm(equation, tuple(x.shape), tuple(y.shape))
        if plan is None or plan["batch"] or plan["x_only"] or plan["y_only"]:
            return None
        ex, ey, ez = plan["ex"], plan["ey"], plan["ez"]
        rows, cols, red, size = plan["rows"], plan["cols"], plan["red"], plan["size"]
        in_axes = [a.name for a in shard[0].axes]
        letter = ex[in_axes.index(name)]
        if letter not in rows or size[letter] % P or rows[0] != letter and False:
            return None
        # the local rows must be whole blocks: every row axis before `letter` is outer
        seg = 1
        for c in rows[rows.index(letter):]:
            seg *= size[c]
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
        a_perm = [ex.index(c) for c in rows + red]
        b_perm = [ey.index(c) for c in red + cols]
        order = rows + cols
        shape = [size[c] for c in order]
        perm = [order.index(c) for c in ez]
        return a_perm, b_perm, m, n, k, seg, seg // P, shape, perm

    def run_gemm_allreduce(self, shard, x, y, group):
        views = self._gemm_views(shard, x, y)
        comm = _comm(group)
        if views is None or (comm is None and self.overlap_chunks <= 1):
            from .einsum import einsum
            from ..parallel.mappings import allreduce_forward_identity_backward
            return allreduce_forward_identity_backward(einsum(shard, x, y), group)
        a, b, shape, perm = views
        if self.overlap_chunks > 1:
            out = _GemmAllReduceOverlap.apply(a, b, group, self.overlap_chunks)
        else:
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


# Measured on B200 (CUDA events, max over ranks), TP-MLP shapes, before the NVLS
# kernel: GEMM + all-reduce, 2 ranks: fused pull epilogue 7.64 ms, fused push
# epilogue 7.51 ms, wide GEMM + NCCL all-reduce 6.16 ms; 8 ranks: fused 31.5 ms,
# GEMM + NCCL 2.6 ms (those epilogues hold the wide kernel's single accumulator
# while tiles cross NVLink).  all-gather + GEMM, 2 ranks: fused (copy warps
# inside the GEMM) 5.48 ms, NCCL all-gather + GEMM 6.12 ms, GEMM alone 5.20 ms.
# So the GEMM + all-reduce runs as the NVLS kernel (gemm_nvls.cu: the partial
# leaves TMEM through the heap, reducer clusters sum it in the switch) wherever
# the group's heap has a multicast mapping; the older epilogue kernels only on
# request (EINSHARD_FUSED_EPILOGUE_MAX_RANKS), and the fused all-gather runs for
# groups up to the size it was measured at.
import os

_FUSED_NVLS = os.environ.get("EINSHARD_FUSED_NVLS", "1") not in ("0", "")
# Who reduces in the fused launch: 0 = the GEMM's own epilogue warps, while
# later tiles' mainloops run (overlap mode, every SM computes); n > 0 = n CTA
# pairs at the front of the launch that only reduce and copy out.  _NVLS_LAG:
# overlap mode's distance in tiles between a tile and its reduction (0: two
# waves of resident CTA pairs).
_NVLS_REDUCER_CLUSTERS = int(os.environ.get("EINSHARD_NVLS_REDUCER_CLUSTERS", "0"))
_NVLS_LAG = int(os.environ.get("EINSHARD_NVLS_LAG", "0"))
_MAX_FUSED_EPILOGUE_RANKS = int(os.environ.get("EINSHARD_FUSED_EPILOGUE_MAX_RANKS", "0"))
_MAX_FUSED_GATHER_RANKS = int(os.environ.get("EINSHARD_FUSED_GATHER_MAX_RANKS", "2"))
# Row-parallel all-reduce overlapped with the GEMM in this many row pieces (0: off,
# the default): piece i's NCCL all-reduce runs while piece i + 1's GEMM runs.
_OVERLAP_AR_CHUNKS = int(os.environ.get("EINSHARD_OVERLAP_AR_CHUNKS", "0"))


def _nvls_comm(comm):
    return comm is not None and comm.nvls and _FUSED_NVLS and not comm.broken


def _fusable(comm, limit):
    return comm is not None and 2 <= comm.size <= limit


def _eligible_tensors(executor):
    x, y = executor.x0, executor.y0
    return x.is_cuda and y.is_cuda and x.dtype == torch.bfloat16 and y.dtype == torch.bfloat16


def provider(executor):
    """Fusion descriptor for a binary executor, or None."""
    if executor.post is not None or not _eligible_tensors(executor):
        return None
    tp = executor.tp
    out_steps = [s for s in tp.output_steps if s.name != "rank_local_einsum"]
    if (len(out_steps) == 1 and out_steps[0].name == "reducescatter_forward_allgather_backward"
            and not tp.input0_steps and not tp.input1_steps):
        name, dim = out_steps[0].args
        comm = _comm(executor.group(dim))
        if _nvls_comm(comm) or _fusable(comm, _MAX_FUSED_EPILOGUE_RANKS):
            return _Fusion("gemm_reducescatter", axis=name)
        return None
    if (not out_steps and len(tp.input0_steps) == 1 and not tp.input1_steps
            and tp.input0_steps[0].name == "allgather_forward_reducescatter_backward"):
        name, dim = tp.input0_steps[0].args
        if _fusable(_comm(executor.group(dim)), _MAX_FUSED_GATHER_RANKS):
            return _Fusion("allgather_gemm", operand=0, axis=name)
        return None
    if (len(out_steps) == 1 and out_steps[0].name == "allreduce_forward_identity_backward"
            and not tp.input0_steps and not tp.input1_steps):
        group = executor.group(out_steps[0].args[0])
        comm = _comm(group)
        if _nvls_comm(comm) or _fusable(comm, _MAX_FUSED_EPILOGUE_RANKS):
            return _Fusion("gemm_allreduce")
        if _OVERLAP_AR_CHUNKS > 1 and dist.get_world_size(group) > 1:
            return _Fusion("gemm_allreduce", overlap_chunks=_OVERLAP_AR_CHUNKS)
        return None
    if out_steps:
        return None
    in0, in1 = tp.input0_steps, tp.input1_steps
    for operand, (mine, other) in enumerate(((in0, in1), (in1, in0))):
        if len(mine) == 1 and not other and mine[0].name == "identity_forward_allreduce_backward":
            comm = _comm(executor.group(mine[0].args[0]))
            if _nvls_comm(comm) or _fusable(comm, _MAX_FUSED_EPILOGUE_RANKS):
                return _Fusion("dgrad_allreduce", operand)
    return None

