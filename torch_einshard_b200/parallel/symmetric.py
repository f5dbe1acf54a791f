"""Native NVLink communicators built on a symmetric device heap.

``activate(mesh)`` creates one :class:`Communicator` per process group of the
mesh (and the world group).  Its heap (``csrc/symm.cpp``) is one ``cuMemCreate``
allocation per rank, shared with the group's other processes as a POSIX file
descriptor over a Unix socket and mapped by every rank, plus, where the
devices support it, an NVLS multicast object bound over all of them.  The heap
is created in phases with an agreement (all-reduce of a status) after each, so
every rank either has the communicator or none has.  The default data capacity
is ``EINSHARD_SYMM_MB`` (64 MiB); collectives that need more ask
:func:`workspace_for_group`, which grows one extra heap per group on demand.

Collectives: with multicast, all-reduce, all-gather(v) and reduce-scatter(v)
run through the NVSwitch (``csrc/nvls.cu``: multimem loads that sum in the
switch, multicast stores); the remaining data movement (uneven boxes,
all-to-all, halo and roll intervals) runs as single kernels that stage the
local input in the heap and pull strided boxes from peers (``csrc/comm.cu``).
Every operation is described on the host, so uneven shards and arbitrary
dimensions need no pack/unpack copies.

A communicator is only created for groups whose ranks all live on this node
and whose devices can access each other; otherwise the collective helpers use
``torch.distributed`` (NCCL).  Set ``EINSHARD_NATIVE_COMM=0`` to disable, and
``EINSHARD_NVLS=0`` to create heaps without multicast.

Native backend of the reference's collective helpers: all_reduce
``src/torch_einshard/helpers.py:27``, broadcast ``:35``, all_gather ``:61``,
reduce_scatter ``:114``, all_to_all_repartition ``:142``, owner_swap ``:184``,
roll ``:224-309``.
"""

import atexit
import os
import socket
import uuid
import warnings

import torch
import torch.distributed as dist

from ..ops import _native

__all__ = ["Communicator", "activate", "deactivate", "communicator_for_group", "communicator_for", "workspace_for",
           "world_communicator", "enabled", "disable", "setup_native_comm", "teardown_native_comm"]

_DEFAULT_MB = int(os.environ.get("EINSHARD_SYMM_MB", "64"))
# Block count of every NVLS collective on a heap (the per-block counters are
# shared by all collectives of the heap, so it is fixed when the heap is made);
# 0: two per SM, which keeps enough 16-byte loads and multimem operations in
# flight to reach the link rate (32 blocks measured 150 GB/s for a 512 MiB
# all-reduce on 2 ranks, a third of NCCL).
_NVLS_BLOCKS = int(os.environ.get("EINSHARD_NVLS_BLOCKS", "0"))
# A two-shot NVLS all-reduce moves N (1 + 1/P) bytes over each GPU's links
# against 2 N (P - 1) / P for a ring: more at P = 2, less from P = 4 on.  Below
# this group size, all-reduces of _NCCL_AR_MIN_BYTES and more go to NCCL.
_NVLS_AR_MIN_RANKS = int(os.environ.get("EINSHARD_NVLS_AR_MIN_RANKS", "4"))
_NVLS = os.environ.get("EINSHARD_NVLS", "1") not in ("0", "")
# Without multicast: 512 MiB all-reduce at 8 ranks on B200, the two-shot copy
# kernel 2.19 ms, NCCL 1.34 ms; NCCL takes the buffers of this size and more.
_NCCL_AR_MIN_BYTES = int(os.environ.get("EINSHARD_NCCL_AR_MIN_BYTES", str(1 << 20)))
# NVLS all-reduce: every rank reduces everything (one launch, one flag round)
# below this size; above it each rank reduces 1/P and multicasts it (two-shot).
_NVLS_ONE_SHOT_MAX = int(os.environ.get("EINSHARD_NVLS_ONE_SHOT_MAX", str(256 << 10)))
# Largest heap an all-reduce grows to; longer tensors run in pieces of it.
_NVLS_AR_PIECE = int(os.environ.get("EINSHARD_NVLS_AR_PIECE_MB", "256")) << 20
# native all-reduce kernel without multicast: "push" (every NVLink transfer a
# store into a peer's region) or "pull" (peers' chunks read over NVLink)
_AR_ALGO = os.environ.get("EINSHARD_AR_ALGO", "push")
_COMMS = {}
_REJECTED = set()
_LARGE = {}  # group key -> the group's on-demand larger communicator


def _agree(group, ok):
    """True when ``ok`` holds on every rank of ``group`` (a collective)."""
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


def _unique_tag(group):
    tag = [f"{os.getpid():x}-{uuid.uuid4().hex[:16]}" if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(tag, src=dist.get_global_rank(group, 0), group=group)
    return tag[0]


def _nvls_blocks(group, device):
    """The heap's NVLS block count, the same on every rank (minimum over ranks)."""
    want = _NVLS_BLOCKS or 2 * torch.cuda.get_device_properties(device).multi_processor_count
    t = torch.tensor([min(1024, max(1, want))], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return int(t.item())


def _create_heap(mod, group, data_bytes, device, want_mc):
    """Collective creation of a heap communicator; its id, or None when any
    rank failed (then no rank keeps one)."""
    rank, size = dist.get_rank(group), dist.get_world_size(group)
    blocks = _nvls_blocks(group, device)
    tag = _unique_tag(group)
    cid, err = mod.symm_prepare(int(data_bytes), device, tag, rank, size, bool(want_mc), blocks)
    phases = (lambda: mod.symm_exchange(cid, 120.0), lambda: mod.symm_bind(cid), lambda: mod.symm_finish(cid))
    errors = [err]
    ok = _agree(group, err == "")
    for phase in phases:
        if not ok:
            break
        err = phase()
        errors.append(err)
        ok = _agree(group, err == "")
    if ok:
        return cid
    mine = "; ".join(e for e in errors if e)
    warnings.warn(f"einshard: symmetric heap ({'with' if want_mc else 'without'} multicast) not created"
                  + (f": {mine}" if mine else " (a peer failed)"), RuntimeWarning, stacklevel=3)
    torch.cuda.synchronize()
    mod.comm_destroy(cid)
    return None


def _contig_strides(shape):
    strides, acc = [], 1
    for size in reversed(shape):
        strides.append(acc)
        acc *= size
    return list(reversed(strides))


def make_box(shape, src_strides, src_off, dst_strides, dst_off, src_rank, esize):
    """4-D copy box (bytes) for an element-wise copy over ``shape``; None if not expressible."""
    dims = [(n, s, d) for n, s, d in zip(shape, src_strides, dst_strides) if n != 1]
    if any(n == 0 for n in shape):
        return "empty"
    merged = []
    for n, s, d in dims:
        if merged and merged[-1][1] == s * n and merged[-1][2] == d * n:
            prev = merged.pop()
            merged.append((prev[0] * n, s, d))
        else:
            merged.append((n, s, d))
    if not merged:
        merged = [(1, 1, 1)]
    if merged[-1][1] != 1 or merged[-1][2] != 1:
        merged.append((1, 1, 1))
    if len(merged) > 4:
        return None
    while len(merged) < 4:
        merged.insert(0, (1, 0, 0))
    sizes = tuple(n for n, _, _ in merged)
    sstr = tuple(s * esize for _, s, _ in merged[:3])
    dstr = tuple(d * esize for _, _, d in merged[:3])
    return (src_rank, sizes, src_off * esize, dst_off * esize, sstr, dstr)


def _view_geometry(view, base):
    return view.storage_offset() - base.storage_offset(), list(view.stride())


def _sent_pieces(table, src):
    """The halo pieces rank ``src`` sends, in packing order (by destination,
    then table order): (dst, (out_off, src, src_off, n))."""
    return [(dst, piece) for dst, pieces in enumerate(table) for piece in pieces if piece[1] == src and dst != src]


def halo_gather_plan(rank, x_shape, dim, table, length, esize):
    """Host plan of ``Communicator.halo_gather`` on rank ``rank``: the slabs
    (offset, rows along ``dim``) it packs into its staged buffer, the copy
    boxes that build its haloed shard (rank -1: from the local input; a peer:
    from that peer's packed buffer) and the haloed shape.  Every rank derives
    every peer's packing from the same table, so no offsets are exchanged."""
    out_shape = list(x_shape)
    out_shape[dim] = length
    out_strides = _contig_strides(out_shape)
    x_strides = _contig_strides(list(x_shape))
    send = [(piece[2], piece[3]) for _, piece in _sent_pieces(table, rank)]
    boxes = []
    for out_off, src, src_off, n in table[rank]:
        shape = list(x_shape)
        shape[dim] = n
        if src == rank:
            boxes.append(make_box(shape, x_strides, src_off * x_strides[dim], out_strides, out_off * out_strides[dim],
                                  -1, esize))
            continue
        packed = _sent_pieces(table, src)
        before = 0
        for dst, piece in packed:
            if dst == rank and piece == (out_off, src, src_off, n):
                break
            before += piece[3]
        packed_shape = list(x_shape)
        packed_shape[dim] = sum(piece[3] for _, piece in packed)
        pstrides = _contig_strides(packed_shape)
        boxes.append(make_box(shape, pstrides, before * pstrides[dim], out_strides, out_off * out_strides[dim], src,
                              esize))
    return send, boxes, out_shape


def halo_ghost_plan(rank, x_shape, dim, table, length, esize):
    """Plan of ``Communicator.halo_ghosts``: only the rows this rank's haloed
    shard takes from peers, as one tensor G whose first ``gtop`` rows (along
    ``dim``) lie above the shard and the other ``gbot`` below it.  Returns
    (send, boxes, G shape, gtop, gbot), or None when the shard's own rows are
    not exactly one piece (a periodic halo wider than the group)."""
    pieces = table[rank]
    own = [i for i, p in enumerate(pieces) if p[1] == rank]
    if len(own) != 1:
        return None
    k = own[0]
    local_n = pieces[k][3]
    mine = [(p[0] if i < k else p[0] - local_n, p[1], p[2], p[3]) for i, p in enumerate(pieces) if i != k]
    gtop = sum(p[3] for p in pieces[:k])
    gbot = sum(p[3] for p in pieces[k + 1:])
    # only this rank's entry changes: every peer packs from its own unchanged
    # table in the same order, so the packed offsets agree
    ghost_table = list(table)
    ghost_table[rank] = mine
    send, boxes, g_shape = halo_gather_plan(rank, x_shape, dim, ghost_table, length - local_n, esize)
    return send, boxes, g_shape, gtop, gbot


def halo_scatter_plan(rank, size, grad_shape, dim, table, in_shape, esize):
    """Host plan of ``Communicator.halo_scatter_add`` on rank ``rank``: the
    ghost slabs of its gradient (offset, rows) it packs and returns to their
    owners, and the accumulate boxes: its own rows from the local gradient
    (rank -1), the rows peers return from their packed buffers."""
    in_strides = _contig_strides(list(in_shape))
    g_strides = _contig_strides(list(grad_shape))

    def returns(q):
        return [p for p in table[q] if p[1] != q]

    send = [(p[0], p[3]) for p in returns(rank)]
    boxes = []
    for out_off, src, src_off, n in table[rank]:
        if src != rank:
            continue
        shape = list(in_shape)
        shape[dim] = n
        boxes.append(make_box(shape, g_strides, out_off * g_strides[dim], in_strides, src_off * in_strides[dim], -1,
                              esize))
    for q in range(size):
        if q == rank:
            continue
        packed = returns(q)
        packed_shape = list(in_shape)
        packed_shape[dim] = sum(p[3] for p in packed)
        pstrides = _contig_strides(packed_shape)
        before = 0
        for out_off, src, src_off, n in packed:
            if src == rank:
                shape = list(in_shape)
                shape[dim] = n
                boxes.append(make_box(shape, pstrides, before * pstrides[dim], in_strides, src_off * in_strides[dim],
                                      q, esize))
            before += n
    return send, boxes


class Communicator:
    def __init__(self, group, data_bytes):
        self.mod = _native.require()
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.device = torch.cuda.current_device()
        self.err = _native.error_word(self.device)
        want_mc = _agree(group, _NVLS and self.mod.symm_multicast_supported(self.device))
        cid = _create_heap(self.mod, group, data_bytes, self.device, want_mc)
        if cid is None and want_mc:
            cid = _create_heap(self.mod, group, data_bytes, self.device, False)
        if cid is None:
            raise RuntimeError("einshard: the symmetric heap could not be created")
        self.cid = cid
        self.nvls = bool(self.mod.comm_has_multicast(cid))
        self.capacity = int(self.mod.comm_data_bytes(cid))
        self.sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self._broken = False
        self.closed = False

    @property
    def broken(self):
        """A communicator that saw a timed-out wait, or whose heap was freed,
        declines every collective (the callers fall back to torch.distributed)."""
        return self._broken or self.closed

    @broken.setter
    def broken(self, value):
        self._broken = bool(value)

    def close(self):
        """Free the heap.  Collective: every rank of the group calls it, after
        its last use (a device synchronisation and a barrier come first)."""
        if self.closed:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.mod.comm_destroy(self.cid)
        self.closed = True

    # -- raw access for fused kernels ----------------------------------------
    @property
    def id(self):
        return self.cid

    @property
    def data_bytes(self):
        return self.capacity

    def enter(self, kind):
        """Order this heap between the protocols that use its data region:
        "copy" (the staged copy kernels, the older fused GEMM kernels and direct
        region writes; per-rank epoch flags), "nvls" (the NVLS collectives;
        per-block counters) and "tile" (the fused GEMM + NVLS all-reduce; per-unit
        epochs).  When the kind changes, a stream-ordered wait makes sure every
        rank finished the previous kind's accesses to this rank's heap: peers'
        reads of a copy op (their done flags), every block of the last NVLS
        collective (its counters).  A fused GEMM + all-reduce needs none: when
        it ends on this rank, no peer touches this rank's heap for it any more."""
        last = getattr(self, "_last_kind", None)
        if last is not None and last != kind:
            if last == "copy":
                self.mod.comm_acquire(self.cid, self.err)
            elif last == "nvls":
                self.mod.nvls_quiesce(self.cid, self.err)
        self._last_kind = kind

    def acquire(self):
        """Stream-ordered wait until every peer finished reading this rank's
        region for the previous op; writes into ``region()`` must follow it."""
        self.enter("copy")
        self.mod.comm_acquire(self.cid, self.err)

    def region(self, nbytes):
        """This rank's symmetric data region (first ``nbytes``) as uint8."""
        return self.mod.comm_region(self.cid, int(nbytes))

    # -- helpers -----------------------------------------------------------
    def _blocks(self, nbytes):
        return int(max(8, min(self.sms, nbytes // (512 * 1024) + 8)))

    def _copy(self, stage, out, boxes, *, reduce=False, accumulate=False, scale=1.0, sequential=False, local=None):
        """Stage ``stage`` in this rank's region, then run the boxes into ``out``:
        a box with a peer rank reads that peer's staged bytes, a box with rank
        -1 reads ``local`` (default: ``stage``)."""
        boxes = [b for b in boxes if b != "empty"]
        if any(b is None for b in boxes) or len(boxes) > 16:
            return False
        stage = stage.contiguous() if stage is not None else None
        stage_bytes = 0 if stage is None else stage.numel() * stage.element_size()
        if stage_bytes > self.capacity:
            return False
        dummy = stage if stage is not None else out
        esize = out.element_size()
        self.enter("copy")
        work = max(stage_bytes, out.numel() * esize)
        self.mod.comm_copy(self.cid, dummy, stage_bytes, out, boxes, esize, reduce, accumulate, float(scale),
                           sequential, self._blocks(work), self.err, local)
        return True

    # -- health -------------------------------------------------------------
    def _skip_injected(self):
        """Host-side fault injection for tests: ``EINSHARD_FAULT_INJECT=skip:<rank>:<n>``
        makes the given global rank skip its n-th native all-reduce (it launches
        nothing, so peers' bounded waits expire).  Returns True to skip."""
        self.calls = getattr(self, "calls", 0) + 1  # native collectives issued on this communicator
        spec = os.environ.get("EINSHARD_FAULT_INJECT", "")
        if not spec.startswith("skip:"):
            return False
        _, rank, nth = spec.split(":")
        return int(rank) == dist.get_rank() and self.calls == int(nth)

    def check_health(self):
        """Synchronise and raise :class:`EinshardCommTimeout` if a kernel of this
        device gave up a wait; the communicator is then marked broken and later
        collectives fall back to ``torch.distributed``."""
        try:
            _native.check_errors(self.device)
        except _native.EinshardCommTimeout:
            self.broken = True
            _native.reset_errors()
            raise

    # -- collectives --------------------------------------------------------
    def all_reduce_(self, t, scale=1.0):
        if self.broken or t.dtype not in (torch.bfloat16, torch.float16, torch.float32) or not t.is_contiguous():
            return False
        if self._skip_injected():
            return True
        nbytes = t.numel() * t.element_size()
        if nbytes == 0:
            return True
        if self.nvls and (self.size >= _NVLS_AR_MIN_RANKS or nbytes < _NCCL_AR_MIN_BYTES):
            return self._nvls_all_reduce(t, scale)
        if nbytes >= _NCCL_AR_MIN_BYTES:
            # without multicast, measured on 2 ranks (bf16): NCCL 0.026 / 0.056 / 0.28 / 0.99 ms
            # against the push kernel 0.043 / 0.078 / 0.31 / 1.14 ms at 1 / 16 / 128 / 512 MiB;
            # on 8 ranks 512 MiB NCCL 1.34 against the pull kernel 2.19 ms.
            return False
        if nbytes % 16 or t.data_ptr() % 16:
            return False
        quantum = 16 * self.size
        push = _AR_ALGO == "push"
        # region per piece: pull stages the piece plus one reduced chunk, push takes two copies
        chunk = ((self.capacity // 2 if push else int(self.capacity / (1.0 + 1.0 / self.size))) // quantum) * quantum
        run = self.mod.comm_all_reduce_push if push else self.mod.comm_all_reduce
        flat = t.view(-1)
        per = chunk // t.element_size()
        self.enter("copy")
        for start in range(0, t.numel(), per):
            piece = flat[start:start + per]
            run(self.cid, piece, float(scale), self._blocks(piece.numel() * t.element_size()), self.err)
        return True

    def _nvls_all_reduce(self, t, scale):
        """In-place all-reduce through the NVSwitch; tensors longer than the
        heap run in pieces (the heap grows up to ``EINSHARD_NVLS_AR_PIECE_MB``)."""
        if t.data_ptr() % 16:
            # every rank takes this path whatever its alignment (the choice must agree)
            tmp = t.clone()
            self._nvls_all_reduce(tmp, scale)
            t.copy_(tmp)
            return True
        nbytes = t.numel() * t.element_size()
        padded = -(-nbytes // 16) * 16
        comm = self
        if padded > self.capacity:
            comm = workspace_for_group(self.group, min(padded, _NVLS_AR_PIECE)) or self
        per = (comm.capacity // 256) * 256 // t.element_size()
        flat = t.view(-1)
        comm.enter("nvls")
        for start in range(0, t.numel(), per):
            piece = flat[start:start + per]
            two_shot = piece.numel() * t.element_size() > _NVLS_ONE_SHOT_MAX
            comm.mod.nvls_all_reduce(comm.cid, piece, piece, float(scale), two_shot, comm.err)
        return True

    def all_reduce_div_(self, t, divisor):
        return self.all_reduce_(t, 1.0 / float(divisor))

    def broadcast_(self, t, src):
        """In place: every rank's ``t`` becomes the group rank ``src``'s.  With
        multicast, the source writes each byte once through the switch into
        every rank's heap (an all-gather in which only the source has a shard)
        and every rank copies it out; otherwise peers pull the staged tensor."""
        if self.broken or not t.is_contiguous():
            return False
        n = t.numel()
        if self.nvls and n > 0:
            lens = [n if q == src else 0 for q in range(self.size)]
            comm = self._nvls_workspace(1, 1, t.element_size(), lens)
            if comm is not None:
                flat = t.view(-1)
                if flat.data_ptr() % 16:
                    tmp = flat.clone()
                    self.broadcast_(tmp, src)
                    flat.copy_(tmp)
                    return True
                mine = flat if self.rank == src else flat[:0]
                comm.enter("nvls")
                comm.mod.nvls_all_gather(comm.cid, mine, flat, 1, 1, lens, comm.err)
                return True
        box = make_box([n], [1], 0, [1], 0, src, t.element_size())
        stage = t if self.rank == src else None
        return self._copy(stage, t, [box])

    @staticmethod
    def _outer_inner(shape, dim):
        outer = 1
        for n in shape[:dim]:
            outer *= n
        inner = 1
        for n in shape[dim + 1:]:
            inner *= n
        return outer, inner

    def _nvls_workspace(self, outer, inner, esize, shapes):
        need = sum(-(-(outer * n * inner * esize) // 256) * 256 for n in shapes)
        if need <= self.capacity:
            return self
        return workspace_for_group(self.group, need)

    def all_gather(self, x, dim, shapes):
        if self.broken:
            return None
        x = x.contiguous()
        if self.nvls:
            outer, inner = self._outer_inner(list(x.shape), dim)
            comm = self._nvls_workspace(outer, inner, x.element_size(), shapes)
            if comm is not None:
                if x.data_ptr() % 16:
                    x = x.clone()
                out_shape = list(x.shape)
                out_shape[dim] = sum(shapes)
                out = x.new_empty(out_shape)
                comm.enter("nvls")
                comm.mod.nvls_all_gather(comm.cid, x, out, outer, inner, [int(n) for n in shapes], comm.err)
                return out
        out_shape = list(x.shape)
        out_shape[dim] = sum(shapes)
        out = x.new_empty(out_shape)
        dst_strides = _contig_strides(out_shape)
        offs = [sum(shapes[:p]) for p in range(self.size)]
        boxes = []
        for p in range(self.size):
            shape = list(x.shape)
            shape[dim] = shapes[p]
            boxes.append(make_box(shape, _contig_strides(shape), 0, dst_strides, offs[p] * dst_strides[dim], p,
                                  x.element_size()))
        return out if self._copy(x, out, boxes) else None

    def reduce_scatter(self, x, dim, shapes, scale=1.0):
        if self.broken or x.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            return None
        x = x.contiguous()
        if self.nvls:
            outer, inner = self._outer_inner(list(x.shape), dim)
            comm = self._nvls_workspace(outer, inner, x.element_size(), shapes)
            if comm is not None:
                out_shape = list(x.shape)
                out_shape[dim] = shapes[self.rank]
                out = x.new_empty(out_shape)
                comm.enter("nvls")
                comm.mod.nvls_reduce_scatter(comm.cid, x, out, outer, inner, [int(n) for n in shapes], float(scale),
                                             comm.err)
                return out
        if scale != 1.0:
            return None
        out_shape = list(x.shape)
        out_shape[dim] = shapes[self.rank]
        out = x.new_empty(out_shape)
        in_strides = _contig_strides(list(x.shape))
        box = make_box(out_shape, in_strides, sum(shapes[:self.rank]) * in_strides[dim], _contig_strides(out_shape), 0,
                       0, x.element_size())
        return out if self._copy(x, out, [box], reduce=True) else None

    def all_to_all(self, x, source_dim, dest_dim, source_shapes, dest_shapes):
        if self.broken:
            return None
        x = x.contiguous()
        out_shape = list(x.shape)
        out_shape[source_dim] = sum(source_shapes)
        out_shape[dest_dim] = dest_shapes[self.rank]
        out = x.new_empty(out_shape)
        dst_strides = _contig_strides(out_shape)
        src_offs = [sum(source_shapes[:p]) for p in range(self.size)]
        my_dst_off = sum(dest_shapes[:self.rank])
        boxes = []
        for p in range(self.size):
            peer_shape = list(x.shape)
            peer_shape[source_dim] = source_shapes[p]
            peer_strides = _contig_strides(peer_shape)
            shape = list(peer_shape)
            shape[dest_dim] = dest_shapes[self.rank]
            boxes.append(make_box(shape, peer_strides, my_dst_off * peer_strides[dest_dim], dst_strides,
                                  src_offs[p] * dst_strides[source_dim], p, x.element_size()))
        return out if self._copy(x, out, boxes) else None

    def send_recv(self, x, send_rank, out, recv_rank):
        """Owner-swap exchange on the world communicator (global ranks)."""
        if self.broken or not out.is_contiguous():
            return False
        box = make_box([out.numel()], [1], 0, [1], 0, recv_rank, out.element_size())
        return self._copy(x, out, [box])

    def interval_exchange(self, x, dim, table, shapes=None):
        """Roll a sharded axis: every (start, length, dst, dst_start) piece lands on its owner."""
        if self.broken:
            return None
        x = x.contiguous()
        out = torch.empty_like(x)
        out_strides = _contig_strides(list(x.shape))
        boxes = []
        for src, pieces in enumerate(table):
            src_shape = list(x.shape)
            if shapes is not None:
                src_shape[dim] = shapes[src]
            src_strides = _contig_strides(src_shape)
            for start, length, dst, dst_start in pieces:
                if dst != self.rank:
                    continue
                shape = list(src_shape)
                shape[dim] = length
                boxes.append(make_box(shape, src_strides, start * src_strides[dim], out_strides,
                                      dst_start * out_strides[dim], src, x.element_size()))
        return out if self._copy(x, out, boxes) else None

    def halo_gather(self, x, dim, table, length, shapes):
        """Haloed shard: this rank's own rows come straight from ``x``; the
        rows peers hold come from a small staged buffer on each peer that packs
        only the slabs it sends (never the whole shard)."""
        if self.broken:
            return None
        x = x.contiguous()
        send, boxes, out_shape = halo_gather_plan(self.rank, list(x.shape), dim, table, length, x.element_size())
        out = x.new_empty(out_shape)
        stage = torch.cat([x.narrow(dim, off, n) for off, n in send], dim) if send else None
        return out if self._copy(stage, out, boxes, local=x) else None

    def halo_ghosts(self, x, dim, table, length, slab=None, shape=None):
        """The rows of this rank's haloed shard that peers hold, without the
        shard itself: (G, gtop, gbot) with G's first gtop rows along ``dim``
        above the shard and the next gbot below it (``halo_ghost_plan``), or
        None.  A consumer that reads x and G in place (the pair conv) needs no
        haloed copy of x.  ``slab(off, n)`` / ``shape``: the rows of a tensor
        of that shape that is never assembled (x with ghost columns on both
        sides); only the rows this rank sends are built."""
        if self.broken:
            return None
        x = x.contiguous()
        shape = list(x.shape) if shape is None else list(shape)
        plan = halo_ghost_plan(self.rank, shape, dim, table, length, x.element_size())
        if plan is None:
            return None
        send, boxes, g_shape, gtop, gbot = plan
        g = x.new_empty(g_shape)
        rows = slab if slab is not None else (lambda off, n: x.narrow(dim, off, n))
        stage = torch.cat([rows(off, n) for off, n in send], dim) if send else None
        # collective: every rank launches the staged copy, with or without boxes
        if not self._copy(stage, g, boxes, local=x):
            return None
        return g, gtop, gbot

    def halo_scatter_add(self, grad, dim, table, in_shape):
        """Adjoint of halo_gather: this rank's own rows of ``grad`` add into the
        result straight from ``grad``; the ghost rows go back to their owners
        through a staged buffer that packs only the slabs this rank returns."""
        if self.broken or grad.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            return None
        grad = grad.contiguous()
        send, boxes = halo_scatter_plan(self.rank, self.size, list(grad.shape), dim, table, list(in_shape),
                                        grad.element_size())
        grad_in = grad.new_zeros(in_shape)
        stage = torch.cat([grad.narrow(dim, off, n) for off, n in send], dim) if send else None
        ok = self._copy(stage, grad_in, boxes, accumulate=True, sequential=True, local=grad)
        return grad_in if ok else None

    def block_exchange(self, z, send_block, out, recv_view):
        """All-to-all of equal blocks described as views (the FFT transposes)."""
        if self.broken or not z.is_contiguous():
            return False
        boxes = []
        mine = send_block(self.rank)
        s_off, s_str = _view_geometry(mine, z)
        for p in range(self.size):
            target = recv_view(out, p)
            d_off, d_str = _view_geometry(target, out)
            boxes.append(make_box(list(target.shape), s_str, s_off, d_str, d_off, p, z.element_size()))
        return self._copy(z, out, boxes)


# ------------------------------------------------------------------ registry

_KEYS = {}


def _group_key(group):
    """Groups with the same ranks share one communicator (a mesh dimension that
    spans every rank and the world group, for instance)."""
    key = _KEYS.get(id(group))
    if key is None:
        key = _KEYS[id(group)] = tuple(dist.get_process_group_ranks(group))
    return key


def _eligible(group):
    """All ranks of ``group`` on this host with mutually accessible CUDA devices."""
    if not (torch.cuda.is_available() and dist.is_initialized()):
        return False
    if dist.get_backend(group) != "nccl":
        return False
    info = (socket.gethostname(), torch.cuda.current_device())
    infos = [None] * dist.get_world_size(group)
    dist.all_gather_object(infos, info, group=group)
    if len({host for host, _ in infos}) != 1 or len({dev for _, dev in infos}) != len(infos):
        return False
    me = torch.cuda.current_device()
    local_ok = all(dev == me or torch.cuda.can_device_access_peer(me, dev) for _, dev in infos)
    flag = torch.tensor([1 if local_ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


def communicator_for_group(group):
    key = _group_key(group)
    if key in _COMMS:
        return _COMMS[key]
    if key in _REJECTED:
        return None
    if group is None or dist.get_world_size(group) == 1 or dist.get_world_size(group) > 8 or not _eligible(group):
        _REJECTED.add(key)
        return None
    comm = Communicator(group, _DEFAULT_MB * (1 << 20))
    _COMMS[key] = comm
    return comm


def workspace_for_group(group, nbytes):
    """A communicator with at least ``nbytes`` of symmetric region: the group's
    default one when large enough, else the group's single larger heap, grown
    (a collective call: every member asks with the same size) by closing the
    previous larger heap on every rank and creating one of the new size, in
    steps of 256 MiB."""
    key = _group_key(group)
    comm = _COMMS.get(key)
    if comm is None:
        return None
    if comm.capacity >= nbytes:
        return comm
    big = _LARGE.get(key)
    if big is not None and big.capacity >= nbytes:
        return big
    if big is not None:
        big.close()
    mb = 256
    size = ((int(nbytes) + (mb << 20) - 1) // (mb << 20)) * (mb << 20)
    big = Communicator(comm.group, size)
    _LARGE[key] = big
    return big


def _mesh_groups(mesh):
    groups = [dist.group.WORLD]
    if mesh is not None:
        for name in getattr(mesh, "mesh_dim_names", None) or ():
            groups.append(mesh[name].get_group())
    return groups


def activate(mesh=None):
    if os.environ.get("EINSHARD_NATIVE_COMM", "1") in ("0", ""):
        return False
    if not _native.available():
        return False
    for group in _mesh_groups(mesh):
        communicator_for_group(group)
    _state["enabled"] = True
    _state["auto_blocked"] = False
    return True


# ------------------------------------------------------------------ lookup used by the collective helpers

_state = {"enabled": False, "auto_blocked": False}
# Opt-in lazy set-up for code that never calls setup_native_comm (drop-in users
# of the reference's API): the first lookup on a CUDA / NCCL group creates that
# group's communicator.  The lookup is collective like the helpers that make it
# (every rank of the group reaches it in the same order).
_AUTO = os.environ.get("EINSHARD_AUTO_NATIVE_COMM", "0") not in ("0", "")


def _auto_activate():
    if (not _AUTO or _state["auto_blocked"] or os.environ.get("EINSHARD_NATIVE_COMM", "1") in ("0", "")
            or not torch.cuda.is_available() or not dist.is_initialized() or not _native.available()):
        return False
    _state["enabled"] = True
    return True


def enabled() -> bool:
    """Whether the native communicators are active (``setup_native_comm``)."""
    return _state["enabled"]


def disable():
    """Route every collective to torch.distributed again (the heaps stay)."""
    _state["enabled"] = False
    _state["auto_blocked"] = True


def communicator_for(group):
    """The native communicator of ``group``, or None (not active, not eligible)."""
    if group is None or (not _state["enabled"] and not _auto_activate()):
        return None
    comm = _COMMS.get(_group_key(group))
    if comm is None and _AUTO and not _state["auto_blocked"]:
        comm = communicator_for_group(group)
    return comm


def workspace_for(group, nbytes):
    """A communicator of ``group`` whose symmetric region holds ``nbytes``
    (collective: every member asks with the same size), or None."""
    if group is None or communicator_for(group) is None:
        return None
    return workspace_for_group(group, nbytes)


def world_communicator():
    return communicator_for(dist.group.WORLD) if _state["enabled"] else None


def setup_native_comm(mesh=None, *, enable=True):
    """Create the native NVLink communicators for every group of ``mesh`` (and
    the world group): CUDA + NCCL process groups only.  Collective over every
    rank.  Returns True when the native path is active; on CPU / gloo it does
    nothing and returns False.  No reference counterpart (the reference only
    uses ``torch.distributed``)."""
    if not enable or not torch.cuda.is_available() or not dist.is_initialized():
        return False
    return activate(mesh)


def teardown_native_comm():
    """Free every symmetric heap (collective while the process group lives)."""
    deactivate()


def _all_comms():
    return list(_COMMS.values()) + list(_LARGE.values())


def deactivate():
    """Free every heap.  With the process group still initialised this is a
    collective close (synchronise, barrier, free); otherwise see _release_at_exit."""
    disable()
    if dist.is_initialized():
        for comm in _all_comms():
            if not comm.closed:
                comm.close()
    else:
        _release_at_exit()
    _COMMS.clear()
    _LARGE.clear()
    _REJECTED.clear()
    _KEYS.clear()


def _release_at_exit():
    """Free the heaps of a process that ends without a collective close: first a
    bounded, stream-ordered wait until every peer finished the collectives that
    touch this rank's memory (the NVLS counters and the copy protocol's done
    flags, written by the peers' kernels, so no process group is needed), then
    unmap, unbind from the multicast object and free."""
    for comm in _all_comms():
        if comm.closed:
            continue
        try:
            comm.mod.nvls_quiesce(comm.cid, comm.err)
            comm.mod.comm_acquire(comm.cid, comm.err)
            torch.cuda.synchronize()
            comm.mod.comm_destroy(comm.cid)
        except Exception:  # noqa: BLE001 - exiting; the driver frees what is left
            pass
        comm.closed = True


atexit.register(_release_at_exit)
