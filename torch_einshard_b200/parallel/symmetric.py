"""Native NVLink communicators built on peer-mapped symmetric buffers.

``activate(mesh)`` creates one :class:`Communicator` per process group of the
mesh (and the world group): every rank allocates a device buffer
(``EINSHARD_SYMM_MB``, default 1280 MiB of data plus 1 MiB of flags), exports
its CUDA IPC handle, gathers the peers' handles through the process group and
maps them.  Collectives then run as single cooperative kernels that stage the
local input into the buffer and pull what they need from peers over NVLink
(``csrc/comm.cu``).  Every operation is described as a list of strided copy
boxes, so uneven shards and arbitrary dimensions need no pack/unpack copies.

A communicator is only created for groups whose ranks all live on this node
and whose devices can access each other; otherwise the collective helpers use
``torch.distributed`` (NCCL).  Set ``EINSHARD_NATIVE_COMM=0`` to disable.

Native backend of the reference's collective helpers: all_reduce
``src/torch_einshard/helpers.py:27``, broadcast ``:35``, all_gather ``:61``,
reduce_scatter ``:114``, all_to_all_repartition ``:142``, owner_swap ``:184``,
roll ``:224-309``.
"""

import os
import socket

import torch
import torch.distributed as dist

from ..ops import _native
from . import native_comm

__all__ = ["Communicator", "activate", "deactivate", "communicator_for_group"]

_DEFAULT_MB = int(os.environ.get("EINSHARD_SYMM_MB", "1280"))
# 512 MiB all-reduce at 8 ranks on B200: this two-shot kernel 2.19 ms, NCCL 1.34 ms.
_NCCL_AR_MIN_BYTES = int(os.environ.get("EINSHARD_NCCL_AR_MIN_BYTES", str(1 << 20)))
# native all-reduce kernel: "push" (every NVLink transfer a store into a peer's region,
# no staging copy; 15-47 % faster than "pull" on 2 ranks from 1 to 512 MiB) or "pull"
# (peers' chunks read over NVLink)
_AR_ALGO = os.environ.get("EINSHARD_AR_ALGO", "push")
_COMMS = {}
_REJECTED = set()
_LARGE = {}  # group key -> larger communicators created on demand (kept until deactivate)


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


class Communicator:
    def __init__(self, group, data_bytes):
        self.mod = _native.require()
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.device = torch.cuda.current_device()
        self.err = _native.error_word(self.device)
        cid, handle = self.mod.comm_create(int(data_bytes), self.device)
        handles = [None] * self.size
        dist.all_gather_object(handles, handle, group=group)
        self.mod.comm_connect(cid, self.rank, handles)
        self.cid = cid
        self.capacity = int(data_bytes)
        self.sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.broken = False

    # -- raw access for fused kernels ----------------------------------------
    @property
    def id(self):
        return self.cid

    @property
    def data_bytes(self):
        return self.capacity

    def acquire(self):
        """Stream-ordered wait until every peer finished reading this rank's
        region for the previous op; writes into ``region()`` must follow it."""
        self.mod.comm_acquire(self.cid, self.err)

    def region(self, nbytes):
        """This rank's symmetric data region (first ``nbytes``) as uint8."""
        return self.mod.comm_region(self.cid, int(nbytes))

    # -- helpers -----------------------------------------------------------
    def _blocks(self, nbytes):
        return int(max(8, min(self.sms, nbytes // (512 * 1024) + 8)))

    def _copy(self, stage, out, boxes, *, reduce=False, accumulate=False, scale=1.0, sequential=False):
        boxes = [b for b in boxes if b != "empty"]
        if any(b is None for b in boxes) or len(boxes) > 16:
            return False
        stage = stage.contiguous() if stage is not None else None
        stage_bytes = 0 if stage is None else stage.numel() * stage.element_size()
        if stage_bytes > self.capacity:
            return False
        dummy = stage if stage is not None else out
        esize = out.element_size()
        self.mod.comm_copy(self.cid, dummy, stage_bytes, out, boxes, esize, reduce, accumulate, float(scale),
                           sequential, self._blocks(max(stage_bytes, out.numel() * esize)), self.err)
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
        if nbytes >= _NCCL_AR_MIN_BYTES:
            # measured on 2 ranks (bf16): NCCL 0.026 / 0.056 / 0.28 / 0.99 ms against the
            # native push kernel 0.043 / 0.078 / 0.31 / 1.14 ms (pull 0.064 / 0.147 / 0.36 /
            # 1.33 ms) at 1 / 16 / 128 / 512 MiB; on 8 ranks 512 MiB NCCL 1.34 against pull
            # 2.19 ms.  A DDP bucket's separate 1/dp scaling pass costs less than that
            # difference.  The native kernel keeps the buffers below 1 MiB.
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
        for start in range(0, t.numel(), per):
            piece = flat[start:start + per]
            run(self.cid, piece, float(scale), self._blocks(piece.numel() * t.element_size()), self.err)
        return True

    def all_reduce_div_(self, t, divisor):
        return self.all_reduce_(t, 1.0 / float(divisor))

    def broadcast_(self, t, src):
        if self.broken or not t.is_contiguous():
            return False
        n = t.numel()
        box = make_box([n], [1], 0, [1], 0, src, t.element_size())
        stage = t if self.rank == src else None
        return self._copy(stage, t, [box])

    def all_gather(self, x, dim, shapes):
        if self.broken:
            return None
        x = x.contiguous()
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

    def reduce_scatter(self, x, dim, shapes):
        if self.broken or x.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            return None
        x = x.contiguous()
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
        if self.broken:
            return None
        x = x.contiguous()
        out_shape = list(x.shape)
        out_shape[dim] = length
        out = x.new_empty(out_shape)
        out_strides = _contig_strides(out_shape)
        boxes = []
        for out_off, src, src_off, n in table[self.rank]:
            src_shape = list(x.shape)
            src_shape[dim] = shapes[src]
            src_strides = _contig_strides(src_shape)
            shape = list(src_shape)
            shape[dim] = n
            boxes.append(make_box(shape, src_strides, src_off * src_strides[dim], out_strides,
                                  out_off * out_strides[dim], src, x.element_size()))
        return out if self._copy(x, out, boxes) else None

    def halo_scatter_add(self, grad, dim, table, in_shape):
        if self.broken or grad.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            return None
        grad = grad.contiguous()
        grad_in = grad.new_zeros(in_shape)
        in_strides = _contig_strides(list(in_shape))
        boxes = []
        for dst, pieces in enumerate(table):
            g_shape = list(grad.shape)
            g_shape[dim] = sum(p[3] for p in pieces)
            g_strides = _contig_strides(g_shape)
            for out_off, src, src_off, n in pieces:
                if src != self.rank:
                    continue
                shape = list(g_shape)
                shape[dim] = n
                boxes.append(make_box(shape, g_strides, out_off * g_strides[dim], in_strides,
                                      src_off * in_strides[dim], dst, grad.element_size()))
        ok = self._copy(grad, grad_in, boxes, accumulate=True, sequential=True)
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

def _group_key(group):
    return id(group)


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
    """A communicator with at least ``nbytes`` of symmetric region.  The default
    one is used when large enough; otherwise a dedicated one is created (a
    collective call: every member asks with the same size) and kept, because
    freeing peer-mapped memory while a peer might still read it is unsafe."""
    comm = _COMMS.get(_group_key(group))
    if comm is None:
        return None
    if comm.capacity >= nbytes:
        return comm
    for big in _LARGE.get(_group_key(group), []):
        if big.capacity >= nbytes:
            return big
    mb = 256
    size = ((int(nbytes) + (mb << 20) - 1) // (mb << 20)) * (mb << 20)
    big = Communicator(group, size)
    _LARGE.setdefault(_group_key(group), []).append(big)
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
    native_comm.enable(lambda group: _COMMS.get(_group_key(group)) if group is not None else None,
                       lambda group, nbytes: workspace_for_group(group, nbytes) if group is not None else None)
    _install_fusions()
    return True


def _install_fusions():
    try:
        from ..ops import fused_native
        fused_native.install()
    except ImportError:
        pass


def deactivate():
    native_comm.disable()
    for comm in list(_COMMS.values()) + [c for cs in _LARGE.values() for c in cs]:
        try:
            comm.mod.comm_destroy(comm.cid)
        except Exception:  # noqa: BLE001
            pass
    _COMMS.clear()
    _LARGE.clear()
    _REJECTED.clear()
