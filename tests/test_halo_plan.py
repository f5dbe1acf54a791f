"""Host plans of the native halo exchange (no GPU): every rank packs only the
slabs it sends, and the copy boxes of every rank, replayed on the host exactly
as the staged copy kernel executes them (byte boxes from the local tensor or a
peer's packed buffer), rebuild the haloed shard and the adjoint scatter-add.
Uneven shards, halos wider than a neighbour's shard, periodic wrap, the halo
along an inner and the outer dimension."""

import numpy as np
import pytest

from torch_einshard_b200.ops.halo import halo_intervals
from torch_einshard_b200.parallel.symmetric import halo_gather_plan, halo_scatter_plan

ESIZE = 4  # float32


def _replay(boxes, locals_bytes, staged, out_bytes, accumulate=False):
    """Apply byte boxes (src_rank, sizes, src_off, dst_off, sstr, dstr) into out."""
    out = out_bytes
    for box in boxes:
        if box == "empty":
            continue
        src_rank, sizes, src_off, dst_off, sstr, dstr = box
        src = locals_bytes if src_rank < 0 else staged[src_rank]
        run = sizes[3] * ESIZE
        for i0 in range(sizes[0]):
            for i1 in range(sizes[1]):
                for i2 in range(sizes[2]):
                    so = src_off + i0 * sstr[0] + i1 * sstr[1] + i2 * sstr[2]
                    do = dst_off + i0 * dstr[0] + i1 * dstr[1] + i2 * dstr[2]
                    chunk = src[so:so + run]
                    if accumulate:
                        cur = np.frombuffer(out[do:do + run].tobytes(), dtype=np.float32)
                        add = np.frombuffer(chunk.tobytes(), dtype=np.float32)
                        out[do:do + run] = np.frombuffer((cur + add).astype(np.float32).tobytes(), dtype=np.uint8)
                    else:
                        out[do:do + run] = chunk
    return out


def _pieces_tensor(xs, dim, pieces):
    return np.concatenate([np.take(xs[src], range(src_off, src_off + n), axis=dim) for _, src, src_off, n in pieces],
                          axis=dim)


CASES = [
    # shapes along the halo dim, left, right, periodic, dim, other dims
    ([5, 4, 6], 1, 1, False, 1, (2, None, 3)),
    ([3, 1, 2, 4], 2, 3, True, 1, (2, None, 2)),
    ([2, 2], 3, 1, True, 0, (None, 3, 2)),
    ([1040 // 40, 1008 // 40], 1, 1, False, 1, (2, None, 4)),
    ([520 // 40, 520 // 40, 504 // 40, 504 // 40], 1, 1, False, 1, (2, None, 4)),
]


@pytest.mark.parametrize("shapes,left,right,periodic,dim,others", CASES)
def test_halo_plans_rebuild_the_haloed_shards_and_the_adjoint(shapes, left, right, periodic, dim, others):
    size = len(shapes)
    rng = np.random.default_rng(0)
    xs = []
    for q in range(size):
        shape = [shapes[q] if o is None else o for o in others]
        xs.append(rng.standard_normal(shape).astype(np.float32))
    table = halo_intervals(shapes, left, right, periodic=periodic)
    # forward: pack, then every rank replays its boxes
    staged = {}
    plans = {}
    for q in range(size):
        length = shapes[q] + left + right if periodic else sum(p[3] for p in table[q])
        send, boxes, out_shape = halo_gather_plan(q, list(xs[q].shape), dim, table, length, ESIZE)
        plans[q] = (boxes, out_shape)
        packed = (np.concatenate([np.take(xs[q], range(o, o + n), axis=dim) for o, n in send], axis=dim)
                  if send else np.zeros(0, np.float32))
        staged[q] = np.frombuffer(np.ascontiguousarray(packed).tobytes(), dtype=np.uint8)
    outs = {}
    for q in range(size):
        boxes, out_shape = plans[q]
        out = np.zeros(int(np.prod(out_shape)) * ESIZE, dtype=np.uint8)
        local = np.frombuffer(np.ascontiguousarray(xs[q]).tobytes(), dtype=np.uint8)
        got = np.frombuffer(_replay(boxes, local, staged, out).tobytes(), dtype=np.float32).reshape(out_shape)
        want = _pieces_tensor(xs, dim, table[q])
        np.testing.assert_array_equal(got, want)
        outs[q] = got
    # backward: every haloed element's gradient goes back to its owner and adds up
    grads = {q: rng.standard_normal(outs[q].shape).astype(np.float32) for q in range(size)}
    want_in = {q: np.zeros_like(xs[q]) for q in range(size)}
    for q in range(size):
        for out_off, src, src_off, n in table[q]:
            idx = [slice(None)] * xs[q].ndim
            idx[dim] = slice(src_off, src_off + n)
            gidx = [slice(None)] * xs[q].ndim
            gidx[dim] = slice(out_off, out_off + n)
            want_in[src][tuple(idx)] += grads[q][tuple(gidx)]
    staged, plans = {}, {}
    for q in range(size):
        send, boxes = halo_scatter_plan(q, size, list(grads[q].shape), dim, table, list(xs[q].shape), ESIZE)
        plans[q] = boxes
        packed = (np.concatenate([np.take(grads[q], range(o, o + n), axis=dim) for o, n in send], axis=dim)
                  if send else np.zeros(0, np.float32))
        staged[q] = np.frombuffer(np.ascontiguousarray(packed).tobytes(), dtype=np.uint8)
    for q in range(size):
        out = np.zeros(xs[q].size * ESIZE, dtype=np.uint8)
        local = np.frombuffer(np.ascontiguousarray(grads[q]).tobytes(), dtype=np.uint8)
        got = np.frombuffer(_replay(plans[q], local, staged, out, accumulate=True).tobytes(),
                            dtype=np.float32).reshape(xs[q].shape)
        np.testing.assert_allclose(got, want_in[q], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("shapes,left,right,periodic,dim,others", CASES)
def test_ghost_plans_rebuild_only_the_peers_rows(shapes, left, right, periodic, dim, others):
    """halo_ghost_plan: every rank's G holds exactly the haloed shard's rows
    that peers own (those above the shard, then those below), nothing of its own."""
    from torch_einshard_b200.parallel.symmetric import halo_ghost_plan
    size = len(shapes)
    rng = np.random.default_rng(1)
    xs = [rng.standard_normal([shapes[q] if o is None else o for o in others]).astype(np.float32) for q in range(size)]
    table = halo_intervals(shapes, left, right, periodic=periodic)
    plans, staged = {}, {}
    for q in range(size):
        length = shapes[q] + left + right if periodic else sum(p[3] for p in table[q])
        plans[q] = halo_ghost_plan(q, list(xs[q].shape), dim, table, length, ESIZE)
        send = plans[q][0] if plans[q] is not None else []
        packed = (np.concatenate([np.take(xs[q], range(o, o + n), axis=dim) for o, n in send], axis=dim)
                  if send else np.zeros(0, np.float32))
        staged[q] = np.frombuffer(np.ascontiguousarray(packed).tobytes(), dtype=np.uint8)
    for q in range(size):
        if plans[q] is None:
            continue
        _, boxes, g_shape, gtop, gbot = plans[q]
        out = np.zeros(int(np.prod(g_shape)) * ESIZE, dtype=np.uint8)
        local = np.frombuffer(np.ascontiguousarray(xs[q]).tobytes(), dtype=np.uint8)
        got = np.frombuffer(_replay(boxes, local, staged, out).tobytes(), dtype=np.float32).reshape(g_shape)
        full = _pieces_tensor(xs, dim, table[q])
        want = np.concatenate([np.take(full, range(0, gtop), axis=dim),
                               np.take(full, range(full.shape[dim] - gbot, full.shape[dim]), axis=dim)], axis=dim)
        np.testing.assert_array_equal(got, want)
        assert g_shape[dim] == gtop + gbot
