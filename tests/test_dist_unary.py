"""Distributed unary einshard on 8 gloo ranks: split/gather, repartition,
owner swaps, partial sums, ellipsis, with the seeded full-tensor oracle."""

import warnings

import pytest
import torch
import torch.distributed as dist

import torch_einshard_b200 as es
from conftest import assert_close
from dist_harness import run_ranks


def _split(full, shapes, dim, rank):
    return torch.split(full, shapes, dim=dim)[rank]


def test_requires_mesh():
    with pytest.raises(ValueError, match="Distributed einshard operations require mesh"):
        es.einshard("a b -> a/dp b", torch.randn(4, 3))


def _split_gather(ctx):
    mesh = ctx.mesh((ctx.world_size,), ("dp",))
    group = mesh["dp"].get_group()
    rank, P = dist.get_rank(group), dist.get_world_size(group)
    rows = P * 2
    shapes = es.compute_split_shapes(rows, P)
    x = torch.randn(rows, 3, requires_grad=True)
    z = es.einshard("a b -> a/dp b", x, mesh=mesh, shapes=shapes)
    assert z.shape == (shapes[rank], 3)
    assert [s.name for s in es.last_plan()] == ["split_forward_allgather_backward"]
    zz = es.einshard("a/dp b -> a b", z, mesh=mesh, shapes=shapes)
    assert_close(zz, x)
    assert [s.name for s in es.last_plan()] == ["allgather_forward_split_backward"]
    (z ** 2).sum().backward()
    assert_close(x.grad, 2 * x)

    # ellipsis on both sides
    x = torch.randn(2, 3, rows, requires_grad=True)
    z = es.einshard("... a -> ... a/dp", x, mesh=mesh, shapes=shapes)
    assert z.shape == (2, 3, shapes[rank])
    assert_close(es.einshard("... a/dp -> ... a", z, mesh=mesh, shapes=shapes), x)

    # split with permutation
    x = torch.randn(3, rows)
    z = es.einshard("b a -> a/dp b", x, mesh=mesh, shapes=shapes)
    assert_close(z, _split(x, shapes, 1, rank).transpose(0, 1).contiguous())

    # uneven gather (BASELINE CPU config shape pattern)
    uneven = es.compute_split_shapes(P * 3 + 1, P)
    full = torch.randn(sum(uneven), 4)
    zz = es.einshard("a/dp c -> a c", _split(full, uneven, 0, rank).contiguous(), mesh=mesh, shapes=uneven)
    assert_close(zz, full)


def test_split_gather_round_trips():
    run_ranks(_split_gather)


def _repartition(ctx):
    mesh = ctx.mesh((ctx.world_size,), ("dp",))
    group = mesh["dp"].get_group()
    rank, P = dist.get_rank(group), dist.get_world_size(group)
    for rows, cols in ((P * 2, P * 3), (P * 2 + 1, P * 3 + 2)):
        rs = es.compute_split_shapes(rows, P)
        cs = es.compute_split_shapes(cols, P)
        full = torch.randn(rows, cols)
        x = _split(full, rs, 0, rank).clone().requires_grad_(True)
        z = es.einshard("a/dp b -> a b/dp", x, mesh=mesh, shapes={"dp": {"a": rs, "b": cs}})
        assert_close(z, _split(full, cs, 1, rank))
        assert [s.name for s in es.last_plan()] == ["alltoall_repartition"]
        z.sum().backward()
        assert_close(x.grad, torch.ones_like(x))
        x = _split(full, cs, 1, rank).clone().requires_grad_(True)
        z = es.einshard("a b/dp -> a/dp b", x, mesh=mesh, shapes={"dp": {"a": rs, "b": cs}})
        assert_close(z, _split(full, rs, 0, rank))


def test_alltoall_repartition_even_and_uneven():
    run_ranks(_repartition)


def _owner_swaps(ctx):
    # (2, 4) mesh: dp and sp have different sizes -> fallback with a warning
    mesh = ctx.mesh((2, ctx.world_size // 2), ("dp", "sp"))
    dp, sp = mesh["dp"].get_group(), mesh["sp"].get_group()
    rows = 16
    dps = es.compute_split_shapes(rows, dist.get_world_size(dp))
    sps = es.compute_split_shapes(rows, dist.get_world_size(sp))
    full = torch.randn(rows, 3)
    x = _split(full, dps, 0, dist.get_rank(dp)).clone()
    with pytest.warns(RuntimeWarning, match="gather/split fallback"):
        z = es.einshard("a/dp b -> a/sp b", x, mesh=mesh, shapes={"dp": {"a": dps}, "sp": {"a": sps}})
    assert_close(z, _split(full, sps, 0, dist.get_rank(sp)))

    # (2, 2, 2) mesh: equal dims -> one owner swap
    mesh = ctx.mesh((2, 2, ctx.world_size // 4), ("dp", "sp", "tp"))
    dp, sp, tp = (mesh[n].get_group() for n in ("dp", "sp", "tp"))
    shapes = es.compute_split_shapes(8, 2)
    full = torch.randn(8, 3)
    x = _split(full, shapes, 0, dist.get_rank(dp)).clone().requires_grad_(True)
    z = es.einshard("a/dp b -> a/sp b", x, mesh=mesh, shapes={"dp": {"a": shapes}, "sp": {"a": shapes}})
    assert_close(z, _split(full, shapes, 0, dist.get_rank(sp)))
    assert [s.name for s in es.last_plan()] == ["owner_swap"]
    z.sum().backward()
    assert_close(x.grad, torch.ones_like(x))

    # swap plus an independent split
    a_s, b_s = es.compute_split_shapes(5, 2), es.compute_split_shapes(7, dist.get_world_size(tp))
    full = torch.randn(5, 7)
    x = _split(full, a_s, 0, dist.get_rank(dp)).clone()
    z = es.einshard("a/dp b -> a/sp b/tp", x, mesh=mesh,
                    shapes={"dp": {"a": a_s}, "sp": {"a": a_s}, "tp": {"b": b_s}})
    assert_close(z, _split(_split(full, a_s, 0, dist.get_rank(sp)), b_s, 1, dist.get_rank(tp)))
    assert [s.name for s in es.last_plan()] == ["owner_swap", "split_forward_allgather_backward"]

    # unchanged axis on an involved dim -> fallback
    a_s, c_s = es.compute_split_shapes(5, 2), es.compute_split_shapes(7, 2)
    full = torch.randn(5, 7, 3)
    x = _split(_split(full, a_s, 0, dist.get_rank(dp)), c_s, 1, dist.get_rank(sp)).clone()
    with pytest.warns(RuntimeWarning, match="gather/split fallback"):
        z = es.einshard("a/dp c/sp b -> a/sp c/sp b", x, mesh=mesh,
                        shapes={"dp": {"a": a_s}, "sp": {"a": a_s, "c": c_s}})
    assert_close(z, _split(_split(full, a_s, 0, dist.get_rank(sp)), c_s, 1, dist.get_rank(sp)))
    assert [s.name for s in es.last_plan()] == ["allgather_forward_split_backward", "split_forward_allgather_backward"]

    # multi-axis swap h/sp1 w/sp2 -> h/sp2 w/sp1
    mesh = ctx.mesh((ctx.world_size // 4, 2, 2), ("dp", "sp1", "sp2"))
    s1, s2 = mesh["sp1"].get_group(), mesh["sp2"].get_group()
    hs, ws = es.compute_split_shapes(5, 2), es.compute_split_shapes(7, 2)
    full = torch.randn(2, 5, 7, 3)
    x = _split(_split(full, hs, 1, dist.get_rank(s1)), ws, 2, dist.get_rank(s2)).clone().requires_grad_(True)
    z = es.einshard("b h/sp1 w/sp2 c -> b h/sp2 w/sp1 c", x, mesh=mesh,
                    shapes={"sp1": {"h": hs, "w": ws}, "sp2": {"h": hs, "w": ws}})
    assert_close(z, _split(_split(full, hs, 1, dist.get_rank(s2)), ws, 2, dist.get_rank(s1)))
    z.sum().backward()
    assert_close(x.grad, torch.ones_like(x))


def test_owner_swaps_and_fallbacks():
    run_ranks(_owner_swaps)


def _partials(ctx):
    mesh = ctx.mesh((ctx.world_size,), ("tp",))
    group = mesh["tp"].get_group()
    rank, P = dist.get_rank(group), dist.get_world_size(group)
    total = float(P * (P + 1) // 2)
    x = torch.full((2, 3), float(rank + 1), requires_grad=True)
    z = es.einshard("a b // tp -> a b", x, mesh=mesh)
    assert_close(z, torch.full_like(x, total))
    z.sum().backward()
    assert_close(x.grad, torch.ones_like(x))

    x = torch.randn(2, 3, requires_grad=True)
    z = es.einshard("a b -> a b // tp", x, mesh=mesh)
    assert_close(z, x)
    z.sum().backward()
    assert_close(x.grad, torch.ones_like(x) * P)

    rows = P * 2
    shapes = es.compute_split_shapes(rows, P)
    x = torch.full((rows, 3), float(rank + 1), requires_grad=True)
    z = es.einshard("a b // tp -> a/tp b", x, mesh=mesh, shapes=shapes)
    assert_close(z, _split(torch.full_like(x, total), shapes, 0, rank))
    z.sum().backward()
    assert_close(x.grad, torch.ones_like(x))

    full = torch.arange(rows * 3, dtype=torch.float32).reshape(rows, 3)
    x = _split(full, shapes, 0, rank).clone().requires_grad_(True)
    z = es.einshard("a/tp b -> a b // tp", x, mesh=mesh, shapes=shapes)
    assert_close(z, full)
    z.sum().backward()
    assert_close(x.grad, torch.ones_like(x) * P)

    mesh2 = es.wrap_mesh(ctx.mesh((2, ctx.world_size // 2), ("dp", "sp")))
    W = dist.get_world_size()
    x = torch.tensor(float(dist.get_rank() + 1), requires_grad=True)
    assert_close(es.einshard("loss // (sp,dp) -> loss", x, mesh=mesh2), torch.tensor(float(W * (W + 1) // 2)))
    z = es.einshard("loss // dp-sp -> loss", x, mesh=mesh2)
    assert_close(z, torch.tensor(float(W * (W + 1) // 2)))
    z.backward()
    assert_close(x.grad, torch.ones_like(x))


def test_partial_sums():
    run_ranks(_partials)
