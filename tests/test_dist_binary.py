"""Distributed binary einshard on 8 gloo ranks (TP/SP/SUMMA/attention patterns,
post-contraction repartition, owner swaps), checked against full-tensor math."""

import pytest
import torch
import torch.distributed as dist

import torch_einshard_b200 as es
from conftest import assert_close
from dist_harness import run_ranks


def _split(full, shapes, dim, rank):
    return torch.split(full, shapes, dim=dim)[rank]


def _names():
    return [s.name for s in es.last_plan()]


def _tp_patterns(ctx):
    mesh = ctx.mesh((ctx.world_size,), ("tp",))
    group = mesh["tp"].get_group()
    rank, P = dist.get_rank(group), dist.get_world_size(group)

    # column parallel is a local operation (every axis keeps its placement):
    # no collective at all, and x.grad holds this rank's contribution only
    hidden = P * 3
    x = torch.randn(2, 4, 5, requires_grad=True)
    w = torch.randn(hidden, 5)
    ws = torch.split(w, hidden // P, dim=0)[rank].contiguous().requires_grad_(True)
    z = es.einshard("b n c, h/tp c -> b n h/tp", x, ws, mesh=mesh)
    assert _names() == ["rank_local_einsum"]
    full = torch.einsum("bnc,hc->bnh", x.detach(), w)
    assert_close(z, torch.split(full, hidden // P, dim=2)[rank])
    g = torch.randn(2, 4, hidden)
    gs = torch.split(g, hidden // P, dim=2)[rank]
    z.backward(gs)
    assert_close(x.grad, torch.einsum("bnh,hc->bnc", gs, ws.detach()), rtol=1e-4, atol=1e-5)

    # row parallel: forward all-reduce; explicit partial keeps local sums
    channels = P * 3
    x = torch.randn(2, 4, channels)
    w = torch.randn(7, channels)
    xs = torch.split(x, channels // P, dim=2)[rank].contiguous()
    wsh = torch.split(w, channels // P, dim=1)[rank].contiguous()
    z = es.einshard("b n c/tp, h c/tp -> b n h", xs, wsh, mesh=mesh)
    assert_close(z, torch.einsum("bnc,hc->bnh", x, w), rtol=1e-4, atol=1e-5)
    assert _names() == ["rank_local_einsum", "allreduce_forward_identity_backward"]
    z = es.einshard("b n c/tp, h c/tp -> b n h // tp", xs, wsh, mesh=mesh)
    assert_close(z, torch.einsum("bnc,hc->bnh", xs, wsh))
    assert _names() == ["rank_local_einsum"]
    assert_close(es.einshard("b n h // tp -> b n h", z, mesh=mesh), torch.einsum("bnc,hc->bnh", x, w),
                 rtol=1e-4, atol=1e-5)

    # sequence parallel: gather l (backward reduce-scatter) / reduce-scatter l
    l_full = torch.randn(P * 4, 6)
    w = torch.randn(6, P * 2)
    xl = _split(l_full, [4] * P, 0, rank).clone().requires_grad_(True)
    wf = torch.split(w, 2, dim=1)[rank].contiguous()
    z = es.einshard("l/tp e, e f/tp -> l f/tp", xl, wf, mesh=mesh)
    assert _names() == ["allgather_forward_reducescatter_backward", "rank_local_einsum"]
    assert_close(z, l_full @ wf)
    a = torch.randn(P * 4, P * 2)
    af = torch.split(a, 2, dim=1)[rank].contiguous()
    w2 = torch.randn(P * 2, 5)
    w2f = torch.split(w2, 2, dim=0)[rank].contiguous()
    z = es.einshard("l f/tp, f/tp e -> l/tp e", af, w2f, mesh=mesh)
    assert _names() == ["rank_local_einsum", "reducescatter_forward_allgather_backward"]
    assert_close(z, _split(a @ w2, [4] * P, 0, rank), rtol=1e-4, atol=1e-5)


def test_tensor_and_sequence_parallel_patterns():
    run_ranks(_tp_patterns)


def _repartition_after_contraction(ctx):
    mesh = ctx.mesh((ctx.world_size,), ("tp",))
    group = mesh["tp"].get_group()
    rank, P = dist.get_rank(group), dist.get_world_size(group)
    rows, cols = P * 2 + 1, P * 3 + 2
    rs, cs = es.compute_split_shapes(rows, P), es.compute_split_shapes(cols, P)
    x_full = torch.randn(rows, 4)
    y = torch.randn(4, cols, requires_grad=True)
    xs = _split(x_full, rs, 0, rank).clone().requires_grad_(True)
    z = es.einshard("l/tp e, e f -> l f/tp", xs, y, mesh=mesh, shapes={"tp": {"l": rs, "f": cs}})
    xr, yr = x_full.clone().requires_grad_(True), y.detach().clone().requires_grad_(True)
    full = xr @ yr
    assert_close(z, _split(full, cs, 1, rank), rtol=1e-4, atol=1e-5)
    g = torch.randn(rows, cols)
    z.backward(_split(g, cs, 1, rank))
    full.backward(g)
    assert_close(xs.grad, _split(xr.grad, rs, 0, rank), rtol=1e-4, atol=1e-5)
    assert_close(y.grad, yr.grad, rtol=1e-4, atol=1e-5)
    assert [(a.name, a.status) for a in es.last_alternatives()] == [
        ("alltoall_repartition", "selected"), ("default", "ranked")]
    assert [(c.name, c.status) for c in es.last_candidates()] == [("alltoall_repartition", "accepted")]
    assert _names() == ["identity_forward_allreduce_backward", "rank_local_einsum", "alltoall_repartition"]

    # without shapes: candidate rejected, gather/split fallback
    xe = _split(x_full[: P * 2], [2] * P, 0, rank)
    z = es.einshard("l/tp e, e f -> l f/tp", xe, y.detach()[:, : P * 3], mesh=mesh)
    assert_close(z, _split(x_full[: P * 2] @ y.detach()[:, : P * 3], [3] * P, 1, rank), rtol=1e-4, atol=1e-5)
    assert [(c.name, c.status) for c in es.last_candidates()] == [("alltoall_repartition", "rejected")]
    assert [(a.name, a.status) for a in es.last_alternatives()] == [
        ("alltoall_repartition", "ranked"), ("default", "selected")]
    assert _names() == ["allgather_forward_reducescatter_backward", "split_forward_allgather_backward",
                        "rank_local_einsum"]

    # invalid split metadata is detected collectively
    bad = list(rs)
    bad[0] += 1
    with pytest.raises(ValueError, match="split metadata"):
        es.einshard("l/tp e, e f -> l f/tp", xs.detach(), y.detach(), mesh=mesh, shapes={"tp": {"l": bad, "f": cs}})
    assert [(c.name, c.status) for c in es.last_candidates()] == [("alltoall_repartition", "rejected")]


def test_post_contraction_repartition():
    run_ranks(_repartition_after_contraction)


def _mesh2d(ctx):
    mesh = ctx.mesh((2, ctx.world_size // 2), ("dp", "sp"))
    sp, dp = mesh["sp"].get_group(), mesh["dp"].get_group()
    # BASELINE CPU config: a/sp b/dp, b/dp c -> a/sp c, then uneven gather of a
    a, b, c = 64, 32, 16
    torch.manual_seed(0)
    xf, yf = torch.randn(a, b), torch.randn(b, c)
    a_sh = es.compute_split_shapes(a, dist.get_world_size(sp))
    b_sh = es.compute_split_shapes(b, dist.get_world_size(dp))
    xs = _split(_split(xf, a_sh, 0, dist.get_rank(sp)), b_sh, 1, dist.get_rank(dp)).contiguous()
    ys = _split(yf, b_sh, 0, dist.get_rank(dp)).contiguous()
    z = es.einshard("a/sp b/dp, b/dp c -> a/sp c", xs, ys, mesh=mesh, shapes={"sp": a_sh, "dp": b_sh})
    assert _names() == ["identity_forward_allreduce_backward", "rank_local_einsum",
                        "allreduce_forward_identity_backward"]
    assert_close(z, _split(xf @ yf, a_sh, 0, dist.get_rank(sp)), rtol=1e-4, atol=1e-5)

    # a/dp k, k b/sp -> a/dp b/sp keeps every placement: a local operation, so
    # y's gradient is this rank's contribution (no replicated-gradient reduction)
    xk = torch.randn(8, 12)
    kb = torch.randn(12, 2 * dist.get_world_size(sp))
    x_s = _split(xk, [4, 4], 0, dist.get_rank(dp)).contiguous().requires_grad_(True)
    y_s = _split(kb, [2] * dist.get_world_size(sp), 1, dist.get_rank(sp)).contiguous().requires_grad_(True)
    z = es.einshard("a/dp k, k b/sp -> a/dp b/sp", x_s, y_s, mesh=mesh)
    full = xk @ kb
    assert_close(z, _split(_split(full, [4, 4], 0, dist.get_rank(dp)), [2] * dist.get_world_size(sp), 1,
                           dist.get_rank(sp)), rtol=1e-4, atol=1e-5)
    z.sum().backward()
    assert _names() == ["rank_local_einsum"]
    assert_close(y_s.grad, x_s.detach().t() @ torch.ones(4, 2), rtol=1e-4, atol=1e-5)

    # attention score pattern: key axis gathered, values contract the key shard
    q = torch.randn(2, 3, 8, 4)
    k = torch.randn(2, 3, 8, 4)
    P = dist.get_world_size(sp)
    qs = _split(q, [8 // P] * P if 8 % P == 0 else es.compute_split_shapes(8, P), 2, dist.get_rank(sp))
    ks = _split(k, [8 // P] * P if 8 % P == 0 else es.compute_split_shapes(8, P), 2, dist.get_rank(sp))
    s = es.einshard("b h q/sp d, b h k/sp d -> b h q/sp k", qs.contiguous(), ks.contiguous(), mesh=mesh)
    ref = torch.einsum("bhqd,bhkd->bhqk", q, k)
    assert_close(s, _split(ref, [8 // P] * P, 2, dist.get_rank(sp)), rtol=1e-4, atol=1e-5)


def test_mesh2d_contractions_and_attention_pattern():
    run_ranks(_mesh2d)


def _binary_owner_swap(ctx):
    mesh = ctx.mesh((ctx.world_size // 4, 2, 2), ("tp", "dp", "sp"))
    dp, sp = mesh["dp"].get_group(), mesh["sp"].get_group()
    k_sh, m_sh = [3, 3], [2, 2]
    xf = torch.randn(5, 6, 4)
    yf = torch.randn(6, 4, 7)
    xs = _split(_split(xf, k_sh, 1, dist.get_rank(dp)), m_sh, 2, dist.get_rank(sp)).contiguous()
    ys = _split(_split(yf, k_sh, 0, dist.get_rank(sp)), m_sh, 1, dist.get_rank(dp)).contiguous()
    z = es.einshard("a k/dp m/sp, k/sp m/dp b -> a b", xs, ys, mesh=mesh,
                    shapes={"dp": {"k": k_sh, "m": m_sh}, "sp": {"k": k_sh, "m": m_sh}})
    assert "owner_swap" in _names()
    assert_close(z, torch.einsum("akm,kmb->ab", xf, yf), rtol=1e-4, atol=1e-5)
    with pytest.raises(NotImplementedError, match="owner-swap-compatible"):
        es.einshard("a k/dp m/sp n/dp, k/sp m/dp n/tp b -> a b", torch.randn(2, 3, 2, 1), torch.randn(3, 2, 1, 4),
                    mesh=mesh)


def test_binary_owner_swap():
    run_ranks(_binary_owner_swap)
