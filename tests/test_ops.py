"""Local and distributed einroll / einhalo / einwindow / einconv / einfft / einsum."""

import pytest
import torch
import torch.distributed as dist
import torch.nn.functional as F

import torch_einshard_b200 as es
from conftest import assert_close
from dist_harness import run_ranks


def _split(full, shapes, dim, rank):
    return torch.split(full, shapes, dim=dim)[rank]


# ------------------------------------------------------------------ local

def test_local_einsum_variants():
    x, y = torch.randn(4, 5, 8, 6), torch.randn(5, 6, 8, 3)
    assert_close(es.einshard("a b k c, b c l d -> k l d a", x, y), torch.einsum("abkc,bcld->klda", x, y))
    assert [s.name for s in es.last_plan()] == ["rank_local_einsum"]
    assert_close(es.einshard("i, j -> i j", torch.ones(3), torch.ones(4), optimize="memory"), torch.ones(3, 4))
    with pytest.raises(ValueError, match="either optimize or policy"):
        es.einshard("i -> i", torch.ones(3), optimize="memory", policy=es.PlanPolicy.from_mode("training"))
    m = torch.randn(5, 5)
    assert_close(es.einshard("i i -> i", m), torch.diagonal(m))
    x, w = torch.randn(2, 3, 4), torch.randn(4, 5)
    assert_close(es.einshard("... c, c o -> ... o", x, w), x @ w)
    assert_close(es.einshard("... c -> c", x), x.sum((0, 1)))
    x = torch.randn(2, 3, 12, 5)
    assert_close(es.einshard("... (h p) c -> ... h p c", x, sizes={"p": 4}), x.reshape(2, 3, 3, 4, 5))
    x = torch.randn(2, 12, 5)
    assert_close(es.einshard("b (h p) c -> b c h p", x, sizes={"h": 3}), x.reshape(2, 3, 4, 5).permute(0, 3, 1, 2))
    assert_close(es.einshard("b h p c -> b (h p) c", x.reshape(2, 3, 4, 5)), x)
    with pytest.raises(ValueError, match="Cannot infer multiple factor sizes"):
        es.einshard("b (h p) c -> b h p c", x)
    with pytest.raises(NotImplementedError, match="local reshape operations"):
        es.einshard("b (h p) c -> b h/sp p c", x, sizes={"p": 4})
    x = torch.randn(2, 3, 8, 10, 5)
    z = es.einshard("b t [*spatial *window] c -> (b *spatial) t *window c", x,
                    families={"spatial": ("h", "w"), "window": ("wh", "ww")}, sizes={"window": (4, 5)})
    assert_close(z, x.reshape(2, 3, 2, 4, 2, 5, 5).permute(0, 2, 4, 1, 3, 5, 6).reshape(8, 3, 4, 5, 5))


def test_local_roll_halo_window():
    x = torch.randn(2, 3, 4, 5, 6, 7)
    z = es.einroll("b t *spatial c", x, {"spatial": (1, -2, 3)}, families={"spatial": ("h", "w", "d")})
    assert_close(z, torch.roll(x, shifts=(1, -2, 3), dims=(2, 3, 4)))
    with pytest.raises(ValueError, match="Distributed einroll operations require mesh"):
        es.einroll("a/dp b", torch.randn(4, 3), {"a": 1})
    v = torch.arange(5, dtype=torch.float32)
    assert_close(es.einhalo("h", v, {"h": (2, 1)}, fill=-1), torch.tensor([-1., -1, 0, 1, 2, 3, 4, -1]))
    assert_close(es.einhalo("h", v, {"h": (2, 1)}, boundary="periodic"), torch.tensor([3., 4, 0, 1, 2, 3, 4, 0]))
    assert_close(es.einhalo("h", v, {"h": (2, 1)}, boundary="replicate"), torch.tensor([0., 0, 0, 1, 2, 3, 4, 4]))
    with pytest.raises(ValueError, match="Halo axis 'w'"):
        es.einhalo("h", v, {"w": 1})
    with pytest.raises(ValueError, match="periodic-pad an empty axis"):
        es.einhalo("h", torch.empty(0), {"h": 1}, boundary="periodic")
    with pytest.raises(NotImplementedError, match="factored axes"):
        es.einhalo("(h p)", torch.randn(6), {"h": 1})
    with pytest.raises(ValueError, match="appears more than once"):
        es.einhalo("h h", torch.randn(3, 3), {"h": 1})
    img = torch.randn(2, 6, 7, 3)
    win = es.einwindow("b h w c -> b h w kh kw c", img, {"h": "kh", "w": "kw"}, {"h": 1, "w": 1})
    padded = F.pad(img, (0, 0, 1, 1, 1, 1))
    ref = padded.unfold(1, 3, 1).unfold(2, 3, 1).permute(0, 1, 2, 4, 5, 3)
    assert_close(win, ref)
    with pytest.raises(ValueError, match="exactly the input axes plus"):
        es.einwindow("b h w c -> b h w c", img, {"h": "kh"}, {"h": 1})


def test_local_conv_matches_torch():
    x = torch.randn(2, 9, 11, 4, requires_grad=True)
    w = torch.randn(5, 4, 3, 3, requires_grad=True)
    bias = torch.randn(5, requires_grad=True)
    z = es.einconv("b h w c, o c kh kw -> b h w o", x, w, {"h": "kh", "w": "kw"}, bias=bias)
    ref = F.conv2d(x.permute(0, 3, 1, 2), w, bias, padding=1).permute(0, 2, 3, 1)
    assert_close(z, ref, rtol=1e-4, atol=1e-5)
    z.sum().backward()
    for mode in ("conv", "none"):
        z2 = es.einconv("b h w c, o c kh kw -> b h w o", x, w, {"h": "kh", "w": "kw"}, checkpoint=mode)
        assert_close(z2, F.conv2d(x.permute(0, 3, 1, 2), w, padding=1).permute(0, 2, 3, 1), rtol=1e-4, atol=1e-5)
    with pytest.raises(NotImplementedError, match="stride=1"):
        es.einconv("b h w c, o c kh kw -> b h w o", x, w, {"h": "kh", "w": "kw"}, stride=2)
    with pytest.raises(ValueError, match="exactly one input channel axis"):
        es.einconv("b h w c d, o c d kh kw -> b h w o", torch.randn(1, 4, 4, 2, 2), torch.randn(3, 2, 2, 3, 3),
                   {"h": "kh", "w": "kw"})
    with pytest.raises(ValueError, match="preserve the spatial length"):
        es.einconv("b h w c, o c kh kw -> b h w o", x, w, {"h": "kh", "w": "kw"}, padding={"h": 0, "w": 1})


def test_local_fft():
    x = torch.randn(3, 8, dtype=torch.complex64)
    assert_close(es.einfft("b x -> b k", x, axes={"x": "k"}), torch.fft.fft(x, dim=1), rtol=1e-4, atol=1e-4)
    assert_close(es.einfft("b x -> b x", x, axes=["x"], inverse=True, norm="ortho"),
                 torch.fft.ifft(x, dim=1, norm="ortho"), rtol=1e-4, atol=1e-4)
    y = torch.randn(4, 6, 8, dtype=torch.complex64)
    assert_close(es.einfft("a b c -> c kb ka", y, axes={"a": "ka", "b": "kb"}),
                 torch.fft.fftn(y, dim=(0, 1)).permute(2, 1, 0), rtol=1e-4, atol=1e-4)
    r = torch.randn(3, 10)
    spec = es.einfft("b t -> b f", r, axes={"t": "f"}, real=True)
    assert_close(spec, torch.fft.rfft(r, dim=1), rtol=1e-4, atol=1e-4)
    back = es.einfft("b f -> b t", spec, axes={"f": "t"}, real=True, inverse=True, signal_sizes={"t": 10})
    assert_close(back, r, rtol=1e-4, atol=1e-4)
    with pytest.raises(ValueError, match="partial"):
        es.einfft("b x // tp -> b k", x, axes={"x": "k"})
    with pytest.raises(TypeError, match="not a string"):
        es.einfft("b t -> b f", x, axes="t")
    info = es.einfft("b x -> x b", torch.randn(2, 3), axes=[], explain=True)
    assert info["path"] == "layout-only"


# ------------------------------------------------------------------ distributed

def _dist_roll_halo(ctx):
    mesh = ctx.mesh((ctx.world_size,), ("dp",))
    group = mesh["dp"].get_group()
    rank, P = dist.get_rank(group), dist.get_world_size(group)
    for rows, shift in ((P * 3, 2), (P * 3, -2), (P * 3 + 1, -3), (P * 3, 3)):
        shapes = es.compute_split_shapes(rows, P)
        full = torch.randn(rows, 5)
        x = _split(full, shapes, 0, rank).clone().requires_grad_(True)
        z = es.einroll("a/dp b", x, {"a": shift}, mesh=mesh, shapes=shapes)
        assert_close(z, _split(torch.roll(full, shifts=shift, dims=0), shapes, 0, rank))
        z.sum().backward()
        assert_close(x.grad, torch.ones_like(x))
    shapes = [3] * P
    full = torch.randn(3 * P, 5)
    with pytest.warns(RuntimeWarning, match="gather/roll/split fallback"):
        z = es.einroll("a/dp b", _split(full, shapes, 0, rank).contiguous(), {"a": 2}, mesh=mesh)
    assert_close(z, _split(torch.roll(full, 2, 0), shapes, 0, rank))

    # halos over uneven shards, including halos wider than a shard
    for boundary in ("constant", "periodic", "replicate"):
        for left, right in ((1, 1), (2, 0), (4, 5)):
            shapes = es.compute_split_shapes(P * 3 + 2, P)
            full = torch.randn(sum(shapes), 3)
            x = _split(full, shapes, 0, rank).clone().requires_grad_(True)
            z = es.einhalo("h/dp c", x, {"h": (left, right)}, boundary=boundary, fill=-2.0, mesh=mesh,
                           shapes=shapes)
            start = sum(shapes[:rank])
            idx = torch.arange(start - left, start + shapes[rank] + right)
            if boundary == "periodic":
                ref = full[idx.remainder(full.shape[0])]
            elif boundary == "replicate":
                ref = full[idx.clamp(0, full.shape[0] - 1)]
            else:
                ref = torch.full((len(idx), 3), -2.0)
                ok = (idx >= 0) & (idx < full.shape[0])
                ref[ok] = full[idx[ok]]
            assert_close(z, ref)
            z.sum().backward()
            counts = torch.zeros(full.shape[0])
            valid = idx if boundary == "periodic" else idx[(idx >= 0) & (idx < full.shape[0])]
            if boundary == "replicate":
                valid = idx.clamp(0, full.shape[0] - 1)
            if boundary == "periodic":
                valid = idx.remainder(full.shape[0])
            counts.index_add_(0, valid, torch.ones(len(valid)))
            total = counts.clone()
            dist.all_reduce(total, group=group)
            assert_close(x.grad[:, 0], _split(total, shapes, 0, rank))


def test_distributed_roll_and_halo():
    run_ranks(_dist_roll_halo)


def _dist_conv_window(ctx):
    mesh = ctx.mesh((2, ctx.world_size // 2), ("sp_h", "sp_w"))
    hg, wg = mesh["sp_h"].get_group(), mesh["sp_w"].get_group()
    H, W = 9, 2 * dist.get_world_size(wg) + 1
    hs, ws = es.compute_split_shapes(H, 2), es.compute_split_shapes(W, dist.get_world_size(wg))
    img = torch.randn(2, H, W, 3)
    weight = torch.randn(4, 3, 3, 3)
    local = _split(_split(img, hs, 1, dist.get_rank(hg)), ws, 2, dist.get_rank(wg)).contiguous()
    shapes = {"sp_h": hs, "sp_w": ws}
    z = es.einconv("b h/sp_h w/sp_w c, o c kh kw -> b h/sp_h w/sp_w o", local, weight, {"h": "kh", "w": "kw"},
                   mesh=mesh, shapes=shapes)
    ref = F.conv2d(img.permute(0, 3, 1, 2), weight, padding=1).permute(0, 2, 3, 1)
    assert_close(z, _split(_split(ref, hs, 1, dist.get_rank(hg)), ws, 2, dist.get_rank(wg)), rtol=1e-4, atol=1e-4)
    win = es.einwindow("b h/sp_h w/sp_w c -> b h/sp_h w/sp_w kh kw c", local, {"h": "kh", "w": "kw"},
                       {"h": 1, "w": 1}, mesh=mesh, shapes=shapes)
    out = es.einshard("b h/sp_h w/sp_w kh kw c, o c kh kw -> b h/sp_h w/sp_w o", win, weight)
    assert_close(out, z, rtol=1e-4, atol=1e-4)


def test_distributed_conv_and_window():
    run_ranks(_dist_conv_window)


def _dist_fft(ctx):
    mesh = ctx.mesh((ctx.world_size,), ("tp",))
    group = mesh["tp"].get_group()
    rank, P = dist.get_rank(group), dist.get_world_size(group)
    size = P * P * 3
    shapes = es.compute_split_shapes(size, P)
    full = torch.randn(2, size, dtype=torch.complex64)
    x = _split(full, shapes, 1, rank).contiguous().requires_grad_(True)
    for inverse in (False, True):
        for norm in (None, "ortho", "forward"):
            z = es.einfft("b x/tp -> b k/tp", x, axes={"x": "k"}, mesh=mesh, shapes={"tp": {"x": shapes, "k": shapes}},
                          inverse=inverse, norm=norm)
            fn = torch.fft.ifftn if inverse else torch.fft.fftn
            assert_close(z, _split(fn(full, dim=(1,), norm=norm), shapes, 1, rank), rtol=1e-4, atol=1e-4)
    info = es.einfft("b x/tp -> b k/tp", x, axes={"x": "k"}, mesh=mesh, shapes={"tp": {"x": shapes, "k": shapes}},
                     explain=True)
    assert info["fast_path"] is True and info["path"] == "distributed-fftn"
    z = es.einfft("b x/tp -> b k/tp", x, axes={"x": "k"}, mesh=mesh, shapes={"tp": {"x": shapes, "k": shapes}})
    g = torch.randn(2, size, dtype=torch.complex64)
    z.backward(_split(g, shapes, 1, rank))
    fr = full.clone().requires_grad_(True)
    torch.fft.fftn(fr, dim=(1,)).backward(g)
    assert_close(x.grad, _split(fr.grad, shapes, 1, rank), rtol=1e-4, atol=1e-4)

    # slab layout (transform axes trade the mesh dim): b x/tp y -> b kx ky/tp
    X, Y = 2 * P, 3 * P
    vol = torch.randn(2, X, Y, dtype=torch.complex64)
    xs_ = es.compute_split_shapes(X, P)
    ys_ = es.compute_split_shapes(Y, P)
    slab = _split(vol, xs_, 1, rank).contiguous()
    z = es.einfft("b x/tp y -> b kx ky/tp", slab, axes={"x": "kx", "y": "ky"}, mesh=mesh,
                  shapes={"tp": {"x": xs_, "ky": ys_}})
    assert_close(z, _split(torch.fft.fftn(vol, dim=(1, 2)), ys_, 2, rank), rtol=1e-4, atol=1e-4)
    info = es.einfft("b x/tp y -> b kx ky/tp", slab, axes={"x": "kx", "y": "ky"}, mesh=mesh,
                     shapes={"tp": {"x": xs_, "ky": ys_}}, explain=True)
    assert info["path"] == "distributed-fftn-slab"
    back = es.einfft("b kx ky/tp -> b x/tp y", z, axes={"kx": "x", "ky": "y"}, mesh=mesh, inverse=True,
                     shapes={"tp": {"ky": ys_, "x": xs_}})
    assert_close(back, slab, rtol=1e-4, atol=1e-4)

    # shared mesh dim with a non-transform axis stays rejected
    with pytest.raises(NotImplementedError, match="cannot share a mesh dimension"):
        es.einfft("b/tp x/tp -> b/tp k/tp", torch.randn(2, 2 * P), axes={"x": "k"}, real=True, mesh=mesh,
                  shapes={"tp": {"b": [1] * P, "x": [2] * P, "k": [2] * P}})


def test_distributed_fft():
    run_ranks(_dist_fft)
