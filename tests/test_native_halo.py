"""Native halo exchange (staged boundary slabs over NVLink) on 2+ GPUs against
the same halo built from the full tensor: uneven shards, a halo wider than a
neighbour's shard, periodic and constant boundaries, forward and the adjoint
scatter-add, and einconv over a sharded spatial axis against a local conv of
the full input: the first image axis sharded (ghost rows read in place, with
gradients) and the second (ghost columns, interior conv plus transposed edge
strips, inference and with gradients)."""

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 or more CUDA devices", allow_module_level=True)

from gpu_harness import run_gpus  # noqa: E402


def _body(rank, world):
    import torch.distributed as dist
    import torch.nn.functional as F
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native
    from torch_einshard_b200.parallel import symmetric

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("sp",))
    assert es.setup_native_comm(mesh)
    calls = []
    comm = symmetric.communicator_for(mesh["sp"].get_group())
    real = comm.halo_gather

    def spy(*a, **k):
        out = real(*a, **k)
        calls.append(out is not None)
        return out
    comm.halo_gather = spy

    shapes = [3 + 2 * p for p in range(world)]
    offs = [sum(shapes[:p]) for p in range(world)]
    total = sum(shapes)
    torch.manual_seed(11)
    full = torch.randn(2, total, 5, device="cuda", dtype=torch.float32)
    mine = full[:, offs[rank]:offs[rank] + shapes[rank]].contiguous().requires_grad_(True)
    for left, right, boundary in ((1, 1, "constant"), (2, 4, "periodic"), (4, 1, "constant")):
        got = es.einhalo("b h/sp c", mine, {"h": (left, right)}, boundary=boundary, mesh=mesh,
                         shapes={"sp": shapes})
        rows = torch.arange(offs[rank] - left, offs[rank] + shapes[rank] + right, device="cuda")
        if boundary == "periodic":
            want = full[:, rows % total]
        else:
            want = F.pad(full, (0, 0, left, right))[:, rows + left]
        torch.testing.assert_close(got, want)
        g = torch.randn_like(got)
        (grad,) = torch.autograd.grad(got, mine, g)
        # the adjoint on the full tensor: every haloed element's gradient returns to its owner
        full_g = torch.zeros_like(full)
        sizes = torch.tensor([g.shape[1]], device="cuda")
        all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
        dist.all_gather(all_sizes, sizes)
        for p in range(world):
            piece = torch.empty(2, int(all_sizes[p].item()), 5, device="cuda")
            if p == rank:
                piece.copy_(g)
            dist.broadcast(piece, p)
            rows = torch.arange(offs[p] - left, offs[p] + shapes[p] + right, device="cuda")
            if boundary == "periodic":
                full_g.index_add_(1, rows % total, piece)
            else:
                keep = (rows >= 0) & (rows < total)
                full_g.index_add_(1, rows[keep], piece[:, keep])
        torch.testing.assert_close(grad, full_g[:, offs[rank]:offs[rank] + shapes[rank]], rtol=1e-5, atol=1e-5)
    assert calls and all(calls), "the native halo exchange declined"

    # einconv over a sharded spatial axis (bf16, native implicit-GEMM conv)
    H, W, C, O = 8 * world, 16, 64, 64
    x = torch.randn(2, H, W, C, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(3, 3, C, O, device="cuda", dtype=torch.bfloat16) * 0.05
    dist.broadcast(x, 0)
    dist.broadcast(w, 0)
    hs = [H // world] * world
    xl = x[:, rank * hs[0]:(rank + 1) * hs[0]].contiguous()
    # forward and backward: the rows are sharded, so the conv reads the shard and
    # its neighbours' ghost rows in place (no haloed copy)
    ghost_calls = []
    from torch_einshard_b200.ops import conv as conv_mod
    real_ghosts = conv_mod.halo_ghost_rows
    conv_mod.halo_ghost_rows = lambda *a, **k: ghost_calls.append(1) or real_ghosts(*a, **k)
    xg = xl.clone().requires_grad_(True)
    wg = w.clone().requires_grad_(True)
    got = es.einconv("b h/sp w c, kh kw c o -> b h/sp w o", xg, wg, {"h": "kh", "w": "kw"}, mesh=mesh,
                     shapes={"sp": hs}, checkpoint=None)
    conv_mod.halo_ghost_rows = real_ghosts
    assert ghost_calls, "the ghost-row conv path was not taken"
    xr = x.float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    ref = F.conv2d(xr.permute(0, 3, 1, 2), wr.permute(3, 2, 0, 1), padding=1).permute(0, 2, 3, 1)
    mine = ref[:, rank * hs[0]:(rank + 1) * hs[0]]
    assert (got.float() - mine).abs().max().item() <= 3e-2 * (mine.abs().max().item() + 1)
    gy = torch.randn(ref.shape, device="cuda", dtype=torch.bfloat16)
    dist.broadcast(gy, 0)
    got.backward(gy[:, rank * hs[0]:(rank + 1) * hs[0]])
    ref.backward(gy.float())
    want_dx = xr.grad[:, rank * hs[0]:(rank + 1) * hs[0]]
    assert (xg.grad.float() - want_dx).abs().max().item() <= 3e-2 * (want_dx.abs().max().item() + 1)
    dw = wg.grad.float()
    dist.all_reduce(dw)  # each rank holds its shard's share of the weight gradient
    assert (dw - wr.grad).abs().max().item() <= 3e-2 * (wr.grad.abs().max().item() + 1)

    # inference with the second image axis sharded: ghost columns exchanged as a
    # thin tensor, interior conv plus transposed edge strips (no haloed copy)
    cols_calls = []
    real_2d = conv_mod.conv_impl.conv2d_ghost_2d
    conv_mod.conv_impl.conv2d_ghost_2d = lambda *a, **k: cols_calls.append(1) or real_2d(*a, **k)
    Wd = 32 * world
    xw = torch.randn(2, 12, Wd, C, device="cuda", dtype=torch.bfloat16)
    dist.broadcast(xw, 0)
    ws_ = [Wd // world] * world
    xwl = xw[:, :, rank * ws_[0]:(rank + 1) * ws_[0]].contiguous()
    with torch.no_grad():
        got = es.einconv("b h w/sp c, kh kw c o -> b h w/sp o", xwl, w, {"h": "kh", "w": "kw"}, mesh=mesh,
                         shapes={"sp": ws_}, checkpoint=None)
    conv_mod.conv_impl.conv2d_ghost_2d = real_2d
    assert cols_calls, "the two-axis ghost conv path was not taken"
    ref = F.conv2d(xw.float().permute(0, 3, 1, 2), w.float().permute(3, 2, 0, 1), padding=1).permute(0, 2, 3, 1)
    ref = ref[:, :, rank * ws_[0]:(rank + 1) * ws_[0]]
    assert (got.float() - ref).abs().max().item() <= 3e-2 * (ref.abs().max().item() + 1)
    # the same with gradients: back through the column exchange's adjoint
    xwg = xwl.clone().requires_grad_(True)
    wwg = w.clone().requires_grad_(True)
    got = es.einconv("b h w/sp c, kh kw c o -> b h w/sp o", xwg, wwg, {"h": "kh", "w": "kw"}, mesh=mesh,
                     shapes={"sp": ws_}, checkpoint=None)
    xr = xw.float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    ref = F.conv2d(xr.permute(0, 3, 1, 2), wr.permute(3, 2, 0, 1), padding=1).permute(0, 2, 3, 1)
    gy = torch.randn(ref.shape, device="cuda", dtype=torch.bfloat16)
    dist.broadcast(gy, 0)
    got.backward(gy[:, :, rank * ws_[0]:(rank + 1) * ws_[0]])
    ref.backward(gy.float())
    want_dx = xr.grad[:, :, rank * ws_[0]:(rank + 1) * ws_[0]]
    assert (xwg.grad.float() - want_dx).abs().max().item() <= 3e-2 * (want_dx.abs().max().item() + 1)
    dw = wwg.grad.float()
    dist.all_reduce(dw)
    assert (dw - wr.grad).abs().max().item() <= 3e-2 * (wr.grad.abs().max().item() + 1)
    torch.cuda.synchronize()
    _native.check_errors()


def test_native_halo_2gpus():
    run_gpus(_body, 2, timeout=300)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_native_halo_4gpus():
    run_gpus(_body, 4, timeout=300)


@pytest.mark.skipif(torch.cuda.device_count() < 8, reason="needs 8 GPUs")
def test_native_halo_8gpus():
    run_gpus(_body, 8, timeout=300)
