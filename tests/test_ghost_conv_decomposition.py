"""The two-axis ghost conv (``conv_impl.conv2d_ghost_2d``) on the host: the
interior conv written into its column range plus the two transposed edge
strips equal a conv of the assembled haloed input, for ghost columns and rows
of any width and zero padding on either side; on 4 gloo ranks (mesh 2 x 2) the
ghost exchanges (columns of x, then rows of the column-haloed tensor that is
never assembled, corners included) feed it the rows and columns a conv of the
full tensor uses, and the training form's gradients (through the exchanges'
adjoints) equal the full conv's.  The conv itself is a torch stand-in with the native
kernel's contract (ghost rows, output column range)."""

import pytest
import torch
import torch.nn.functional as F

from dist_harness import run_ranks
from torch_einshard_b200.ops.conv_impl import conv2d_ghost_2d


def _torch_run(x, w, bias, ph, pw, ghosts=None, gtop=0, gbot=0, ghost_w0=0, out=None, out_w0=0):
    """The native conv's contract in torch (fp32): ghost rows above / below x
    taken from columns ghost_w0 .. of ``ghosts``; result into ``out``'s columns."""
    v = x
    if ghosts is not None:
        g = ghosts.narrow(2, ghost_w0, x.shape[2])
        v = torch.cat([g.narrow(1, 0, gtop), x, g.narrow(1, gtop, gbot)], 1)
    vp = F.pad(v.permute(0, 3, 1, 2), (pw[0], pw[1], ph[0], ph[1]))
    y = F.conv2d(vp, w.permute(0, 3, 1, 2), bias).permute(0, 2, 3, 1)
    if out is None:
        return y
    out[:, :, out_w0:out_w0 + y.shape[2]] = y
    return out


@pytest.mark.parametrize("gl,gr,gtop,gbot,ph,pw,K", [
    (1, 1, 1, 1, (0, 0), (0, 0), 3),
    (1, 0, 0, 1, (1, 0), (0, 1), 3),
    (0, 1, 1, 0, (0, 1), (1, 0), 3),
    (2, 2, 2, 2, (0, 0), (0, 0), 5),
    (0, 2, 0, 0, (2, 2), (2, 0), 5),
])
def test_interior_plus_strips_equal_the_assembled_conv(gl, gr, gtop, gbot, ph, pw, K):
    torch.manual_seed(0)
    B, H, W, C, O = 2, 7, 9, 3, 4
    full = torch.randn(B, gtop + H + gbot, gl + W + gr, C)
    x = full[:, gtop:gtop + H, gl:gl + W].contiguous()
    cols = torch.cat([full[:, gtop:gtop + H, :gl], full[:, gtop:gtop + H, gl + W:]], 2)
    ghosts = torch.cat([full[:, :gtop], full[:, gtop + H:]], 1) if gtop + gbot else None
    w = torch.randn(O, K, K, C)
    bias = torch.randn(O)
    got = conv2d_ghost_2d(x, ghosts, gtop, gbot, cols, gl, gr, w, bias, ph, pw, run=_torch_run)
    want = _torch_run(full, w, bias, ph, pw)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


def _mesh_body(ctx):
    from torch_einshard_b200.notation.parser import parse_sharding
    from torch_einshard_b200.ops.halo import _axes, halo_ghost_rows
    mesh = ctx.mesh((2, 2), ("sh", "sw"))
    rh, rw = mesh["sh"].get_local_rank(), mesh["sw"].get_local_rank()
    hs, ws = [5, 4], [6, 7]
    B, C, O, K = 2, 3, 4, 3
    full = torch.randn(B, sum(hs), sum(ws), C)  # the same on every rank (seeded)
    w = torch.randn(O, K, K, C)
    x = full[:, sum(hs[:rh]):sum(hs[:rh + 1]), sum(ws[:rw]):sum(ws[:rw + 1])].contiguous()
    spec = parse_sharding("b h/sh w/sw c -> b h/sh w/sw c")[0]
    axes = {a.name: a for a in _axes(spec)}
    shapes = {"sh": {"h": hs}, "sw": {"w": ws}}
    cols, gl, gr, zl, zr, _ = halo_ghost_rows(x, axes["w"], 2, 1, 1, mesh=mesh, shapes=shapes)
    vshape = list(x.shape)
    vshape[2] = gl + x.shape[2] + gr

    def slab(off, n):
        c = cols.narrow(1, off, n)
        return torch.cat([c.narrow(2, 0, gl), x.narrow(1, off, n), c.narrow(2, gl, gr)], 2)
    g, gtop, gbot, mlo, mhi, _ = halo_ghost_rows(x, axes["h"], 1, 1, 1, mesh=mesh, shapes=shapes, slab=slab,
                                                 shape=vshape)
    got = conv2d_ghost_2d(x, g, gtop, gbot, cols, gl, gr, w, None, (mlo, mhi), (zl, zr), run=_torch_run)
    want = _torch_run(full, w, None, (1, 1), (1, 1))
    want = want[:, sum(hs[:rh]):sum(hs[:rh + 1]), sum(ws[:rw]):sum(ws[:rw + 1])]
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)

    # training: the gradient of the haloed input goes back through the row
    # exchange's adjoint, then the column exchange's
    from torch_einshard_b200.ops.conv_impl import conv2d_ghost_2d_train
    _, _, _, _, _, adjoint_cols = halo_ghost_rows(x, axes["w"], 2, 1, 1, mesh=mesh, shapes=shapes)
    _, _, _, _, _, adjoint_rows = halo_ghost_rows(x, axes["h"], 1, 1, 1, mesh=mesh, shapes=shapes, slab=slab,
                                                  shape=vshape)
    xg = x.clone().requires_grad_(True)
    wg = w.clone().requires_grad_(True)
    bias = torch.randn(O, requires_grad=True)
    y = conv2d_ghost_2d_train(xg, g, gtop, gbot, cols, gl, gr, lambda dv: adjoint_cols(adjoint_rows(dv)), wg, bias,
                              (mlo, mhi), (zl, zr), run=_torch_run)
    fullg = full.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    br = bias.detach().clone().requires_grad_(True)
    yr = _torch_run(fullg, wr, br, (1, 1), (1, 1))
    dy_full = torch.randn_like(yr)  # the same on every rank (seeded)
    rows = slice(sum(hs[:rh]), sum(hs[:rh + 1]))
    colsl = slice(sum(ws[:rw]), sum(ws[:rw + 1]))
    y.backward(dy_full[:, rows, colsl])
    yr.backward(dy_full)
    torch.testing.assert_close(xg.grad, fullg.grad[:, rows, colsl], rtol=1e-4, atol=1e-4)
    dw, db = wg.grad.clone(), bias.grad.clone()
    torch.distributed.all_reduce(dw)
    torch.distributed.all_reduce(db)
    torch.testing.assert_close(dw, wr.grad, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(db, br.grad, rtol=1e-4, atol=1e-4)


def test_ghost_exchanges_on_a_2x2_mesh_feed_the_decomposition():
    run_ranks(_mesh_body, 4)
