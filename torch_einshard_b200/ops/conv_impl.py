"""Native implicit-GEMM conv2d for ``einconv`` (``_C.conv2d_implicit``).

The einconv path hands this module the halo-extended input (padding 0 from
here on), so the forward is a valid convolution.  Tensors are brought to NHWC
(batch axes flattened), weights to [O][KH][KW][C]; the kernel reads the input
windows straight from the NHWC tensor with shifted TMA boxes (no im2col).

Zero padding may differ per side (``pads`` values are ``p`` or ``(lo, hi)``):
the einconv path pads only where a sharded axis has no neighbour (the global
edge) and lets the kernel read zeros there.  Where the weights fit in shared
memory the forward runs on the CTA-pair kernel with resident weights
(``csrc/conv_pair.cu``), else on the weights-streaming kernel (``csrc/conv.cu``;
``EINSHARD_CONV_KERNEL=1`` forces it).

Backward: the input gradient runs on the same kernels as a full correlation of
dY with the flipped, channel-transposed weights (zero padding KH-1-lo, KH-1-hi
done by the TMA zero fill); the weight gradient runs on the split-K implicit-GEMM
kernel (``_C.conv2d_wgrad``: dY and the shifted input windows as MN-major
operands, fp32 partial tiles added atomically) when both channel counts are
multiples of 64, else ``torch.nn.grad.conv2d_weight``; the bias gradient is a
reduction.

Replaces the reference's ``F.conv2d`` call in ``einconv`` (``src/torch_einshard/conv.py:48-52``).
"""

import os

import torch

from . import _native

__all__ = ["conv2d_nhwc", "conv2d_native", "conv2d_ghost_rows", "conv2d_nhwc_ghost_rows", "conv2d_ghost_2d",
           "conv2d_ghost_2d_train", "pair_kernel_fits",
           "try_conv", "kernel_padding_ok"]

_KERNEL = int(os.environ.get("EINSHARD_CONV_KERNEL", "0"))


def _lohi(p):
    return (int(p[0]), int(p[1])) if isinstance(p, (tuple, list)) else (int(p), int(p))


def _run(mod, x, w, bias, ph, pw, ghosts=None, gtop=0, gbot=0, ghost_w0=0, out=None, out_w0=0):
    """ph, pw: (lo, hi) zero padding of the rows and the columns; ghosts: rows
    that continue x above (gtop) and below (gbot), [B, gtop + gbot, Wg, C] with
    x's columns at ghost_w0 .. ghost_w0 + W; out: write the result into
    columns out_w0 .. of this (wider) tensor instead of a new one."""
    B, H, W, _ = x.shape
    O, KH, KW, _ = w.shape
    Hv = H + gtop + gbot
    Ho, Wo = Hv + ph[0] + ph[1] - KH + 1, W + pw[0] + pw[1] - KW + 1
    if out is None:
        out = torch.empty(B, Ho, Wo, O, dtype=x.dtype, device=x.device)
    b = bias if bias is not None else torch.empty(0, dtype=torch.float32, device=x.device)
    g = ghosts.contiguous() if ghosts is not None else torch.empty(0, dtype=x.dtype, device=x.device)
    mod.conv2d_implicit(x, w, b, out, ph[0], pw[0], ph[1], pw[1], _KERNEL, g, gtop, gbot, ghost_w0, out_w0,
                        _native.error_word(x.device))
    return out


# Shared-memory budget of the CTA-pair kernel's resident weights (csrc/conv_pair.cu:
# 227 KB per block less 4 input stages of 17 KB, alignment and barriers).
_PAIR_WEIGHT_BYTES = 232448 - 1024 - 4 * 136 * 128 - 256


def pair_kernel_fits(C, O, KH, KW):
    """Whether the CTA-pair kernel (the only one that reads ghost rows) takes
    this shape: channels as its boxes need, and some output-channel tile whose
    weight slice fits in shared memory.  The extension answers when it is
    loaded (``conv_pair_otile``, the kernel's own choice); the same rule is
    restated here for hosts without it."""
    mod = _native.module()
    if mod is not None and hasattr(mod, "conv_pair_otile"):
        return mod.conv_pair_otile(int(C), int(O), int(KH), int(KW)) > 0
    if C % 64 or O % 16 or KW > 9:
        return False
    return any(ot <= O and O % ot == 0 and KH * KW * (C // 64) * (ot // 2) * 128 <= _PAIR_WEIGHT_BYTES
               for ot in (128, 64, 32, 16))


def _haloed_input_grad(grad, w, ph, pw, haloed):
    """Gradient of a conv's (haloed) input: the conv of dY with the flipped,
    channel-transposed kernel on the native kernels, else torch.  ``haloed()``
    builds the input (only the torch path needs it)."""
    O, KH, KW, C = w.shape
    if O % 64 == 0 and KH - 1 >= max(ph) and KW - 1 >= max(pw):
        wt = w.flip(1, 2).permute(3, 1, 2, 0).contiguous()  # [C][KH][KW][O]
        return _run(_native.require(), grad, wt, None, (KH - 1 - ph[0], KH - 1 - ph[1]),
                    (KW - 1 - pw[0], KW - 1 - pw[1]))
    v = haloed()
    xt = torch.nn.functional.pad(v.permute(0, 3, 1, 2), (pw[0], pw[1], ph[0], ph[1]))
    dv = torch.nn.grad.conv2d_input(xt.shape, w.permute(0, 3, 1, 2), grad.permute(0, 3, 1, 2))
    return dv[:, :, ph[0]:ph[0] + v.shape[1], pw[0]:pw[0] + v.shape[2]].permute(0, 2, 3, 1).contiguous()


def _haloed_weight_grad(v, grad, w, ph, pw):
    """Weight gradient of a conv over the haloed input ``v``."""
    O, KH, KW, C = w.shape
    if O % 64 == 0:
        dw = torch.empty(O, KH, KW, C, dtype=torch.float32, device=v.device)
        _native.require().conv2d_wgrad(v.contiguous(), grad, dw, ph[0], pw[0], ph[1], pw[1],
                                       _native.error_word(v.device))
        return dw.to(w.dtype)
    xt = torch.nn.functional.pad(v.permute(0, 3, 1, 2), (pw[0], pw[1], ph[0], ph[1]))
    return torch.nn.grad.conv2d_weight(xt, w.permute(0, 3, 1, 2).shape, grad.permute(0, 3, 1, 2)).permute(0, 2, 3, 1)


class _Conv2dGhostRows(torch.autograd.Function):
    """NHWC conv2d of the rows [ghosts above; x; ghosts below] without
    assembling them: the pair kernel reads x and the ghost tensor in place.
    Backward: the gradient of the whole haloed input from the flipped-kernel
    conv, handed to ``adjoint`` (the halo exchange's adjoint, which returns the
    ghost rows' share to their owners); the weight gradient over the haloed
    input, assembled only here."""

    @staticmethod
    def forward(ctx, x, ghosts, w, bias, gtop, gbot, ph, pw, adjoint):
        ctx.save_for_backward(x, ghosts, w)
        ctx.meta = (gtop, gbot, ph, pw, adjoint)
        ctx.has_bias = bias is not None
        ctx.bias_dtype = bias.dtype if bias is not None else None
        return _run(_native.require(), x, w, None if bias is None else bias.float().contiguous(), ph, pw,
                    ghosts, gtop, gbot)

    @staticmethod
    def backward(ctx, grad):
        x, g, w = ctx.saved_tensors
        gtop, gbot, ph, pw, adjoint = ctx.meta
        grad = grad.contiguous()
        gx = gw = gb = None

        def assembled():
            return torch.cat([g.narrow(1, 0, gtop), x, g.narrow(1, gtop, gbot)], 1)
        if ctx.needs_input_grad[0]:
            gx = adjoint(_haloed_input_grad(grad, w, ph, pw, assembled))
        if ctx.needs_input_grad[2]:
            gw = _haloed_weight_grad(assembled(), grad, w, ph, pw)
        if ctx.has_bias and ctx.needs_input_grad[3]:
            gb = grad.float().sum(dim=(0, 1, 2)).to(ctx.bias_dtype)
        return gx, None, gw, gb, None, None, None, None, None


def conv2d_ghost_rows(x, ghosts, gtop, gbot, adjoint, w, bias=None, ph=0, pw=0):
    """NHWC conv2d of [ghosts[:, :gtop]; x; ghosts[:, gtop:]] along the rows
    with zero padding ph / pw beyond them, on the CTA-pair kernel."""
    ph, pw = _lohi(ph), _lohi(pw)
    x, w = x.contiguous(), w.contiguous()
    return _Conv2dGhostRows.apply(x, ghosts.detach().contiguous(), w, bias, gtop, gbot, ph, pw, adjoint)


def _torch_pads(ph, pw):
    """F.pad / conv padding for the torch fallbacks: symmetric pads as conv padding,
    asymmetric ones as an explicit F.pad of the NCHW input."""
    return (ph[0], pw[0]) if ph[0] == ph[1] and pw[0] == pw[1] else None


class _Conv2dNHWC(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, bias, ph, pw):
        ctx.save_for_backward(x, w)
        ctx.pad = (ph, pw)
        ctx.has_bias = bias is not None
        ctx.bias_dtype = bias.dtype if bias is not None else None
        return _run(_native.require(), x, w, None if bias is None else bias.float().contiguous(), ph, pw)

    @staticmethod
    def backward(ctx, grad):
        x, w = ctx.saved_tensors
        grad = grad.contiguous()
        gx = gw = gb = None
        O, KH, KW, C = w.shape
        ph, pw = ctx.pad
        sym = _torch_pads(ph, pw)
        xt = x.permute(0, 3, 1, 2)
        if sym is None and not (O % 64 == 0 and KH - 1 >= max(ph) and KW - 1 >= max(pw)):
            # the torch fallbacks take symmetric padding only: pad the input explicitly
            xt = torch.nn.functional.pad(xt, (pw[0], pw[1], ph[0], ph[1]))
            sym = (0, 0)
        if ctx.needs_input_grad[0]:
            if O % 64 == 0 and KH - 1 >= max(ph) and KW - 1 >= max(pw):
                # full correlation with the flipped, channel-transposed kernel, cropped by the padding
                wt = w.flip(1, 2).permute(3, 1, 2, 0).contiguous()  # [C][KH][KW][O]
                gx = _run(_native.require(), grad, wt, None, (KH - 1 - ph[0], KH - 1 - ph[1]),
                          (KW - 1 - pw[0], KW - 1 - pw[1]))
            else:
                gx = torch.nn.grad.conv2d_input(xt.shape, w.permute(0, 3, 1, 2), grad.permute(0, 3, 1, 2),
                                                padding=sym)
                if xt.shape[2:] != x.shape[1:3]:
                    gx = gx[:, :, ph[0]:ph[0] + x.shape[1], pw[0]:pw[0] + x.shape[2]]
                gx = gx.permute(0, 2, 3, 1)
        if ctx.needs_input_grad[1] and O % 64 == 0:
            dw = torch.empty(O, KH, KW, C, dtype=torch.float32, device=x.device)
            _native.require().conv2d_wgrad(x, grad, dw, ph[0], pw[0], ph[1], pw[1], _native.error_word(x.device))
            gw = dw.to(w.dtype)
        elif ctx.needs_input_grad[1]:
            gw = torch.nn.grad.conv2d_weight(xt, w.permute(0, 3, 1, 2).shape, grad.permute(0, 3, 1, 2),
                                             padding=sym).permute(0, 2, 3, 1)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            gb = grad.float().sum(dim=(0, 1, 2)).to(ctx.bias_dtype)
        return gx, gw, gb, None, None


def supported(x, w_dtype, cin_size, ndim, dilation):
    """1-D convs run as 2-D ones of height 1 (``conv2d_nhwc``)."""
    return (x.is_cuda and ndim in (1, 2) and all(d == 1 for d in dilation) and x.dtype in (torch.bfloat16, torch.float16)
            and w_dtype == x.dtype and cin_size % 64 == 0)


def conv2d_native(x, w, bias=None, ph=0, pw=0):
    """NHWC conv2d with zero padding ph, pw (``p`` or ``(lo, hi)``): x [B, H, W, C],
    w [O, KH, KW, C] -> [B, H + lo + hi - KH + 1, W + lo + hi - KW + 1, O]."""
    ph, pw = _lohi(ph), _lohi(pw)
    x, w = x.contiguous(), w.contiguous()
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad or (bias is not None and bias.requires_grad)):
        return _Conv2dNHWC.apply(x, w, bias, ph, pw)
    return _run(_native.require(), x, w, None if bias is None else bias.float().contiguous(), ph, pw)


def conv2d_nhwc(mod, x, weight, bias, in_names, w_names, out_names, spatial, kernel, cin, cout, dilation,
                pads=None):
    """``pads``: {spatial name: zero padding ``p`` or ``(lo, hi)`` done by the kernel (TMA zero fill)}."""
    if not weight.is_cuda or not supported(x, weight.dtype, x.shape[in_names.index(cin)], len(spatial), dilation):
        return None
    pads = pads or {}
    batch = [n for n in in_names if n not in spatial and n != cin]
    xn = x.permute([in_names.index(n) for n in batch + list(spatial) + [cin]])
    lead = xn.shape[:len(batch)]
    xn = xn.reshape(-1, *xn.shape[len(batch):])
    wn = weight.permute([w_names.index(n) for n in [cout] + list(kernel) + [cin]])
    if len(spatial) == 1:  # a row of height 1: [B, L, C] -> [B, 1, L, C], [O, K, C] -> [O, 1, K, C]
        out = conv2d_native(xn.unsqueeze(1), wn.unsqueeze(1), bias, 0, pads.get(spatial[0], 0)).squeeze(1)
    else:
        out = conv2d_native(xn, wn, bias, pads.get(spatial[0], 0), pads.get(spatial[1], 0))
    out = out.reshape(*lead, *out.shape[1:])
    produced = batch + list(spatial) + [cout]
    return out.permute([produced.index(n) for n in out_names]).contiguous()


def conv2d_ghost_2d(x, ghosts, gtop, gbot, cols, gl, gr, w, bias, ph, pw, run=None):
    """Inference conv of a shard haloed along both image axes, without
    assembling the haloed shard.  x [B, H, W, C]; ghosts [B, gtop + gbot,
    gl + W + gr, C]: the rows above / below, including the corners; cols
    [B, H, gl + gr, C]: the columns left / right of x; ph / pw: zero padding
    beyond the ghosts.  The interior columns are one conv over x with ghost
    rows, written into its column range of the output; the P = gl + pw[0]
    left and Q = gr + pw[1] right output columns come from thin strips of the
    haloed input (KW - 1 + ghost columns wide), convolved transposed so that
    their long axis runs along the kernel's 256-pixel tiles.  ``run``: the
    conv of ``_run``'s contract (default: the native kernels)."""
    run = run or (lambda *a, **k: _run(_native.require(), *a, **k))
    B, H, W, C = x.shape
    O, KH, KW, _ = w.shape
    Hv = H + gtop + gbot
    Ho, Wo = Hv + ph[0] + ph[1] - KH + 1, gl + W + gr + pw[0] + pw[1] - KW + 1
    P, Q = gl + pw[0], gr + pw[1]
    bias32 = None if bias is None else bias.float().contiguous()
    out = torch.empty(B, Ho, Wo, O, dtype=x.dtype, device=x.device)
    run(x, w, bias32, ph, (0, 0), ghosts if gtop + gbot else None, gtop, gbot, gl, out, P)

    def strip(c0, c1):
        """Columns [c0, c1) of the haloed input (x's column 0 at index 0), all rows."""
        parts = []
        if c0 < 0:
            parts.append(cols.narrow(2, gl + c0, min(c1, 0) - c0))
        if c1 > 0 and c0 < W:
            parts.append(x.narrow(2, max(c0, 0), min(c1, W) - max(c0, 0)))
        if c1 > W:
            parts.append(cols.narrow(2, gl + max(c0, W) - W, c1 - max(c0, W)))
        mid = torch.cat(parts, 2)
        if gtop + gbot == 0:
            return mid
        g = ghosts.narrow(2, gl + c0, c1 - c0)
        return torch.cat([g.narrow(1, 0, gtop), mid, g.narrow(1, gtop, gbot)], 1)
    wt = w.transpose(1, 2).contiguous()  # [O][KW][KH][C]: the strips run transposed
    if P > 0:
        s = strip(-gl, KW - 1).transpose(1, 2).contiguous()
        out[:, :, :P] = run(s, wt, bias32, (pw[0], 0), ph).transpose(1, 2)
    if Q > 0:
        s = strip(W - KW + 1, W + gr).transpose(1, 2).contiguous()
        out[:, :, Wo - Q:] = run(s, wt, bias32, (0, pw[1]), ph).transpose(1, 2)
    return out


def _assemble_2d(x, ghosts, gtop, gbot, cols, gl, gr):
    """The haloed input [rows above; [cols left | x | cols right]; rows below]."""
    mid = torch.cat([cols.narrow(2, 0, gl), x, cols.narrow(2, gl, gr)], 2)
    if ghosts is None or gtop + gbot == 0:
        return mid
    return torch.cat([ghosts.narrow(1, 0, gtop), mid, ghosts.narrow(1, gtop, gbot)], 1)


class _Conv2dGhost2D(torch.autograd.Function):
    """Training form of ``conv2d_ghost_2d``: backward forms the gradient of the
    whole haloed input (one flipped-kernel conv), hands it to ``adjoint`` (the
    row exchange's adjoint, then the column exchange's, which return every
    ghost's share to its owner) and takes the weight gradient over the haloed
    input, assembled only in backward.  ``grads``: the input- and weight-
    gradient functions (the native ones by default)."""

    @staticmethod
    def forward(ctx, x, ghosts, cols, w, bias, meta, adjoint):
        gtop, gbot, gl, gr, ph, pw, run, grads = meta
        ctx.save_for_backward(x, ghosts, cols, w)
        ctx.meta, ctx.adjoint = meta, adjoint
        ctx.has_bias = bias is not None
        ctx.bias_dtype = bias.dtype if bias is not None else None
        return conv2d_ghost_2d(x, ghosts, gtop, gbot, cols, gl, gr, w, bias, ph, pw, run=run)

    @staticmethod
    def backward(ctx, grad):
        x, g, cols, w = ctx.saved_tensors
        gtop, gbot, gl, gr, ph, pw, _, grads = ctx.meta
        input_grad, weight_grad = grads or (_haloed_input_grad, _haloed_weight_grad)
        grad = grad.contiguous()
        gx = gw = gb = None
        v = None

        def assembled():
            return _assemble_2d(x, g, gtop, gbot, cols, gl, gr)
        if ctx.needs_input_grad[0]:
            gx = ctx.adjoint(input_grad(grad, w, ph, pw, assembled))
        if ctx.needs_input_grad[3]:
            v = assembled() if v is None else v
            gw = weight_grad(v, grad, w, ph, pw)
        if ctx.has_bias and ctx.needs_input_grad[4]:
            gb = grad.float().sum(dim=(0, 1, 2)).to(ctx.bias_dtype)
        return gx, None, None, gw, gb, None, None


def conv2d_ghost_2d_train(x, ghosts, gtop, gbot, cols, gl, gr, adjoint, w, bias=None, ph=0, pw=0, run=None,
                          grads=None):
    """``conv2d_ghost_2d`` with gradients: ``adjoint(dv)`` maps the gradient of
    the haloed input to x's (the exchanges' adjoints).  ``run`` / ``grads``:
    stand-ins for the native conv and its input / weight gradients."""
    ph, pw = _lohi(ph), _lohi(pw)
    ghosts = ghosts.detach().contiguous() if ghosts is not None else None
    meta = (gtop, gbot, gl, gr, ph, pw, run, grads)
    return _Conv2dGhost2D.apply(x.contiguous(), ghosts, cols.detach().contiguous(), w.contiguous(), bias, meta,
                                adjoint)


def conv2d_nhwc_ghost_rows(x, ghosts, gtop, gbot, adjoint, weight, bias, in_names, w_names, out_names, spatial,
                           kernel, cin, cout, pads):
    """einconv's named-axis call with ghost rows along ``spatial[0]`` (the NHWC
    H axis): x and ghosts in ``in_names`` order; ``adjoint`` maps a gradient of
    the haloed input (in ``in_names`` order) to x's gradient."""
    batch = [n for n in in_names if n not in spatial and n != cin]
    order = [in_names.index(n) for n in batch + list(spatial) + [cin]]
    inverse = [order.index(d) for d in range(len(order))]
    xn = x.permute(order)
    lead = xn.shape[:len(batch)]
    xn = xn.reshape(-1, *xn.shape[len(batch):])
    gn = ghosts.permute(order).reshape(-1, *ghosts.permute(order).shape[len(batch):])

    def adjoint_nhwc(dv):
        d = adjoint(dv.reshape(*lead, *dv.shape[1:]).permute(inverse))
        return d.permute(order).reshape(-1, *d.permute(order).shape[len(batch):])
    wn = weight.permute([w_names.index(n) for n in [cout] + list(kernel) + [cin]])
    out = conv2d_ghost_rows(xn, gn, gtop, gbot, adjoint_nhwc, wn, bias, pads.get(spatial[0], 0),
                            pads.get(spatial[1], 0))
    out = out.reshape(*lead, *out.shape[1:])
    produced = batch + list(spatial) + [cout]
    return out.permute([produced.index(n) for n in out_names]).contiguous()


def try_conv(x, weight, bias, in_names, w_names, out_names, spatial, kernel, cin, cout, dilation, pads=None):
    """The native implicit-GEMM convolution of einconv's named-axis call, or
    None outside its envelope (not CUDA bf16/fp16, not 2-D, dilation != 1,
    channel counts the TMA boxes cannot address); einconv then uses
    ``torch.nn.functional``."""
    mod = _native.module()
    if mod is None or not hasattr(mod, "conv2d_implicit") or not x.is_cuda:
        return None
    return conv2d_nhwc(mod, x, weight, bias, in_names, w_names, out_names, spatial, kernel, cin, cout, dilation,
                       pads)


def kernel_padding_ok(x, weight, cin_size, spatial, dilation):
    """True when the native kernel would run and can zero-pad by itself."""
    mod = _native.module()
    if mod is None or not hasattr(mod, "conv2d_implicit") or not x.is_cuda:
        return False
    return supported(x, weight.dtype, cin_size, len(spatial), dilation)
