"""``einconv``: halo exchange followed by a same-length convolution.

A call is handled in three stages.

1. Analysis (``_Analysis``): the named-axis formula, the windows mapping and the
   numeric arguments are reduced to roles: batch axes, spatial (window source)
   axes, kernel (window) axes, one input and one output channel axis, plus the
   per-axis padding.  The checks form one ordered rule table (``_RULES``); the
   first rule that fails raises.  The table keeps the reference's error types,
   texts and order (user code and tests match them): one input channel axis,
   one output channel axis, local weight and channel axes, stride 1, groups 1,
   padding that preserves every spatial length.
2. Layout (``_Layout``): the permutations that bring the operands into the
   order the chosen kernel reads.  The native implicit-GEMM kernel
   (``csrc/conv.cu``, tcgen05, no im2col) reads channels-last operands:
   input [batch, spatial..., C], weight [O, taps..., C] and writes
   [batch, spatial..., O]; ``torch.nn.functional.conv{1,2,3}d`` (every case
   outside the native envelope) reads channels-first ones.  Local spatial axes
   with a zero boundary are padded by the native kernel itself (TMA zero fill),
   so no padded copy of the input is made for them; every other axis gets its
   halo (``ops/halo.py``) first.
3. Execution with the checkpoint mode: ``"full"`` (default; halo and conv
   recomputed in backward), ``"conv"`` (only the convolution) or off.

Contract of ``src/torch_einshard/conv.py:64-210``.
"""

from dataclasses import dataclass
from functools import cached_property

import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as torch_checkpoint

from ..notation.families import cached_expand_axis_families, expand_family_mapping
from ..notation.parser import parse_sharding
from ..notation.spec import EllipsisAxis
from . import conv_impl
from .halo import halo_ghost_rows, halo_tensor, halo_tensor_unpadded, normalize_halo, pad_dim

__all__ = ["einconv"]

_TORCH_CONV = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}


def _axes(spec):
    return spec.axes if hasattr(spec, "axes") else spec


def _per_dim(value, ndim, label):
    values = (value,) * ndim if isinstance(value, int) else tuple(value)
    if len(values) != ndim:
        raise ValueError(f"{label} must have {ndim} values")
    return values


class _Analysis:
    """Roles of every axis of an einconv call, derived on demand (the rules
    below read them in order, so a property is only computed once the rules
    before it have passed)."""

    def __init__(self, specs, windows, weight, padding, stride, dilation, groups, families):
        self.in_spec, self.w_spec, self.out_spec = specs
        self.windows, self.weight = windows, weight
        self.padding, self.stride_arg, self.dilation_arg = padding, stride, dilation
        self.groups, self.families = groups, families

    def names(self, spec, label):
        seen = []
        for axis in _axes(spec):
            if isinstance(axis, EllipsisAxis):
                raise NotImplementedError(f"einconv does not support ellipsis axes in {label}")
            if not hasattr(axis, "name"):
                raise NotImplementedError(f"einconv does not support factored axes in {label}")
            if axis.name in seen:
                raise ValueError(f"Axis {axis.name!r} appears more than once in {label}")
            seen.append(axis.name)
        return seen

    @cached_property
    def in_names(self):
        return self.names(self.in_spec, "input")

    @cached_property
    def w_names(self):
        return self.names(self.w_spec, "weight")

    @cached_property
    def out_names(self):
        return self.names(self.out_spec, "output")

    @property
    def spatial(self):
        return list(self.windows)

    @property
    def kernel(self):
        return list(self.windows.values())

    def axis(self, spec, name):
        return {a.name: a for a in _axes(spec)}[name]

    @cached_property
    def cin_candidates(self):
        return [n for n in self.in_names if n in self.w_names and n not in self.spatial and n not in self.out_names]

    @cached_property
    def cout_candidates(self):
        return [n for n in self.w_names if n in self.out_names and n not in self.in_names]

    @property
    def cin(self):
        return self.cin_candidates[0]

    @property
    def cout(self):
        return self.cout_candidates[0]

    @cached_property
    def ndim(self):
        return len(self.spatial)

    @cached_property
    def stride(self):
        return _per_dim(self.stride_arg, self.ndim, "stride")

    @cached_property
    def dilation(self):
        return _per_dim(self.dilation_arg, self.ndim, "dilation")

    @cached_property
    def pads(self):
        """Padding per spatial axis as given (an int or a (left, right) pair)."""
        kdims = [self.w_names.index(n) for n in self.kernel]
        if self.padding is None:
            pads = []
            for kd, dil in zip(kdims, self.dilation):
                span = dil * (self.weight.shape[kd] - 1)
                if span % 2:
                    raise ValueError("Default einconv padding requires odd effective kernel sizes")
                pads.append(span // 2)
            return tuple(pads)
        pads = expand_family_mapping(self.padding, self.families, label="Padding")
        if not isinstance(pads, dict):
            return _per_dim(pads, self.ndim, "padding")
        unknown = set(pads) - set(self.spatial)
        if unknown:
            raise ValueError(f"Padding axis {sorted(unknown)[0]!r} has no matching window")
        missing = [n for n in self.spatial if n not in pads]
        if missing:
            raise ValueError(f"Missing padding for window source axis {missing[0]!r}")
        return tuple(pads[n] for n in self.spatial)


def _first(items):
    return items[0] if items else None


# Ordered rule table: (condition that must hold, error raised when it does not).
# Each condition may itself raise (name checks, per-dim lengths, padding forms).
_RULES = (
    (lambda a: a.w_spec is not None, lambda a: ValueError("einconv expects a binary sharding expression")),
    (lambda a: not (a.in_spec.partials or a.w_spec.partials or a.out_spec.partials),
     lambda a: ValueError("einconv does not support partial tensor specs")),
    (lambda a: a.groups == 1, lambda a: NotImplementedError("einconv currently supports only groups=1")),
    # the name checks raise their own errors (ellipsis, factored, repeated axes)
    (lambda a: (a.in_names, a.w_names, a.out_names) is not None, None),
    (lambda a: a.ndim in (1, 2, 3), lambda a: ValueError("einconv supports 1D, 2D, and 3D convolutions")),
    (lambda a: len(set(a.kernel)) == len(a.kernel), lambda a: ValueError("Window axes must be distinct")),
    (lambda a: _first([n for n in a.spatial if n not in a.in_names]) is None,
     lambda a: ValueError(f"Window source axis {_first([n for n in a.spatial if n not in a.in_names])!r} "
                          "is not present in the input")),
    (lambda a: _first([n for n in a.kernel if n not in a.w_names]) is None,
     lambda a: ValueError(f"Window axis {_first([n for n in a.kernel if n not in a.w_names])!r} "
                          "is not present in the weight")),
    (lambda a: not any(n in a.in_names or n in a.out_names for n in a.kernel),
     lambda a: ValueError("Window axes must be weight-only axes")),
    (lambda a: all(axis.local() for axis in _axes(a.w_spec)), lambda a: ValueError("einconv weight axes must be local")),
    (lambda a: all(a.axis(a.out_spec, x.name) == x for x in _axes(a.in_spec) if x.name in a.out_names),
     lambda a: ValueError("einconv output must preserve input axis sharding")),
    (lambda a: len(a.cin_candidates) == 1, lambda a: ValueError("einconv expects exactly one input channel axis")),
    (lambda a: a.axis(a.in_spec, a.cin).local(), lambda a: ValueError("einconv input channel axis must be local")),
    (lambda a: len(a.cout_candidates) == 1, lambda a: ValueError("einconv expects exactly one output channel axis")),
    (lambda a: a.axis(a.out_spec, a.cout).local(), lambda a: ValueError("einconv output channel axis must be local")),
    (lambda a: _first([n for n in a.w_names if n not in {a.cout, a.cin, *a.kernel}]) is None,
     lambda a: ValueError(f"Unexpected weight axis {_first([n for n in a.w_names if n not in {a.cout, a.cin, *a.kernel}])!r}")),
    (lambda a: set(a.out_names) == (set(a.in_names) - {a.cin}) | {a.cout},
     lambda a: ValueError("einconv output axes must be input axes with the channel axis replaced by the output "
                          "channel axis")),
    (lambda a: a.stride is not None and a.dilation is not None and all(s == 1 for s in a.stride),
     lambda a: NotImplementedError("einconv currently supports only stride=1")),
)


def _preserving(a):
    """Raise unless every spatial axis keeps its length (left + right = dilated span)."""
    for name, pad, kd, dil in zip(a.spatial, a.pads, [a.w_names.index(n) for n in a.kernel], a.dilation):
        left, right = normalize_halo(pad)
        expected = dil * (a.weight.shape[kd] - 1)
        if left + right != expected:
            raise ValueError(
                f"Padding for axis {name!r} must preserve the spatial length; "
                f"got left + right = {left + right}, expected {expected}"
            )


def _validate(a):
    for holds, error in _RULES:
        if not holds(a):
            raise error(a)
    _preserving(a)


@dataclass
class _Layout:
    """Operand and result permutations of one einconv call."""

    batch: list
    spatial: list
    kernel: list
    cin: str
    cout: str
    in_names: list
    w_names: list
    out_names: list

    def x_order(self, channels_last):
        order = self.batch + self.spatial + [self.cin] if channels_last else self.batch + [self.cin] + self.spatial
        return [self.in_names.index(n) for n in order]

    def w_order(self, channels_last):
        order = [self.cout] + self.kernel + [self.cin] if channels_last else [self.cout, self.cin] + self.kernel
        return [self.w_names.index(n) for n in order]

    def out_order(self, channels_last):
        produced = self.batch + self.spatial + [self.cout] if channels_last else self.batch + [self.cout] + self.spatial
        return [produced.index(n) for n in self.out_names]


def _mesh_dim_size(mesh, dim):
    try:
        return mesh[dim].size()
    except Exception:  # noqa: BLE001 - compound or unknown names: not treated as trivial
        return 0


def _kernel_padded_axes(a, x, mesh, boundary, fill):
    """Spatial axes whose zero padding (before, after) the native kernel
    applies itself: local axes (and axes sharded over a one-rank mesh dim,
    which have no neighbours), when the boundary is a zero constant."""
    if boundary != "constant" or fill != 0:
        return {}
    if not conv_impl.kernel_padding_ok(x, a.weight, x.shape[a.in_names.index(a.cin)], a.spatial, a.dilation):
        return {}
    pads = {}
    for name, pad in zip(a.spatial, a.pads):
        left, right = normalize_halo(pad)
        axis = a.axis(a.in_spec, name)
        alone = not axis.local() and mesh is not None and _mesh_dim_size(mesh, axis.shard_dim) == 1
        if axis.local() or alone:
            pads[name] = (left, right)
    return pads


def _checkpointed(function, tensors, mode, use_reentrant):
    if mode in (False, None, "none"):
        return function(*tensors)
    if mode in (True, "full", "conv"):
        return torch_checkpoint(function, *tensors, use_reentrant=use_reentrant)
    raise ValueError("checkpoint must be one of 'full', 'conv', 'none', True, or False")


def einconv(shard, x, weight, windows, *, bias=None, padding=None, stride=1, dilation=1, groups=1,
            boundary="constant", fill=0, mesh=None, shapes=None, families=None, checkpoint="full",
            use_reentrant=False):
    """Sharding-aware halo exchange followed by a convolution."""
    shard, _ = cached_expand_axis_families(shard, families=families)
    windows = expand_family_mapping(windows, families, label="Window")
    a = _Analysis(parse_sharding(shard), windows, weight, padding, stride, dilation, groups, families)
    _validate(a)
    layout = _Layout([n for n in a.in_names if n not in a.spatial and n != a.cin], a.spatial, a.kernel, a.cin,
                     a.cout, a.in_names, a.w_names, a.out_names)
    kernel_pads = _kernel_padded_axes(a, x, mesh, boundary, fill)
    exchanged = {n: p for n, p in zip(a.spatial, a.pads) if n not in kernel_pads}
    halo_args = dict(mesh=mesh, shapes=shapes, boundary=boundary, fill=fill)
    # with a zero boundary the native kernel also supplies the fill at the
    # global edges of sharded axes: the exchange adds only the neighbours' rows
    edges_in_kernel = (bool(exchanged) and boundary == "constant" and fill == 0 and
                       conv_impl.kernel_padding_ok(x, weight, x.shape[a.in_names.index(a.cin)], a.spatial, a.dilation))
    pads = dict(kernel_pads)
    native_shape = groups == 1 and all(s == 1 for s in a.stride)  # the native kernels: stride 1, one group
    # the first spatial axis (the NHWC rows) sharded: the pair conv reads the
    # shard and its neighbours' rows in place, so no haloed copy is made along it
    row = a.spatial[0]
    ghost_rows = (edges_in_kernel and native_shape and a.ndim == 2 and row in exchanged and
                  conv_impl.pair_kernel_fits(x.shape[a.in_names.index(a.cin)], weight.shape[a.w_names.index(a.cout)],
                                             weight.shape[a.w_names.index(a.kernel[0])],
                                             weight.shape[a.w_names.index(a.kernel[1])]))

    # the second image axis sharded too (channels-last input): ghost columns
    # and ghost rows (with the corners) are exchanged as thin tensors and the
    # conv runs as an interior part plus two transposed strips
    # (conv_impl.conv2d_ghost_2d_train), so no haloed copy of the shard is made
    col = a.spatial[1] if a.ndim == 2 else None
    ghost_cols = (ghost_rows or (edges_in_kernel and native_shape and a.ndim == 2 and row in kernel_pads)) and (
        col in exchanged and a.in_names[-3:] == [row, col, a.cin] and
        x.shape[a.in_names.index(col)] >= weight.shape[a.w_names.index(a.kernel[1])] and
        conv_impl.pair_kernel_fits(x.shape[a.in_names.index(a.cin)], weight.shape[a.w_names.index(a.cout)],
                                   weight.shape[a.w_names.index(a.kernel[0])],
                                   weight.shape[a.w_names.index(a.kernel[1])]))

    def ghost_2d(xa, wa, ba):
        dim_h, dim_w = a.in_names.index(row), a.in_names.index(col)
        lw, rw = normalize_halo(exchanged[col])
        cols_g, gl, gr, zl, zr, adjoint_cols = halo_ghost_rows(xa, a.axis(a.in_spec, col), dim_w, lw, rw,
                                                                mesh=mesh, shapes=shapes)
        adjoint_rows = None
        if row in exchanged:
            lh, rh = normalize_halo(exchanged[row])
            vshape = list(xa.shape)
            vshape[dim_w] = gl + xa.shape[dim_w] + gr

            def slab(off, n):  # rows of [ghost columns left | x | ghost columns right]
                c = cols_g.narrow(dim_h, off, n)
                return torch.cat([c.narrow(dim_w, 0, gl), xa.narrow(dim_h, off, n), c.narrow(dim_w, gl, gr)], dim_w)
            g, gtop, gbot, mlo, mhi, adjoint_rows = halo_ghost_rows(xa, a.axis(a.in_spec, row), dim_h, lh, rh,
                                                                    mesh=mesh, shapes=shapes, slab=slab, shape=vshape)
        else:
            g, gtop, gbot = None, 0, 0
            mlo, mhi = kernel_pads[row]
        lead = xa.shape[:-3]
        flat = lambda t: t.reshape(-1, *t.shape[-3:]).contiguous()  # noqa: E731

        def adjoint(dv):  # haloed-input gradient (flat NHWC) -> the shard's, through both exchanges
            d = dv.reshape(*lead, *dv.shape[1:])
            if adjoint_rows is not None:
                d = adjoint_rows(d)
            return flat(adjoint_cols(d))
        wn = wa.permute([a.w_names.index(n) for n in [a.cout, a.kernel[0], a.kernel[1], a.cin]])
        out = conv_impl.conv2d_ghost_2d_train(flat(xa), flat(g) if g is not None else None, gtop, gbot,
                                              flat(cols_g), gl, gr, adjoint, wn, ba, (mlo, mhi), (zl, zr))
        out = out.reshape(*lead, *out.shape[1:])
        produced = list(a.in_names[:-3]) + [row, col, a.cout]
        return out.permute([produced.index(n) for n in a.out_names]).contiguous()

    def conv(xa, wa, ba=None):
        out = None
        if native_shape:
            out = conv_impl.try_conv(xa, wa, ba, a.in_names, a.w_names, a.out_names, a.spatial, a.kernel, a.cin,
                                     a.cout, a.dilation, pads)
        if out is not None:
            return out
        for name, (lo, hi) in pads.items():  # the torch path pads explicitly
            xa = pad_dim(xa, a.in_names.index(name), lo, hi, boundary="constant", fill=0)
        xc = xa.permute(layout.x_order(False)).contiguous()
        lead = xc.shape[:len(layout.batch)]
        xc = xc.reshape((-1, *xc.shape[len(layout.batch):]))
        wc = wa.permute(layout.w_order(False)).contiguous()
        out = _TORCH_CONV[a.ndim](xc, wc, ba, stride=a.stride, padding=0, dilation=a.dilation, groups=groups)
        return out.reshape((*lead, *out.shape[1:])).permute(layout.out_order(False)).contiguous()

    def halo_then_conv(xa, wa, *maybe_bias):
        if ghost_cols:
            return ghost_2d(xa, wa, maybe_bias[0] if maybe_bias else None)
        if ghost_rows:
            others = {n: p for n, p in exchanged.items() if n != row}
            za, edges = (halo_tensor_unpadded(a.in_spec, xa, others, mesh=mesh, shapes=shapes) if others
                         else (xa, {}))
            pads.update(edges)
            left, right = normalize_halo(exchanged[row])
            g, gtop, gbot, missing_lo, missing_hi, adjoint = halo_ghost_rows(
                za, a.axis(a.in_spec, row), a.in_names.index(row), left, right, mesh=mesh, shapes=shapes)
            pads[row] = (missing_lo, missing_hi)
            return conv_impl.conv2d_nhwc_ghost_rows(za, g, gtop, gbot, adjoint, wa, maybe_bias[0] if maybe_bias else None,
                                                    a.in_names, a.w_names, a.out_names, a.spatial, a.kernel, a.cin,
                                                    a.cout, pads)
        if edges_in_kernel:
            haloed, edges = halo_tensor_unpadded(a.in_spec, xa, exchanged, mesh=mesh, shapes=shapes)
            pads.update(edges)
        else:
            haloed = halo_tensor(a.in_spec, xa, exchanged, **halo_args)
        args = (haloed, wa, *maybe_bias)
        if checkpoint == "conv":
            return _checkpointed(conv, args, "conv", use_reentrant)
        return conv(*args)

    tensors = (x, weight) if bias is None else (x, weight, bias)
    if checkpoint == "conv":
        return halo_then_conv(*tensors)
    return _checkpointed(halo_then_conv, tensors, checkpoint, use_reentrant)
