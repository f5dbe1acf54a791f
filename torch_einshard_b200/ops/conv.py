"""``einconv``: halo exchange followed by a same-length convolution.

Validates the named-axis formula (one input channel axis, one output channel
axis, local weight/kernel axes, stride 1, groups 1, padding that preserves the
spatial length), exchanges halos of the sharded spatial axes and runs the
convolution with zero padding on the haloed tensor.  ``checkpoint`` selects
activation checkpointing: ``"full"`` (default: halo + conv recomputed in
backward), ``"conv"`` (only the convolution), or off.  Contract of
``src/torch_einshard/conv.py:64-210``.

The 2-D bf16/fp16 CUDA case with a 3x3-style odd kernel runs as an implicit
GEMM on the tcgen05 kernel (``ops.conv_native``): each kernel tap is one GEMM
over shifted views of the haloed NHWC input, accumulated in fp32, so no
im2col tensor is materialised.  Other cases use ``torch.nn.functional.conv*d``.
"""

import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as torch_checkpoint

from ..notation.families import cached_expand_axis_families, expand_family_mapping
from ..notation.parser import parse_sharding
from ..notation.spec import EllipsisAxis
from .halo import halo_tensor, normalize_halo

__all__ = ["einconv"]


def _axes(spec):
    return spec.axes if hasattr(spec, "axes") else spec


def _names(axes, *, label):
    names = []
    for axis in axes:
        if isinstance(axis, EllipsisAxis):
            raise NotImplementedError(f"einconv does not support ellipsis axes in {label}")
        if not hasattr(axis, "name"):
            raise NotImplementedError(f"einconv does not support factored axes in {label}")
        if axis.name in names:
            raise ValueError(f"Axis {axis.name!r} appears more than once in {label}")
        names.append(axis.name)
    return names


def _per_dim(value, ndim, *, label):
    if isinstance(value, int):
        return (value,) * ndim
    values = tuple(value)
    if len(values) != ndim:
        raise ValueError(f"{label} must have {ndim} values")
    return values


def _conv_fn(ndim):
    try:
        return {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}[ndim]
    except KeyError:
        raise ValueError("einconv supports 1D, 2D, and 3D convolutions") from None


def _mesh_dim_size(mesh, dim):
    try:
        return mesh[dim].size()
    except Exception:  # noqa: BLE001 - compound or unknown names: not treated as trivial
        return 0


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
    in_spec, w_spec, out_spec = parse_sharding(shard)
    if w_spec is None:
        raise ValueError("einconv expects a binary sharding expression")
    if in_spec.partials or w_spec.partials or out_spec.partials:
        raise ValueError("einconv does not support partial tensor specs")
    if groups != 1:
        raise NotImplementedError("einconv currently supports only groups=1")

    in_axes, w_axes, out_axes = _axes(in_spec), _axes(w_spec), _axes(out_spec)
    in_names = _names(in_axes, label="input")
    w_names = _names(w_axes, label="weight")
    out_names = _names(out_axes, label="output")
    spatial = list(windows.keys())
    kernel = list(windows.values())
    if len(spatial) not in (1, 2, 3):
        raise ValueError("einconv supports 1D, 2D, and 3D convolutions")
    if len(set(kernel)) != len(kernel):
        raise ValueError("Window axes must be distinct")
    missing = [n for n in spatial if n not in in_names]
    if missing:
        raise ValueError(f"Window source axis {missing[0]!r} is not present in the input")
    missing = [n for n in kernel if n not in w_names]
    if missing:
        raise ValueError(f"Window axis {missing[0]!r} is not present in the weight")
    if any(n in in_names or n in out_names for n in kernel):
        raise ValueError("Window axes must be weight-only axes")
    if not all(axis.local() for axis in w_axes):
        raise ValueError("einconv weight axes must be local")
    out_by = {a.name: a for a in out_axes}
    for axis in in_axes:
        if axis.name in out_by and out_by[axis.name] != axis:
            raise ValueError("einconv output must preserve input axis sharding")
    shared = [n for n in in_names if n in w_names and n not in spatial]
    in_channels = [n for n in shared if n not in out_names]
    if len(in_channels) != 1:
        raise ValueError("einconv expects exactly one input channel axis")
    cin = in_channels[0]
    if not in_axes[in_names.index(cin)].local():
        raise ValueError("einconv input channel axis must be local")
    out_channels = [n for n in w_names if n in out_names and n not in in_names]
    if len(out_channels) != 1:
        raise ValueError("einconv expects exactly one output channel axis")
    cout = out_channels[0]
    if not out_by[cout].local():
        raise ValueError("einconv output channel axis must be local")
    extra = [n for n in w_names if n not in {cout, cin, *kernel}]
    if extra:
        raise ValueError(f"Unexpected weight axis {extra[0]!r}")
    if set(out_names) != (set(in_names) - {cin}) | {cout}:
        raise ValueError("einconv output axes must be input axes with the channel axis replaced by the output channel axis")

    ndim = len(spatial)
    stride = _per_dim(stride, ndim, label="stride")
    dilation = _per_dim(dilation, ndim, label="dilation")
    if any(s != 1 for s in stride):
        raise NotImplementedError("einconv currently supports only stride=1")
    kdims = tuple(w_names.index(n) for n in kernel)
    if padding is None:
        pads = []
        for kd, dil in zip(kdims, dilation):
            span = dil * (weight.shape[kd] - 1)
            if span % 2:
                raise ValueError("Default einconv padding requires odd effective kernel sizes")
            pads.append(span // 2)
        pads = tuple(pads)
    else:
        pads = expand_family_mapping(padding, families, label="Padding")
        if isinstance(pads, dict):
            unknown = set(pads) - set(spatial)
            if unknown:
                raise ValueError(f"Padding axis {sorted(unknown)[0]!r} has no matching window")
            missing = [n for n in spatial if n not in pads]
            if missing:
                raise ValueError(f"Missing padding for window source axis {missing[0]!r}")
            pads = tuple(pads[n] for n in spatial)
        else:
            pads = _per_dim(pads, ndim, label="padding")
    for name, pad, kd, dil in zip(spatial, pads, kdims, dilation):
        left, right = normalize_halo(pad)
        expected = dil * (weight.shape[kd] - 1)
        if left + right != expected:
            raise ValueError(
                f"Padding for axis {name!r} must preserve the spatial length; "
                f"got left + right = {left + right}, expected {expected}"
            )

    halos = dict(zip(spatial, pads))
    conv = _conv_fn(ndim)
    batch = [n for n in in_names if n not in spatial and n != cin]
    x_perm = [in_names.index(n) for n in batch + [cin] + spatial]
    w_perm = [w_names.index(n) for n in [cout, cin] + kernel]
    conv_out = batch + [cout] + spatial
    out_perm = [conv_out.index(n) for n in out_names]

    from . import conv_native
    # Local spatial axes with a zero boundary are padded by the native kernel itself
    # (TMA zero fill), so no padded copy of the input is made for them.
    kernel_pads = {}
    if conv_native.kernel_padding_ok(x, weight, x.shape[in_names.index(cin)], spatial, dilation) and \
            boundary == "constant" and fill == 0:
        for name in spatial:
            left, right = normalize_halo(halos[name])
            axis = in_axes[in_names.index(name)]
            # an axis sharded over a one-rank mesh dim has no neighbours: its halo is the zero boundary
            alone = not axis.local() and mesh is not None and _mesh_dim_size(mesh, axis.shard_dim) == 1
            if (axis.local() or alone) and left == right:
                kernel_pads[name] = left
    other_halos = {n: h for n, h in halos.items() if n not in kernel_pads}

    def run_conv(xa, wa, ba=None):
        native = conv_native.try_conv(xa, wa, ba, in_names, w_names, out_names, spatial, kernel, cin, cout,
                                      dilation, kernel_pads)
        if native is not None:
            return native
        if kernel_pads:
            xa = halo_tensor(in_spec, xa, kernel_pads, mesh=mesh, shapes=shapes, boundary=boundary, fill=fill)
        xc = xa.permute(x_perm).contiguous()
        lead = xc.shape[:len(batch)]
        xc = xc.reshape((-1, xc.shape[len(batch)], *xc.shape[len(batch) + 1:]))
        wc = wa.permute(w_perm).contiguous()
        out = conv(xc, wc, ba, stride=stride, padding=0, dilation=dilation, groups=groups)
        out = out.reshape((*lead, *out.shape[1:]))
        return out.permute(out_perm).contiguous()

    def run_full(xa, wa, *maybe_bias):
        ba = maybe_bias[0] if maybe_bias else None
        haloed = halo_tensor(in_spec, xa, other_halos, mesh=mesh, shapes=shapes, boundary=boundary, fill=fill)
        if checkpoint == "conv":
            args = (haloed, wa) if ba is None else (haloed, wa, ba)
            return _checkpointed(lambda *a: run_conv(*a), args, "conv", use_reentrant)
        return run_conv(haloed, wa, ba)

    tensors = (x, weight) if bias is None else (x, weight, bias)
    if checkpoint == "conv":
        return run_full(*tensors)
    return _checkpointed(lambda *a: run_full(*a), tensors, checkpoint, use_reentrant)
