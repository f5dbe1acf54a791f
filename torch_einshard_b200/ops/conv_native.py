"""Native implicit-GEMM convolution for ``einconv`` (tcgen05, NHWC, no im2col).

``try_conv`` returns ``None`` when the call is outside the native envelope
(not CUDA bf16/fp16, not 2-D, dilation != 1, channel counts the TMA boxes
cannot address) and ``einconv`` then uses ``torch.nn.functional``.

Replaces the reference's ``F.conv2d`` call in ``einconv`` (``src/torch_einshard/conv.py:48-52``).
"""

__all__ = ["try_conv"]


def try_conv(x, weight, bias, in_names, w_names, out_names, spatial, kernel, cin, cout, dilation, pads=None):
    from . import _native
    mod = _native.module()
    if mod is None or not hasattr(mod, "conv2d_implicit") or not x.is_cuda:
        return None
    from .conv_impl import conv2d_nhwc
    return conv2d_nhwc(mod, x, weight, bias, in_names, w_names, out_names, spatial, kernel, cin, cout, dilation,
                       pads)


def kernel_padding_ok(x, weight, cin_size, spatial, dilation):
    """True when the native kernel would run and can zero-pad by itself."""
    from . import _native
    mod = _native.module()
    if mod is None or not hasattr(mod, "conv2d_implicit") or not x.is_cuda:
        return False
    from .conv_impl import supported
    return supported(x, weight.dtype, cin_size, len(spatial), dilation)
