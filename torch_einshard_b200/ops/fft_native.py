"""Native Stockham FFT along one axis for CUDA complex tensors.

``try_fft`` returns ``None`` when the native kernels do not cover the call
(not CUDA complex64, length not a supported power of two) and the caller then
uses ``torch.fft``.

Replaces the reference's ``torch.fft`` calls (``src/torch_einshard/fft.py:202-205``).
"""

__all__ = ["try_fft"]


def try_fft(x, dim, inverse, scale=1.0):
    from . import _native
    if not x.is_cuda:
        return None
    mod = _native.module()
    if mod is None or not hasattr(mod, "fft_c2c"):
        return None
    from .fft_impl import fft_c2c
    return fft_c2c(mod, x, dim, inverse, scale)
