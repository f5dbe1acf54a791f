"""Host rule of the CTA-pair conv (no GPU): which shapes it takes and with
which output-channel tile, from the extension (``conv_pair_otile``), and the
same rule restated in ``conv_impl.pair_kernel_fits`` for hosts without it."""

import pytest

from torch_einshard_b200.ops import _native, conv_impl

mod = _native.module()
if mod is None or not hasattr(mod, "conv_pair_otile"):
    pytest.skip("the extension is not built", allow_module_level=True)


@pytest.mark.parametrize("C,O,KH,KW,tile", [
    (128, 128, 3, 3, 128),   # the halo-conv config: 147 KB of weights per CTA
    (64, 256, 3, 3, 128),
    (128, 256, 5, 5, 32),    # weights too large for a 128- or 64-channel tile
    (192, 256, 5, 5, 32),
    (64, 96, 3, 3, 32),      # 96 is no multiple of 64
    (64, 8, 3, 3, 0),        # O not a multiple of 16
    (96, 128, 3, 3, 0),      # C not a multiple of 64
    (64, 128, 3, 11, 0),     # wider than the 8 extra rows of an input box
    (512, 512, 3, 3, 32),
])
def test_pair_tile_choice(C, O, KH, KW, tile):
    assert mod.conv_pair_otile(C, O, KH, KW) == tile


def test_python_restatement_agrees(monkeypatch):
    shapes = [(C, O, K, K) for C in (64, 128, 192, 256, 512) for O in (16, 48, 64, 96, 128, 256, 512)
              for K in (1, 3, 5, 7, 9)]
    native = {s: mod.conv_pair_otile(*s) > 0 for s in shapes}
    monkeypatch.setattr(_native, "module", lambda: None)
    for s in shapes:
        assert conv_impl.pair_kernel_fits(*s) == native[s], s
