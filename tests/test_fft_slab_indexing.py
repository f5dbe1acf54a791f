"""Index math of the fused slab exchange (host walk of the kernel's loader, no
GPU): gathering every rank's staged input through the walked (rank, offset)
pairs must produce the transposed slab of the reference layout."""

import pytest
import torch

from torch_einshard_b200.ops import _native

mod = _native.module()
pytestmark = pytest.mark.skipif(mod is None, reason="native extension not built")


@pytest.mark.parametrize("P", [2, 4, 8])
@pytest.mark.parametrize("A,B,C,Sl,D", [(1, 1, 1, 4, 8), (2, 3, 5, 2, 16), (1, 2, 4, 8, 8)])
def test_mode0_gathered_axis_before_split_axis(P, A, B, C, Sl, D):
    # rank r stages x_r [A, Sl, B, D, C] (its Sl rows of the gathered axis S = P * Sl);
    # rank `me` outputs [A, S, B, Dl, C], its block of D
    if D % P:
        pytest.skip("D must split evenly")
    n, Dl = P * Sl, D // P
    full = torch.randn(A, n, B, D, C, dtype=torch.float64)
    staged = [full[:, r * Sl:(r + 1) * Sl].contiguous() for r in range(P)]
    for me in range(P):
        out_off, src_rank, src_off = mod.fft_slab_sources(0, n, A, B, C, D, Dl, me * Dl, P)
        out = torch.empty(A * n * B * Dl * C, dtype=torch.float64)
        src = torch.stack([staged[r].reshape(-1) for r in range(P)])
        out[out_off] = src[src_rank.long(), src_off]
        want = full[:, :, :, me * Dl:(me + 1) * Dl].contiguous().reshape(-1)
        assert torch.equal(out, want)


@pytest.mark.parametrize("P", [2, 4])
@pytest.mark.parametrize("A,B,C,Sl,D", [(1, 1, 1, 4, 8), (2, 3, 5, 2, 4)])
def test_mode1_split_axis_before_gathered_axis(P, A, B, C, Sl, D):
    # rank r stages [A, D, B, Sl, C]; rank `me` outputs [A, Dl, B, S, C]
    if D % P:
        pytest.skip("D must split evenly")
    n, Dl = P * Sl, D // P
    full = torch.randn(A, D, B, n, C, dtype=torch.float64)
    staged = [full[:, :, :, r * Sl:(r + 1) * Sl].contiguous() for r in range(P)]
    for me in range(P):
        out_off, src_rank, src_off = mod.fft_slab_sources(1, n, A, B, C, D, Dl, me * Dl, P)
        out = torch.empty(A * Dl * B * n * C, dtype=torch.float64)
        src = torch.stack([staged[r].reshape(-1) for r in range(P)])
        out[out_off] = src[src_rank.long(), src_off]
        want = full[:, me * Dl:(me + 1) * Dl].contiguous().reshape(-1)
        assert torch.equal(out, want)
