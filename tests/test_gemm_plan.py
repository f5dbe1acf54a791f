"""Kernel choice of the native GEMM (host-side plan, no GPU needed): the
measured policy for the training and TP-MLP shapes."""

import pytest

from torch_einshard_b200.ops import _native

mod = _native.module()
pytestmark = pytest.mark.skipif(mod is None, reason="native extension not built")

SMS = 148


def plan(m, n, k, a_mn=False, b_mn=False):
    return mod.gemm_plan(m, n, k, 1, a_mn, b_mn, SMS)


def test_full_waves_use_the_wide_kernel():
    p = plan(32768, 28672, 8192)            # TP-MLP forward at tp = 1: 7168 pair tiles
    assert p["kernel"] == 2 and p["tail_tiles"] == 0 and p["persistent"] == 0


def test_short_k_runs_persistent_clusters():
    p = plan(65536, 2048, 2048)             # transformer q/k/v/o forward
    assert p["kernel"] == 2 and p["persistent"] == 1 and p["tail_tiles"] == 0


def test_partial_last_wave_gets_a_stream_k_tail():
    p = plan(3584, 8192, 32768, True, True)  # TP-MLP weight gradient at tp = 8: 224 pair tiles
    assert p["kernel"] == 2
    assert p["sk_first"] == 222 and p["tail_tiles"] == 2
    assert p["clusters"] - p["sk_first"] <= SMS // 2
    assert p["sk_iters"] * (p["clusters"] - p["sk_first"]) >= 2 * 512
    q = plan(14336, 8192, 32768, True, True)  # the same at tp = 2: 896 pair tiles, 8 left over
    assert q["sk_first"] == 888 and q["tail_tiles"] == 8


def test_remainders_above_a_ninth_of_a_wave_stay_whole_tiles():
    assert plan(28672, 8192, 32768, True, True)["tail_tiles"] == 0   # tp = 1: 16 left over


def test_large_remainder_stays_whole_tiles():
    # transformer MLP weight gradient: 128 pair tiles, 54 left over (the tail
    # phase would stream from DRAM: measured slower)
    p = plan(8192, 2048, 65536, True, True)
    assert p["kernel"] == 2 and p["tail_tiles"] == 0


def test_underfilled_long_k_uses_the_pair_kernel():
    p = plan(2048, 2048, 65536, True, True)  # 32 wide tiles, 64 pair tiles
    assert p["kernel"] == 1 and p["tail_tiles"] == 0


def test_small_problems_use_the_one_sm_kernel():
    assert plan(256, 256, 512)["kernel"] == 0
    assert plan(4096, 64, 4096)["swapped"] == 1   # narrow N runs transposed


def test_stream_k_modes():
    try:
        mod.set_gemm_streamk(0)
        assert plan(3584, 8192, 32768, True, True)["tail_tiles"] == 0
        mod.set_gemm_streamk(1)
        p = plan(512, 1024, 8192)
        assert p["sk_first"] == 0 and p["tail_tiles"] == 4
    finally:
        mod.set_gemm_streamk(-1)
