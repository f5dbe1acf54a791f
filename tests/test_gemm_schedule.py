"""The wide GEMM kernel's work partition, walked on the host with the same
schedule functions the kernel runs (no GPU): every pair tile's K blocks are
covered exactly once, in every mode (whole tiles, persistent clusters,
stream-K tail, every tile split)."""

import itertools

import pytest

from torch_einshard_b200.ops import _native

mod = _native.module()
pytestmark = pytest.mark.skipif(mod is None, reason="native extension not built")

SHAPES = [(3584, 8192, 32768), (2500, 4000, 4608), (2048, 2048, 65536), (65536, 2048, 2048), (512, 1024, 8192),
          (1000, 1536, 4160), (768, 2048, 4100), (14336, 8192, 32768), (257, 513, 65),
          (32768, 3584, 8192), (7168, 8192, 32768), (32768, 8192, 3584)]   # TP-MLP GEMMs at tp = 8 and 4


def _check(m, n, k, sms=148):
    segs = mod.gemm_wide_schedule(m, n, k, sms)
    pairs = -(-m // 256) * -(-n // 512)
    nkb = -(-k // 64)
    cover = {}
    origin = {}
    for launch, cluster, p, m0, n0, kb0, kb1 in segs:
        assert 0 <= p < pairs and 0 <= kb0 < kb1 <= nkb
        assert m0 % 256 == 0 and n0 % 512 == 0 and m0 < m and n0 < n
        assert origin.setdefault(p, (m0, n0)) == (m0, n0)
        cover.setdefault(p, []).append((kb0, kb1))
    assert sorted(cover) == list(range(pairs))
    for p, ranges in cover.items():
        ranges.sort()
        assert ranges[0][0] == 0 and ranges[-1][1] == nkb
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:])), (p, ranges)  # no gap, no overlap
    assert len(set(origin.values())) == pairs
    return segs


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("streamk,persistent", list(itertools.product([-1, 0, 1], [-1, 0, 1])))
def test_every_k_block_once(shape, streamk, persistent):
    mod.set_gemm_pair_mode(-1)
    mod.set_gemm_streamk(streamk)
    mod.set_gemm_persistent(persistent)
    try:
        _check(*shape)
    finally:
        mod.set_gemm_streamk(-1)
        mod.set_gemm_persistent(-1)


def test_stream_k_tail_layout():
    mod.set_gemm_pair_mode(-1)
    mod.set_gemm_streamk(-1)
    plan = mod.gemm_plan(3584, 8192, 32768, 1, True, True, 148)
    segs = _check(3584, 8192, 32768)
    whole = [s for s in segs if s[0] == 0]
    tail = [s for s in segs if s[0] == 1]
    assert len(whole) == plan["sk_first"] == 222
    assert all(c == p and (k0, k1) == (0, 512) for _, c, p, _, _, k0, k1 in whole)  # one whole tile per cluster
    assert {p for _, _, p, _, _, _, _ in tail} == {222, 223}
    per_cluster = {}
    for _, c, _, _, _, k0, k1 in tail:
        per_cluster[c] = per_cluster.get(c, 0) + k1 - k0
    assert len(per_cluster) <= 74 and max(per_cluster.values()) <= plan["sk_iters"]


def test_tp8_forward_gets_a_tail_of_eight_tiles():
    mod.set_gemm_pair_mode(-1)
    mod.set_gemm_streamk(-1)
    plan = mod.gemm_plan(32768, 3584, 8192, 1, False, False, 148)
    assert plan["sk_first"] == 888 and plan["tail_tiles"] == 8


def test_persistent_clusters_walk_strided_tiles():
    mod.set_gemm_pair_mode(-1)
    mod.set_gemm_persistent(1)
    try:
        segs = _check(65536, 2048, 2048)
        assert len({c for _, c, *_ in segs}) == 74
        for _, c, p, *_ in segs:
            assert p % 74 == c
    finally:
        mod.set_gemm_persistent(-1)
