"""Row-block order of the fused all-gather -> GEMM kernel (host walk of the
kernel's mapping, no GPU): every rank visits every 256-row block of the
gathered operand exactly once, its own shard first, then rank + 1, rank + 2, ..."""

import pytest

from torch_einshard_b200.ops import _native

mod = _native.module()
pytestmark = pytest.mark.skipif(mod is None, reason="native extension not built")


@pytest.mark.parametrize("size", [2, 4, 8])
@pytest.mark.parametrize("segments,shard", [(1, 256), (1, 4096), (3, 512), (8, 1024)])
def test_each_rank_visits_every_block_once_local_first(size, segments, shard):
    rows = segments * size * shard
    for rank in range(size):
        order = mod.gemm_allgather_row_order(rank, size, segments, shard)
        assert sorted(order) == list(range(0, rows, 256))
        per_owner = segments * shard // 256           # blocks each owner holds
        owners = [(m0 // shard) % size for m0 in order]
        for k in range(size):                         # owner rank + k's blocks come k-th
            assert set(owners[k * per_owner:(k + 1) * per_owner]) == {(rank + k) % size}
