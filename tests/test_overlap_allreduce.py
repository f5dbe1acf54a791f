"""Row-parallel all-reduce overlapped with the GEMM in row pieces (host logic
on gloo ranks, torch matmul for the pieces): the result equals the GEMM
followed by one all-reduce, for piece counts that do and do not divide the
rows."""

import torch
import torch.distributed as dist

from dist_harness import run_ranks


def _overlap(ctx):
    from torch_einshard_b200.ops.fused_native import gemm_allreduce_overlapped

    def gemm_into(a, b, out):
        torch.matmul(a, b, out=out)

    for m, chunks in [(1024, 4), (1000, 3), (300, 8), (256, 1)]:
        a = torch.randn(1, m, 24) + ctx.rank   # a different partial product on every rank
        b = torch.randn(1, 24, 40)
        want = torch.matmul(a, b)
        dist.all_reduce(want)
        got = gemm_allreduce_overlapped(a, b, None, chunks, gemm_into)
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-4)


def test_overlapped_allreduce_matches_gemm_then_allreduce():
    run_ranks(_overlap, world_size=2)
