"""NVLS collectives (multimem through the NVSwitch) against NCCL on 2+ GPUs.

Covers all-reduce below and above the one-shot/two-shot switch, an odd byte
count, a tensor larger than the default heap (the heap grows and the
all-reduce runs in pieces), the three dtypes with and without scaling, broadcasts from every rank,
all-gather and reduce-scatter with uneven shards along inner and outer
dimensions (vector and byte paths), many collectives in a row (the per-block
counters), and NVLS collectives interleaved with the copy-protocol kernels on
the same heap.
"""

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 or more CUDA devices", allow_module_level=True)

from gpu_harness import run_gpus  # noqa: E402


def _body(rank, world):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native
    from torch_einshard_b200.parallel import symmetric

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    assert es.setup_native_comm(mesh)
    group = mesh["tp"].get_group()
    comm = symmetric.communicator_for(group)
    assert comm is not None
    assert comm.nvls, "the heap has no NVLS multicast mapping on this machine"
    symmetric._NVLS_AR_MIN_RANKS = 1  # the kernels themselves at every group size
    g = torch.Generator(device="cuda").manual_seed(100 + rank)

    def nccl_sum(x, scale=1.0):
        """The fp32 sum over ranks (the oracle: a bf16 ring rounds at every step)."""
        y = x.to(torch.float32, copy=True)  # never x itself: the input stays for the native call
        dist.all_reduce(y, group=group)
        return (y * scale if scale != 1.0 else y)

    tol = {torch.bfloat16: 2e-2, torch.float16: 5e-3, torch.float32: 1e-5}
    sizes = [8, 500, 128 << 10, (1 << 20) + 9, 3 << 20]
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        for n in sizes:
            x = torch.randn(n, device="cuda", dtype=dtype, generator=g)
            want = nccl_sum(x)
            got = x.clone()
            assert comm.all_reduce_(got)
            torch.testing.assert_close(got.float(), want, rtol=tol[dtype], atol=tol[dtype] * world)
        x = torch.randn(4096, 33, device="cuda", dtype=dtype, generator=g)
        got = x.clone()
        assert comm.all_reduce_(got, 1.0 / world)
        torch.testing.assert_close(got.float(), nccl_sum(x, 1.0 / world), rtol=tol[dtype], atol=tol[dtype])

    # larger than the default heap: grows the group's workspace, runs in pieces
    big = torch.randn(80 << 20, device="cuda", dtype=torch.bfloat16, generator=g)
    want = nccl_sum(big)
    assert comm.all_reduce_(big)
    torch.testing.assert_close(big.float(), want, rtol=2e-2, atol=2e-2 * world)

    # uneven all-gather / reduce-scatter along an inner (byte path) and the outer dimension
    for dtype in (torch.bfloat16, torch.float32):
        for dim, inner in ((1, 6), (0, 64)):
            shapes = [5 + 3 * p for p in range(world)]
            shp = [4, shapes[rank], inner] if dim == 1 else [shapes[rank], 3, inner]
            shard = torch.randn(shp, device="cuda", dtype=dtype, generator=g) + rank
            got = comm.all_gather(shard, dim, shapes)
            parts = [torch.empty([4, s, inner] if dim == 1 else [s, 3, inner], device="cuda", dtype=dtype)
                     for s in shapes]
            for p in range(world):
                src = shard if p == rank else torch.empty_like(parts[p])
                dist.broadcast(src, dist.get_global_rank(group, p), group=group)
                parts[p] = src
            torch.testing.assert_close(got, torch.cat(parts, dim))

            full_shape = [4, sum(shapes), inner] if dim == 1 else [sum(shapes), 3, inner]
            full = torch.randn(full_shape, device="cuda", dtype=dtype, generator=g) * (rank + 1)
            got = comm.reduce_scatter(full, dim, shapes)
            want = nccl_sum(full).narrow(dim, sum(shapes[:rank]), shapes[rank])
            t = 2e-2 if dtype == torch.bfloat16 else 1e-5
            torch.testing.assert_close(got.float(), want, rtol=t, atol=t * want.abs().max().item())

    # broadcast from each rank (NVLS: the source multicasts, every rank copies out)
    for src in range(world):
        for n in (5, 4096 + 3, 3 << 20):
            t = torch.full((n,), float(rank + 10), device="cuda", dtype=torch.bfloat16)
            assert comm.broadcast_(t, src)
            assert torch.all(t == float(src + 10))

    # many collectives in a row, alternating with the copy protocol on the same heap
    rs = [3 + p for p in range(world)]
    cs = [2 * world + 1 - p for p in range(world)]
    for it in range(40):
        x = torch.full((1000 + it,), float(rank + 1), device="cuda", dtype=torch.float32)
        assert comm.all_reduce_(x)
        assert torch.all(x == world * (world + 1) / 2)
        if it % 5 == 0:
            part = torch.randn(rs[rank], sum(cs), 5, device="cuda", generator=g) + rank
            out = comm.all_to_all(part, 0, 1, rs, cs)
            assert out is not None and out.shape == (sum(rs), cs[rank], 5)
    torch.cuda.synchronize()
    _native.check_errors("cuda")


def test_nvls_collectives_match_nccl_2gpus():
    run_gpus(_body, 2, timeout=300)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_nvls_collectives_match_nccl_4gpus():
    run_gpus(_body, 4, timeout=300)


@pytest.mark.skipif(torch.cuda.device_count() < 8, reason="needs 8 GPUs")
def test_nvls_collectives_match_nccl_8gpus():
    run_gpus(_body, 8, timeout=300)
