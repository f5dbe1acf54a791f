"""Fused GEMM + NVLS all-reduce (one launch: wide tcgen05 GEMM, partial units
through the symmetric heap, sums in the NVSwitch) against an fp32 product
all-reduced by NCCL, on 2, 4 and 8 GPUs.

Ragged shapes (rows and columns that end inside a unit), both operand
layouts, calls of alternating shapes on one heap (the per-unit epochs), the
fused call between NVLS collectives and copy-protocol kernels on the same heap,
the reduce-scatter mode (row segments), both reduction modes (dedicated
reducer CTA pairs; the GEMM's epilogue warps with several lags, the product
spanning more than one wave of CTA pairs), and the TP-MLP through the public API
(forward and backward) against the unfused NCCL path.
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
    from torch_einshard_b200.models.tp_mlp import TPMLP
    from torch_einshard_b200.ops import _native, fused_native
    from torch_einshard_b200.parallel import symmetric

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    assert es.setup_native_comm(mesh)
    group = mesh["tp"].get_group()
    comm = symmetric.communicator_for(group)
    assert comm is not None and comm.nvls, "no NVLS multicast heap"
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    defaults = fused_native._NVLS_REDUCER_CLUSTERS, fused_native._NVLS_LAG

    def check(a, b):
        got = fused_native.gemm_allreduce_nvls(comm, a, b)
        assert got is not None
        want = a.float() @ b.float()
        dist.all_reduce(want, group=group)
        scale = want.abs().max().item() + 1.0
        err = (got.float() - want).abs().max().item()
        assert err <= 2e-2 * scale, (tuple(a.shape), tuple(b.shape), err, scale)

    shapes = [(512, 1024, 256), (300, 712, 136), (2048, 4096, 1024), (256, 512, 64), (777, 1032, 320),
              (4096, 4096, 256)]
    # (reducer CTA pairs, lag): dedicated reducers, and overlap mode (the GEMM's
    # epilogue warps reduce) with the automatic lag and lags inside one wave
    modes = [(12, 0), (0, 0), (0, 1), (0, 5)]
    for rep in range(2 * len(modes)):
        fused_native._NVLS_REDUCER_CLUSTERS, fused_native._NVLS_LAG = modes[rep % len(modes)]
        for m, n, k in shapes:
            a = torch.randn(1, m, k, device="cuda", dtype=torch.bfloat16, generator=g)
            b_kn = torch.randn(1, k, n, device="cuda", dtype=torch.bfloat16, generator=g)
            b_nk = torch.randn(1, n, k, device="cuda", dtype=torch.bfloat16, generator=g).transpose(1, 2)
            check(a, b_kn)
            check(a, b_nk)
            # other protocols on the same heap between fused calls
            x = torch.full((4096,), float(rank), device="cuda")
            assert comm.all_reduce_(x) and torch.all(x == world * (world - 1) / 2)
            part = torch.randn(3, 2 * world, 5, device="cuda", generator=g)
            assert comm.all_to_all(part, 0, 1, [3] * world, [2] * world) is not None
    # reduce-scatter mode: each rank keeps its rows of every segment
    for (reducers, lag), (m, n, k, seg) in [(md, sh) for md in modes for sh in
                                            [(1024 * world, 1024, 256, 64 * world), (256 * world, 520, 136, 32 * world)]]:
        fused_native._NVLS_REDUCER_CLUSTERS, fused_native._NVLS_LAG = reducers, lag
        a = torch.randn(1, m, k, device="cuda", dtype=torch.bfloat16, generator=g)
        b = torch.randn(1, n, k, device="cuda", dtype=torch.bfloat16, generator=g).transpose(1, 2)
        shard = seg // world
        got = fused_native.gemm_reducescatter_nvls(comm, a, b, seg, shard)
        want = a.float() @ b.float()
        dist.all_reduce(want, group=group)
        want = want.reshape(1, m // seg, seg, n)[:, :, rank * shard:(rank + 1) * shard].reshape(1, m // world, n)
        scale = want.abs().max().item() + 1.0
        assert (got.float() - want).abs().max().item() <= 2e-2 * scale, (m, n, k, seg)
    torch.cuda.synchronize()
    _native.check_errors()
    fused_native._NVLS_REDUCER_CLUSTERS, fused_native._NVLS_LAG = defaults

    # the TP-MLP through the public API: fused NVLS path against NCCL only
    model = TPMLP(1024, 4096, mesh, device="cuda")
    x = torch.randn(2, 512, 1024, device="cuda", dtype=torch.bfloat16, generator=torch.Generator(device="cuda").manual_seed(0))
    dy = torch.randn(2, 512, 1024, device="cuda", dtype=torch.bfloat16, generator=torch.Generator(device="cuda").manual_seed(1))

    def run():
        xi = x.detach().clone().requires_grad_(True)
        model.w1.grad = model.w2.grad = None
        y = model(xi)
        y.backward(dy)
        return y.detach().float(), xi.grad.float(), model.w1.grad.float(), model.w2.grad.float()

    fused = run()
    assert [s.name for s in es.last_plan()] == ["rank_local_einsum", "allreduce_forward_identity_backward"]
    symmetric.disable()
    plain = run()
    symmetric._state["enabled"] = True
    for got, want in zip(fused, plain):
        scale = want.abs().max().item() + 1e-3
        assert (got - want).abs().max().item() <= 3e-2 * scale
    torch.cuda.synchronize()
    _native.check_errors()


def test_gemm_nvls_allreduce_2gpus():
    run_gpus(_body, 2, timeout=300)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_gemm_nvls_allreduce_4gpus():
    run_gpus(_body, 4, timeout=300)


@pytest.mark.skipif(torch.cuda.device_count() < 8, reason="needs 8 GPUs")
def test_gemm_nvls_allreduce_8gpus():
    run_gpus(_body, 8, timeout=300)
