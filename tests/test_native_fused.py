"""Fused GEMM + NVLink all-reduce and the TP-MLP path on 2+ GPUs."""

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 or more CUDA devices", allow_module_level=True)

from gpu_harness import run_gpus  # noqa: E402


def _fused(rank, world):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native, fused_native, gemm
    from torch_einshard_b200.ops.fused_native import gemm_allreduce
    from torch_einshard_b200.parallel import symmetric
    from torch_einshard_b200.models.tp_mlp import TPMLP

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    assert es.setup_native_comm(mesh)
    group = mesh["tp"].get_group()
    comm = symmetric.communicator_for(group)

    # raw fused kernel: ragged shapes, repeated calls (epochs), both operand layouts
    for (m, n, k) in [(256, 512, 128), (300, 700, 136), (1024, 2048, 512)]:
        for _ in range(2):
            a = torch.randn(1, m, k, device="cuda", dtype=torch.bfloat16) * (rank + 1)
            b = torch.randn(1, n, k, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
            got = gemm_allreduce(comm, a, b)
            want = gemm.native_bmm(a, b).float()
            dist.all_reduce(want, group=group)
            scale = want.abs().max().item() + 1
            err = (got.float() - want).abs().max().item()
            assert err < 3e-2 * scale, (m, n, k, err, scale)
    torch.cuda.synchronize()
    _native.check_errors()

    # push-model fused kernel (wide GEMM): ragged shapes, repeated calls
    for (m, n, k) in [(512, 1024, 128), (300, 700, 136), (2048, 2048, 512)]:
        for _ in range(2):
            a = torch.randn(1, m, k, device="cuda", dtype=torch.bfloat16) * (rank + 1)
            b = torch.randn(1, n, k, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
            got = fused_native.gemm_allreduce_push(comm, a, b)
            want = gemm.native_bmm(a, b).float()
            dist.all_reduce(want, group=group)
            scale = want.abs().max().item() + 1
            err = (got.float() - want).abs().max().item()
            assert err < 3e-2 * scale, ("push", m, n, k, err, scale)
    torch.cuda.synchronize()
    _native.check_errors()

    # TP-MLP through the public API: fused native path vs the NCCL-only path
    torch.manual_seed(0)
    model = TPMLP(512, 2048, mesh, device="cuda")
    x = torch.randn(2, 256, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    dy = torch.randn(2, 256, 512, device="cuda", dtype=torch.bfloat16)
    runs = []
    for fused_limit in (0, world):  # default policy (GEMM, then the all-reduce) and the fused kernel
        fused_native._MAX_FUSED_EPILOGUE_RANKS = fused_limit
        xi = x.detach().clone().requires_grad_(True)
        model.w1.grad = model.w2.grad = None
        y = model(xi)
        assert [s.name for s in es.last_plan()] == ["rank_local_einsum", "allreduce_forward_identity_backward"]
        y.backward(dy)
        runs.append((y.detach().float(), xi.grad.float(), model.w1.grad.float(), model.w2.grad.float()))
    fused_native._MAX_FUSED_EPILOGUE_RANKS = 0

    symmetric.disable()
    x2 = x.detach().clone().requires_grad_(True)
    model.w1.grad = model.w2.grad = None
    y2 = model(x2)
    y2.backward(dy)
    want = (y2.detach().float(), x2.grad.float(), model.w1.grad.float(), model.w2.grad.float())
    symmetric._state["enabled"] = True
    for got in runs:
        for g, w in zip(got, want):
            scale = w.abs().max().item() + 1e-3
            assert (g - w).abs().max().item() < 3e-2 * scale
    torch.cuda.synchronize()
    _native.check_errors()


def test_fused_gemm_allreduce_2gpu():
    run_gpus(_fused, 2)


def test_fused_gemm_allreduce_all_gpus():
    n = torch.cuda.device_count()
    if n < 4:
        pytest.skip("needs 4+ GPUs")
    run_gpus(_fused, min(n, 8))


def _sequence_parallel(rank, world):
    """Megatron sequence parallelism: AG(x) -> GEMM and GEMM -> RS, fused, against NCCL."""
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native, fused_native
    from torch_einshard_b200.parallel import symmetric

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    assert es.setup_native_comm(mesh)
    group = mesh["tp"].get_group()
    comm = symmetric.communicator_for(group)

    # raw fused GEMM + reduce-scatter of row segments
    torch.manual_seed(1)
    for (segs, seg, n, k) in [(2, 256 * world, 512, 128), (1, 128 * world, 300, 64)]:
        a = torch.randn(1, segs * seg, k, device="cuda", dtype=torch.bfloat16) * (rank + 1)
        b = torch.randn(1, n, k, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
        for _ in range(2):
            got = fused_native.gemm_reducescatter(comm, a, b, seg, seg // world)
            full = (a.float() @ b.float())
            dist.all_reduce(full, group=group)
            shard = seg // world
            want = full.reshape(segs, seg, n)[:, rank * shard:(rank + 1) * shard].reshape(1, -1, n)
            scale = want.abs().max().item() + 1
            assert (got.float() - want).abs().max().item() < 3e-2 * scale
    _native.check_errors()

    # raw fused all-gather -> GEMM (copy warps inside the GEMM), two calls in a row
    for (segs, shard, n, k) in [(2, 256, 1024, 256), (1, 512, 512, 128)]:
        a_local = torch.randn(1, segs * shard, k, device="cuda", dtype=torch.bfloat16) * (rank + 1)
        b = torch.randn(1, n, k, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
        parts = [torch.empty_like(a_local) for _ in range(world)]
        dist.all_gather(parts, a_local, group=group)
        want_a = torch.cat([p.reshape(segs, shard, k) for p in parts], dim=1).reshape(1, segs * shard * world, k)
        for _ in range(2):
            out, gathered = fused_native.gemm_allgather(comm, a_local, b, shard * world, shard)
            assert torch.equal(gathered, want_a)
            want = want_a.float() @ b.float()
            assert (out.float() - want).abs().max().item() < 3e-2 * (want.abs().max().item() + 1)
    _native.check_errors()

    # through einshard: l/tp e, e f/tp -> l f/tp (AG -> GEMM) and back l f/tp, f/tp e -> l/tp e (GEMM -> RS)
    torch.manual_seed(0)
    L, E, F_ = 256 * world, 256, 512 * world
    x_full = torch.randn(2, L, E, device="cuda", dtype=torch.bfloat16)
    w1 = torch.randn(F_ // world, E, device="cuda", dtype=torch.bfloat16) * 0.05
    w2 = torch.randn(E, F_ // world, device="cuda", dtype=torch.bfloat16) * 0.05
    dy = torch.randn(2, L // world, E, device="cuda", dtype=torch.bfloat16)

    def run():
        x = x_full[:, rank * (L // world):(rank + 1) * (L // world)].clone().requires_grad_(True)
        a = w1.clone().requires_grad_(True)
        b = w2.clone().requires_grad_(True)
        h = es.einshard("s l/tp e, f/tp e -> s l f/tp", x, a, mesh=mesh)
        plan1 = [s.name for s in es.last_plan()]
        y = es.einshard("s l f/tp, e f/tp -> s l/tp e", h, b, mesh=mesh)
        plan2 = [s.name for s in es.last_plan()]
        y.backward(dy)
        return (h.detach().float(), y.detach().float(), x.grad.float(), a.grad.float(), b.grad.float()), plan1, plan2

    fused_native._MAX_FUSED_EPILOGUE_RANKS = world  # also run the fused GEMM -> reduce-scatter
    got, p1, p2 = run()
    fused_native._MAX_FUSED_EPILOGUE_RANKS = 0
    assert p1 == ["allgather_forward_reducescatter_backward", "rank_local_einsum"], p1
    assert p2 == ["rank_local_einsum", "reducescatter_forward_allgather_backward"], p2
    symmetric.disable()
    want, q1, q2 = run()
    symmetric._state["enabled"] = True
    assert (p1, p2) == (q1, q2)
    for g, w in zip(got, want):
        scale = w.abs().max().item() + 1e-3
        assert (g - w).abs().max().item() < 3e-2 * scale
    torch.cuda.synchronize()
    _native.check_errors()


def test_sequence_parallel_fused_2gpu():
    run_gpus(_sequence_parallel, 2)


def _overlap_ar(rank, world):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native, fused_native, gemm
    from torch_einshard_b200.models.tp_mlp import TPMLP

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    assert es.setup_native_comm(mesh)
    group = mesh["tp"].get_group()
    # the row pieces on the native GEMM, all-reduced on NCCL while the next piece runs
    for m, chunks in [(2048, 4), (1000, 3)]:
        a = torch.randn(1, m, 256, device="cuda", dtype=torch.bfloat16) * (rank + 1)
        b = torch.randn(1, 384, 256, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
        got = fused_native.gemm_allreduce_overlapped(a, b, group, chunks, fused_native._native_gemm_into)
        want = gemm.native_bmm(a, b).float()
        dist.all_reduce(want, group=group)
        scale = want.abs().max().item() + 1
        assert (got.float() - want).abs().max().item() < 3e-2 * scale
    # the TP-MLP with the overlap path selected, forward and backward against the plain path
    old = fused_native._OVERLAP_AR_CHUNKS
    try:
        results = []
        for chunks in (0, 4):
            fused_native._OVERLAP_AR_CHUNKS = chunks
            torch.manual_seed(7)
            model = TPMLP(512, 2048, mesh, device="cuda")
            x = torch.randn(4, 512, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
            y = model(x)
            y.float().square().mean().backward()
            results.append((y.float(), model.w1.grad.float(), model.w2.grad.float()))
        for plain, overlapped in zip(*results):
            scale = plain.abs().max().item() + 1
            assert (plain - overlapped).abs().max().item() < 2e-2 * scale
    finally:
        fused_native._OVERLAP_AR_CHUNKS = old
    torch.cuda.synchronize()
    _native.check_errors()


def test_overlapped_row_parallel_allreduce_2gpu():
    run_gpus(_overlap_ar, 2)
