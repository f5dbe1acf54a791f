"""Native NVLink collectives against torch.distributed (NCCL) on 2+ GPUs."""

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 or more CUDA devices", allow_module_level=True)

from gpu_harness import run_gpus  # noqa: E402


def _collectives(rank, world):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native
    from torch_einshard_b200.parallel import collectives as C
    from torch_einshard_b200.parallel import symmetric

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    assert es.setup_native_comm(mesh)
    group = mesh["tp"].get_group()
    assert symmetric.communicator_for(group) is not None

    def ref(fn):
        symmetric.disable()
        try:
            return fn()
        finally:
            symmetric._state["enabled"] = True

    for dtype in (torch.bfloat16, torch.float32):
        x = torch.randn(3, 1000 + 8 * rank * 0, 24, device="cuda", dtype=dtype) * (rank + 1)
        got = C.all_reduce(x, group)
        want = ref(lambda: C.all_reduce(x, group))
        tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
        torch.testing.assert_close(got, want, rtol=tol, atol=tol)

        shapes = [5 + p for p in range(world)]
        shard = torch.randn(4, shapes[rank], 6, device="cuda", dtype=dtype) + rank
        got = C.all_gather(shard, group, 1, shapes)
        want = ref(lambda: C.all_gather(shard, group, 1, shapes))
        torch.testing.assert_close(got, want)

        full = torch.randn(4, sum(shapes), 6, device="cuda", dtype=dtype) * (rank + 1)
        got = C.reduce_scatter(full, group, 1, shapes)
        want = ref(lambda: C.reduce_scatter(full, group, 1, shapes))
        torch.testing.assert_close(got, want, rtol=tol, atol=tol)

        rs, cs = [3 + p for p in range(world)], [2 * world + 1 - p for p in range(world)]
        part = torch.randn(rs[rank], sum(cs), 5, device="cuda", dtype=dtype) + rank
        got = C.all_to_all_repartition(part, group, 0, 1, rs, cs)
        want = ref(lambda: C.all_to_all_repartition(part, group, 0, 1, rs, cs))
        torch.testing.assert_close(got, want)

        b = torch.full((7, 9), float(rank + 3), device="cuda", dtype=dtype)
        torch.testing.assert_close(C.broadcast(b, group, 1), torch.full_like(b, 4.0))

        roll_shapes = [4 + (p % 2) for p in range(world)]
        r = torch.randn(roll_shapes[rank], 3, device="cuda", dtype=dtype)
        for shift in (1, -3, sum(roll_shapes) + 2):
            got = C.roll_sharded(r, group, 0, shift, roll_shapes)
            want = ref(lambda: C.roll_sharded(r, group, 0, shift, roll_shapes))
            torch.testing.assert_close(got, want)

    # the same collectives twice more: epochs and buffer reuse
    for _ in range(3):
        y = torch.randn(1 << 20, device="cuda", dtype=torch.bfloat16)
        torch.testing.assert_close(C.all_reduce(y, group), ref(lambda: C.all_reduce(y, group)), rtol=2e-2, atol=2e-2)
    torch.cuda.synchronize()
    _native.check_errors()


def test_native_collectives_match_nccl_2gpu():
    run_gpus(_collectives, 2)


def test_native_collectives_match_nccl_all_gpus():
    n = torch.cuda.device_count()
    if n < 4:
        pytest.skip("needs 4+ GPUs")
    run_gpus(_collectives, min(n, 8))
