"""Push-model native all-reduce (every NVLink transfer a store) against NCCL,
on 2 GPUs: dtypes, ragged sizes, the fused scale, pieces larger than the
symmetric region, and alternation with the pull kernel on the same epochs."""

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 GPUs", allow_module_level=True)

from gpu_harness import run_gpus  # noqa: E402


def _push(rank, world):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native
    from torch_einshard_b200.parallel import symmetric

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    assert es.setup_native_comm(mesh)
    comm = symmetric.communicator_for(mesh["tp"].get_group())
    mod = _native.require()
    for dtype, n in [(torch.bfloat16, 8 * 7), (torch.float16, 4096 * 3 + 8), (torch.float32, 4 * 1001),
                     (torch.bfloat16, 1 << 20)]:
        for scale in (1.0, 0.5):
            x = torch.randn(n, device="cuda", dtype=dtype) * (rank + 1)
            want = x.float().clone()
            dist.all_reduce(want)
            want = want * scale
            got = x.clone()
            mod.comm_all_reduce_push(comm.cid, got, scale, 16, comm.err)
            tol = 1e-5 if dtype == torch.float32 else 2e-2
            torch.testing.assert_close(got.float(), want, rtol=tol, atol=tol)
            # the pull kernel on the next epochs of the same region
            got2 = x.clone()
            mod.comm_all_reduce(comm.cid, got2, scale, 16, comm.err)
            torch.testing.assert_close(got2.float(), want, rtol=tol, atol=tol)
    # through the communicator, in pieces larger than the region allows at once
    old_algo, old_min = symmetric._AR_ALGO, symmetric._NCCL_AR_MIN_BYTES
    symmetric._AR_ALGO, symmetric._NCCL_AR_MIN_BYTES = "push", 1 << 62
    try:
        n = comm.capacity // 2 + (1 << 20)  # bf16 elements: more than one piece
        x = torch.randn(n, device="cuda", dtype=torch.bfloat16)
        want = x.float().clone()
        dist.all_reduce(want)
        got = x.clone()
        assert comm.all_reduce_(got)
        torch.testing.assert_close(got.float(), want, rtol=2e-2, atol=2e-2)
    finally:
        symmetric._AR_ALGO, symmetric._NCCL_AR_MIN_BYTES = old_algo, old_min
    comm.check_health()


def test_push_all_reduce_matches_nccl_2gpu():
    run_gpus(_push, 2, timeout=240)
