"""Failure detection without faulting a GPU.

* A bounded device wait on a flag that nothing sets expires, records its code
  in the error word, and returns: the host raises EinshardCommTimeout and the
  CUDA context keeps working.
* On 2 GPUs (heaps without NVLS multicast, NCCL with NVLS off) a rank skips one
  native all-reduce (host-side injection); its peer's kernel gives up after the wait limit, the peer's host sees the timeout, the
  communicator is marked broken and the next all-reduce falls back to NCCL.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200.ops import _native, gemm  # noqa: E402


def test_bounded_wait_expires_and_context_survives():
    mod = _native.require()
    _native.reset_errors()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    result = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    mod.wait_probe(flag, 1, 50_000_000, result, _native.error_word("cuda"))  # 50 ms, nothing sets the flag
    assert int(result.item()) == 0
    with pytest.raises(_native.EinshardCommTimeout, match="peer flag never set"):
        _native.check_errors("cuda")
    _native.reset_errors()
    # the context is intact: a native GEMM still runs and is correct
    a = torch.randn(1, 256, 128, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1, 128, 256, device="cuda", dtype=torch.bfloat16)
    c = gemm.native_bmm(a, b)
    assert (c.float() - a.float() @ b.float()).abs().max().item() < 0.5
    # once the flag is set the same wait succeeds
    flag.fill_(1)
    mod.wait_probe(flag, 1, 50_000_000, result, _native.error_word("cuda"))
    assert int(result.item()) == 1
    _native.check_errors("cuda")


def _skip_one_allreduce(rank, world):
    import os
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    import torch_einshard_b200 as es
    from torch_einshard_b200.ops import _native
    from torch_einshard_b200.parallel import symmetric

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    assert es.setup_native_comm(mesh)
    comm = symmetric.communicator_for(mesh["tp"].get_group())
    x = torch.ones(1024, device="cuda")
    assert comm.all_reduce_(x)           # call 1: everyone
    comm.check_health()
    assert torch.all(x == world)
    os.environ["EINSHARD_FAULT_INJECT"] = "skip:1:2"
    previous = _native.wait_timeout_us()
    _native.set_wait_timeout_us(300_000)  # the peer wait gives up after 0.3 s
    y = torch.ones(1024, device="cuda")
    comm.all_reduce_(y)                  # call 2: rank 1 launches nothing
    os.environ.pop("EINSHARD_FAULT_INJECT")
    _native.set_wait_timeout_us(previous)
    if rank == 0:
        with pytest.raises(_native.EinshardCommTimeout):
            comm.check_health()
    else:
        comm.broken = True               # the skipping rank knows it left the protocol
        torch.cuda.synchronize()
    assert comm.broken
    # both ranks continue on NCCL
    z = torch.ones(1024, device="cuda")
    dist.all_reduce(z)
    assert torch.all(z == world)
    assert not comm.all_reduce_(z)       # a broken communicator declines


@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_that_skips_a_collective_is_detected():
    from gpu_harness import run_gpus
    # plain peer loads only: no NVLS multicast object in a test where a rank leaves a protocol
    run_gpus(_skip_one_allreduce, 2, timeout=120, env={"EINSHARD_NVLS": "0"})
