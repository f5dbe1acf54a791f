"""The fused-path policy of the binary executor (host logic, no GPU): which
plans get a fused kernel, the overlapped all-reduce or the unfused steps, for
each group size, with fakes of the executor and the communicator."""

from types import SimpleNamespace

import pytest
import torch

from torch_einshard_b200.ops import fused_native as fn
from torch_einshard_b200.plan.state import PlanStep


class FakeTensor:
    is_cuda = True
    dtype = torch.bfloat16


def executor(output_steps=(), input0_steps=(), input1_steps=()):
    tp = SimpleNamespace(output_steps=[PlanStep("rank_local_einsum")] + list(output_steps),
                         input0_steps=list(input0_steps), input1_steps=list(input1_steps))
    return SimpleNamespace(post=None, x0=FakeTensor(), y0=FakeTensor(), tp=tp, group=lambda dim: ("group", dim))


@pytest.fixture
def ranks(monkeypatch):
    """Set the size of every group (and its native communicator: with or
    without an NVLS multicast mapping)."""
    def set_size(size, nvls=False):
        monkeypatch.setattr(fn, "_comm", lambda group: SimpleNamespace(size=size, nvls=nvls, broken=False))
        monkeypatch.setattr(fn.dist, "get_world_size", lambda group=None: size)
    return set_size


AR = PlanStep("allreduce_forward_identity_backward", ("tp",))
RS = PlanStep("reducescatter_forward_allgather_backward", ("n", "tp"))
AG = PlanStep("allgather_forward_reducescatter_backward", ("n", "tp"))
DX = PlanStep("identity_forward_allreduce_backward", ("tp",))


@pytest.mark.parametrize("size", [2, 4, 8])
def test_nvls_groups_fuse_the_allreduce_by_default(ranks, monkeypatch, size):
    """With a multicast heap, the row-parallel GEMM + all-reduce, the replicated
    operand's gradient all-reduce and the row reduce-scatter output run as the
    fused NVLS kernel at every group size."""
    ranks(size, nvls=True)
    monkeypatch.setattr(fn, "_MAX_FUSED_EPILOGUE_RANKS", 0)
    monkeypatch.setattr(fn, "_FUSED_NVLS", True)
    assert fn.provider(executor(output_steps=[AR])).kind == "gemm_allreduce"
    f = fn.provider(executor(input0_steps=[DX]))
    assert f.kind == "dgrad_allreduce" and f.operand == 0
    assert fn.provider(executor(output_steps=[RS])).kind == "gemm_reducescatter"


def test_nvls_fusion_can_be_switched_off(ranks, monkeypatch):
    ranks(8, nvls=True)
    monkeypatch.setattr(fn, "_MAX_FUSED_EPILOGUE_RANKS", 0)
    monkeypatch.setattr(fn, "_OVERLAP_AR_CHUNKS", 0)
    monkeypatch.setattr(fn, "_FUSED_NVLS", False)
    assert fn.provider(executor(output_steps=[AR])) is None


@pytest.mark.parametrize("size", [2, 4, 8])
def test_defaults_keep_gemm_then_collective(ranks, monkeypatch, size):
    ranks(size)
    monkeypatch.setattr(fn, "_MAX_FUSED_EPILOGUE_RANKS", 0)
    monkeypatch.setattr(fn, "_OVERLAP_AR_CHUNKS", 0)
    assert fn.provider(executor(output_steps=[AR])) is None
    assert fn.provider(executor(output_steps=[RS])) is None
    assert fn.provider(executor(input0_steps=[DX])) is None


@pytest.mark.parametrize("size,fused", [(2, True), (4, False), (8, False)])
def test_fused_allgather_gemm_up_to_two_ranks(ranks, monkeypatch, size, fused):
    ranks(size)
    monkeypatch.setattr(fn, "_MAX_FUSED_GATHER_RANKS", 2)
    f = fn.provider(executor(input0_steps=[AG]))
    assert (f is not None and f.kind == "allgather_gemm") == fused


def test_epilogue_fusion_on_request(ranks, monkeypatch):
    ranks(2)
    monkeypatch.setattr(fn, "_MAX_FUSED_EPILOGUE_RANKS", 2)
    assert fn.provider(executor(output_steps=[AR])).kind == "gemm_allreduce"
    assert fn.provider(executor(output_steps=[RS])).kind == "gemm_reducescatter"
    f = fn.provider(executor(input1_steps=[DX]))
    assert f.kind == "dgrad_allreduce" and f.operand == 1


def test_overlapped_allreduce_on_request(ranks, monkeypatch):
    ranks(8)
    monkeypatch.setattr(fn, "_MAX_FUSED_EPILOGUE_RANKS", 0)
    monkeypatch.setattr(fn, "_OVERLAP_AR_CHUNKS", 4)
    f = fn.provider(executor(output_steps=[AR]))
    assert f.kind == "gemm_allreduce" and f.overlap_chunks == 4


def test_non_cuda_or_fp32_operands_are_never_fused(ranks, monkeypatch):
    ranks(2)
    monkeypatch.setattr(fn, "_MAX_FUSED_EPILOGUE_RANKS", 8)
    ex = executor(output_steps=[AR])
    ex.x0 = SimpleNamespace(is_cuda=True, dtype=torch.float32)
    assert fn.provider(ex) is None


def test_fused_nvls_kernel_reduces_in_the_gemm_epilogue_by_default(monkeypatch):
    """Unless overridden, the fused GEMM + NVLS launch has no dedicated reducer
    CTA pairs (overlap mode: the GEMM's epilogue warps reduce) and the kernel
    picks its lag (two waves of CTA pairs); both reach the extension call."""
    import importlib
    monkeypatch.delenv("EINSHARD_NVLS_REDUCER_CLUSTERS", raising=False)
    monkeypatch.delenv("EINSHARD_NVLS_LAG", raising=False)
    mod = importlib.reload(fn)
    try:
        assert mod._NVLS_REDUCER_CLUSTERS == 0 and mod._NVLS_LAG == 0
        calls = []

        class Ext:
            def gemm_allreduce_nvls(self, cid, a, b, out, reducers, lag, err):
                calls.append((reducers, lag))

        ws = SimpleNamespace(nvls=True, broken=False, cid=3, enter=lambda kind: None)
        monkeypatch.setattr(mod._native, "require", lambda: Ext())
        monkeypatch.setattr(mod._native, "error_word", lambda device: None)
        monkeypatch.setattr(mod, "_prepare", lambda t: t)
        from torch_einshard_b200.parallel import symmetric
        monkeypatch.setattr(symmetric, "workspace_for", lambda group, nbytes: ws)
        a = torch.zeros(1, 4, 8, dtype=torch.bfloat16)
        b = torch.zeros(1, 8, 16, dtype=torch.bfloat16)
        out = mod.gemm_allreduce_nvls(SimpleNamespace(group=None), a, b)
        assert out is not None and out.shape == (1, 4, 16) and calls == [(0, 0)]
    finally:
        importlib.reload(fn)
