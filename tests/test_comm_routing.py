"""Host-side routing of the native all-reduce (no GPU): which calls the native
kernel takes and which go back to torch.distributed, with a recording fake of
the extension."""

import pytest
import torch

from torch_einshard_b200.parallel import symmetric


class FakeMod:
    def __init__(self):
        self.calls = []

    def comm_all_reduce(self, cid, piece, scale, blocks, err):
        self.calls.append(("pull", piece.numel() * piece.element_size(), scale))

    def comm_all_reduce_push(self, cid, piece, scale, blocks, err):
        self.calls.append(("push", piece.numel() * piece.element_size(), scale))

    def nvls_all_reduce(self, cid, inp, out, scale, two_shot, err):
        assert inp is out
        self.calls.append(("nvls2" if two_shot else "nvls1", inp.numel() * inp.element_size(), scale))

    def comm_acquire(self, cid, err):
        self.calls.append(("acquire",))

    def nvls_quiesce(self, cid, err):
        self.calls.append(("quiesce",))


def make_comm(size=2, capacity=64 << 20):
    comm = object.__new__(symmetric.Communicator)
    comm.mod = FakeMod()
    comm.cid = 0
    comm.size = size
    comm.capacity = capacity
    comm.broken = False
    comm.closed = False
    comm.nvls = False
    comm.sms = 148
    comm.err = None
    return comm


@pytest.mark.parametrize("size", [2, 4, 8])
def test_small_buffers_take_the_native_kernel(size, monkeypatch):
    monkeypatch.delenv("EINSHARD_FAULT_INJECT", raising=False)
    comm = make_comm(size)
    t = torch.zeros(1 << 16, dtype=torch.bfloat16)   # 128 KiB
    assert comm.all_reduce_(t, 0.5) is True
    assert comm.mod.calls == [("push", 1 << 17, 0.5)]   # the push kernel is the default


def test_pull_kernel_on_request(monkeypatch):
    monkeypatch.delenv("EINSHARD_FAULT_INJECT", raising=False)
    monkeypatch.setattr(symmetric, "_AR_ALGO", "pull")
    comm = make_comm(2)
    assert comm.all_reduce_(torch.zeros(1 << 16, dtype=torch.bfloat16)) is True
    assert comm.mod.calls == [("pull", 1 << 17, 1.0)]


def test_push_pieces_fit_two_copies_in_the_region(monkeypatch):
    monkeypatch.delenv("EINSHARD_FAULT_INJECT", raising=False)
    monkeypatch.setattr(symmetric, "_NCCL_AR_MIN_BYTES", 1 << 62)
    comm = make_comm(2, capacity=1 << 20)
    assert comm.all_reduce_(torch.zeros(1 << 20, dtype=torch.bfloat16)) is True   # 2 MiB through a 1 MiB region
    sizes = [c[1] for c in comm.mod.calls]
    assert sum(sizes) == 2 << 20 and all(2 * b <= comm.capacity for b in sizes)


@pytest.mark.parametrize("size", [2, 4, 8])
def test_buffers_from_one_mib_go_to_nccl(size, monkeypatch):
    monkeypatch.delenv("EINSHARD_FAULT_INJECT", raising=False)
    comm = make_comm(size)
    t = torch.zeros(1 << 19, dtype=torch.bfloat16)   # 1 MiB
    assert comm.all_reduce_(t) is False
    assert comm.mod.calls == []


def test_declines_what_the_kernel_cannot_take(monkeypatch):
    monkeypatch.delenv("EINSHARD_FAULT_INJECT", raising=False)
    comm = make_comm()
    assert comm.all_reduce_(torch.zeros(7, dtype=torch.float32)) is False          # not a multiple of 16 bytes
    assert comm.all_reduce_(torch.zeros(8, 8).t()) is False                        # not contiguous
    assert comm.all_reduce_(torch.zeros(16, dtype=torch.int32)) is False           # dtype
    comm.broken = True
    assert comm.all_reduce_(torch.zeros(16)) is False                              # after a timeout
    assert comm.mod.calls == []


@pytest.mark.parametrize("size", [2, 4, 8])
def test_nvls_heaps_take_every_size(size, monkeypatch):
    """With a multicast mapping every all-reduce runs through the switch:
    one-shot up to the switch-over size, two-shot above it."""
    monkeypatch.delenv("EINSHARD_FAULT_INJECT", raising=False)
    comm = make_comm(size)
    comm.nvls = True
    small = torch.zeros(symmetric._NVLS_ONE_SHOT_MAX // 2, dtype=torch.bfloat16)
    large = torch.zeros(8 << 20, dtype=torch.bfloat16)       # 16 MiB
    assert comm.all_reduce_(small, 0.5)
    if size < symmetric._NVLS_AR_MIN_RANKS:
        # a two-shot NVLS all-reduce moves more bytes than a ring at 2 ranks: NCCL takes it
        assert not comm.all_reduce_(large)
        assert comm.mod.calls == [("nvls1", symmetric._NVLS_ONE_SHOT_MAX, 0.5)]
    else:
        assert comm.all_reduce_(large)
        assert comm.mod.calls == [("nvls1", symmetric._NVLS_ONE_SHOT_MAX, 0.5), ("nvls2", 16 << 20, 1.0)]


def test_nvls_pieces_when_larger_than_the_workspace(monkeypatch):
    monkeypatch.delenv("EINSHARD_FAULT_INJECT", raising=False)
    comm = make_comm(4, capacity=4 << 20)
    comm.nvls = True
    monkeypatch.setattr(symmetric, "workspace_for_group", lambda group, nbytes: comm)
    comm.group = None
    assert comm.all_reduce_(torch.zeros(5 << 20, dtype=torch.float32))   # 20 MiB through 4 MiB
    sizes = [c[1] for c in comm.mod.calls]
    assert sum(sizes) == 20 << 20 and all(b <= comm.capacity for b in sizes)


def test_protocol_switch_waits_for_the_other_kind(monkeypatch):
    """A copy-protocol kernel after NVLS collectives waits for their completion
    on every rank (quiesce), and an NVLS collective after copy kernels waits for
    peers' reads (acquire)."""
    monkeypatch.delenv("EINSHARD_FAULT_INJECT", raising=False)
    comm = make_comm(2)
    comm.nvls = True
    comm.all_reduce_(torch.zeros(64, dtype=torch.float32))
    comm.enter("copy")
    comm.enter("copy")
    comm.all_reduce_(torch.zeros(64, dtype=torch.float32))
    kinds = [c[0] for c in comm.mod.calls]
    assert kinds == ["nvls1", "quiesce", "acquire", "nvls1"]


def test_automatic_set_up_is_opt_in_and_needs_cuda(monkeypatch):
    """EINSHARD_AUTO_NATIVE_COMM lets the first lookup create a group's
    communicator; off by default, never on CPU / gloo, and disable() blocks it."""
    from torch_einshard_b200.parallel import symmetric
    monkeypatch.setitem(symmetric._state, "enabled", False)
    monkeypatch.setitem(symmetric._state, "auto_blocked", False)
    assert symmetric._AUTO is False or "EINSHARD_AUTO_NATIVE_COMM" in __import__("os").environ
    monkeypatch.setattr(symmetric, "_AUTO", False)
    assert symmetric.communicator_for(object()) is None and not symmetric.enabled()
    monkeypatch.setattr(symmetric, "_AUTO", True)
    monkeypatch.setattr(symmetric.torch.cuda, "is_available", lambda: False)
    assert symmetric.communicator_for(object()) is None and not symmetric.enabled()
    monkeypatch.setattr(symmetric.torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(symmetric.dist, "is_initialized", lambda: True)
    monkeypatch.setattr(symmetric._native, "available", lambda: True)
    made = []
    monkeypatch.setattr(symmetric, "_group_key", lambda group: ("k",))
    monkeypatch.setattr(symmetric, "communicator_for_group", lambda group: made.append(group) or "comm")
    group = object()
    assert symmetric.communicator_for(group) == "comm" and made == [group] and symmetric.enabled()
    symmetric.disable()
    assert symmetric.communicator_for(group) is None
