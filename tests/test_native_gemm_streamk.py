"""Stream-K on the wide GEMM against a plain fp32 PyTorch matmul: every tile
split (forced) and the default hybrid (whole tiles for the full waves, the
partial last wave split over all SM pairs, fp32 partials reduce-added by TMA)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from torch_einshard_b200.ops import _native, gemm  # noqa: E402


@pytest.fixture
def streamk():
    mod = _native.require()
    mod.set_gemm_pair_mode(-1)
    mod.set_gemm_streamk(1)
    yield mod
    mod.set_gemm_streamk(-1)


def _check(a, b, out_dtype=None, act=None):
    _native.reset_errors()
    before = _native.require().launch_count()
    c = gemm.native_bmm(a, b, out_dtype=out_dtype, act=act)
    torch.cuda.synchronize()
    _native.check_errors(a.device)
    # the tail kernel and its finishing pass, plus the whole-tile launch when there are full waves
    assert _native.require().launch_count() - before in (2, 3)
    ref = torch.matmul(a.float(), b.float())
    if act == "silu":
        ref = torch.nn.functional.silu(ref)
    scale = ref.abs().max().item() + 1.0
    tol = 1e-3 if c.dtype == torch.float32 else 1e-2
    err = (c.float() - ref).abs().max().item()
    assert err <= tol * scale, f"max err {err} (scale {scale})"


@pytest.mark.parametrize("m,n,k", [(512, 1024, 8192), (1000, 1536, 4160), (768, 2048, 4100), (2048, 512, 16384)])
def test_streamk_shapes(streamk, m, n, k):
    torch.manual_seed(m + n + k)
    a = torch.randn(1, m, k, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1, k, n, device="cuda", dtype=torch.bfloat16)
    _check(a, b)


@pytest.mark.parametrize("a_t,b_t", [(True, False), (False, True), (True, True)])
def test_streamk_operand_layouts(streamk, a_t, b_t):
    m, n, k = 640, 1024, 6144
    a = torch.randn(1, k, m, device="cuda", dtype=torch.bfloat16).transpose(1, 2) if a_t else \
        torch.randn(1, m, k, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1, n, k, device="cuda", dtype=torch.bfloat16).transpose(1, 2) if b_t else \
        torch.randn(1, k, n, device="cuda", dtype=torch.bfloat16)
    _check(a, b)


def test_streamk_fp32_out_and_silu(streamk):
    a = torch.randn(1, 520, 4096, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1, 4096, 1030, device="cuda", dtype=torch.bfloat16)
    _check(a, b, out_dtype=torch.float32)
    _check(a, b, act="silu")


def test_streamk_weight_gradient_shape(streamk):
    """2048 x 2048 output with K = 65536 (a transformer weight gradient): 32
    pair tiles for 74 SM pairs, every pair gets an equal K slice."""
    g = torch.randn(1, 65536, 2048, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(1, 65536, 2048, device="cuda", dtype=torch.bfloat16)
    _check(g.transpose(1, 2), x)


def test_streamk_tail_by_default():
    """80 pair tiles for 74 SM pairs and 72 K blocks: one whole wave (a plain
    launch), the other 6 tiles split over all pairs (ragged M and N)."""
    mod = _native.require()
    mod.set_gemm_pair_mode(-1)
    mod.set_gemm_streamk(-1)
    torch.manual_seed(5)
    a = torch.randn(1, 2500, 4608, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1, 4608, 4000, device="cuda", dtype=torch.bfloat16)
    _check(a, b)
    _check(a, b, act="silu")


def test_streamk_not_for_short_k():
    mod = _native.require()
    mod.set_gemm_pair_mode(-1)
    mod.set_gemm_streamk(-1)
    a = torch.randn(1, 2500, 2048, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1, 2048, 4000, device="cuda", dtype=torch.bfloat16)
    before = mod.launch_count()
    gemm.native_bmm(a, b)
    torch.cuda.synchronize()
    assert mod.launch_count() - before == 1


def test_streamk_off_under_deterministic_algorithms(streamk):
    a = torch.randn(1, 512, 8192, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1, 8192, 1024, device="cuda", dtype=torch.bfloat16)
    torch.use_deterministic_algorithms(True)
    try:
        before = streamk.launch_count()
        c1 = gemm.native_bmm(a, b)
        c2 = gemm.native_bmm(a, b)
        torch.cuda.synchronize()
        assert streamk.launch_count() - before == 2  # one plain launch each
        assert torch.equal(c1, c2)
    finally:
        torch.use_deterministic_algorithms(False)
