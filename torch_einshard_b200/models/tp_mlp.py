"""Tensor-parallel MLP written with einshard formulas (the flagship benchmark model).

    a   = einshard("b n c, h/tp c -> b n h/tp", x, w1,        column parallel, SiLU
                   activation="silu")                          in the GEMM's epilogue
    y_p = einshard("b n h/tp, c h/tp -> b n c // tp", a, w2)  row parallel, partial sums
    y   = einshard("b n c // tp -> b n c", y_p)                all-reduce over tp

The column-parallel step is a rank-local contraction (no collective; the
gradient of the replicated x stays a partial sum over tp, as in the
reference's executor) and the row-parallel step ends with one all-reduce over
tp.  Which kernel runs that all-reduce is decided by the fusion policy in
``ops/fused_native.py`` (group size, shapes, environment overrides).

The pattern is the reference's tensor-parallel MLP
(``docs/user-guide/tensor-parallel.md``, ``tests/test_scigpt_patterns.py``);
the reference ships no model class.
"""

import torch

from ..api import einshard

__all__ = ["TPMLP", "tp_mlp_flops"]


class TPMLP(torch.nn.Module):
    def __init__(self, c, h, mesh, *, tp_dim="tp", dtype=torch.bfloat16, device=None, std=0.02, seed=0,
                 single_formula=True):
        super().__init__()
        # single_formula: write the row-parallel step as one formula
        # ("b n h/tp, c h/tp -> b n c"), whose plan is the same local contraction
        # followed by the same all-reduce as the two-call chain below, so the
        # executor can run both as one fused kernel.
        self.single_formula = single_formula
        tp = mesh[tp_dim].size() if hasattr(mesh[tp_dim], "size") else 1
        if h % tp:
            raise ValueError(f"hidden size {h} is not divisible by tp={tp}")
        self.mesh, self.tp_dim, self.tp = mesh, tp_dim, tp
        local = h // tp
        gen = torch.Generator(device="cpu").manual_seed(seed)
        rank = mesh[tp_dim].get_local_rank() if hasattr(mesh[tp_dim], "get_local_rank") else 0
        # every rank draws the full weights from the same seed and keeps its shard
        full1 = torch.empty(h, c, dtype=torch.float32).normal_(0.0, std, generator=gen)
        full2 = torch.empty(c, h, dtype=torch.float32).normal_(0.0, std, generator=gen)
        self.w1 = torch.nn.Parameter(full1[rank * local:(rank + 1) * local].to(device=device, dtype=dtype))
        self.w2 = torch.nn.Parameter(full2[:, rank * local:(rank + 1) * local].contiguous().to(device=device, dtype=dtype))

    def forward(self, x):
        t = self.tp_dim
        a = einshard(f"b n c, h/{t} c -> b n h/{t}", x, self.w1, mesh=self.mesh, activation="silu")
        if self.single_formula:
            return einshard(f"b n h/{t}, c h/{t} -> b n c", a, self.w2, mesh=self.mesh)
        y = einshard(f"b n h/{t}, c h/{t} -> b n c // {t}", a, self.w2, mesh=self.mesh)
        return einshard(f"b n c // {t} -> b n c", y, mesh=self.mesh)


def tp_mlp_flops(b, n, c, h, *, backward=True):
    """Whole-job FLOPs of one step (2 GEMMs forward, 4 more in backward)."""
    gemm = 2.0 * b * n * c * h
    return gemm * (6 if backward else 2)
