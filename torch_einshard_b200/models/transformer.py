"""Decoder-only transformer with tensor parallelism written in einshard notation.

Every block is Megatron-style over the ``tp`` mesh dimension:

    x_t  = einshard("b s d -> b s d // tp", x)                   identity fwd, all-reduce of dx bwd
    q    = einshard("b s d, e/tp d -> b s e/tp", x_t, wq)         column parallel (local)
    ...  causal attention on the local heads (torch SDPA / flash)
    o    = einshard("b s e/tp, d e/tp -> b s d", attn, wo)       row parallel: fused GEMM + all-reduce
    a    = einshard("b s d, f/tp d -> b s f/tp", x_t, w_up,       column parallel, SiLU in
                    activation="silu")                            the GEMM's epilogue
    y    = einshard("b s f/tp, d f/tp -> b s d", a, w_dn)        row parallel: fused GEMM + all-reduce

Data parallelism over ``dp`` uses PyTorch DDP with
:func:`register_grad_reduction_hook_`: the hook averages every bucket over
``dp`` (the DDP group); parameters carry their einshard layouts (tp-sharded
or replicated) and need no extra reduction groups.  The
embedding, norms and LM head are replicated over ``tp``; their gradients are
identical on every tp rank because activations entering them are replicated.

Built from the reference's tensor-parallel patterns
(``docs/user-guide/tensor-parallel.md``); the reference ships no model.
"""

import math

import torch
import torch.utils.checkpoint
import torch.nn.functional as F

from ..api import einshard
from ..params import register_parameter_layout

__all__ = ["TransformerConfig", "TPTransformer", "transformer_flops_per_token"]


class TransformerConfig:
    def __init__(self, layers=24, d=2048, heads=16, mlp=8192, vocab=32000, seq=8192, dtype=torch.bfloat16):
        self.layers, self.d, self.heads, self.mlp, self.vocab, self.seq, self.dtype = \
            layers, d, heads, mlp, vocab, seq, dtype


def transformer_flops_per_token(cfg, *, backward=True):
    """Matmul FLOPs per token (dense projections, attention scores/values, LM head)."""
    dense = 2 * (4 * cfg.d * cfg.d + 2 * cfg.d * cfg.mlp)
    attention = 2 * 2 * cfg.seq * cfg.d / 2  # causal: half of QK^T and PV
    per_layer = dense + attention
    total = cfg.layers * per_layer + 2 * cfg.d * cfg.vocab
    return total * (3 if backward else 1)


class _Block(torch.nn.Module):
    def __init__(self, cfg, tp, tp_rank, gen, device):
        super().__init__()
        d, hd = cfg.d, cfg.d // cfg.heads
        self.local_heads = cfg.heads // tp
        self.head_dim = hd
        e = self.local_heads * hd
        f = cfg.mlp // tp

        def shard(rows, cols, std, *, dim):
            full = torch.empty(rows, cols).normal_(0.0, std, generator=gen)
            if dim == 0:
                piece = full[tp_rank * (rows // tp):(tp_rank + 1) * (rows // tp)]
            else:
                piece = full[:, tp_rank * (cols // tp):(tp_rank + 1) * (cols // tp)]
            return torch.nn.Parameter(piece.contiguous().to(device=device, dtype=cfg.dtype))

        std = 0.02
        self.wq = shard(d, d, std, dim=0)
        self.wk = shard(d, d, std, dim=0)
        self.wv = shard(d, d, std, dim=0)
        self.wo = shard(d, d, std / math.sqrt(2 * cfg.layers), dim=1)
        self.w_up = shard(cfg.mlp, d, std, dim=0)
        self.w_dn = shard(d, cfg.mlp, std / math.sqrt(2 * cfg.layers), dim=1)
        self.ln1 = torch.nn.LayerNorm(d, device=device, dtype=cfg.dtype)
        self.ln2 = torch.nn.LayerNorm(d, device=device, dtype=cfg.dtype)
        assert e == self.wq.shape[0] and f == self.w_up.shape[0]

    def forward(self, x, mesh):
        b, s, _ = x.shape
        h = einshard("b s d -> b s d // tp", self.ln1(x), mesh=mesh)
        q = einshard("b s d, e/tp d -> b s e/tp", h, self.wq, mesh=mesh)
        k = einshard("b s d, e/tp d -> b s e/tp", h, self.wk, mesh=mesh)
        v = einshard("b s d, e/tp d -> b s e/tp", h, self.wv, mesh=mesh)
        shape = (b, s, self.local_heads, self.head_dim)
        q, k, v = (t.reshape(shape).transpose(1, 2) for t in (q, k, v))
        attn = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        attn = attn.transpose(1, 2).reshape(b, s, self.local_heads * self.head_dim)
        x = x + einshard("b s e/tp, d e/tp -> b s d", attn, self.wo, mesh=mesh)
        h = einshard("b s d -> b s d // tp", self.ln2(x), mesh=mesh)
        act = einshard("b s d, f/tp d -> b s f/tp", h, self.w_up, mesh=mesh, activation="silu")
        return x + einshard("b s f/tp, d f/tp -> b s d", act, self.w_dn, mesh=mesh)


class TPTransformer(torch.nn.Module):
    def __init__(self, cfg, mesh, *, tp_dim="tp", device=None, seed=0, checkpoint=False):
        super().__init__()
        self.cfg, self.mesh = cfg, mesh
        self.checkpoint = checkpoint  # recompute each block in backward (activation checkpointing)
        tp_mesh = mesh[tp_dim]
        tp = tp_mesh.size()
        tp_rank = tp_mesh.get_local_rank()
        if cfg.heads % tp or cfg.mlp % tp:
            raise ValueError("heads and mlp must be divisible by tp")
        gen = torch.Generator(device="cpu").manual_seed(seed)
        self.embed = torch.nn.Parameter(
            torch.empty(cfg.vocab, cfg.d).normal_(0.0, 0.02, generator=gen).to(device=device, dtype=cfg.dtype))
        self.blocks = torch.nn.ModuleList(_Block(cfg, tp, tp_rank, gen, device) for _ in range(cfg.layers))
        self.ln_f = torch.nn.LayerNorm(cfg.d, device=device, dtype=cfg.dtype)
        self._register_metadata(mesh)

    def _register_metadata(self, mesh):
        names = tuple(mesh.mesh_dim_names)
        for block in self.blocks:
            for w in (block.wq, block.wk, block.wv, block.w_up):
                register_parameter_layout(w, "o/tp i", mesh_dim_names=names)
            for w in (block.wo, block.w_dn):
                register_parameter_layout(w, "o i/tp", mesh_dim_names=names)
            for ln in (block.ln1, block.ln2):
                for p in ln.parameters():
                    register_parameter_layout(p, "c", mesh_dim_names=names)
        register_parameter_layout(self.embed, "v d", mesh_dim_names=names)
        for p in self.ln_f.parameters():
            register_parameter_layout(p, "c", mesh_dim_names=names)

    def forward(self, tokens, targets=None):
        x = F.embedding(tokens, self.embed)
        for block in self.blocks:
            if self.checkpoint and torch.is_grad_enabled():
                x = torch.utils.checkpoint.checkpoint(block, x, self.mesh, use_reentrant=False)
            else:
                x = block(x, self.mesh)
        x = self.ln_f(x)
        logits = einshard("b s d, v d -> b s v", x, self.embed)
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().flatten(0, 1), targets.flatten())
