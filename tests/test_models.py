"""Model families on CPU gloo ranks: the TP MLP and the dp x tp transformer,
each checked against a plain single-process PyTorch computation."""

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch.nn.parallel import DistributedDataParallel

import torch_einshard_b200 as es
from conftest import assert_close
from dist_harness import run_ranks
from torch_einshard_b200.models.tp_mlp import TPMLP
from torch_einshard_b200.models.transformer import TPTransformer, TransformerConfig


def _mlp(ctx):
    mesh = ctx.mesh((ctx.world_size,), ("tp",))
    c, h = 16, 8 * ctx.world_size
    for single in (True, False):
        model = TPMLP(c, h, mesh, dtype=torch.float32, single_formula=single)
        gen = torch.Generator().manual_seed(0)
        w1 = torch.empty(h, c).normal_(0.0, 0.02, generator=gen)
        w2 = torch.empty(c, h).normal_(0.0, 0.02, generator=gen)
        x = torch.randn(2, 5, c)
        y = model(x)
        assert_close(y, F.silu(x @ w1.t()) @ w2.t(), rtol=1e-4, atol=1e-6)


def test_tp_mlp_matches_dense():
    run_ranks(_mlp, world_size=4)


def _reference_weights(cfg, seed=0):
    gen = torch.Generator().manual_seed(seed)
    embed = torch.empty(cfg.vocab, cfg.d).normal_(0.0, 0.02, generator=gen)
    blocks = []
    std = 0.02
    for _ in range(cfg.layers):
        w = {}
        for name, (rows, cols, s) in (("wq", (cfg.d, cfg.d, std)), ("wk", (cfg.d, cfg.d, std)),
                                      ("wv", (cfg.d, cfg.d, std)),
                                      ("wo", (cfg.d, cfg.d, std / math.sqrt(2 * cfg.layers))),
                                      ("w_up", (cfg.mlp, cfg.d, std)),
                                      ("w_dn", (cfg.d, cfg.mlp, std / math.sqrt(2 * cfg.layers)))):
            w[name] = torch.empty(rows, cols).normal_(0.0, s, generator=gen)
        blocks.append(w)
    return embed, blocks


def _reference_loss(cfg, embed, blocks, tokens, targets):
    x = F.embedding(tokens, embed)
    b, s, _ = x.shape
    hd = cfg.d // cfg.heads
    for w in blocks:
        h = F.layer_norm(x, (cfg.d,))
        q, k, v = (h @ w[n].t() for n in ("wq", "wk", "wv"))
        q, k, v = (t.reshape(b, s, cfg.heads, hd).transpose(1, 2) for t in (q, k, v))
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(b, s, cfg.d)
        x = x + a @ w["wo"].t()
        h = F.layer_norm(x, (cfg.d,))
        x = x + F.silu(h @ w["w_up"].t()) @ w["w_dn"].t()
    x = F.layer_norm(x, (cfg.d,))
    logits = x @ embed.t()
    return F.cross_entropy(logits.flatten(0, 1), targets.flatten())


def _transformer(ctx):
    mesh = ctx.mesh((2, ctx.world_size // 2), ("dp", "tp"))
    tp = mesh["tp"].size()
    cfg = TransformerConfig(layers=2, d=16, heads=4, mlp=32, vocab=24, seq=6, dtype=torch.float32)
    model = TPTransformer(cfg, mesh)
    dp_group = mesh["dp"].get_group()
    ddp = DistributedDataParallel(model, process_group=dp_group)
    es.register_grad_reduction_hook_(ddp, mesh, ddp_group="dp")
    gen = torch.Generator().manual_seed(1)
    all_tokens = torch.randint(0, cfg.vocab, (4, cfg.seq + 1), generator=gen)
    dp_rank = dist.get_rank(dp_group)
    tokens = all_tokens[2 * dp_rank:2 * dp_rank + 2, :-1]
    targets = all_tokens[2 * dp_rank:2 * dp_rank + 2, 1:]
    loss = ddp(tokens, targets)
    loss.backward()

    embed, blocks = _reference_weights(cfg)
    embed.requires_grad_(True)
    for w in blocks:
        for t in w.values():
            t.requires_grad_(True)
    ref_local = _reference_loss(cfg, embed, blocks, tokens, targets)
    assert_close(loss.detach(), ref_local.detach(), rtol=1e-4, atol=1e-5)
    # DDP averages over dp: the reference gradient is the mean of both dp halves
    ref_full = 0.5 * (_reference_loss(cfg, embed, blocks, all_tokens[:2, :-1], all_tokens[:2, 1:])
                      + _reference_loss(cfg, embed, blocks, all_tokens[2:, :-1], all_tokens[2:, 1:]))
    ref_full.backward()
    tp_rank = mesh["tp"].get_local_rank()
    rows = cfg.d // tp
    got = model.blocks[0].wq.grad
    want = blocks[0]["wq"].grad[tp_rank * rows:(tp_rank + 1) * rows]
    assert_close(got, want, rtol=1e-3, atol=1e-5)
    got = model.blocks[1].w_dn.grad
    cols = cfg.mlp // tp
    want = blocks[1]["w_dn"].grad[:, tp_rank * cols:(tp_rank + 1) * cols]
    assert_close(got, want, rtol=1e-3, atol=1e-5)
    assert_close(model.embed.grad, embed.grad, rtol=1e-3, atol=1e-5)


def test_dp_tp_transformer_matches_dense_reference():
    run_ranks(_transformer, world_size=4)
