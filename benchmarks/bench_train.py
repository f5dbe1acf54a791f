"""Transformer training benchmark (the BASELINE training config).

    torchrun --nproc-per-node N benchmarks/bench_train.py [--impl native|reference]

24 layers, d=2048, 16 heads, MLP 8192, seq 8192, batch 8 per dp rank, vocab
32000, bf16 parameters and activations, AdamW, tokens uniform in [0, 32000)
from seed 0.  Mesh (dp, tp) = (1,1), (2,1), (2,2), (2,4) for N = 1, 2, 4, 8.
Tensor parallelism is Megatron-style through einshard formulas (column
parallel q/k/v/up, row parallel o/down); data parallelism is DDP with
``register_grad_reduction_hook_``.  With tp = 1 every block is activation
checkpointed in both arms (the full-sequence activations of 24 layers do not
fit next to the optimizer otherwise).

Native arm: ``torch_einshard_b200.models.TPTransformer`` (tcgen05 GEMMs, fused
GEMM + NVLink all-reduce for the row-parallel steps).  Reference arm: the
same network written with the reference's ``einshard`` and parameter API.

Prints one JSON line (rank 0): tokens/s over the whole job from CUDA events
around K steps (max over ranks) and the model TFLOP/s it implies.
"""

import argparse
import json
import math
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.nn.functional as F
import torch.utils.checkpoint
from torch.nn.parallel import DistributedDataParallel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from common import ClockSampler, visible_gpu_indices  # noqa: E402
MESHES = {1: (1, 1), 2: (2, 1), 4: (2, 2), 8: (2, 4)}


class Cfg:
    def __init__(self, small=False):
        if small:
            self.layers, self.d, self.heads, self.mlp, self.vocab, self.seq, self.batch = 2, 512, 8, 2048, 4096, 1024, 2
        else:
            self.layers, self.d, self.heads, self.mlp, self.vocab, self.seq, self.batch = 24, 2048, 16, 8192, 32000, 8192, 8
        self.dtype = torch.bfloat16


def flops_per_token(cfg):
    dense = 2 * (4 * cfg.d * cfg.d + 2 * cfg.d * cfg.mlp)
    attention = 2 * 2 * cfg.seq * cfg.d / 2
    return 3 * (cfg.layers * (dense + attention) + 2 * cfg.d * cfg.vocab)


def reference_model(es, cfg, mesh, device):
    """The same network as the native model, written with the reference's API."""
    tp = mesh["tp"].size()
    tp_rank = mesh["tp"].get_local_rank()
    names = tuple(mesh.mesh_dim_names)
    gen = torch.Generator(device="cpu").manual_seed(0)

    def shard(rows, cols, std, dim):
        full = torch.empty(rows, cols).normal_(0.0, std, generator=gen)
        piece = full.chunk(tp, dim=dim)[tp_rank]
        return torch.nn.Parameter(piece.contiguous().to(device=device, dtype=cfg.dtype))

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            std, d = 0.02, cfg.d
            self.wq, self.wk, self.wv = (shard(d, d, std, 0) for _ in range(3))
            self.wo = shard(d, d, std / math.sqrt(2 * cfg.layers), 1)
            self.w_up = shard(cfg.mlp, d, std, 0)
            self.w_dn = shard(d, cfg.mlp, std / math.sqrt(2 * cfg.layers), 1)
            self.ln1 = torch.nn.LayerNorm(d, device=device, dtype=cfg.dtype)
            self.ln2 = torch.nn.LayerNorm(d, device=device, dtype=cfg.dtype)
            for w in (self.wq, self.wk, self.wv, self.w_up):
                es.register_parameter_layout(w, "o/tp i", mesh_dim_names=names)
            for w in (self.wo, self.w_dn):
                es.register_parameter_layout(w, "o i/tp", mesh_dim_names=names)
            for p in list(self.ln1.parameters()) + list(self.ln2.parameters()):
                es.register_parameter_layout(p, "c", mesh_dim_names=names)

        def forward(self, x):
            b, s, _ = x.shape
            hl, hd = cfg.heads // tp, cfg.d // cfg.heads
            h = es.einshard("b s d -> b s d // tp", self.ln1(x), mesh=mesh)
            q, k, v = (es.einshard("b s d, e/tp d -> b s e/tp", h, w, mesh=mesh) for w in (self.wq, self.wk, self.wv))
            q, k, v = (t.reshape(b, s, hl, hd).transpose(1, 2) for t in (q, k, v))
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(b, s, hl * hd)
            x = x + es.einshard("b s e/tp, d e/tp -> b s d", a, self.wo, mesh=mesh)
            h = es.einshard("b s d -> b s d // tp", self.ln2(x), mesh=mesh)
            up = es.einshard("b s d, f/tp d -> b s f/tp", h, self.w_up, mesh=mesh)
            return x + es.einshard("b s f/tp, d f/tp -> b s d", F.silu(up), self.w_dn, mesh=mesh)

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = torch.nn.Parameter(
                torch.empty(cfg.vocab, cfg.d).normal_(0.0, 0.02, generator=gen).to(device=device, dtype=cfg.dtype))
            self.blocks = torch.nn.ModuleList(Block() for _ in range(cfg.layers))
            self.ln_f = torch.nn.LayerNorm(cfg.d, device=device, dtype=cfg.dtype)
            es.register_parameter_layout(self.embed, "v d", mesh_dim_names=names)
            for p in self.ln_f.parameters():
                es.register_parameter_layout(p, "c", mesh_dim_names=names)
            self.checkpoint = False

        def forward(self, tokens, targets):
            x = F.embedding(tokens, self.embed)
            for block in self.blocks:
                if self.checkpoint:
                    x = torch.utils.checkpoint.checkpoint(block, x, use_reentrant=False)
                else:
                    x = block(x)
            logits = es.einshard("b s d, v d -> b s v", self.ln_f(x), self.embed)
            return F.cross_entropy(logits.float().flatten(0, 1), targets.flatten())

    return Model()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--small", action="store_true", help="reduced model for smoke runs (not a bench number)")
    p.add_argument("--checkpoint", choices=("auto", "on", "off"), default="auto")
    p.add_argument("--kernel-table", type=int, default=0, metavar="N",
                   help="after the timed steps, run one more step under torch.profiler and print the N kernels "
                        "with the most device time to stderr (a breakdown, not a bench number)")
    args = p.parse_args()
    if "RANK" not in os.environ:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT="29651", RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=600))
    world, rank = dist.get_world_size(), dist.get_rank()
    from torch.distributed.device_mesh import init_device_mesh
    dp, tp = MESHES[world]
    mesh = init_device_mesh("cuda", (dp, tp), mesh_dim_names=("dp", "tp"))
    cfg = Cfg(args.small)
    checkpoint = args.checkpoint == "on" or (args.checkpoint == "auto" and tp == 1 and not args.small)

    if args.impl == "native":
        sys.path.insert(0, ROOT)
        import torch_einshard_b200 as es
        from torch_einshard_b200.models.transformer import TPTransformer, TransformerConfig
        es.setup_native_comm(mesh)
        tcfg = TransformerConfig(cfg.layers, cfg.d, cfg.heads, cfg.mlp, cfg.vocab, cfg.seq, cfg.dtype)
        model = TPTransformer(tcfg, mesh, device="cuda", checkpoint=checkpoint)
    else:
        ref = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref, "torch_einshard")):
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}))
            dist.destroy_process_group()
            return
        sys.path.insert(0, ref)
        sys.path.insert(0, os.path.join(ROOT, "baseline", "parsley_shim"))
        import torch_einshard as es
        model = reference_model(es, cfg, mesh, "cuda")
        model.checkpoint = checkpoint

    ddp = DistributedDataParallel(model, process_group=mesh["dp"].get_group(), bucket_cap_mb=25)
    es.register_grad_reduction_hook_(ddp, mesh, ddp_group="dp")
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)

    gen = torch.Generator(device="cpu").manual_seed(0)
    dp_rank = mesh["dp"].get_local_rank()
    host = torch.randint(0, cfg.vocab, (dp, cfg.batch, cfg.seq + 1), generator=gen)[dp_rank].pin_memory()
    tokens_dev = torch.empty(cfg.batch, cfg.seq + 1, dtype=torch.int64, device="cuda")

    def step():
        tokens_dev.copy_(host, non_blocking=True)   # host -> device input every step
        loss = ddp(tokens_dev[:, :-1], tokens_dev[:, 1:])
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    sampler = ClockSampler(visible_gpu_indices(world)) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.mark_start()
    t0.record()
    losses = []
    for _ in range(args.steps):
        losses.append(step().detach())
    t1.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.mark_end()
    clocks = sampler.stop() if sampler else None
    dist.barrier()
    ms = torch.tensor([t0.elapsed_time(t1) / args.steps], device="cuda", dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = ms.item()
    if args.kernel_table and rank == 0:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=args.kernel_table, max_name_column_width=90),
              file=sys.stderr, flush=True)
    elif args.kernel_table:
        step()
        torch.cuda.synchronize()
    global_tokens = dp * cfg.batch * cfg.seq
    tok_s = global_tokens / (ms / 1e3)
    if rank == 0:
        print(json.dumps({"metric": "train tok/s", "value": round(tok_s, 1), "unit": "tokens/s",
                          "higher_is_better": True, "n_gpus": world, "impl": args.impl, "ms_per_step": round(ms, 2),
                          "model_tflops_all_gpus": round(tok_s * flops_per_token(cfg) / 1e12, 1),
                          "loss": round(float(losses[-1].item()), 4), "clocks": clocks, "activation_checkpointing": checkpoint,
                          "config": {"layers": cfg.layers, "d": cfg.d, "heads": cfg.heads, "mlp": cfg.mlp,
                                     "vocab": cfg.vocab, "seq_len": cfg.seq, "batch_per_dp": cfg.batch,
                                     "mesh": [dp, tp], "dtype": "bf16", "optimizer": "AdamW (fused)",
                                     "small": bool(args.small)}}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
