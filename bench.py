"""Flagship benchmark: tensor-parallel MLP forward+backward through the einshard API.

Config (the reference's TP-contraction benchmark): b=8, n=4096, c=8192,
h=28672, bf16, activations ~N(0,1), weights ~N(0,0.02), seed 0, tp = number of
GPUs (one rank per GPU).  The global problem is fixed, so scaling is strong.

    python bench.py --gpus N --steps K --warmup W [--impl native|reference]

Prints one JSON line on rank 0.  ``value`` is whole-job TFLOP/s from CUDA
events around exactly K steps (barrier + synchronize on both sides, max over
ranks).  Inputs (x: 512 MiB bf16 per rank) are larger than the 126 MB L2, so
no explicit flush is needed between steps.  ``e2e`` repeats the measurement
end to end through the public API: each rank copies its b/tp slice of the
step's input from pinned host memory, the step gathers x with
``einshard("b/tp n c -> b n c")`` (both arms, each with its own framework), and
the loss is read back to the host.
"""

import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

from benchmarks.common import ClockSampler, visible_gpu_indices

HERE = os.path.dirname(os.path.abspath(__file__))
CFG = dict(b=8, n=4096, c=8192, h=28672)
METRIC = "TP-contraction TFLOP/s"
BASELINE_VALUE = None  # the reference publishes no number (BASELINE.json "published": {})


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["native", "reference"], default="native")
    p.add_argument("--small", action="store_true", help="reduced shapes for smoke runs (not a bench number)")
    p.add_argument("--kernel-table", type=int, default=0, metavar="N",
                   help="after the timed steps, profile one more step (torch.profiler) and print the N kernels "
                        "with the most device time to stderr (a breakdown, not a bench number)")
    return p.parse_args()


def init_dist(args):
    if "RANK" not in os.environ:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29000 + os.getpid() % 2000))
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    world = dist.get_world_size()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    return dist.get_rank(), world, local


def max_over_ranks(value):
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(step, steps):
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    return max_over_ranks(start.elapsed_time(end))


def build_native(cfg, world, rank):
    sys.path.insert(0, HERE)
    import torch_einshard_b200 as es
    from torch_einshard_b200.models.tp_mlp import TPMLP
    from torch.distributed.device_mesh import init_device_mesh
    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    es.setup_native_comm(mesh)
    model = TPMLP(cfg["c"], cfg["h"], mesh, device="cuda")
    return es, model, mesh


def build_reference(cfg, world, rank):
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "torch_einshard")):
        return None, "reference is not installed under baseline/_ref", None
    sys.path.insert(0, ref)
    shim = os.path.join(HERE, "baseline", "parsley_shim")
    sys.path.insert(0, shim)
    try:
        import torch_einshard as es  # noqa: F401
    except Exception as error:  # noqa: BLE001
        return None, f"reference import failed: {error!r}", None
    from torch.distributed.device_mesh import init_device_mesh
    import torch.nn.functional as F
    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    local = cfg["h"] // world
    gen = torch.Generator(device="cpu").manual_seed(0)
    full1 = torch.empty(cfg["h"], cfg["c"]).normal_(0.0, 0.02, generator=gen)
    full2 = torch.empty(cfg["c"], cfg["h"]).normal_(0.0, 0.02, generator=gen)
    w1 = torch.nn.Parameter(full1[rank * local:(rank + 1) * local].to("cuda", torch.bfloat16))
    w2 = torch.nn.Parameter(full2[:, rank * local:(rank + 1) * local].contiguous().to("cuda", torch.bfloat16))

    class RefMLP(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w1, self.w2 = w1, w2

        def forward(self, x):
            h = es.einshard("b n c, h/tp c -> b n h/tp", x, self.w1, mesh=mesh)
            y = es.einshard("b n h/tp, c h/tp -> b n c // tp", F.silu(h), self.w2, mesh=mesh)
            return es.einshard("b n c // tp -> b n c", y, mesh=mesh)

    return es, RefMLP(), mesh


def native_launches(impl):
    """Kernel launches of this framework so far (its extension's counter).  The
    reference arm never imports this package, so its count is 0."""
    if impl != "native":
        return 0
    from torch_einshard_b200.ops import _native
    mod = _native.module()
    return int(mod.launch_count()) if mod is not None else 0


def main():
    args = parse()
    rank, world, local = init_dist(args)
    cfg = dict(CFG)
    if args.small:
        cfg = dict(b=2, n=512, c=1024, h=4096)
    if args.impl == "reference":
        es, model, mesh = build_reference(cfg, world, rank)
        if es is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": model}), flush=True)
            dist.destroy_process_group()
            return
    else:
        es, model, mesh = build_native(cfg, world, rank)

    torch.manual_seed(0)
    b, n, c, h = cfg["b"], cfg["n"], cfg["c"], cfg["h"]
    x = torch.randn(b, n, c, device="cuda", dtype=torch.bfloat16).requires_grad_(True)
    dy = torch.randn(b, n, c, device="cuda", dtype=torch.bfloat16)

    def step():
        x.grad = None
        for p in model.parameters():
            p.grad = None
        y = model(x)
        y.backward(dy)

    # ---------------------------------------------------------------- device-timed
    sampler = ClockSampler(visible_gpu_indices(world)) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches0 = native_launches(args.impl)
    if sampler:
        sampler.mark_start()
    ms = timed(step, args.steps)
    if sampler:
        sampler.mark_end()
    clocks = sampler.stop() if sampler else None
    launches = native_launches(args.impl) - launches0
    flops = 12.0 * b * n * c * h  # 2 forward GEMMs + 4 backward GEMMs of 2*b*n*c*h each
    value = flops * args.steps / (ms / 1e3) / 1e12

    if args.kernel_table:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        if rank == 0:
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=args.kernel_table,
                                            max_name_column_width=90), file=sys.stderr, flush=True)

    # ---------------------------------------------------------------- end to end
    # Each rank loads only its b/tp slice of the step's input from pinned host
    # memory (one step ahead, on a side stream), and the step gathers the full x
    # over NVLink through the framework's own API ("b/tp n c -> b n c"): the job
    # reads every input byte from the host once, not once per rank.
    b_local = b // world if b % world == 0 else b
    host_x = torch.randn(b_local, n, c, dtype=torch.bfloat16).pin_memory()
    copy_stream = torch.cuda.Stream()
    bufs = [torch.empty(b_local, n, c, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    losses = []

    def prefetch(i):
        with torch.cuda.stream(copy_stream):
            bufs[i % 2].copy_(host_x, non_blocking=True)
            ready[i % 2].record(copy_stream)

    def e2e_step(i):
        torch.cuda.current_stream().wait_event(ready[i % 2])
        xin = bufs[i % 2].requires_grad_(True)
        for p in model.parameters():
            p.grad = None
        xfull = xin if b_local == b else es.einshard("b/tp n c -> b n c", xin, mesh=mesh)
        y = model(xfull)
        loss = y.float().square().mean()
        loss.backward()
        xin.grad = None
        xin.requires_grad_(False)
        if i + 1 < total_e2e:
            prefetch(i + 1)  # next input streams in while this step's kernels run
        losses.append(loss.item())

    total_e2e = args.warmup + args.steps
    prefetch(0)
    for i in range(args.warmup):
        e2e_step(i)
    dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.warmup, total_e2e):
        e2e_step(i)
    t1.record()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1))
    e2e_value = flops * args.steps / (e2e_ms / 1e3) / 1e12

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 4),
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) random-init weights)",
            "config": {
                "model": "tp_mlp (b n c, h/tp c -> b n h/tp; silu; b n h/tp, c h/tp -> b n c // tp -> b n c)",
                "global_batch": b,
                "seq_len": n,
                "c": c,
                "h": h,
                "parallelism": f"tp{world}",
                "fwd_bwd": True,
                "l2": "inputs larger than L2 (x is 512 MiB bf16 per rank); no flush",
                "small": bool(args.small),
            },
            "clocks": clocks,
            "e2e": {
                "value": round(e2e_value, 2),
                "unit": "TFLOP/s",
                "h2d_bytes_per_step": host_x.numel() * host_x.element_size(),
                "d2h_bytes_per_step": 4,
                "ms_per_step": round(e2e_ms / args.steps, 4),
                "input": ("per rank: its b/tp slice of x copied from pinned host memory, then gathered "
                          "with einshard('b/tp n c -> b n c'); bytes are per rank") if b_local != b else
                         "x copied from pinned host memory",
            },
            "gpu_launches": launches,
            "impl": args.impl,
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    if args.impl == "native":
        from torch_einshard_b200.parallel import symmetric
        symmetric.deactivate()  # collective close of the symmetric heaps before the group goes
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
