"""Halo-exchange convolution benchmark (the BASELINE halo-conv config).

    torchrun --nproc-per-node N benchmarks/bench_halo_conv.py [--impl native|reference] [--path conv|window]

Global input b=16, h=w=2048, c=128 bf16 ~N(0,1); 3x3x128x128 kernel ~N(0,0.02);
output 'b h/sp_h w/sp_w o'.  Mesh (sp_h, sp_w) = (1,1), (2,1), (2,2), (2,4) for
N = 1, 2, 4, 8; the h split over sp_h = 2 is uneven, [1040, 1008].

  --path conv    einconv 'b h/sp_h w/sp_w c, kh kw c o -> b h/sp_h w/sp_w o'
                 (native: halo exchange + implicit-GEMM tcgen05 conv; reference:
                 halo exchange + cuDNN)
  --path window  einwindow 'b h/sp_h w/sp_w c -> b h/sp_h w/sp_w kh kw c' (halo 1)
                 then einshard 'b h w kh kw c, kh kw c o -> b h w o' (the window
                 tensor is materialised: 9x the input)

Prints one JSON line (rank 0): ms per forward as the max over ranks (CUDA
events), TFLOP/s over all GPUs, and the fraction of the measured bf16 peak.
"""

import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from common import ClockSampler, peaks, visible_gpu_indices  # noqa: E402

MESHES = {1: (1, 1), 2: (2, 1), 4: (2, 2), 8: (2, 4)}


def split(n, parts, uneven=None):
    if parts == 1:
        return [n]
    if uneven is not None and parts == 2:
        return list(uneven)
    return [n // parts] * parts


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--path", choices=("conv", "window"), default="conv")
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--hw", type=int, default=2048)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--breakdown", action="store_true",
                   help="after the timed steps, one more step under torch.profiler: every rank's kernels with their "
                        "device time, one JSON line per rank (not a timing run)")
    args = p.parse_args()
    if "RANK" not in os.environ:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT="29631", RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    world, rank = dist.get_world_size(), dist.get_rank()
    from torch.distributed.device_mesh import init_device_mesh
    mh, mw = MESHES[world]
    mesh = init_device_mesh("cuda", (mh, mw), mesh_dim_names=("sp_h", "sp_w"))
    B, H, W, C, O = args.batch, args.hw, args.hw, 128, 128
    hs = split(H, mh, uneven=(H * 1040 // 2048, H - H * 1040 // 2048))
    ws = split(W, mw)
    shapes = {"sp_h": {"h": hs}, "sp_w": {"w": ws}}
    rh, rw = mesh["sp_h"].get_local_rank(), mesh["sp_w"].get_local_rank()
    gen = torch.Generator(device="cuda").manual_seed(0 + rank)
    x = torch.randn(B, hs[rh], ws[rw], C, device="cuda", generator=gen).to(torch.bfloat16)
    gw = torch.Generator(device="cuda").manual_seed(1234)
    w = (torch.randn(3, 3, C, O, device="cuda", generator=gw) * 0.02).to(torch.bfloat16)

    if args.impl == "native":
        sys.path.insert(0, ROOT)
        import torch_einshard_b200 as es
        es.setup_native_comm(mesh)
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

    if args.path == "conv":
        def step():
            return es.einconv("b h/sp_h w/sp_w c, kh kw c o -> b h/sp_h w/sp_w o", x, w, {"h": "kh", "w": "kw"},
                              mesh=mesh, shapes=shapes, checkpoint=None)
    else:
        def step():
            win = es.einwindow("b h/sp_h w/sp_w c -> b h/sp_h w/sp_w kh kw c", x, {"h": "kh", "w": "kw"},
                               {"h": 1, "w": 1}, mesh=mesh, shapes=shapes)
            return es.einshard("b h w kh kw c, kh kw c o -> b h w o", win, w)

    sampler = ClockSampler(visible_gpu_indices(world)) if rank == 0 else None
    if sampler:
        sampler.start()
    with torch.no_grad():
        for _ in range(args.warmup):
            y = step()
        del y
        dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if sampler:
            sampler.mark_start()
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        torch.cuda.synchronize()
        if sampler:
            sampler.mark_end()
        dist.barrier()
    if args.breakdown:
        from torch.profiler import ProfilerActivity, profile
        with torch.no_grad(), profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        kernels = {}
        for ev in prof.events():
            if ev.device_type.name == "CUDA":
                k = kernels.setdefault(ev.name[:90], [0, 0.0])
                k[0] += 1
                k[1] += ev.device_time_total / 1e3
        top = sorted(kernels.items(), key=lambda kv: -kv[1][1])[:12]
        line = json.dumps({"breakdown_rank": rank, "mesh_rank": [rh, rw],
                           "kernels_ms": [[name, n, round(t, 3)] for name, (n, t) in top],
                           "total_ms": round(sum(t for _, t in kernels.values()), 3)})
        lines = [None] * world
        dist.all_gather_object(lines, line)
        if rank == 0:
            for entry in lines:
                print(entry, flush=True)
    ms = torch.tensor([t0.elapsed_time(t1) / args.steps], device="cuda", dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = ms.item()
    flops = 2.0 * B * H * W * 9 * C * O
    tflops = flops / (ms / 1e3) / 1e12
    if rank == 0:
        print(json.dumps({"metric": "halo-conv ms (forward)", "value": round(ms, 3), "unit": "ms",
                          "higher_is_better": False, "n_gpus": world, "impl": args.impl, "path": args.path,
                          "clocks": sampler.stop() if sampler else None, "tflops_all_gpus": round(tflops, 1),
                          "roofline_frac": round(tflops / world / peaks()["bf16_tflops"], 3),
                          "roofline_of": f"{peaks()['source']} bf16_tflops per GPU",
                          "config": {"b": B, "h": H, "w": W, "c": C, "o": O, "mesh": [mh, mw], "h_split": hs,
                                     "dtype": "bf16", "l2": "inputs larger than L2; no flush"}}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
