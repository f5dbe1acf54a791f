"""CPU / gloo benchmark (the BASELINE CPU config; runs without a GPU).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/bench_cpu_gloo.py [--impl native|reference]

Mesh (2, 4) named (dp, sp).  x: [1024, 2048], y: [2048, 512] fp32 ~N(0,1) from
seed 0; ``einshard("a/sp b/dp, b/dp c -> a/sp c")`` then the uneven gather
``einshard("a/sp c -> a c")`` with sp shapes [300, 250, 250, 224], both
checked against a local ``torch.einsum``.  One step = both calls (forward).
Prints one JSON line (rank 0): median ms per step over ranks' max.
"""

import argparse
import json
import os
import statistics
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    args = p.parse_args()
    dist.init_process_group("gloo")
    world, rank = dist.get_world_size(), dist.get_rank()
    if args.impl == "native":
        sys.path.insert(0, ROOT)
        import torch_einshard_b200 as es
    else:
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        sys.path.insert(0, os.path.join(ROOT, "baseline", "parsley_shim"))
        import torch_einshard as es
    from torch.distributed.device_mesh import init_device_mesh
    mesh = init_device_mesh("cpu", (2, world // 2), mesh_dim_names=("dp", "sp"))
    sp = mesh["sp"].size()
    a_shapes = [300, 250, 250, 224] if sp == 4 else es.compute_split_shapes(1024, sp)
    b_shapes = es.compute_split_shapes(2048, 2)
    shapes = {"sp": {"a": a_shapes}, "dp": {"b": b_shapes}}
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1024, 2048, generator=g)
    y = torch.randn(2048, 512, generator=g)
    rs, rd = mesh["sp"].get_local_rank(), mesh["dp"].get_local_rank()
    xs = torch.split(torch.split(x, a_shapes, 0)[rs], b_shapes, 1)[rd].contiguous()
    ys = torch.split(y, b_shapes, 0)[rd].contiguous()

    def step():
        z = es.einshard("a/sp b/dp, b/dp c -> a/sp c", xs, ys, mesh=mesh, shapes=shapes)
        return es.einshard("a/sp c -> a c", z, mesh=mesh, shapes=shapes)

    out = step()
    want = torch.einsum("ab,bc->ac", x, y)
    err = (out - want).abs().max().item() / want.abs().max().item()
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        dist.barrier()
        t0 = time.perf_counter()
        step()
        dist.barrier()
        times.append((time.perf_counter() - t0) * 1e3)
    med = torch.tensor([statistics.median(times)], dtype=torch.float64)
    dist.all_reduce(med, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(json.dumps({"metric": "cpu gloo einshard ms (contraction + uneven gather)", "value": round(med.item(), 3),
                          "unit": "ms", "higher_is_better": False, "n_procs": world, "impl": args.impl,
                          "max_rel_err_vs_torch_einsum": err,
                          "config": {"x": [1024, 2048], "y": [2048, 512], "dtype": "fp32", "mesh": [2, world // 2],
                                     "sp_shapes": a_shapes}}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
