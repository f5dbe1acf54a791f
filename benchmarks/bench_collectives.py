"""Collective bandwidth: this framework's native collectives against NCCL.

    torchrun --nproc-per-node N benchmarks/bench_collectives.py [--ops all_reduce,all_gather,reduce_scatter]
        [--sizes 4K,1M,64M,512M] [--dtype bf16] [--iters 20] [--warmup 5]

For every operation and message size (bytes of the full tensor: the
all-reduce buffer, the all-gather output, the reduce-scatter input), both arms
run on the same tensors: ``native`` is the communicator the einshard helpers
use (NVLS multimem kernels when the heap has a multicast mapping), ``nccl`` is
``torch.distributed`` on the same group.  Each call is timed with CUDA events
after warm-up; the per-iteration median is taken as the maximum over ranks.
One JSON line per (op, size, arm) on rank 0 with algbw (bytes / time) and
busbw (NCCL's convention: all-reduce x 2(P-1)/P, all-gather and
reduce-scatter x (P-1)/P), and a final line with the clock record of the run.
No reference counterpart (the reference has no collective benchmark); the
baseline arm is NCCL, which the reference's helpers call
(``src/torch_einshard/helpers.py:27-139``).
"""

import json
import os
import statistics
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from benchmarks.common import ClockSampler, visible_gpu_indices  # noqa: E402

DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def parse_size(text):
    text = text.strip().upper()
    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    return int(float(text[:-1]) * mult[text[-1]]) if text[-1] in mult else int(text)


def time_ms(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    times = []
    for _ in range(iters):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    med = torch.tensor([statistics.median(times)], dtype=torch.float64, device="cuda")
    dist.all_reduce(med, op=dist.ReduceOp.MAX)
    return float(med.item())


def main():
    import argparse
    p = argparse.ArgumentParser()
    p.add_argument("--ops", default="all_reduce,all_gather,reduce_scatter")
    p.add_argument("--sizes", default="4K,64K,1M,4M,16M,64M,256M,512M")
    p.add_argument("--dtype", default="bf16", choices=sorted(DTYPES))
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--arms", default="native,nccl")
    args = p.parse_args()

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    import torch_einshard_b200 as es
    from torch.distributed.device_mesh import init_device_mesh
    from torch_einshard_b200.ops import _native
    from torch_einshard_b200.parallel import symmetric
    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    es.setup_native_comm(mesh)
    symmetric._NVLS_AR_MIN_RANKS = 1  # time the native kernels at every group size
    group = mesh["tp"].get_group()
    comm = symmetric.communicator_for(group)
    dtype = DTYPES[args.dtype]
    esize = torch.tensor([], dtype=dtype).element_size()
    sampler = ClockSampler(visible_gpu_indices(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        sampler.mark_start()
    arms = args.arms.split(",")
    for op in args.ops.split(","):
        for size in [parse_size(s) for s in args.sizes.split(",")]:
            n = max(world, size // esize) // world * world
            full = torch.randn(n, device="cuda", dtype=dtype)
            shard = torch.randn(n // world, device="cuda", dtype=dtype)
            shapes = [n // world] * world
            for arm in arms:
                if arm == "native" and comm is None:
                    continue
                if op == "all_reduce":
                    buf = full.clone()
                    fn = (lambda: comm.all_reduce_(buf)) if arm == "native" else (lambda: dist.all_reduce(buf, group=group))
                    factor = 2.0 * (world - 1) / world
                elif op == "all_gather":
                    out = torch.empty(n, device="cuda", dtype=dtype)
                    fn = ((lambda: comm.all_gather(shard, 0, shapes)) if arm == "native"
                          else (lambda: dist.all_gather_into_tensor(out, shard, group=group)))
                    factor = (world - 1) / world
                else:
                    out = torch.empty(n // world, device="cuda", dtype=dtype)
                    fn = ((lambda: comm.reduce_scatter(full, 0, shapes)) if arm == "native"
                          else (lambda: dist.reduce_scatter_tensor(out, full, group=group)))
                    factor = (world - 1) / world
                ms = time_ms(fn, args.warmup, args.iters)
                nbytes = n * esize
                if rank == 0:
                    print(json.dumps({"name": f"{op}", "arm": arm, "bytes": nbytes, "world_size": world,
                                      "dtype": args.dtype, "max_over_ranks_ms": round(ms, 5),
                                      "algbw_gbs": round(nbytes / ms / 1e6, 2),
                                      "busbw_gbs": round(nbytes * factor / ms / 1e6, 2),
                                      "nvls": bool(comm is not None and comm.nvls) if arm == "native" else None}),
                          flush=True)
    torch.cuda.synchronize()
    _native.check_errors("cuda")
    if sampler:
        sampler.mark_end()
        print(json.dumps({"name": "clocks", "clocks": sampler.stop()}), flush=True)
    dist.barrier()
    from torch_einshard_b200.parallel import symmetric
    symmetric.deactivate()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
