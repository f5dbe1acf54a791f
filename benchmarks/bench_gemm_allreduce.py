"""Row-parallel contraction + all-reduce at the TP-MLP shape, four ways.

    torchrun --nproc-per-node N benchmarks/bench_gemm_allreduce.py [--m 32768 --n 8192 --h 28672]

Per rank: A [m, h/N] @ B [h/N, n], summed over the N ranks into every rank's
[m, n] output (bf16).  Arms, on the same tensors:
  fused      - one launch: wide GEMM + NVLS all-reduce (csrc/gemm_nvls.cu)
  gemm+nvls  - the native GEMM, then the native NVLS all-reduce
  gemm+nccl  - the native GEMM, then NCCL
  torch+nccl - torch.matmul (cuBLAS), then NCCL: what the reference runs
               (src/torch_einshard/einsum.py:132, helpers.py:27-32)
CUDA events per call after warm-up; inputs are larger than L2.  The median is
taken as the maximum over ranks.  Roofline of the fused call: the slower of the
FLOPs at the measured sustained bf16 peak and 9/8 of the output bytes over
NVLink at 770 GB/s per direction.  One JSON line per arm, then a clock record.
"""

import argparse
import json
import os
import statistics
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from benchmarks.common import ClockSampler, peaks, visible_gpu_indices  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--m", type=int, default=32768)
    p.add_argument("--n", type=int, default=8192)
    p.add_argument("--h", type=int, default=28672)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--arms", default="fused,gemm+nvls,gemm+nccl,torch+nccl")
    p.add_argument("--reducers", default="", help="comma list of reducer CTA-pair counts to time the fused arm with "
                                                   "(arms fused-R<n>; 0 = overlap mode); empty: the default")
    p.add_argument("--lags", default="", help="comma list of overlap-mode lags (arms fused-L<n>; 0 = auto)")
    args = p.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    import torch_einshard_b200 as es
    from torch.distributed.device_mesh import init_device_mesh
    from torch_einshard_b200.ops import _native, fused_native, gemm
    from torch_einshard_b200.parallel import symmetric
    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("tp",))
    es.setup_native_comm(mesh)
    symmetric._NVLS_AR_MIN_RANKS = 1  # time the native kernels at every group size
    group = mesh["tp"].get_group()
    comm = symmetric.communicator_for(group)
    k = args.h // world
    g = torch.Generator(device="cuda").manual_seed(rank)
    a = torch.randn(1, args.m, k, device="cuda", dtype=torch.bfloat16, generator=g)
    b = torch.randn(1, args.n, k, device="cuda", dtype=torch.bfloat16, generator=g).transpose(1, 2)

    default_mode = fused_native._NVLS_REDUCER_CLUSTERS, fused_native._NVLS_LAG

    def fused():
        fused_native._NVLS_REDUCER_CLUSTERS, fused_native._NVLS_LAG = default_mode
        return fused_native.gemm_allreduce_nvls(comm, a, b)

    def gemm_nvls():
        out = gemm.native_bmm(a, b)
        comm.all_reduce_(out)
        return out

    def gemm_nccl():
        out = gemm.native_bmm(a, b)
        dist.all_reduce(out, group=group)
        return out

    def torch_nccl():
        out = torch.matmul(a, b)
        dist.all_reduce(out, group=group)
        return out

    arms = {"fused": fused, "gemm+nvls": gemm_nvls, "gemm+nccl": gemm_nccl, "torch+nccl": torch_nccl}
    names = args.arms.split(",")
    for r in [int(v) for v in args.reducers.split(",") if v]:
        def fused_r(r=r):
            fused_native._NVLS_REDUCER_CLUSTERS, fused_native._NVLS_LAG = r, default_mode[1]
            return fused_native.gemm_allreduce_nvls(comm, a, b)
        arms[f"fused-R{r}"] = fused_r
        names.append(f"fused-R{r}")
    for lag in [int(v) for v in args.lags.split(",") if v]:
        def fused_l(lag=lag):
            fused_native._NVLS_REDUCER_CLUSTERS = 0
            fused_native._NVLS_LAG = lag
            return fused_native.gemm_allreduce_nvls(comm, a, b)
        arms[f"fused-L{lag}"] = fused_l
        names.append(f"fused-L{lag}")
    sampler = ClockSampler(visible_gpu_indices(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        sampler.mark_start()
    pk = peaks()
    flops = 2.0 * args.m * args.n * k
    out_bytes = args.m * args.n * 2
    t_compute = flops / (pk["bf16_tflops_sustained"] * 1e12) * 1e3
    t_link = (9.0 / 8.0 if world > 1 else 0.0) * out_bytes / 770e9 * 1e3
    roof = max(t_compute, t_link)
    results = {}
    names = [n for n in names if comm is not None or not (n.startswith("fused") or n == "gemm+nvls")]
    for name in list(names):
        for _ in range(args.warmup):
            if arms[name]() is None:  # the fused path declined (no NVLS heap): nothing to time
                names.remove(name)
                break
    torch.cuda.synchronize()
    dist.barrier()
    # arms interleaved call by call, so that clock and power drift reach every arm alike
    times = {name: [] for name in names}
    for _ in range(args.iters):
        for name in names:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            arms[name]()
            e.record()
            torch.cuda.synchronize()
            times[name].append(s.elapsed_time(e))
    for name in names:
        med = torch.tensor([statistics.median(times[name])], dtype=torch.float64, device="cuda")
        dist.all_reduce(med, op=dist.ReduceOp.MAX)
        results[name] = float(med.item())
    # numerics of the fused call against the unfused native path
    ref = gemm_nccl().float()
    got = fused().float() if comm is not None and comm.nvls else ref
    err = (got - ref).abs().max().item() / (ref.abs().max().item() + 1e-6)
    torch.cuda.synchronize()
    _native.check_errors()
    if rank == 0:
        for name, ms in results.items():
            print(json.dumps({"name": "gemm_allreduce", "arm": name, "world_size": world, "m": args.m, "n": args.n,
                              "k_per_rank": k, "max_over_ranks_ms": round(ms, 4),
                              "tflops_per_gpu": round(flops / ms / 1e9, 1),
                              "roofline_ms": round(roof, 4), "roofline_frac": round(roof / ms, 3),
                              "roofline_of": f"{pk['source']} bf16_tflops_sustained, 770 GB/s NVLink"}), flush=True)
        print(json.dumps({"name": "gemm_allreduce_check", "fused_vs_unfused_rel_err": err}), flush=True)
    if sampler:
        sampler.mark_end()
        clocks = sampler.stop()
        if rank == 0:
            print(json.dumps({"name": "clocks", "clocks": clocks}), flush=True)
    dist.barrier()
    symmetric.deactivate()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
