"""Distributed 3D FFT benchmark (the BASELINE FFT config).

    torchrun --nproc-per-node N benchmarks/bench_fft.py [--impl native|reference] [--n 1024]

One step = forward ``einfft("b x/sp y z -> b kx ky/sp kz")`` plus the inverse
back to ``b x/sp y z``; b=1, x=y=z=n complex64 with real/imag ~N(0,1) from
seed 0, sp = number of GPUs.  The reference rejects this literal layout
(NotImplementedError in its einfft), so its arm runs the equivalent slab
pipeline from reference primitives: einfft over (y, z), the all-to-all
repartition ``b x/sp ky kz -> b x ky/sp kz`` (shapes given), einfft over x;
and the mirror image for the inverse.

Prints one JSON line (rank 0): ms per step as the max over ranks of CUDA-event
time, and the fraction of a roofline built from measured peaks: every local
FFT pass reads and writes the local tensor once (HBM), and (P-1)/P of it
crosses NVLink per transpose.
"""

import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from common import ClockSampler, peaks, visible_gpu_indices  # noqa: E402

NVLINK_GBS = 770.0  # measured peer copy per direction on this machine class


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--n", type=int, default=1024)
    p.add_argument("--nx", type=int, default=0, help="length of the x axis (default n); smaller for profiling")
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--breakdown", action="store_true",
                   help="after the timed steps, one more step under torch.profiler: rank 0's kernels with their "
                        "device time (not a timing run)")
    args = p.parse_args()
    if "RANK" not in os.environ:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT="29611", RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    world, rank = dist.get_world_size(), dist.get_rank()
    from torch.distributed.device_mesh import init_device_mesh
    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("sp",))
    n = args.n
    nx = args.nx or n
    xl = nx // world
    shapes = {"sp": {"x": [xl] * world, "ky": [n // world] * world, "y": [n // world] * world,
                     "kx": [xl] * world}}
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = torch.complex(torch.randn(1, xl, n, n, device="cuda", generator=gen),
                      torch.randn(1, xl, n, n, device="cuda", generator=gen))

    if args.impl == "native":
        sys.path.insert(0, ROOT)
        import torch_einshard_b200 as es
        es.setup_native_comm(mesh)

        def step():
            y = es.einfft("b x/sp y z -> b kx ky/sp kz", x, {"x": "kx", "y": "ky", "z": "kz"}, mesh=mesh)
            return es.einfft("b kx ky/sp kz -> b x/sp y z", y, {"kx": "x", "ky": "y", "kz": "z"}, inverse=True,
                             mesh=mesh)
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

        def step():
            y = es.einfft("b x/sp y z -> b x/sp ky kz", x, {"y": "ky", "z": "kz"}, mesh=mesh)
            y = es.einshard("b x/sp ky kz -> b x ky/sp kz", y, mesh=mesh, shapes=shapes)
            y = es.einfft("b x ky/sp kz -> b kx ky/sp kz", y, {"x": "kx"}, mesh=mesh)
            z = es.einfft("b kx ky/sp kz -> b x ky/sp kz", y, {"kx": "x"}, inverse=True, mesh=mesh)
            z = es.einshard("b x ky/sp kz -> b x/sp ky kz", z, mesh=mesh, shapes=shapes)
            return es.einfft("b x/sp ky kz -> b x/sp y z", z, {"ky": "y", "kz": "z"}, inverse=True, mesh=mesh)

    sampler = ClockSampler(visible_gpu_indices(world)) if rank == 0 else None
    if sampler:
        sampler.start()
    with torch.no_grad():
        out = step()
        err = ((out - x).abs().max() / x.abs().max()).item()
        for _ in range(args.warmup):
            step()
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
        kernels = []
        for ev in prof.events():
            if ev.device_type.name == "CUDA":
                kernels.append([ev.name[:80], round(ev.device_time_total / 1e3, 3)])
        if rank == 0:
            print(json.dumps({"breakdown_rank": rank, "kernels_ms_in_order": kernels[:40]}), flush=True)
    ms = torch.tensor([t0.elapsed_time(t1) / args.steps], device="cuda", dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = ms.item()
    local_bytes = x.numel() * 8
    hbm_s = 2 * 3 * 2 * local_bytes / (peaks()["hbm_gbs"] * 1e9)      # 3 passes each way, read + write
    link_s = 2 * local_bytes * (world - 1) / world / (NVLINK_GBS * 1e9) if world > 1 else 0.0
    roofline_ms = 1e3 * max(hbm_s, link_s)
    if rank == 0:
        print(json.dumps({"metric": "dist-FFT ms (forward + inverse)", "value": round(ms, 3), "unit": "ms",
                          "higher_is_better": False, "n_gpus": world, "impl": args.impl,
                          "config": {"shape": [1, nx, n, n], "dtype": "complex64", "layout": "b x/sp y z <-> b kx ky/sp kz",
                                     "l2": "inputs larger than L2; no flush"},
                          "clocks": sampler.stop() if sampler else None, "roundtrip_rel_err": err, "roofline_ms": round(roofline_ms, 3),
                          "roofline_frac": round(roofline_ms / ms, 3),
                          "roofline_of": f"{peaks()['source']} hbm_gbs; NVLink 770 GB/s"}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
