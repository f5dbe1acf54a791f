"""Distributed einshard step benchmarks (CPU gloo or CUDA/NCCL + native comm).

    torchrun --nproc-per-node N benchmarks/bench_distributed.py [--device cuda] [--size medium]

Cases: uneven split/gather round trip, all-to-all repartition with shape
metadata, owner swap on a 2-D mesh, tensor-parallel MLP contraction, sharded
roll.  One JSONL record per case (``benchmarks/common.py`` schema).
"""

import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from common import ROOT, Writer, init_distributed, parser  # noqa: E402
from common import benchmark as _benchmark  # noqa: E402



def load_impl(impl):
    """The package under test: this framework, or the unmodified reference from
    baseline/_ref (its parser dependency supplied by baseline/parsley_shim)."""
    if impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        sys.path.insert(0, os.path.join(ROOT, "baseline", "parsley_shim"))
        import torch_einshard
        return torch_einshard
    sys.path.insert(0, ROOT)
    import torch_einshard_b200
    return torch_einshard_b200

IMPL = {"impl": "native"}


def benchmark(name, fn, **kw):
    kw["extra"] = dict(kw.get("extra") or {}, **IMPL)
    return _benchmark(name, fn, **kw)


SHAPES = {"small": dict(rows=128, cols=96, hidden=128, batch=4, seq=16),
          "medium": dict(rows=1024, cols=768, hidden=1024, batch=8, seq=64),
          "large": dict(rows=4096, cols=3072, hidden=4096, batch=16, seq=128)}


def main():
    p = parser(__doc__)
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    args = p.parse_args()
    es = load_impl(args.impl)
    device = torch.device(args.device)
    init_distributed(device)
    from torch.distributed.device_mesh import init_device_mesh
    world = dist.get_world_size()
    if device.type == "cuda":
        dev = device
    else:
        dev = torch.device("cpu")
    mesh1 = init_device_mesh(device.type, (world,), mesh_dim_names=("dp",))
    side = int(round(world ** 0.5))
    mesh2 = init_device_mesh(device.type, (side, world // side), mesh_dim_names=("dp", "sp")) if side * side == world \
        else None
    if device.type == "cuda" and args.impl == "native":
        es.setup_native_comm(mesh1)
    torch.manual_seed(args.seed)
    cfg = SHAPES[args.size]
    writer = Writer(args.output)
    IMPL["impl"] = args.impl
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    group = mesh1["dp"].get_group()
    rank = dist.get_rank(group)

    rows = cfg["rows"] + 1
    row_shapes = es.compute_split_shapes(rows, world)
    x = torch.randn(rows, cfg["cols"], device=dev, dtype=dtype)

    def round_trip():
        z = es.einshard("a b -> a/dp b", x, mesh=mesh1, shapes=row_shapes)
        return es.einshard("a/dp b -> a b", z, mesh=mesh1, shapes=row_shapes)
    benchmark("distributed_split_gather_round_trip", round_trip, args=args, device=device, writer=writer,
              extra={"global_shape": [rows, cfg["cols"]]})

    r, c = cfg["rows"], cfg["cols"]
    rs, cs = es.compute_split_shapes(r, world), es.compute_split_shapes(c, world)
    full = torch.randn(r, c, device=dev, dtype=dtype)
    xl = torch.split(full, rs, 0)[rank].contiguous()
    benchmark("distributed_repartition_axis_metadata",
              lambda: es.einshard("a/dp b -> a b/dp", xl, mesh=mesh1, shapes={"dp": {"a": rs, "b": cs}}),
              args=args, device=device, writer=writer, extra={"global_shape": [r, c]})

    if mesh2 is not None:
        p, q = mesh2["dp"].size(), mesh2["sp"].size()
        a = torch.randn(r // p, c // q, device=dev, dtype=dtype)
        benchmark("distributed_owner_swap", lambda: es.einshard("a/dp b/sp -> a/sp b/dp", a, mesh=mesh2),
                  args=args, device=device, writer=writer, extra={"global_shape": [r, c], "mesh": [p, q]})

    b, n, h = cfg["batch"], cfg["seq"], cfg["hidden"]
    xin = torch.randn(b, n, h, device=dev, dtype=dtype)
    w1 = torch.randn(4 * h // world, h, device=dev, dtype=dtype) * 0.02
    w2 = torch.randn(h, 4 * h // world, device=dev, dtype=dtype) * 0.02

    def mlp():
        y = es.einshard("b n c, f/dp c -> b n f/dp", xin, w1, mesh=mesh1)
        return es.einshard("b n f/dp, c f/dp -> b n c", y, w2, mesh=mesh1)
    benchmark("distributed_tp_mlp_contract", mlp, args=args, device=device, writer=writer,
              flops=2 * 2 * b * n * h * 4 * h // world if device.type == "cuda" else None,
              extra={"batch": b, "seq": n, "hidden": h})

    roll_x = torch.split(full, rs, 0)[rank].contiguous()
    benchmark("distributed_roll_sharded",
              lambda: es.einroll("a/dp b", roll_x, {"a": 3}, mesh=mesh1, shapes=rs),
              args=args, device=device, writer=writer, extra={"global_shape": [r, c], "shift": 3})
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
