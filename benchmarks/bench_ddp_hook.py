"""DDP gradient-reduction hook benchmark (CPU gloo or CUDA).

    torchrun --nproc-per-node N benchmarks/bench_ddp_hook.py [--device cuda] [--mode per_spec|combined|mixed]

A stack of linear layers whose parameters carry einshard layouts; DDP over the
data-parallel mesh dim with ``register_grad_reduction_hook_``.  ``per_spec``:
every parameter has an extra replicated reduction group; ``combined``: the
compound-group fast path; ``mixed``: half the parameters without extra groups.
One fwd+bwd step per timed iteration.
"""

import os
import sys

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from common import ROOT, Writer, benchmark, init_distributed, parser  # noqa: E402



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

WIDTH = {"small": (256, 4), "medium": (1024, 8), "large": (4096, 8)}


class Stack(torch.nn.Module):
    def __init__(self, width, depth, device, dtype):
        super().__init__()
        self.layers = torch.nn.ModuleList(torch.nn.Linear(width, width, device=device, dtype=dtype)
                                          for _ in range(depth))

    def forward(self, x):
        for layer in self.layers:
            x = torch.relu(layer(x))
        return x


def main():
    p = parser(__doc__)
    p.add_argument("--mode", choices=("per_spec", "combined", "mixed"), default="combined")
    p.add_argument("--bucket-cap-mb", type=int, default=25)
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    args = p.parse_args()
    es = load_impl(args.impl)
    device = torch.device(args.device)
    init_distributed(device)
    from torch.distributed.device_mesh import init_device_mesh
    world = dist.get_world_size()
    dp = 2 if world % 2 == 0 else 1
    mesh = init_device_mesh(device.type, (dp, world // dp), mesh_dim_names=("dp", "sp"))
    wrapped = es.wrap_mesh(mesh)
    if device.type == "cuda" and args.impl == "native":
        es.setup_native_comm(mesh)
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    width, depth = WIDTH[args.size]
    model = Stack(width, depth, device, dtype)
    for i, param in enumerate(model.parameters()):
        axes = "o c" if param.dim() == 2 else "o"
        extra = args.mode != "mixed" or i % 2 == 0
        spec = f"{axes} [param, grad=sp] -> {axes}" if extra else f"{axes} [param, grad=none] -> {axes}"
        es.set_parameter_state(param, es.ParameterState.from_spec(es.parse_sharding(spec)[0]))
    ddp = DistributedDataParallel(model, process_group=mesh["dp"].get_group(), bucket_cap_mb=args.bucket_cap_mb)
    if args.mode == "combined":
        es.register_grad_reduction_hook_(ddp, wrapped, ddp_group="dp", combined_reduce_group="dp-sp",
                                         combined_reduce="sp")
    else:
        es.register_grad_reduction_hook_(ddp, mesh, ddp_group="dp")
    x = torch.randn(32, width, device=device, dtype=dtype)

    def step():
        ddp(x).float().square().mean().backward()
        for param in model.parameters():
            param.grad = None

    benchmark(f"ddp_hook_{args.mode}", step, args=args, device=device, writer=Writer(args.output), grad=True,
              extra={"impl": args.impl, "mode": args.mode, "bucket_cap_mb": args.bucket_cap_mb, "width": width, "depth": depth,
                     "params": sum(p.numel() for p in model.parameters())})
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
