"""Sharded checkpoints built on :class:`ParamShardMetadata`.

``save_sharded`` writes one file per rank holding every registered parameter
shard with its metadata (global shape, local slices, local shape, shard dims).
``load_sharded`` reads all shard files, reassembles each parameter from the
recorded slices and copies the slice that this rank owns under the *current*
layout, so a checkpoint can be loaded on a different mesh or world size.
Parameters without attached metadata are saved whole by rank 0.

Builds on the reference's ``ParamShardMetadata``
(``src/torch_einshard/params.py:557-562,1660-1669``); the reference itself has
no save/load.
"""

import dataclasses
import glob
import os

import torch
import torch.distributed as dist

from .registry import get_parameter_state
from .shard_meta import param_shard_metadata

__all__ = ["save_sharded", "load_sharded", "global_shape_of"]


def _groups_and_dims(param, state, mesh):
    for dim, axis in enumerate(state.axes):
        if getattr(axis, "shard_dim", ""):
            yield dim, mesh[axis.shard_dim].get_group()


def global_shape_of(param, state, mesh):
    """Global shape of a sharded parameter: local sizes summed over each shard group."""
    shape = list(param.shape)
    for dim, group in _groups_and_dims(param, state, mesh):
        size = torch.tensor([param.shape[dim]], dtype=torch.int64,
                            device=param.device if param.is_cuda else "cpu")
        dist.all_reduce(size, group=group)
        shape[dim] = int(size.item())
    return tuple(shape)


def save_sharded(module, path, mesh=None):
    os.makedirs(path, exist_ok=True)
    rank = dist.get_rank() if dist.is_initialized() else 0
    payload = {}
    for name, param in module.named_parameters():
        state = get_parameter_state(param)
        if state is None or state.spec is None or mesh is None:
            if rank == 0:
                payload[name] = {"tensor": param.detach().cpu(), "meta": None}
            continue
        meta = param_shard_metadata(param, global_shape_of(param, state, mesh), mesh)
        payload[name] = {"tensor": param.detach().cpu(), "meta": dataclasses.asdict(meta)}
    torch.save({"rank": rank, "params": payload}, os.path.join(path, f"shard_{rank:05d}.pt"))
    if dist.is_initialized():
        dist.barrier()


def load_sharded(module, path, mesh=None):
    files = sorted(glob.glob(os.path.join(path, "shard_*.pt")))
    if not files:
        raise FileNotFoundError(f"no shard files under {path!r}")
    pieces = {}
    for file in files:
        blob = torch.load(file, map_location="cpu", weights_only=False)
        for name, item in blob["params"].items():
            pieces.setdefault(name, []).append(item)
    for name, param in module.named_parameters():
        if name not in pieces:
            raise KeyError(f"checkpoint has no entry for parameter {name!r}")
        items = pieces[name]
        meta = items[0]["meta"]
        if meta is None:
            full = items[0]["tensor"]
        else:
            full = torch.empty(meta["global_shape"], dtype=items[0]["tensor"].dtype)
            for item in items:
                full[tuple(item["meta"]["local_slices"])] = item["tensor"]
        state = get_parameter_state(param)
        if state is not None and state.spec is not None and mesh is not None and meta is not None:
            mine = param_shard_metadata(param, tuple(full.shape), mesh)
            local = full[mine.local_slices]
        else:
            local = full
        with torch.no_grad():
            param.copy_(local.to(param.device, param.dtype))
    return module
