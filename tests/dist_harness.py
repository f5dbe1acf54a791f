"""Run a test body on N CPU ranks (forked processes, gloo, 127.0.0.1).

``run_ranks(body, world_size)`` forks ``world_size`` processes; each
initialises a gloo process group, seeds torch with 333 (so every rank draws
the same full tensors, the oracle pattern) and calls ``body(ctx)`` with
``ctx.rank``, ``ctx.world_size`` and mesh builders.  Failures (exceptions,
timeouts, non-zero exits) are re-raised in the parent with the rank's
traceback.  A rank that raises is reported; the others are stopped by the
process-group timeout or by the parent's deadline.
"""

import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta
from types import SimpleNamespace

import torch
import torch.distributed as dist


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _mesh(shape, names):
    from torch.distributed.device_mesh import init_device_mesh
    return init_device_mesh("cpu", shape, mesh_dim_names=names)


def _worker(rank, world_size, port, body, queue):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world_size), LOCAL_RANK=str(rank))
        torch.set_num_threads(1)
        dist.init_process_group("gloo", rank=rank, world_size=world_size, timeout=timedelta(seconds=60))
        torch.manual_seed(333)
        ctx = SimpleNamespace(rank=rank, world_size=world_size, mesh=_mesh)
        body(ctx)
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, None))
    except BaseException:  # noqa: BLE001 - forwarded to the parent
        queue.put((rank, traceback.format_exc()))


def run_ranks(body, world_size=8, timeout=240):
    ctx = mp.get_context("fork")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world_size, port, body, queue)) for r in range(world_size)]
    for proc in procs:
        proc.start()
    results = {}
    try:
        for _ in range(world_size):
            rank, err = queue.get(timeout=timeout)
            results[rank] = err
            if err is not None:
                break
    except Exception:  # noqa: BLE001
        pass
    for proc in procs:
        proc.join(timeout=5)
    for proc in procs:
        if proc.is_alive():
            proc.kill()
            proc.join()
    failures = {r: e for r, e in results.items() if e is not None}
    if failures:
        rank = min(failures)
        raise AssertionError(f"rank {rank} failed:\n{failures[rank]}")
    if len(results) != world_size:
        raise AssertionError(f"only {len(results)} of {world_size} ranks reported (timeout or crash)")
