"""Run a test body on N GPUs: one spawned process per device, NCCL, 127.0.0.1.

Ranks that fail report their traceback; a short process-group timeout ends
collectives whose peer died, and the parent kills (by PID) any rank that
outlives the deadline.
"""

import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _worker(rank, world, port, body, queue, env):
    try:
        import torch
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
        os.environ.update(env or {})
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        torch.manual_seed(333)
        body(rank, world)
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, None))
    except BaseException:  # noqa: BLE001
        queue.put((rank, traceback.format_exc()))


def run_gpus(body, world, timeout=300, env=None):
    """``env``: extra environment variables of every rank (set before the body runs)."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, body, queue, env)) for r in range(world)]
    for proc in procs:
        proc.start()
    results = {}
    try:
        for _ in range(world):
            rank, err = queue.get(timeout=timeout)
            results[rank] = err
            if err is not None:
                break
    except Exception:  # noqa: BLE001
        pass
    for proc in procs:
        proc.join(timeout=30)
    for proc in procs:
        if proc.is_alive():
            proc.kill()
            proc.join()
    failures = {r: e for r, e in results.items() if e is not None}
    if failures:
        rank = min(failures)
        raise AssertionError(f"rank {rank} failed:\n{failures[rank]}")
    if len(results) != world:
        raise AssertionError(f"only {len(results)} of {world} ranks reported")
