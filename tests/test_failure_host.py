"""Host-level failure detection on CPU (gloo): a rank that leaves between
steps makes its peers' next einshard collective end with an error after the
process-group timeout, instead of waiting forever."""

import multiprocessing as mp
import os
import socket
import time
from datetime import timedelta

import torch
import torch.distributed as dist


def _port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _report(queue, rank, text):
    queue.put((rank, text))
    queue.close()
    queue.join_thread()      # flushed before os._exit


def _rank(rank, port, queue):
    try:
        _body(rank, port, queue)
    except BaseException as err:  # noqa: BLE001 - reported to the parent
        _report(queue, rank, f"setup failed: {err!r}")
        os._exit(1)


def _body(rank, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=3))
    import torch_einshard_b200 as es
    from torch.distributed.device_mesh import init_device_mesh
    mesh = init_device_mesh("cpu", (2,), mesh_dim_names=("tp",))
    y = torch.ones(8, 4)                                  # this rank's partial sum
    # step 1: both ranks
    z = es.einshard("a b // tp -> a b", y, mesh=mesh)
    assert torch.equal(z, torch.full((8, 4), 2.0))
    dist.barrier()
    if rank == 1:
        _report(queue, rank, "left")
        os._exit(0)                # leaves between steps, nothing in flight
    t0 = time.time()
    try:
        es.einshard("a b // tp -> a b", y, mesh=mesh)    # step 2: the peer is gone
        text = "no error"
    except Exception as err:  # noqa: BLE001 - any error ends the wait; the point is that it ends
        text = f"error after {time.time() - t0:.1f}s: {type(err).__name__}"
    _report(queue, rank, text)
    os._exit(0)


def test_peer_that_leaves_ends_the_next_collective_with_an_error():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, port, queue)) for r in range(2)]
    for proc in procs:
        proc.start()
    results = dict(queue.get(timeout=120) for _ in range(2))
    for proc in procs:
        proc.join(timeout=10)
        if proc.is_alive():
            proc.kill()
    assert results[1] == "left"
    assert results[0].startswith("error after"), results[0]
    assert float(results[0].split()[2].rstrip("s:")) < 60
