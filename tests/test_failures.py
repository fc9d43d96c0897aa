"""Host-side failure detection for the multi-rank paths (CPU, gloo; no GPU involved).

A peer that dies between steps must surface as an error on the surviving
rank within the process group's timeout, never as a hang: the disaggregated
protocol's only host synchronisation points are collectives with a bounded
timeout.
"""

from __future__ import annotations

import datetime
import os
import socket
import time

import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, q) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    dist.barrier()  # both ranks are up
    if rank == 1:
        os._exit(3)  # the decode peer dies before the "push complete" barrier
    t0 = time.perf_counter()
    try:
        dist.barrier()
        q.put(("no error", time.perf_counter() - t0))
    except Exception as exc:  # gloo reports the lost peer or the timeout
        q.put((type(exc).__name__, time.perf_counter() - t0))
    q.close()
    q.join_thread()  # flush the queue's feeder thread before the hard exit
    os._exit(0)


def test_peer_death_is_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, waited = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert kind != "no error"
    assert waited < 60
    assert procs[1].exitcode == 3
