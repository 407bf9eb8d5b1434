"""Failure detection across ranks, on the host: a rank that leaves between
steps (here: exits right after joining) must make the surviving rank's next
collective end with an error within the process group's deadline instead of
hanging. Two gloo ranks on CPU; no GPU is involved."""

import os
import socket
import time
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)                       # step 1: both ranks present
    if rank == 1:
        os._exit(0)                          # leaves between steps, no goodbye
    t0 = time.time()
    try:
        dist.all_reduce(t)                   # step 2: the peer is gone
        q.put(("no error", time.time() - t0))
    except Exception as e:                   # the expected outcome
        q.put((type(e).__name__, time.time() - t0))


def test_survivor_gets_an_error_not_a_hang():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outcome, seconds = q.get(timeout=120)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert outcome != "no error"
    assert seconds < 60
