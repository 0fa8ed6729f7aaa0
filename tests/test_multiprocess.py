"""Multi-process host logic on CPU ranks (gloo, world size 2): the bench's cross-rank reduction (max of the
device time, sum of the tokens) and the rank-0-only reference arm."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path.insert(0, ROOT)
    import bench
    ms, toks = bench.reduce_time_and_count(10.0 + rank, 100 + rank, torch.device("cpu"), world)
    out[rank] = (ms, toks)
    dist.barrier()
    dist.destroy_process_group()


def test_reduce_time_and_count_two_ranks():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert out[0] == out[1] == (11.0, 201)


def test_reduce_identity_on_one_rank():
    sys.path.insert(0, ROOT)
    import bench
    import torch
    assert bench.reduce_time_and_count(3.5, 7, torch.device("cpu"), 1) == (3.5, 7)
