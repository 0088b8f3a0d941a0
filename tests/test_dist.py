"""Multi-rank plumbing of bench.py on CPU: world_size 2 over gloo.

bench.py runs one process per GPU (torchrun); every timed number is the max
over ranks, taken after a barrier.  Here two ranks report different times and
both must see the larger one; the replicas mode needs no other collective.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, ws, port, q):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(ws),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "CWEN_DIST_BACKEND": "gloo"})
    import torch.distributed as dist

    import bench
    w, r, local = bench.dist_init(None)
    bench.barrier(w)
    got = bench.barrier_max(w, 1.5 + rank)
    q.put((r, w, got))
    dist.destroy_process_group()


def test_barrier_max_two_ranks():
    ws = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(ws))
    assert res == [(0, 2, 2.5), (1, 2, 2.5)]
