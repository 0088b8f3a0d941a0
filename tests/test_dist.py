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


def test_reference_arm_under_torchrun_prints_one_line():
    """`bench.py --impl reference` launched like the driver's N>1 runs: rank 0
    alone times the reference and prints one JSON line; the other rank exits
    0 without work."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    import bench
    if not bench.ref_lib_path()[0].exists():
        pytest.skip("reference library (oracle/_ref) not built")
    root = Path(__file__).resolve().parents[1]
    env = {**os.environ, "CWEN_DIST_BACKEND": "gloo", "OMP_NUM_THREADS": "2"}
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "bench.py",
                        "--gpus", "2", "--impl", "reference", "--workload", "gemv", "--steps", "2", "--warmup", "3"],
                       cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["unit"] == "GB/s" and rec["value"] > 0
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["cpu_baseline"]["kind"] == "reference"


def test_shard_rows_partition():
    """cwen_shard_rows: for every group size the ranks' row ranges are
    contiguous, disjoint, cover [0, M) in rank order, and start on multiples
    of the alignment (the FFN and lm_head row split of the sharded decode)."""
    import ctypes as C

    import cwen_b200
    L = cwen_b200.lib()
    r0, r1 = C.c_int(), C.c_int()
    for M in (0, 16, 512, 1024, 5120, 17408, 248320, 1000):
        for world in range(1, 9):
            for align in (1, 16):
                edge = 0
                for rank in range(world):
                    assert L.cwen_shard_rows(M, align, rank, world, C.byref(r0), C.byref(r1)) == 0
                    assert r0.value == edge and r1.value >= r0.value, (M, world, align, rank)
                    assert r0.value % align == 0 or r0.value == M
                    edge = r1.value
                assert edge == M, (M, world, align)
    assert L.cwen_shard_rows(10, 1, 2, 2, C.byref(r0), C.byref(r1)) < 0  # rank outside the group


def _shard_exchange_main(rank, ws, port, q):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(ws),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "CWEN_DIST_BACKEND": "gloo"})
    import torch.distributed as dist

    import bench
    w, r, _ = bench.dist_init(None)
    blob = bytes([r]) * bench.SHARD_HANDLE
    q.put((r, bench.shard_exchange(blob, w)))
    dist.destroy_process_group()


def test_shard_handle_exchange_two_ranks():
    """The sharded decode's set-up step over a process group: every rank ends
    with all ranks' handle blobs concatenated in rank order."""
    import bench
    ws = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_shard_exchange_main, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    want = b"".join(bytes([r]) * bench.SHARD_HANDLE for r in range(ws))
    res = dict(q.get(timeout=10) for _ in range(ws))
    assert res == {0: want, 1: want}
