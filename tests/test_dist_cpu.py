"""The multi-process host logic of bench.py on the CPU: two ranks over gloo
(127.0.0.1) -- the max over ranks that every timing goes through, the
whole-job rate (all ranks' frames over the slowest rank's time), the
broadcast of the tensor-parallel group id, and the barrier; and the
single-process fall-throughs."""
import multiprocessing as mp
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    try:
        import bench
        assert bench.dist_env() == (rank, world, rank)
        dist = bench.init_dist(world, rank, backend="gloo")
        mx = bench.reduce_max(dist, 1.5 + rank)
        gid = bench.broadcast_bytes(dist, bytes(range(128)) if rank == 0 else b"", 128)
        value, ms = bench.whole_job_rate(dist, world, 10.0 * (rank + 1))
        bench.barrier(dist)
        dist.destroy_process_group()
        q.put((rank, (mx, gid, value, ms)))
    except Exception as ex:  # reported to the parent
        q.put((rank, repr(ex)))


def test_two_gloo_ranks_share_max_rate_and_group_id():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert not isinstance(got[r], str), f"rank {r}: {got[r]}"
        mx, gid, value, ms = got[r]
        assert mx == 2.5                       # max over ranks, on every rank
        assert gid == bytes(range(128))        # rank 0's id on every rank
        assert ms == 20.0 and value == pytest.approx(100.0)  # 2 ranks x 1000 / slowest 20 ms


def test_single_process_fall_throughs():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.init_dist(1, 0) is None
    assert bench.reduce_max(None, 3.25) == 3.25
    assert bench.broadcast_bytes(None, b"abc", 3) == b"abc"
    assert bench.whole_job_rate(None, 1, 4.0) == (250.0, 4.0)
    bench.barrier(None)
