"""The cross-rank half of bench.py's byte check (`exchange_rows`) on CPU: world_size 2 `gloo`
ranks each host a segment (here plain host memory, as with --pool host), ask for rows of the
other rank's segment, and get back exactly those bytes, read by the hosting rank. No GPU."""
import os
import socket

import numpy as np
import pytest

ROW = 1152


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Cl:
    """The parts of bench.Cluster exchange_rows uses."""

    def __init__(self, dist, rank, world):
        self.dist, self.rank, self.world, self.seg_dev = dist, rank, world, -1

    def all_gather(self, obj):
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out


def _worker(rank, world, port, q):
    import sys

    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows = 64
        seg = np.random.default_rng(rank).integers(0, 256, rows * ROW, dtype=np.uint8)
        # rank h hosts node h of the other rank's pool ("others" placement, world 2)
        hosted = {(1 - rank, 0): seg.ctypes.data}
        want = [3, 0, 63, 7, 3]
        ask = {(rank, 0): want}  # node 0 of my pool lives on the other rank
        bench.ROW_BYTES = ROW
        got = bench.exchange_rows(torch, _Cl(dist, rank, world), hosted, ask, rows * ROW)
        exp = np.random.default_rng(1 - rank).integers(0, 256, rows * ROW, dtype=np.uint8).reshape(rows, ROW)[want]
        q.put((rank, bool(np.array_equal(got[(rank, 0)], exp))))
        with pytest.raises(RuntimeError):
            bench.exchange_rows(torch, _Cl(dist, rank, world), hosted, {(rank, 0): [rows]}, rows * ROW)
    finally:
        dist.destroy_process_group()


def test_exchange_rows_two_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == {0: True, 1: True}
