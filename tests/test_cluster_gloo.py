"""Multi-rank host logic of the pool placement (kv_offload_proto_b200.cluster) on CPU:
world_size 2 and 4 `gloo` process groups exchange placeholder segment handles; no GPU."""
import os
import socket

import pytest

from kv_offload_proto_b200 import cluster


@pytest.mark.parametrize("placement", ["others", "all"])
def test_placement_covers_every_node_once(placement):
    for world in (1, 2, 4, 8):
        seen = {}
        for rank in range(world):
            for owner, idx in cluster.hosted_segments(rank, world, placement):
                assert (owner, idx) not in seen
                seen[(owner, idx)] = rank
                assert cluster.pool_nodes(owner, world, placement)[idx] == rank
        for owner in range(world):
            nodes = cluster.pool_nodes(owner, world, placement)
            if placement == "others":
                assert len(nodes) == (1 if world == 1 else world - 1)
                assert owner not in nodes or world == 1
            else:
                assert nodes == list(range(world))
            assert all((owner, i) in seen for i in range(len(nodes)))
        # every rank hosts the same number of segments (balanced placement)
        assert len({len(cluster.hosted_segments(r, world, placement)) for r in range(world)}) == 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, placement="others"):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        handles = {(o, i): "h:{}:{}:{}".format(rank, o, i).encode()
                   for o, i in cluster.hosted_segments(rank, world, placement)}
        mine = cluster.exchange_handles(dist, rank, world, handles, placement)
        t = cluster.max_over_ranks(dist, world, 1.5 + rank)
        q.put((rank, mine, t))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,placement", [(2, "others"), (4, "others"), (2, "all")])
def test_handle_exchange_gloo(world, placement):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, placement)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, mine, t = q.get(timeout=120)
        out[rank] = (mine, t)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, (mine, t) in out.items():
        nodes = cluster.pool_nodes(rank, world, placement)
        assert mine == ["h:{}:{}:{}".format(host, rank, i).encode() for i, host in enumerate(nodes)]
        assert t == 1.5 + world - 1
