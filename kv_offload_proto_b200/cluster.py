"""Placement of striped pools over the GPUs of one node, one process per GPU.

Each rank owns the requests it decodes and their pool. Two placements:
  * "others": with N > 1 ranks, rank h's pool is striped over the N-1 other GPUs ("over the
    other GPUs' HBM"): node i of rank h's pool lives on the i-th GPU other
    than h, and every rank hosts one segment of every other rank's pool;
  * "all": every rank's pool is striped over all N GPUs, its own included (node i on GPU i),
    so 1/N of its rows are local (BASELINE configs 3 and 4).
With one rank both are the rank's own GPU. Segments are shared as CUDA IPC handles gathered
over the process group (host plumbing only; no collective touches the data path).
"""
from typing import Dict, List, Tuple

__all__ = ["pool_nodes", "hosted_segments", "exchange_handles", "max_over_ranks"]


PLACEMENTS = ("others", "all")


def pool_nodes(owner: int, world: int, placement: str = "others") -> List[int]:
    """GPU of each node of `owner`'s pool, in node order."""
    if placement not in PLACEMENTS:
        raise ValueError("placement must be one of {}".format(PLACEMENTS))
    if world == 1:
        return [owner]
    if placement == "all":
        return list(range(world))
    return [g for g in range(world) if g != owner]


def hosted_segments(rank: int, world: int, placement: str = "others") -> List[Tuple[int, int]]:
    """(owner, node index) of every segment that `rank` allocates and fills."""
    out = []
    for owner in range(world):
        nodes = pool_nodes(owner, world, placement)
        if rank in nodes:
            out.append((owner, nodes.index(rank)))
    return out


def exchange_handles(dist, rank: int, world: int, handles: Dict[Tuple[int, int], bytes],
                     placement: str = "others") -> List[bytes]:
    """All-gather every rank's {(owner, node): handle} and return this rank's pool handles in
    node order (world == 1: the rank's own handle list)."""
    n = len(pool_nodes(rank, world, placement))
    if world == 1:
        return [handles[(rank, i)] for i in range(n)]
    gathered = [None] * world
    dist.all_gather_object(gathered, handles)
    mine: List[bytes] = [None] * n  # type: ignore[list-item]
    for hd in gathered:
        for (owner, idx), h in hd.items():
            if owner == rank:
                mine[idx] = h
    missing = [i for i, h in enumerate(mine) if h is None]
    if missing:
        raise RuntimeError("rank {}: no handle for pool node(s) {}".format(rank, missing))
    return mine


def max_over_ranks(dist, world: int, value: float) -> float:
    """Largest `value` over all ranks (device times are reported as the max)."""
    if world == 1:
        return value
    out = [None] * world
    dist.all_gather_object(out, float(value))
    return max(out)
