"""RowAllocator (kv_offload_proto_b200.pool): the pool-row allocator's contiguity contract
(xds/xds_ems_pool.py:54-106, exercised by the reference's test/test_allocator.py): fresh
allocations are contiguous and in row order, freed rows are reused from the lowest run,
single freed rows merge back into runs, exhaustion and bad rows raise. A seeded random
history is checked step by step against a brute-force model of the same rules."""
import numpy as np
import pytest

from kv_offload_proto_b200.pool import RowAllocator


def test_fresh_allocations_are_contiguous_and_ordered():
    a = RowAllocator(1000)
    assert a.alloc(300) == list(range(300))
    assert a.alloc(200) == list(range(300, 500))
    assert a.free_rows() == 500 and a.used_rows() == 500


def test_freed_block_is_reused_from_its_start():
    a = RowAllocator(600)
    first, second = a.alloc(200), a.alloc(200)
    a.free(first)
    assert a.alloc(50) == list(range(50))          # the lowest run that fits
    assert a.alloc(180) == list(range(400, 580))    # [50, 200) is too small: next run in order
    a.free(second)
    assert a.free_runs() == [(50, 400), (580, 600)]


def test_single_rows_merge_back_into_one_run():
    a = RowAllocator(12)
    rows = [a.alloc(1)[0] for _ in range(12)]
    assert rows == list(range(12))
    for r in (3, 5, 4, 2, 6):  # out of order: neighbours on both sides merge
        a.free([r])
    assert a.free_runs() == [(2, 7)]
    assert a.alloc(5) == [2, 3, 4, 5, 6]


def test_fragmented_request_takes_the_lowest_rows():
    a = RowAllocator(10)
    a.alloc(10)
    a.free([1, 2, 5, 8, 9])
    assert a.alloc(4) == [1, 2, 5, 8]
    assert a.free_runs() == [(9, 10)]


def test_exhaustion_and_bad_rows():
    a = RowAllocator(4)
    with pytest.raises(MemoryError):
        a.alloc(5)
    with pytest.raises(ValueError):
        a.alloc(0)
    rows = a.alloc(4)
    with pytest.raises(ValueError):
        a.free([4])
    with pytest.raises(ValueError):
        a.free([-1])
    a.free(rows[:2])
    with pytest.raises(ValueError):
        a.free([0])  # already free
    with pytest.raises(ValueError):
        a.free([2, 2])
    assert a.used_rows() == 2


def test_alloc_free_cycles_leave_no_leak():
    a = RowAllocator(64)
    blocks = [a.alloc(16) for _ in range(4)]
    for b in reversed(blocks):
        a.free(b)
    assert a.used_rows() == 0 and a.free_runs() == [(0, 64)]


def _model_alloc(free, n):
    """Brute force of the contract on a boolean free map."""
    idx = np.flatnonzero(free)
    runs, start = [], None
    for i in range(len(free) + 1):
        f = i < len(free) and free[i]
        if f and start is None:
            start = i
        if not f and start is not None:
            runs.append((start, i))
            start = None
    for lo, hi in runs:
        if hi - lo >= n:
            return list(range(lo, lo + n))
    return [int(x) for x in idx[:n]]


def test_random_history_matches_brute_force_model():
    rng = np.random.default_rng(2024)
    cap = 300
    a = RowAllocator(cap)
    free = np.ones(cap, bool)
    live = []
    for _ in range(2000):
        if live and (rng.random() < 0.45 or free.sum() == 0):
            blk = live.pop(int(rng.integers(len(live))))
            part = [r for r in blk if rng.random() < 0.7] or blk  # free some or all of a block
            rest = [r for r in blk if r not in part]
            if rest:
                live.append(rest)
            a.free(part)
            free[part] = True
        else:
            n = int(rng.integers(1, 40))
            if n > free.sum():
                with pytest.raises(MemoryError):
                    a.alloc(n)
                continue
            got = a.alloc(n)
            assert got == _model_alloc(free, n)
            free[got] = False
            live.append(got)
        assert a.free_rows() == int(free.sum())
        runs = a.free_runs()
        assert all(hi > lo for lo, hi in runs)
        assert all(runs[i][1] < runs[i + 1][0] for i in range(len(runs) - 1))  # disjoint, not adjacent
