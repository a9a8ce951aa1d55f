"""CPU model of the SIEVE kernels' table update (phases 4-5 of sieve_fast_kernel): evicted keys
deleted with backward shift, then the step's new keys inserted by priority rounds in which a
pending key passes every cell held by a surviving key or by an earlier (higher-priority) key
and claims the next one by compare-and-swap. The rounds are replayed with random interleavings
of the keys' single-cell reads and CAS operations, and the final table must equal the
reference's order: every erase, then every insert in priority order, each by linear probing
(hisp_kernel_common.h:40-94; hisp_sieve_update.cpp:140-163). The GPU tests compare the
kernels' table bytes with the C restatement; this test pins the argument behind the insertion
rounds on its own."""
import random

import pytest

EMPTY = None


def home(key, size):
    return (key * 2654435761 >> 7) % size


def insert_seq(table, key):
    i = home(key, len(table))
    while table[i] is not EMPTY:
        i = (i + 1) % len(table)
    table[i] = key


def erase_seq(table, key):
    """Backward-shift deletion (Knuth 6.4, Algorithm R)."""
    n = len(table)
    i = table.index(key)
    table[i] = EMPTY
    j = i
    while True:
        j = (j + 1) % n
        k = table[j]
        if k is EMPTY:
            return
        h = home(k, n)
        # k may move to i when i lies cyclically in [h, j)
        if (j > i and (h <= i or h > j)) or (j < i and h <= i and h > j):
            table[i] = k
            table[j] = EMPTY
            i = j


def insert_rounds(table, keys, prio, rng):
    """The kernel's phase 5: keys ordered by prio (lower wins). Returns the number of rounds."""
    n = len(table)
    at = {k: home(k, n) for k in keys}
    placed = {k: False for k in keys}

    def closed(k, occupant):  # a survivor, or an earlier new key
        return occupant not in prio or prio[occupant] < prio[k]

    def step(k):
        if placed[k]:
            if table[at[k]] == k:
                return
            placed[k] = False  # displaced by an earlier key: moves on
            at[k] = (at[k] + 1) % n
        changed[0] = True
        e = table[at[k]]
        for _ in range(n):
            if e is EMPTY or not closed(k, e):
                break
            at[k] = (at[k] + 1) % n
            yield  # another key may act between two cell reads
            e = table[at[k]]
        yield
        if table[at[k]] == e:  # compare-and-swap
            table[at[k]] = k
            placed[k] = True

    rounds = 0
    while True:
        changed = [False]
        gens = [g for g in (step(k) for k in keys) if g is not None]
        live = list(gens)
        while live:
            g = rng.choice(live)
            try:
                next(g)
            except StopIteration:
                live.remove(g)
        rounds += 1
        if not changed[0]:
            return rounds
        assert rounds < 4 * n, "insertion rounds did not converge"


@pytest.mark.parametrize("seed", range(40))
def test_insert_rounds_equal_sequential_order(seed):
    rng = random.Random(seed)
    size = rng.choice([64, 128, 256])
    load = rng.uniform(0.1, 0.45)
    survivors = rng.sample(range(1, 10 * size), int(load * size))
    table = [EMPTY] * size
    for k in survivors:
        insert_seq(table, k)
    evicted = rng.sample(survivors, rng.randint(0, len(survivors) // 2))
    pool = [k for k in range(10 * size, 20 * size)]
    new = rng.sample(pool, min(len(evicted) + rng.randint(0, 4), size // 2 - len(survivors) + len(evicted)))
    prio = {k: p for p, k in enumerate(rng.sample(new, len(new)))}  # miss positions

    expect = list(table)
    for k in evicted:
        erase_seq(expect, k)
    for k in sorted(new, key=prio.get):
        insert_seq(expect, k)

    got = list(table)
    for k in rng.sample(evicted, len(evicted)):  # deletions in any order give the same table
        erase_seq(got, k)
    insert_rounds(got, new, prio, rng)
    assert got == expect
