"""Shared helpers for the SIEVE parity tests: fixture loading, the KAT replay and the
hash-table invariant check. Used by both the CPU (oracle) and GPU test files."""
import json
import os

import numpy as np

from conftest import GOLDEN

RANDOM_CASES = ["mixed_small", "mid", "wrap_heavy", "dbs_unaligned", "c2_like"]


def load_kats():
    with open(os.path.join(GOLDEN, "sieve_kat.json")) as f:
        return json.load(f)


def load_npz(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def kat_top_k(case):
    """One fixed top_k per KAT state: the longest row, rounded up; rows are padded with -1
    (invalid positions: outputs -1/0 and no state change, hisp_sieve_update.cpp:119-122)."""
    return max(8, max(len(s["topk"]) for s in case["steps"]))


def pad_row(row, k):
    return np.array(list(row) + [-1] * (k - len(row)), dtype=np.int32)


def resident_map(tokens_row, dbs):
    """token -> slot for the occupied hot slots of one request (the oracle's t2s)."""
    return {int(t): s for s, t in enumerate(tokens_row[:dbs]) if t >= 0}


def hash32(t):
    return ((int(t) & 0xFFFFFFFF) * 2654435761 & 0xFFFFFFFF) >> 16


def check_ht_invariants(ht_row, tokens_row, dbs):
    """The table holds exactly one entry per resident token, each reachable from its home
    by a gap-free probe run (linear probing with backward-shift deletion keeps this)."""
    ht = np.asarray(ht_row).view(np.uint16)
    mask = len(ht) - 1
    res = resident_map(tokens_row, dbs)
    entries = {}
    for idx in np.nonzero(ht)[0]:
        slot = int(ht[idx]) - 1
        tok = int(tokens_row[slot])
        assert tok >= 0, "entry at {} points to empty slot {}".format(idx, slot)
        assert tok not in entries, "token {} twice in table".format(tok)
        entries[tok] = slot
        h = hash32(tok) & mask
        i = h
        while i != idx:
            assert ht[i] != 0, "gap between home {} and entry {}".format(h, idx)
            i = (i + 1) & mask
    assert entries == res
