"""Pin the C restatement (oracle/kvoracle.c) against the golden vectors recorded from the
reference's own Python oracle (xds/xds_decode.py:66-118) and the reference's SIEVE KATs
(test/test_sieve_oracle.py:24-83). CPU only."""
import numpy as np
import pytest

import oracle
from sieve_cases import (RANDOM_CASES, check_ht_invariants, kat_top_k, load_kats, load_npz, pad_row,
                         resident_map)


@pytest.mark.parametrize("case", load_kats(), ids=lambda c: c["name"])
def test_kat(case):
    K = kat_top_k(case)
    st = oracle.SieveState(1, case["num_reqs"], case["dbs"], K)
    for r in range(case["num_reqs"]):
        st.admit(r, case["prefill"])
    for step in case["steps"]:
        n = len(step["topk"])
        slots, miss = st.update(0, pad_row(step["topk"], K)[None], np.array([step["pool_idx"]]),
                                np.array([step["seq_len"]]))
        assert slots[0, :n].tolist() == step["slots"]
        assert miss[0, :n].tolist() == step["is_miss"]
        assert (slots[0, n:] == -1).all() and (miss[0, n:] == 0).all()
    for r, fin in enumerate(case["final"]):
        assert int(st.hand[0, r, 0]) == fin["hand"]
        assert sorted(resident_map(st.tokens[0, r], case["dbs"]).items()) == [tuple(x) for x in fin["t2s"]]
        check_ht_invariants(st.ht[0, r], st.tokens[0, r], case["dbs"])


def test_c1_ref_sampler():
    fx = load_npz("sieve_c1_ref_sampler.npz")
    R, K, dbs, L = int(fx["req"]), int(fx["top_k"]), int(fx["dbs"]), int(fx["layers"])
    st = oracle.SieveState(L, R, dbs, K)
    for r in range(R):
        st.admit(r, int(fx["prefill"]))
    seq = np.full(R, int(fx["prefill"]), np.int32)
    for s in range(int(fx["steps"])):
        slots, miss = st.update(s % L, fx["topk"][s], np.arange(R), seq)
        np.testing.assert_array_equal(slots, fx["slots"][s])
        np.testing.assert_array_equal(miss, fx["is_miss"][s])


@pytest.mark.parametrize("name", RANDOM_CASES)
@pytest.mark.parametrize("nthreads", [1, 3])
def test_random_fixture(name, nthreads):
    fx = load_npz("sieve_{}.npz".format(name))
    R, K, dbs, L = int(fx["req"]), int(fx["top_k"]), int(fx["dbs"]), int(fx["layers"])
    st = oracle.SieveState(L, R, dbs, K)
    for r in range(R):
        st.admit(r, int(fx["prefill"]))
    seq = np.full(R, int(fx["seq_len"]), np.int32)
    for s in range(int(fx["steps"])):
        for l in range(L):
            slots, miss = st.update(l, fx["topk"][s, l], np.arange(R), seq, nthreads=nthreads)
            np.testing.assert_array_equal(slots, fx["slots"][s, l])
            np.testing.assert_array_equal(miss, fx["is_miss"][s, l])
    for l in range(L):
        for r in range(R):
            check_ht_invariants(st.ht[l, r], st.tokens[l, r], dbs)


def test_padding_and_bad_pool_rows():
    """Rows >= num_real and rows whose pool index is out of range get -1/0 and leave the
    state untouched (hisp_sieve_update.cpp:72-88)."""
    st = oracle.SieveState(1, 4, 32, 16)
    for r in range(4):
        st.admit(r, 100)
    before = st.copy()
    topk = np.tile(np.arange(40, 56, dtype=np.int32), (4, 1))
    slots, miss = st.update(0, topk, np.array([0, 9, -1, 3]), np.full(4, 100), num_real=3)
    assert (miss[0] == 1).all()
    for b in (1, 2, 3):
        assert (slots[b] == -1).all() and (miss[b] == 0).all()
    for r in (1, 2, 3):
        np.testing.assert_array_equal(st.tokens[0, r], before.tokens[0, r])
        np.testing.assert_array_equal(st.ht[0, r], before.ht[0, r])


def test_dirty_hand_clamped():
    """A hand outside [0, dbs) restarts the sweep at slot 0 (hisp_sieve_update.cpp:108-111)."""
    st = oracle.SieveState(1, 1, 8, 8)
    st.admit(0, 100)
    st.hand[0, 0, 0] = 12345
    slots, miss = st.update(0, pad_row([50], 8)[None], np.array([0]), np.array([100]))
    assert slots[0, 0] == 0 and miss[0, 0] == 1
    assert st.hand[0, 0, 0] == 1


def test_hash_matches_reference_formula():
    for t in (0, 1, 7, 4095, 65535, 2 ** 31 - 1, -1, -12345):
        assert oracle.hash32(t) == ((t & 0xFFFFFFFF) * 2654435761 & 0xFFFFFFFF) >> 16
