"""GPU parity of the large-table SIEVE tier (sieve_big_kernel): slots / is_miss and every
persisted state byte (tokens, visited bitmap, hash-table bytes, hand) against the C restatement
of the reference kernel, step after step. The tier is forced (kvops_set_sieve_tier) on the
shapes the shared-memory tier also runs, so that many states are compared cheaply, and runs by
itself at the stress shape (hot buffer 65518 slots, 262144-cell table: BASELINE config 5,
fewer requests and steps). States the tier refuses (a token row holding a token twice, a sweep
that would pass a slot twice) must fall back to the position-ordered loop with the same bytes."""
import numpy as np
import pytest

import oracle
from gpu_util import DeviceSieve, config_topk, kv

pytestmark = pytest.mark.gpu


@pytest.fixture
def tier():
    mod = kv()
    yield mod.set_sieve_tier
    mod.set_sieve_tier("auto")


def _run(rng, st, steps, K, miss, prefill, ext=16, invalid=0.01, dup=0.01, reqs=None, num_real=None, expect="large"):
    mod = kv()
    ds = DeviceSieve(st)
    R = st.pool_size if reqs is None else len(reqs)
    reqs = np.arange(R) if reqs is None else np.asarray(reqs)
    for _ in range(steps):
        topk = config_topk(rng, st, 0, reqs, K, miss, ext=ext, invalid=invalid, dup=dup)
        seq = np.full(len(reqs), prefill + ext, np.int32)
        got_s, got_m = ds.update(0, topk, reqs, seq, num_real=num_real)
        assert mod.last_sieve_tier() == expect
        exp_s, exp_m = st.update(0, topk, reqs, seq, num_real=num_real)
        np.testing.assert_array_equal(got_m, exp_m)
        np.testing.assert_array_equal(got_s, exp_s)
        ds.assert_state_equal()


# (dbs, top_k, requests, steps, miss ratio): config 1, 2 and 3 shapes, an unaligned hot buffer
# and a sweep that wraps (more misses than unvisited slots: the fallback).
FORCED = [(64, 64, 8, 6, 0.5), (4096, 2048, 6, 4, 0.2), (8192, 2048, 3, 3, 0.5), (1000, 300, 5, 8, 0.9),
          (64, 256, 4, 4, 0.9)]


@pytest.mark.parametrize("dbs,K,R,steps,miss", FORCED, ids=lambda v: str(v))
def test_forced_large_tier_vs_oracle(tier, dbs, K, R, steps, miss):
    tier("large")
    rng = np.random.default_rng(dbs * 3 + K)
    prefill = max(2 * dbs, 3 * K)
    st = oracle.SieveState(1, R, dbs, K)
    for r in range(R):
        st.admit(r, prefill)
    _run(rng, st, steps, K, miss, prefill)


def test_forced_large_tier_padding_rows_and_bad_pool(tier):
    tier("large")
    st = oracle.SieveState(1, 6, 256, 128)
    for r in range(6):
        st.admit(r, 2000)
    st.hand[0, 1, 0] = -5
    _run(np.random.default_rng(3), st, 3, 128, 0.6, 2000, reqs=[0, 1, 2, 77, -1, 5, 4, 3], num_real=6)


def test_forced_large_tier_duplicate_tokens_fall_back(tier):
    """A token held by two slots (only the first has a table entry): the table check refuses
    the state and the position-ordered loop runs; the bytes still equal the reference's."""
    tier("large")
    R, dbs, K = 3, 300, 100
    prefill = 900
    st = oracle.SieveState(1, R, dbs, K)
    for r in range(R):
        st.admit(r, prefill)
    st.tokens[0, :, 5] = st.tokens[0, :, 2]
    st.tokens[0, :, 9] = st.tokens[0, :, 7]
    _run(np.random.default_rng(11), st, 5, K, 0.3, prefill, ext=0, invalid=0.0, dup=0.0)


@pytest.mark.parametrize("dist", ["uniform", "zipf"])
def test_stress_shape_runs_large_tier(dist):
    """BASELINE config 5's shape (dbs 65518, topK 2048, context 131072) with the stress draws
    (90% misses, or Zipf(0.8) popularity): the automatic choice is the large-table tier, and
    after a few steps the reference's 16-bit homes have packed the table's first quarter into
    long probe runs that every erase and insert crosses."""
    from kv_offload_proto_b200.workload import stress_topk_uniform, stress_topk_zipf, zipf_cdf
    mod = kv()
    R, dbs, K, ctx, steps = 4, 65518, 2048, 131072, 4
    st = oracle.SieveState(1, R, dbs, K)
    for r in range(R):
        st.admit(r, ctx)
    ds = DeviceSieve(st)
    rng = np.random.default_rng(5)
    cdf, perm = zipf_cdf(ctx, 0.8, 5)
    reqs, seq = np.arange(R), np.full(R, ctx, np.int32)
    for _ in range(steps):
        topk = stress_topk_uniform(rng, st.tokens[0], dbs, ctx, K, 0.9) if dist == "uniform" else \
            stress_topk_zipf(rng, R, ctx, K, cdf, perm)
        got_s, got_m = ds.update(0, topk, reqs, seq)
        assert mod.last_sieve_tier() == "large"
        exp_s, exp_m = st.update(0, topk, reqs, seq, nthreads=R)
        np.testing.assert_array_equal(got_m, exp_m)
        np.testing.assert_array_equal(got_s, exp_s)
    ds.assert_state_equal()


def test_tier_choice_validation():
    mod = kv()
    with pytest.raises(Exception):
        mod.set_sieve_tier("fastest")
    mod.set_sieve_tier("auto")
