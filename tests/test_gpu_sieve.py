"""GPU parity of the CUDA SIEVE (hisp_sieve_update / hisp_sieve_ht_init) through the C ABI:
bit-exact slots / is_miss against the reference oracle's golden vectors, and bit-exact
persisted state (tokens, visited bitmap, hash-table bytes, hand) against the C restatement,
across the shared-memory and global-memory state tiers."""
import numpy as np
import pytest

import oracle
from gpu_util import DeviceSieve, config_topk, dev, host, kv
from sieve_cases import RANDOM_CASES, check_ht_invariants, kat_top_k, load_kats, load_npz, pad_row

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", load_kats(), ids=lambda c: c["name"])
def test_kat_gpu(case):
    K = kat_top_k(case)
    st = oracle.SieveState(1, case["num_reqs"], case["dbs"], K)
    for r in range(case["num_reqs"]):
        st.admit(r, case["prefill"])
    ds = DeviceSieve(st)
    for step in case["steps"]:
        n = len(step["topk"])
        row = pad_row(step["topk"], K)[None]
        slots, miss = ds.update(0, row, [step["pool_idx"]], [step["seq_len"]])
        assert slots[0, :n].tolist() == step["slots"]
        assert miss[0, :n].tolist() == step["is_miss"]
        st.update(0, row, np.array([step["pool_idx"]]), np.array([step["seq_len"]]))
    ds.assert_state_equal()


def test_c1_through_coordinator():
    """BASELINE config 1 (reference sampler, seed 42) driven through the coordinator API."""
    import torch
    from kv_offload_proto_b200.offload import XdsOffloadCoordinator
    kv()
    fx = load_npz("sieve_c1_ref_sampler.npz")
    R, K, dbs, L, pre = int(fx["req"]), int(fx["top_k"]), int(fx["dbs"]), int(fx["layers"]), int(fx["prefill"])
    co = XdsOffloadCoordinator("cuda:0", L, R, dbs, K, R, pre)
    for r in range(R):
        co.admit_request(r, r, pre, r * pre)
    co.set_batch(torch.arange(R, dtype=torch.int64, device="cuda"), torch.full((R,), pre, dtype=torch.int32,
                                                                                device="cuda"))
    for s in range(int(fx["steps"])):
        co.sieve_update(s % L, dev(fx["topk"][s]))
        np.testing.assert_array_equal(host(co.top_k_device_slots), fx["slots"][s])
        np.testing.assert_array_equal(host(co.is_miss), fx["is_miss"][s])
    assert int(co.miss_count().item()) == int(fx["is_miss"][-1].sum())


@pytest.mark.parametrize("name", RANDOM_CASES)
def test_random_fixture_gpu(name):
    import torch
    from kv_offload_proto_b200.offload import XdsOffloadCoordinator
    kv()
    fx = load_npz("sieve_{}.npz".format(name))
    R, K, dbs, L, pre = int(fx["req"]), int(fx["top_k"]), int(fx["dbs"]), int(fx["layers"]), int(fx["prefill"])
    co = XdsOffloadCoordinator("cuda:0", L, R, dbs, K, R, int(fx["seq_len"]))
    co.admit_all([pre] * R, [r * pre for r in range(R)])
    co.set_batch(torch.arange(R, dtype=torch.int64, device="cuda"),
                 torch.full((R,), int(fx["seq_len"]), dtype=torch.int32, device="cuda"))
    for s in range(int(fx["steps"])):
        for l in range(L):
            co.sieve_update(l, dev(fx["topk"][s, l]))
            np.testing.assert_array_equal(host(co.top_k_device_slots), fx["slots"][s, l])
            np.testing.assert_array_equal(host(co.is_miss), fx["is_miss"][s, l])
    tok, ht = host(co.device_buffer_tokens), host(co.device_buffer_ht).view(np.uint16)
    for l in range(L):
        for r in range(R):
            check_ht_invariants(ht[l, r], tok[l, r], dbs)


# (dbs, top_k, requests, steps, miss_ratio): shared-memory tier (c2 / c3 shapes) and the
# global-memory tier (hot buffer at the uint16 limit, c5 shape).
TIERS = [(64, 64, 8, 6, 0.5), (4096, 2048, 6, 3, 0.2), (8192, 2048, 4, 3, 0.5), (1000, 300, 5, 8, 0.9),
         (65518, 2048, 2, 2, 0.9)]


@pytest.mark.parametrize("dbs,K,R,steps,miss", TIERS, ids=lambda v: str(v))
def test_state_bytes_vs_oracle(dbs, K, R, steps, miss):
    kv()
    rng = np.random.default_rng(dbs + K)
    prefill = max(2 * dbs, 3 * K)
    st = oracle.SieveState(1, R + 1, dbs, K)
    for r in range(R + 1):
        st.admit(r, prefill)
    ds = DeviceSieve(st)
    reqs = np.arange(R)
    for s in range(steps):
        topk = config_topk(rng, st, 0, reqs, K, miss, ext=16, invalid=0.01, dup=0.01)
        seq = np.full(R, prefill + 16, np.int32)
        got_s, got_m = ds.update(0, topk, reqs, seq)
        exp_s, exp_m = st.update(0, topk, reqs, seq)
        np.testing.assert_array_equal(got_m, exp_m)
        np.testing.assert_array_equal(got_s, exp_s)
        ds.assert_state_equal()


def test_padding_rows_bad_pool_and_dirty_hand():
    kv()
    st = oracle.SieveState(1, 6, 256, 128)
    for r in range(6):
        st.admit(r, 2000)
    st.hand[0, 1, 0] = -5
    st.hand[0, 2, 0] = 99999
    ds = DeviceSieve(st)
    rng = np.random.default_rng(3)
    reqs = np.array([0, 1, 2, 77, -1, 5, 4, 3])
    topk = config_topk(rng, st, 0, reqs, 128, 0.6)
    seq = np.full(len(reqs), 2000, np.int32)
    got = ds.update(0, topk, reqs, seq, num_real=6)
    exp = st.update(0, topk, reqs, seq, num_real=6)
    for g, e in zip(got, exp):
        np.testing.assert_array_equal(g, e)
    for b in (3, 4, 6, 7):  # bad pool index, negative index, padding rows
        assert (got[0][b] == -1).all() and (got[1][b] == 0).all()
    ds.assert_state_equal()


def test_num_real_above_max_is_clamped():
    kv()
    st = oracle.SieveState(1, 2, 64, 32)
    for r in range(2):
        st.admit(r, 500)
    ds = DeviceSieve(st)
    topk = config_topk(np.random.default_rng(1), st, 0, [0, 1], 32, 0.5)
    got = ds.update(0, topk, [0, 1], [500, 500], num_real=50)
    exp = st.update(0, topk, np.array([0, 1]), np.array([500, 500]), num_real=50)
    np.testing.assert_array_equal(got[0], exp[0])
    ds.assert_state_equal()


@pytest.mark.parametrize("dbs,K,block_dim", [(64, 64, 0), (4096, 2048, 0), (65518, 2048, 0), (300, 40, 5)])
def test_ht_init_matches_oracle(dbs, K, block_dim):
    """Admission build from arbitrary token rows (holes and duplicates included), with the
    reference's block -> (layer, request) mapping and partial block counts."""
    import torch
    kv()
    L, P = 3, 4
    st = oracle.SieveState(L, P, dbs, K)
    rng = np.random.default_rng(dbs)
    st.tokens[:] = rng.integers(-1, 3 * dbs, size=st.tokens.shape).astype(np.int32)
    st.tokens[:, :, ::7] = st.tokens[:, :, 3:4]  # duplicates: first slot must win
    st.ht[:] = 0xBEEF
    ds = DeviceSieve(st)
    kv().sieve_ht_init(ds.tokens.data_ptr(), ds.ht.data_ptr(), ds.prefill.data_ptr(), 1, 2, L, P, dbs, st.padded,
                       st.ht_size, 0, block_dim)
    torch.cuda.synchronize()
    st.ht_init(1, 2, block_dim if block_dim else L * 2)
    np.testing.assert_array_equal(host(ds.ht).view(np.uint16), st.ht)


@pytest.mark.parametrize("kw,msg", [
    (dict(padded=72), "multiple of 16"),
    (dict(padded=65536, dbs=65530, vis=8192), "<= 65534"),
    (dict(vis=32), "64B aligned"),
    (dict(vis=0), "64B aligned"),
    (dict(dbs=100), "device_buffer_size"),
    (dict(block_dim=0), "block_dim"),
])
def test_sieve_update_validation(kw, msg):
    mod = kv()
    a = dict(padded=64, dbs=64, vis=64, block_dim=8)
    a.update(kw)
    with pytest.raises(RuntimeError, match=msg):
        mod.sieve_update(8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 64, a["dbs"], a["padded"], a["vis"], 1, 1, 0,
                         a["block_dim"])


@pytest.mark.parametrize("dbs,K", [(300, 100), (4096, 2048)])
def test_duplicate_token_state_matches_oracle(dbs, K):
    """A token row holding the same token twice (only its first slot is in the table) is
    outside the parallel path's assumptions: such steps must still match the reference."""
    kv()
    R = 3
    rng = np.random.default_rng(dbs * 7)
    prefill = max(2 * dbs, 3 * K)
    st = oracle.SieveState(1, R, dbs, K)
    for r in range(R):
        st.admit(r, prefill)
    st.tokens[0, :, 5] = st.tokens[0, :, 2]
    st.tokens[0, :, 9] = st.tokens[0, :, 7]
    ds = DeviceSieve(st)
    for s in range(6):
        topk = config_topk(rng, st, 0, np.arange(R), K, 0.3)
        seq = np.full(R, prefill, np.int32)
        got = ds.update(0, topk, np.arange(R), seq)
        exp = st.update(0, topk, np.arange(R), seq)
        np.testing.assert_array_equal(got[1], exp[1])
        np.testing.assert_array_equal(got[0], exp[0])
        ds.assert_state_equal()


@pytest.mark.parametrize("seed", range(4))
def test_c2_shape_many_steps(seed):
    """Config-2 shape, 12 steps at 20% and 60% misses: long runs through the parallel path."""
    kv()
    R, dbs, K = 4, 4096, 2048
    rng = np.random.default_rng(100 + seed)
    st = oracle.SieveState(1, R, dbs, K)
    for r in range(R):
        st.admit(r, 8192)
    ds = DeviceSieve(st)
    for s in range(12):
        topk = config_topk(rng, st, 0, np.arange(R), K, 0.2 if s % 3 else 0.6)
        seq = np.full(R, 8192, np.int32)
        got = ds.update(0, topk, np.arange(R), seq)
        exp = st.update(0, topk, np.arange(R), seq)
        np.testing.assert_array_equal(got[1], exp[1])
        np.testing.assert_array_equal(got[0], exp[0])
    ds.assert_state_equal()
