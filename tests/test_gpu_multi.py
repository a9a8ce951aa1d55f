"""Parity of the layer-step with pool segments in another GPU's HBM (needs >= 2 GPUs; skipped
otherwise): the rows are read in-kernel over NVLink/NVSwitch, either through a peer mapping in
the same process or through a CUDA IPC mapping of a segment that another process allocated
and filled (the one-process-per-GPU layout of bench.py). Slots, miss flags, SIEVE state and
every hot-row byte are checked against the C restatement."""
import multiprocessing as mp

import numpy as np
import pytest

import oracle
from gpu_util import config_topk, dev, host, kv

pytestmark = pytest.mark.gpu

RB = 1152


def _gpus():
    import torch
    return torch.cuda.device_count()


def _seg_bytes(seed, n):
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8)


def _steps(mod, seg_addrs, segs_h, path, R=16, K=512, ctx=4096, dbs=1024, S=1, steps=3, miss=0.25, seed=0):
    """`steps` layer-steps through sieve_import with the given segments (node order), each
    checked against the C restatement (sieve, then the gather over host copies of the segments)."""
    import torch
    rng = np.random.default_rng(seed)
    N = len(seg_addrs)
    st = oracle.SieveState(1, R, dbs, K)
    for r in range(R):
        st.admit(r, ctx)
    tokens, vis, ht, hand = dev(st.tokens[0]), dev(st.visited[0]), dev(st.ht[0].view(np.int16)), dev(st.hand[0])
    pre = dev(st.prefill_lens)
    pool_idx, seq, base = np.arange(R, dtype=np.int64), np.full(R, ctx, np.int32), np.arange(R, dtype=np.int64) * ctx
    t_pool, t_seq, t_base, t_nr = dev(pool_idx), dev(seq), dev(base), dev(np.array([R], np.int32))
    plsr = oracle.per_layer_seg_rows(R * ctx, N)
    hot = torch.zeros(R * dbs * RB, dtype=torch.uint8, device="cuda")
    exp_hot = np.zeros(R * dbs * RB, np.uint8)
    slots = torch.empty((R, K), dtype=torch.int32, device="cuda")
    missf = torch.empty((R, K), dtype=torch.int8, device="cuda")
    status = mod.alloc_status(8 * N)
    ran = set()
    for _ in range(steps):
        topk = config_topk(rng, st, 0, pool_idx, K, miss)
        t_topk = dev(topk)
        mod.sieve_import(t_topk.data_ptr(), t_pool.data_ptr(), t_seq.data_ptr(), pre.data_ptr(), tokens.data_ptr(),
                         vis.data_ptr(), ht.data_ptr(), hand.data_ptr(), slots.data_ptr(), missf.data_ptr(),
                         t_nr.data_ptr(), K, dbs, st.padded, st.vis_stride, R, R, seg_addrs, 0, plsr, RB,
                         t_base.data_ptr(), hot.data_ptr(), S, status, 0, 1, hot_req_stride_rows=dbs, path=path)
        ran.add(mod.last_step_path())
        rcs = [mod.poll_status(status + s * 64, 10_000_000) for s in range(N)]
        torch.cuda.synchronize()
        assert rcs == [0] * N
        exp_slots, exp_miss = st.update(0, topk, pool_idx, seq)
        np.testing.assert_array_equal(host(slots), exp_slots)
        np.testing.assert_array_equal(host(missf), exp_miss)
        np.testing.assert_array_equal(host(tokens), st.tokens[0])
        np.testing.assert_array_equal(host(ht).view(np.uint16), st.ht[0])
        n = oracle.gather_all(segs_h, 0, RB, topk, pool_idx, base, exp_slots, exp_miss, R, exp_hot, K, R, S,
                              hot_req_stride_rows=dbs)
        assert n == int(exp_miss.sum()) > 0
        np.testing.assert_array_equal(host(hot), exp_hot)
    return ran


@pytest.mark.parametrize("path", ["coop", "split"])
def test_peer_segments_in_one_process(path):
    """Node 0 of the pool in GPU 1's HBM (peer mapping), node 1 in GPU 0's own HBM."""
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    import torch
    from kv_offload_proto_b200.pool import device_view
    mod = kv()
    R, ctx = 16, 4096
    plsr = oracle.per_layer_seg_rows(R * ctx, 2)
    nbytes = plsr * RB
    mod.enable_peer_access(0, 1)
    peer = mod.segment_alloc(1, nbytes)
    local = mod.segment_alloc(0, nbytes)
    segs_h = [_seg_bytes(1, nbytes), _seg_bytes(2, nbytes)]
    device_view(peer, nbytes, "cuda:1").copy_(torch.from_numpy(segs_h[0]).to("cuda:1"))
    device_view(local, nbytes, "cuda:0").copy_(torch.from_numpy(segs_h[1]).to("cuda:0"))
    torch.cuda.synchronize(1)
    try:
        assert _steps(mod, [peer, local], segs_h, path) == {path}
    finally:
        torch.cuda.synchronize()
        mod.segment_free(peer)
        mod.segment_free(local)


def _host_segment(q_handle, q_done, nbytes, seed):
    """Second process: owns GPU 1, allocates and fills one segment, exports its IPC handle and
    keeps it alive until told (or until a bounded wait runs out)."""
    import queue

    import torch
    import kv_offload_proto_b200 as kp
    from kv_offload_proto_b200.pool import device_view
    torch.cuda.set_device(1)
    mod = kp.install_kvops_ext()
    mod.init(1, "")
    addr = mod.segment_alloc(1, nbytes)
    device_view(addr, nbytes, "cuda:1").copy_(torch.from_numpy(_seg_bytes(seed, nbytes)).to("cuda:1"))
    torch.cuda.synchronize()
    q_handle.put(mod.ipc_get_handle(addr))
    try:
        q_done.get(timeout=300)
    except queue.Empty:
        pass
    mod.segment_free(addr)


def test_ipc_segment_from_another_process():
    """The pool's only node is a segment that another process allocated on GPU 1; this process
    maps it through its CUDA IPC handle and runs cooperative layer-steps reading it over NVLink."""
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    import torch
    mod = kv()
    R, ctx = 16, 4096
    plsr = oracle.per_layer_seg_rows(R * ctx, 1)
    nbytes = plsr * RB
    ctx_mp = mp.get_context("spawn")
    q_handle, q_done = ctx_mp.Queue(), ctx_mp.Queue()
    proc = ctx_mp.Process(target=_host_segment, args=(q_handle, q_done, nbytes, 7))
    proc.start()
    try:
        handle = q_handle.get(timeout=300)
        addr = mod.ipc_open_handle(0, handle)
        try:
            assert _steps(mod, [addr], [_seg_bytes(7, nbytes)], "coop") == {"coop"}
        finally:
            torch.cuda.synchronize()
            mod.ipc_close_handle(addr)
    finally:
        q_done.put(1)
        proc.join(timeout=120)
    assert proc.exitcode == 0
