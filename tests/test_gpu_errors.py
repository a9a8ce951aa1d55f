"""Device-side error reporting on the GPU without any GPU fault (no trap, no bad address, no
unbounded wait): the cooperative copy CTAs' bounded wait made to run out, the error word of
launches that publish no status words (CUDA-graph replays), and device-memory status words
cleared in stream order. The errCode bands are the reference's (kvops/kernel/kvc_common.h:24)."""
import numpy as np
import pytest

import oracle
from gpu_util import config_topk, dev, host, kv

pytestmark = pytest.mark.gpu

RB = 1152
COPY_TIMEOUT = 0x102
SEG_NULL = 0x101


def _coordinator(R, ctx, K, dbs, L):
    import torch
    from kv_offload_proto_b200.offload import XdsOffloadCoordinator
    co = XdsOffloadCoordinator("cuda:0", L, R, dbs, K, R, ctx)
    co.admit_all([ctx] * R, [r * ctx for r in range(R)])
    co.set_batch(torch.arange(R, dtype=torch.int64, device="cuda"),
                 torch.full((R,), ctx, dtype=torch.int32, device="cuda"))
    return co


def test_coop_copy_wait_that_runs_out_reports_copy_timeout():
    """copy_wait_polls=1: every copy CTA polls its walk lists once, finds them unfinished (the
    hand sweeps take tens of microseconds) and gives up. The step must still complete, report
    KVOPS_ERR_COPY_TIMEOUT in its status words and error word, and leave SIEVE outputs and state
    equal to the C restatement; the next step with the default bound copies every row."""
    import torch
    from kv_offload_proto_b200.pool import DevicePool, device_view
    mod = kv()
    R, ctx, K, dbs, L = 8, 4096, 512, 1024, 1
    rng = np.random.default_rng(5)
    st = oracle.SieveState(L, R, dbs, K)
    for r in range(R):
        st.admit(r, ctx)
    co = _coordinator(R, ctx, K, dbs, L)
    pool = DevicePool(0, L, R * ctx, RB, 1, segment_devices=(0,))
    seg_h = rng.integers(0, 256, pool.segment_bytes, dtype=np.uint8)
    device_view(pool.seg_bases[0], pool.segment_bytes, "cuda:0").copy_(dev(seg_h))
    hot = torch.zeros(R * dbs * RB, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pool_idx, seq, base = np.arange(R, dtype=np.int64), np.full(R, ctx, np.int32), np.arange(R, dtype=np.int64) * ctx
    for step, polls in enumerate((1, 0)):
        topk = config_topk(rng, st, 0, pool_idx, K, 0.3)
        status = pool.sieve_and_read(co, 0, dev(topk), hot, 0, 1, hot_req_stride_rows=dbs, path="coop",
                                     err_word=err, copy_wait_polls=polls)
        assert mod.last_step_path() == "coop"
        rc = mod.poll_status(status, 10_000_000)
        torch.cuda.synchronize()
        exp_slots, exp_miss = st.update(0, topk, pool_idx, seq)
        np.testing.assert_array_equal(host(co.top_k_device_slots), exp_slots)
        np.testing.assert_array_equal(host(co.is_miss), exp_miss)
        np.testing.assert_array_equal(host(co.device_buffer_ht)[0].view(np.uint16), st.ht[0])
        np.testing.assert_array_equal(host(co.device_buffer_tokens)[0], st.tokens[0])
        if polls == 1:
            assert exp_miss.sum() > 0
            assert rc == COPY_TIMEOUT, hex(rc)
            assert int(err.item()) == COPY_TIMEOUT
            err.zero_()
        else:
            assert rc == 0 and int(err.item()) == 0
            hot_exp = host(hot).copy()
            oracle.gather_rows(seg_h, 0, RB, topk, pool_idx, base, exp_slots, exp_miss, R, hot_exp, K, R, 1, 1, 0,
                               dbs)
            np.testing.assert_array_equal(host(hot), hot_exp)


@pytest.mark.parametrize("path", ["auto", "split"])
def test_step_graph_error_word_reports_null_segment(path):
    """A pool whose second segment base is 0: every replay's launches record
    KVOPS_ERR_SEG_NULL in the graph's error word (no status words exist in a replay), the rows
    of the other segment still land, and clear_error() resets the word."""
    import torch
    from kv_offload_proto_b200.graph import StepGraph
    from kv_offload_proto_b200.pool import DevicePool
    from kv_offload_proto_b200.workload import sample_topk_device
    kv()
    R, ctx, K, dbs, L = 8, 2048, 256, 512, 2
    good = DevicePool(0, L, R * ctx, RB, 1, segment_devices=(0,))
    pool = DevicePool(0, L, R * ctx, RB, 1, segment_devices=(0, 0), segment_addrs=[good.seg_bases[0], 0])
    co = _coordinator(R, ctx, K, dbs, L)
    hot = torch.zeros((L, R * dbs * RB), dtype=torch.uint8, device="cuda")
    g = StepGraph(pool, co, hot, path=path, hot_req_stride_rows=dbs)
    gen = torch.Generator(device="cuda").manual_seed(3)
    for _ in range(2):
        for layer in range(L):
            g.topk[layer] = sample_topk_device(co.device_buffer_tokens[layer, :R], ctx, dbs, K, 0.3, gen)
        assert g.error() == 0
        g.replay()
        torch.cuda.synchronize()
        assert g.error() == SEG_NULL
        g.clear_error()
    good.destroy()


def test_device_memory_status_words_are_cleared_in_stream_order():
    """Status words in device memory: two gathers in a row on the legacy stream publish into the
    same device slot; each poll (which reads on the legacy stream) sees only its own launch's
    done word, because the clear runs on the launch stream before the kernel."""
    import torch
    mod = kv()
    R, K, ctx, dbs, N = 4, 128, 1024, 256, 2
    rng = np.random.default_rng(9)
    plsr = oracle.per_layer_seg_rows(R * ctx, N)
    segs_h = [rng.integers(0, 256, plsr * RB, dtype=np.uint8) for _ in range(N)]
    segs = [dev(h) for h in segs_h]
    status = torch.zeros(8 * N * 8, dtype=torch.int64, device="cuda")  # 8 slots per node, device memory
    pool_idx, base = np.arange(R, dtype=np.int64), np.arange(R, dtype=np.int64) * ctx
    t_pool, t_base, t_nr = dev(pool_idx), dev(base), dev(np.array([R], np.int32))
    hot = torch.zeros(R * dbs * RB, dtype=torch.uint8, device="cuda")
    exp = np.zeros(R * dbs * RB, np.uint8)
    for call in range(2):
        topk = np.stack([rng.choice(ctx, K, replace=False) for _ in range(R)]).astype(np.int32)
        miss = (rng.random((R, K)) < 0.4).astype(np.int8)
        slots = np.stack([rng.permutation(dbs)[:K] for _ in range(R)]).astype(np.int32)
        miss_ok = miss.copy()
        if call == 1:  # a row past its segment (node 0, segRow R*ctx >= plsr): the 0x2xx band, not copied
            topk[0, 0], miss[0, 0], miss_ok[0, 0] = 2 * R * ctx, 1, 0
        t_topk, t_slots, t_miss = dev(topk), dev(slots), dev(miss)
        mod.import_multi([s.data_ptr() for s in segs], 0, plsr, RB, t_topk.data_ptr(), t_pool.data_ptr(),
                         t_base.data_ptr(), t_slots.data_ptr(), t_miss.data_ptr(), t_nr.data_ptr(), hot.data_ptr(),
                         K, R, 1, status.data_ptr(), 0, 2, hot_req_stride_rows=dbs)
        rcs = [mod.poll_status(status.data_ptr() + s * 64 + b * 8, 10_000_000) for s in range(N) for b in range(2)]
        if call == 0:
            assert rcs == [0] * (2 * N)
        else:
            assert all((rc & ~0xFF) == 0x10200 for rc in rcs), [hex(r) for r in rcs]
        torch.cuda.synchronize()
        oracle.gather_all(segs_h, 0, RB, topk, pool_idx, base, slots, miss_ok, R, exp, K, R, 1,
                          hot_req_stride_rows=dbs)
    np.testing.assert_array_equal(host(hot), exp)
