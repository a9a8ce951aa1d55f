"""GPU parity of CUDA-graph replay (kv_offload_proto_b200.graph.StepGraph): decode steps
replayed from a graph must leave exactly the state, outputs and hot rows that the reference's
per-layer call pair (sieve_update then batch_read, xds_decode.py:225-233) leaves."""
import numpy as np
import pytest

from gpu_util import kv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", ["auto", "split"])
def test_step_graph_replay_equals_reference_call_pair(path):
    import torch
    from kv_offload_proto_b200.graph import StepGraph
    from kv_offload_proto_b200.offload import XdsOffloadCoordinator
    from kv_offload_proto_b200.pool import DevicePool, device_view
    from kv_offload_proto_b200.workload import sample_topk_device
    kv()
    R, ctx, K, dbs, L, RB = 16, 2048, 256, 512, 3, 1152
    pool = DevicePool(0, L, R * ctx, RB, 1, segment_devices=(0, 0))
    for s in range(2):
        v = torch.as_tensor(np.arange(pool.segment_bytes // 4, dtype=np.int32) * (s + 3)).cuda()
        device_view(pool.seg_bases[s], pool.segment_bytes, "cuda:0").copy_(v.view(torch.uint8))
    cos, hots = [], []
    for _ in range(2):
        co = XdsOffloadCoordinator("cuda:0", L, R, dbs, K, R, ctx)
        co.admit_all([ctx] * R, [r * ctx for r in range(R)])
        co.set_batch(torch.arange(R, dtype=torch.int64, device="cuda"),
                     torch.full((R,), ctx, dtype=torch.int32, device="cuda"))
        cos.append(co)
        hots.append(torch.zeros((L, R * dbs * RB), dtype=torch.uint8, device="cuda"))
    counts = torch.zeros(L, dtype=torch.int64, device="cuda")  # filled inside the graph (after_layer)
    graph = StepGraph(pool, cos[1], hots[1], path=path, hot_req_stride_rows=dbs,
                      after_layer=lambda l: counts[l].copy_(cos[1].is_miss.sum()))
    assert graph.path == ("coop" if path == "auto" else "split")
    torch.cuda.synchronize()
    # capture launched nothing: both sides still start from the admitted state
    assert torch.equal(cos[0].device_buffer_ht, cos[1].device_buffer_ht)
    gen = torch.Generator(device="cuda").manual_seed(6)
    for step in range(4):
        topk = torch.empty((L, R, K), dtype=torch.int32, device="cuda")
        co = cos[0]
        ref_counts = []
        for layer in range(L):
            topk[layer] = sample_topk_device(co.device_buffer_tokens[layer, :R], ctx, dbs, K, 0.25, gen)
            co.sieve_update(layer, topk[layer])
            st = pool.batch_read(layer, topk[layer], co._req_pool_indices, co.req_host_base, co.top_k_device_slots,
                                 co.is_miss, co.num_real, hots[0][layer], R, K, 0, 1, hot_req_stride_rows=dbs)
            pool.wait(st)
            ref_counts.append(int(co.is_miss.sum()))
        graph.topk.copy_(topk)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(cos[0].top_k_device_slots, cos[1].top_k_device_slots)
        assert torch.equal(cos[0].is_miss, cos[1].is_miss)
        for name in ("device_buffer_tokens", "device_buffer_visited", "device_buffer_ht", "sieve_hand"):
            assert torch.equal(getattr(cos[0], name), getattr(cos[1], name)), (step, name)
        assert torch.equal(hots[0], hots[1]), step
        assert counts.tolist() == ref_counts, step  # per-layer outputs seen by the captured hook
        assert int(cos[1].is_miss.sum()) > 0
    pool.destroy()


def test_step_graph_1000_replays_with_num_real_padding_and_growing_seq_lens():
    """1000 replays of one captured step while num_real (batch padding) and seq_lens (decode
    growth) change in place between replays, against the reference's call pair on a twin."""
    import torch
    from kv_offload_proto_b200.graph import StepGraph
    from kv_offload_proto_b200.offload import XdsOffloadCoordinator
    from kv_offload_proto_b200.pool import DevicePool, device_view
    from kv_offload_proto_b200.workload import sample_topk_device
    kv()
    R, ctx, K, dbs, L, RB = 8, 512, 64, 128, 1, 1152
    pool = DevicePool(0, L, R * ctx, RB, 1, segment_devices=(0,))
    v = torch.as_tensor(np.arange(pool.segment_bytes // 4, dtype=np.int32)).cuda()
    device_view(pool.seg_bases[0], pool.segment_bytes, "cuda:0").copy_(v.view(torch.uint8))
    cos, hots = [], []
    for _ in range(2):
        co = XdsOffloadCoordinator("cuda:0", L, R, dbs, K, R, ctx + 1100)
        co.admit_all([ctx] * R, [r * ctx for r in range(R)])
        co.set_batch(torch.arange(R, dtype=torch.int64, device="cuda"),
                     torch.full((R,), ctx, dtype=torch.int32, device="cuda"))
        cos.append(co)
        hots.append(torch.zeros((L, R * dbs * RB), dtype=torch.uint8, device="cuda"))
    graph = StepGraph(pool, cos[1], hots[1], hot_req_stride_rows=dbs)
    gen = torch.Generator(device="cuda").manual_seed(9)
    pads = [R, R - 3, R, 1, R - 1]
    for step in range(1000):
        nr = pads[step % len(pads)]
        for co in cos:
            co.num_real.fill_(nr)
            co._seq_lens.add_(1)
        co = cos[0]
        topk = sample_topk_device(co.device_buffer_tokens[0, :R], ctx, dbs, K, 0.3, gen)
        ext = torch.rand((R, K), device="cuda", generator=gen) < 0.05  # some decode-extension positions
        topk = torch.where(ext, ctx + step % 7, topk).to(torch.int32)
        co.sieve_update(0, topk)
        st = pool.batch_read(0, topk, co._req_pool_indices, co.req_host_base, co.top_k_device_slots, co.is_miss,
                             co.num_real, hots[0][0], R, K, 0, 1, hot_req_stride_rows=dbs)
        pool.wait(st)
        graph.topk[0].copy_(topk)
        graph.replay()
        if step % 50 == 49 or step == 999:
            torch.cuda.synchronize()
            assert torch.equal(cos[0].top_k_device_slots[:nr], cos[1].top_k_device_slots[:nr]), step
            assert torch.equal(cos[0].is_miss[:nr], cos[1].is_miss[:nr]), step
            for name in ("device_buffer_tokens", "device_buffer_visited", "device_buffer_ht", "sieve_hand"):
                assert torch.equal(getattr(cos[0], name), getattr(cos[1], name)), (step, name)
            assert torch.equal(hots[0], hots[1]), step
    pool.destroy()
