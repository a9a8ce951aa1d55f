"""GPU parity of the miss-row gather (kvc_gather_rows) and the striped export
(kvc_scatter_rows_alllayer) through the C ABI: every destination byte against the C
restatement on host copies, the status-slot protocol, and the device-side errCodes."""
import numpy as np
import pytest

import oracle
from gpu_util import dev, host, host_view, kv

pytestmark = pytest.mark.gpu

RB = 1152


def make_batch(rng, R, K, ctx, dbs, miss_ratio, stride):
    """Sieve-shaped inputs: topk positions, is_miss, slots. Miss destinations never collide
    (unique slots per request; unique across requests when the hot buffer is shared)."""
    topk = np.stack([rng.choice(ctx, K, replace=False) for _ in range(R)]).astype(np.int32)
    miss = (rng.random((R, K)) < miss_ratio).astype(np.int8)
    slots = np.full((R, K), -1, np.int32)
    if stride:
        for r in range(R):
            slots[r] = rng.permutation(dbs)[:K]
    else:
        perm = rng.permutation(dbs)
        cnt = 0
        for r in range(R):
            for k in range(K):
                if miss[r, k]:
                    slots[r, k] = perm[cnt]
                    cnt += 1
    topk[rng.random((R, K)) < 0.01] = -1  # invalid entries are skipped even when flagged
    return topk, miss, slots


def run_gather(N, S, injective, stride, fused, block_dim=1, num_real=None, R=6, K=96, ctx=4096, dbs=1024,
               layers=3, layer=1, seed=0, segs_on_host=False, row_bytes=RB):
    import torch
    mod = kv()
    rng = np.random.default_rng(seed)
    layer_rows = R * ctx
    plsr = oracle.per_layer_seg_rows_injective(layer_rows, S, N) if (injective and S) else \
        oracle.per_layer_seg_rows(layer_rows, N)
    seg_bytes = layers * plsr * row_bytes
    segs_h = [rng.integers(0, 256, seg_bytes, dtype=np.uint8) for _ in range(N)]
    if segs_on_host:
        addrs = [mod.segment_alloc(-1, seg_bytes) for _ in range(N)]
        for a, h in zip(addrs, segs_h):
            host_view(a, seg_bytes)[:] = h
        keep = addrs
    else:
        keep = [dev(h) for h in segs_h]
        addrs = [t.data_ptr() for t in keep]
    topk, miss, slots = make_batch(rng, R, K, ctx, dbs, 0.3, stride)
    req_pool = np.arange(R, dtype=np.int64)
    req_pool[1] = -1  # a request without a pool row is skipped
    host_base = (np.arange(R, dtype=np.int64) * ctx)
    hot_rows = (R * dbs) if stride else dbs
    hot_h = rng.integers(0, 256, hot_rows * row_bytes, dtype=np.uint8)
    hot_d = dev(hot_h)
    t_topk, t_pool, t_base, t_slots, t_miss = dev(topk), dev(req_pool), dev(host_base), dev(slots), dev(miss)
    nr = R if num_real is None else num_real
    t_nr = dev(np.array([nr], np.int32))
    status = mod.alloc_status(8 * N)
    off = layer * plsr
    common = (off, plsr, row_bytes, t_topk.data_ptr(), t_pool.data_ptr(), t_base.data_ptr(), t_slots.data_ptr(),
              t_miss.data_ptr(), t_nr.data_ptr(), hot_d.data_ptr(), K, R, S)
    if fused:
        mod.import_multi(addrs, *common, status, 0, block_dim, hot_req_stride_rows=dbs if stride else 0,
                         injective=injective)
    else:
        for s in range(N):
            mod.import_seg(0, addrs[s], *common, N, s, status, 0, block_dim,
                           hot_req_stride_rows=dbs if stride else 0, injective=injective)
    for s in range(N):
        for b in range(block_dim):
            assert mod.poll_status(status + s * 64 + b * 8, 10_000_000) == 0
    torch.cuda.synchronize()
    exp = hot_h.copy()
    for s in range(N):
        oracle.gather_rows(segs_h[s], off, row_bytes, topk, req_pool, host_base, slots, miss, nr, exp, K, R, S, N, s,
                           dbs if stride else 0, injective)
    got = host(hot_d)
    np.testing.assert_array_equal(got, exp)
    if segs_on_host:
        for a in addrs:
            mod.segment_free(a)
    return int(((miss != 0) & (topk >= 0)).sum())


@pytest.mark.parametrize("N,S,injective", [(1, 1, False), (2, 1, False), (3, 1, False), (8, 1, False),
                                           (8, 16, False), (4, 64, False), (8, 16, True), (3, 64, True),
                                           (1, 0, False)])
@pytest.mark.parametrize("fused", [False, True])
def test_gather_parity(N, S, injective, fused):
    assert run_gather(N, S, injective, stride=True, fused=fused) > 0


def test_gather_shared_hot_buffer_reference_layout():
    run_gather(2, 1, False, stride=False, fused=False)


@pytest.mark.parametrize("block_dim", [1, 3, 8])
def test_gather_status_words(block_dim):
    run_gather(2, 1, False, stride=True, fused=True, block_dim=block_dim)


def test_gather_num_real_padding():
    run_gather(2, 1, False, stride=True, fused=True, num_real=3)
    run_gather(2, 1, False, stride=True, fused=True, num_real=0)


def test_gather_from_pinned_host_segments():
    run_gather(2, 1, False, stride=True, fused=True, segs_on_host=True)


@pytest.mark.parametrize("row_bytes", [1100, 1150, 136, 128])
def test_gather_odd_row_sizes(row_bytes):
    run_gather(2, 1, False, stride=True, fused=True, row_bytes=row_bytes, K=40, ctx=512, dbs=256)


def test_gather_large_c2_shape():
    """One layer at the DSA shape (64 x 2048 positions, 20% miss) on a local segment."""
    run_gather(1, 1, False, stride=True, fused=True, R=64, K=2048, ctx=8192, dbs=4096, layers=1, layer=0)


def _gather_args(mod, R=2, K=16, ctx=64, plsr=None, N=1, seg=None):
    topk = np.tile(np.arange(K, dtype=np.int32), (R, 1))
    miss = np.ones((R, K), np.int8)
    slots = np.tile(np.arange(K, dtype=np.int32), (R, 1))
    t = [dev(topk), dev(np.arange(R, dtype=np.int64)), dev(np.arange(R, dtype=np.int64) * ctx), dev(slots),
         dev(miss), dev(np.array([R], np.int32))]
    hot = dev(np.zeros(R * K * RB, np.uint8))
    return t, hot


def test_gather_null_segment_reports_init_band():
    mod = kv()
    t, hot = _gather_args(mod)
    status = mod.alloc_status(8)
    mod.import_seg(0, 0, 0, 128, RB, *[x.data_ptr() for x in t], hot.data_ptr(), 16, 2, 1, 1, 0, status, 0, 1)
    assert mod.poll_status(status, 10_000_000) == 0x101
    assert int(host(hot).max()) == 0  # nothing touched


def test_gather_row_outside_segment_reports_row_band():
    mod = kv()
    t, hot = _gather_args(mod)
    seg = dev(np.zeros(4 * RB, np.uint8))
    status = mod.alloc_status(8)
    # plsr = 4 rows but requests span 2 x 64 rows: rows past the segment are refused
    mod.import_seg(0, seg.data_ptr(), 0, 4, RB, *[x.data_ptr() for x in t], hot.data_ptr(), 16, 2, 1, 1, 0, status,
                   0, 1)
    rc = mod.poll_status(status, 10_000_000)
    assert rc & 0xFF00 == 0x200 and rc >> 16 == 1


def test_poll_timeout_on_never_launched_slot():
    mod = kv()
    status = mod.alloc_status(4)
    assert mod.poll_status(status + 64, 2000) == -0x2000


def test_poll_device_memory_status_word():
    import torch
    mod = kv()
    word = torch.zeros(8, dtype=torch.int64, device="cuda")
    word[0] = (1 << 32) | 0x1234
    torch.cuda.synchronize()
    assert mod.poll_status(word.data_ptr(), 1000) == 0x1234


def test_import_validation():
    mod = kv()
    with pytest.raises(RuntimeError, match="<= 8"):
        mod.import_seg(0, 8, 0, 1, RB, 8, 8, 8, 8, 8, 8, 8, 1, 1, 1, 1, 0, 0, 0, 9)
    with pytest.raises(RuntimeError, match="my_node"):
        mod.import_seg(0, 8, 0, 1, RB, 8, 8, 8, 8, 8, 8, 8, 1, 1, 1, 2, 2, 0, 0, 1)
    with pytest.raises(RuntimeError, match="address is 0"):
        mod.import_seg(0, 8, 0, 1, RB, 0, 8, 8, 8, 8, 8, 8, 1, 1, 1, 1, 0, 0, 0, 1)


# ---- export --------------------------------------------------------------------------

def run_export(N, S, injective, row_lo, row_cnt, layer_rows=600, layers=3, block_dim=1, on_host=False, seed=1,
               row_bytes=RB):
    import torch
    mod = kv()
    rng = np.random.default_rng(seed)
    src_h = rng.integers(0, 256, layers * layer_rows * row_bytes, dtype=np.uint8)
    src_d = dev(src_h)
    plsr = oracle.per_layer_seg_rows_injective(layer_rows, S, N) if (injective and S) else \
        oracle.per_layer_seg_rows(layer_rows, N)
    seg_bytes = layers * plsr * row_bytes
    init = [rng.integers(0, 256, seg_bytes, dtype=np.uint8) for _ in range(N)]
    if on_host:
        addrs = [mod.segment_alloc(-1, seg_bytes) for _ in range(N)]
        for a, h in zip(addrs, init):
            host_view(a, seg_bytes)[:] = h
        keep = None
    else:
        keep = [dev(h) for h in init]
        addrs = [x.data_ptr() for x in keep]
    status = mod.alloc_status(8 * N)
    for s in range(N):
        mod.export_seg_alllayer(0, addrs[s], plsr, row_bytes, row_lo, row_cnt, layers, src_d.data_ptr(),
                                layer_rows * row_bytes, S, N, s, status, 0, block_dim, injective=injective)
    for s in range(N):
        for b in range(block_dim):
            assert mod.poll_status(status + s * 64 + b * 8, 10_000_000) == 0
    torch.cuda.synchronize()
    for s in range(N):
        exp = init[s].copy()
        oracle.export_alllayer(exp, plsr, row_bytes, row_lo, row_cnt, layers, src_h, layer_rows * row_bytes, S, N,
                               s, injective)
        got = host_view(addrs[s], seg_bytes).copy() if on_host else host(keep[s])
        np.testing.assert_array_equal(got, exp)
    if on_host:
        for a in addrs:
            mod.segment_free(a)


@pytest.mark.parametrize("N,S,injective", [(1, 1, False), (2, 1, False), (3, 1, False), (8, 1, False),
                                           (2, 16, False), (3, 64, False), (8, 16, True), (3, 64, True),
                                           (1, 0, False)])
@pytest.mark.parametrize("lo,cnt", [(0, 600), (37, 401), (5, 1)])
def test_export_parity(N, S, injective, lo, cnt):
    run_export(N, S, injective, lo, cnt)


def test_export_to_pinned_host_segments():
    run_export(2, 64, False, 0, 600, on_host=True)
    run_export(2, 1, False, 3, 500, on_host=True, block_dim=4)


def test_export_odd_row_size():
    run_export(2, 1, False, 0, 300, layer_rows=300, row_bytes=1100)


def test_export_then_gather_round_trip():
    """Injective (or S=1) layout: export every row, gather all of them back."""
    import torch
    mod = kv()
    R, ctx, L, N, S = 4, 512, 2, 3, 16
    layer_rows = R * ctx
    rng = np.random.default_rng(9)
    src = dev(rng.integers(0, 256, L * layer_rows * RB, dtype=np.uint8))
    plsr = oracle.per_layer_seg_rows_injective(layer_rows, S, N)
    segs = [torch.zeros(L * plsr * RB, dtype=torch.uint8, device="cuda") for _ in range(N)]
    st = mod.alloc_status(8 * N)
    for s in range(N):
        mod.export_seg_alllayer(0, segs[s].data_ptr(), plsr, RB, 0, layer_rows, L, src.data_ptr(), layer_rows * RB,
                                S, N, s, st, 0, 1, injective=True)
    K = ctx
    topk = np.tile(np.arange(ctx, dtype=np.int32), (R, 1))
    t = [dev(topk), dev(np.arange(R, dtype=np.int64)), dev(np.arange(R, dtype=np.int64) * ctx), dev(topk),
         dev(np.ones((R, K), np.int8)), dev(np.array([R], np.int32))]
    for layer in range(L):
        hot = torch.zeros(R * ctx * RB, dtype=torch.uint8, device="cuda")
        mod.import_multi([x.data_ptr() for x in segs], layer * plsr, plsr, RB, *[x.data_ptr() for x in t],
                         hot.data_ptr(), K, R, S, st + 64 * N, 0, 1, hot_req_stride_rows=ctx, injective=True)
        for s in range(N):
            assert mod.poll_status(st + 64 * N + 64 * s, 10_000_000) == 0
        want = src.view(L, layer_rows * RB)[layer]
        assert torch.equal(hot, want)


def test_export_null_segment():
    mod = kv()
    src = dev(np.zeros(10 * RB, np.uint8))
    st = mod.alloc_status(8)
    mod.export_seg_alllayer(0, 0, 10, RB, 0, 10, 1, src.data_ptr(), 10 * RB, 1, 1, 0, st, 0, 1)
    assert mod.poll_status(st, 10_000_000) == 0x101
