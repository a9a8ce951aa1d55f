"""GPU parity of the single-layer indexed export (kvops_export_seg, kvc_scatter_rows: the
gather's rules with hot rows -> segment rows) against the C restatement, its errCodes, and the
round trip export -> import."""
import numpy as np
import pytest

import oracle
from gpu_util import dev, host, kv

pytestmark = pytest.mark.gpu
RB = 1152


def make_inputs(rng, R, K, ctx, dbs, stride):
    """Export positions with pairwise distinct pool rows (so no two writes race)."""
    topk = np.stack([rng.choice(ctx, K, replace=False) for _ in range(R)]).astype(np.int32)
    flags = (rng.random((R, K)) < 0.4).astype(np.int8)
    slots = np.stack([rng.permutation(dbs)[:K] for _ in range(R)]).astype(np.int32)
    topk[rng.random((R, K)) < 0.02] = -1
    return topk, flags, slots


@pytest.mark.parametrize("N,S,injective", [(1, 1, False), (3, 2, True), (2, 0, False), (4, 1, False)])
def test_export_seg_parity(N, S, injective):
    import torch
    mod = kv()
    rng = np.random.default_rng(N * 10 + S)
    R, K, ctx, dbs, layers, layer = 5, 96, 2048, 512, 2, 1
    layer_rows = R * ctx
    if S == 0:
        N = 1
    plsr = oracle.per_layer_seg_rows_injective(layer_rows, S, N) if (injective and S) else \
        oracle.per_layer_seg_rows(layer_rows, N)
    segs_h = [rng.integers(0, 256, layers * plsr * RB, dtype=np.uint8) for _ in range(N)]
    segs = [dev(h) for h in segs_h]
    topk, flags, slots = make_inputs(rng, R, K, ctx, dbs, True)
    req_pool = np.arange(R, dtype=np.int64)
    req_pool[2] = -1
    base = np.arange(R, dtype=np.int64) * ctx
    hot_h = rng.integers(0, 256, R * dbs * RB, dtype=np.uint8)
    hot = dev(hot_h)
    t = [dev(a) for a in (topk, req_pool, base, slots, flags, np.array([R - 1], np.int32))]
    status = mod.alloc_status(8 * N)
    for s in range(N):
        mod.export_seg(0, segs[s].data_ptr(), layer * plsr, plsr, RB, *[x.data_ptr() for x in t], hot.data_ptr(), K,
                       R, S, N, s, status, 0, 1, hot_req_stride_rows=dbs, injective=injective)
    for s in range(N):
        assert mod.poll_status(status + s * 64, 10_000_000) == 0
    torch.cuda.synchronize()
    n = 0
    for s in range(N):
        n += oracle.scatter_rows(segs_h[s], layer * plsr, RB, topk, req_pool, base, slots, flags, R - 1, hot_h, K, R,
                                 S, N, s, dbs, injective)
        np.testing.assert_array_equal(host(segs[s]), segs_h[s])
    assert n > 0


def test_export_then_import_round_trip():
    import torch
    mod = kv()
    rng = np.random.default_rng(7)
    R, K, ctx, dbs = 4, 128, 1024, 256
    plsr = R * ctx
    seg = dev(np.zeros(plsr * RB, np.uint8))
    topk, flags, slots = make_inputs(rng, R, K, ctx, dbs, True)
    t = [dev(a) for a in (topk, np.arange(R, dtype=np.int64), np.arange(R, dtype=np.int64) * ctx, slots, flags,
                          np.array([R], np.int32))]
    src = dev(rng.integers(0, 256, R * dbs * RB, dtype=np.uint8))
    back = dev(np.zeros(R * dbs * RB, np.uint8))
    status = mod.alloc_status(8)
    mod.export_seg(0, seg.data_ptr(), 0, plsr, RB, *[x.data_ptr() for x in t], src.data_ptr(), K, R, 1, 1, 0, status,
                   0, 1, hot_req_stride_rows=dbs)
    assert mod.poll_status(status, 10_000_000) == 0
    mod.import_seg(0, seg.data_ptr(), 0, plsr, RB, *[x.data_ptr() for x in t], back.data_ptr(), K, R, 1, 1, 0, status,
                   0, 1, hot_req_stride_rows=dbs)
    assert mod.poll_status(status, 10_000_000) == 0
    torch.cuda.synchronize()
    b, sh = host(back).reshape(R, dbs, RB), host(src).reshape(R, dbs, RB)
    for r in range(R):
        for k in range(K):
            if flags[r, k] and topk[r, k] >= 0:
                np.testing.assert_array_equal(b[r, slots[r, k]], sh[r, slots[r, k]])


def test_export_seg_error_bands_and_validation():
    import torch
    mod = kv()
    R, K = 2, 16
    topk = np.tile(np.arange(K, dtype=np.int32), (R, 1))
    t = [dev(a) for a in (topk, np.arange(R, dtype=np.int64), np.arange(R, dtype=np.int64) * 64,
                          np.tile(np.arange(K, dtype=np.int32), (R, 1)), np.ones((R, K), np.int8),
                          np.array([R], np.int32))]
    hot = dev(np.zeros(R * K * RB, np.uint8))
    status = mod.alloc_status(8)
    mod.export_seg(0, 0, 0, 128, RB, *[x.data_ptr() for x in t], hot.data_ptr(), K, R, 1, 1, 0, status, 0, 1)
    assert mod.poll_status(status, 10_000_000) == 0x101
    seg = dev(np.zeros(4 * RB, np.uint8))
    mod.export_seg(0, seg.data_ptr(), 0, 4, RB, *[x.data_ptr() for x in t], hot.data_ptr(), K, R, 1, 1, 0, status, 0,
                   1)
    rc = mod.poll_status(status, 10_000_000)
    assert rc & 0xFF00 == 0x200 and rc >> 16 == 1
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="export_seg my_node"):
        mod.export_seg(0, 1, 0, 4, RB, *[x.data_ptr() for x in t], hot.data_ptr(), K, R, 1, 1, 1, status, 0, 1)
    with pytest.raises(RuntimeError, match="export_seg blockDim"):
        mod.export_seg(0, 1, 0, 4, RB, *[x.data_ptr() for x in t], hot.data_ptr(), K, R, 1, 1, 0, status, 0, 9)
