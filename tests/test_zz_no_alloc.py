"""The no-allocation gather entry point, kvops_import_multi_noalloc, through the C ABI.

It exists for callers that cannot allocate device memory: an inference engine whose HBM
is owned by its own allocator or fixed budget, or a decode loop that cannot pay for
cudaMalloc/cudaFree. Its scratch is a static device array shared by all calls, so the
test checks two calls in a row against the regular kvops_import_multi, byte for byte, on
the hot buffer and on every status word. This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RB = 1152


class Opts(ctypes.Structure):
    _fields_ = [("hot_req_stride_rows", ctypes.c_uint64), ("injective", ctypes.c_uint32),
                ("step_path", ctypes.c_uint32)]


def _lib():
    import kv_offload_proto_b200 as kp
    lib = kp.load_library()
    u64, u32 = ctypes.c_uint64, ctypes.c_uint32
    sig = [u32, ctypes.POINTER(u64), u32, u32, u32] + [u64] * 7 + [u32, u32, u32, u64, u64, u32, ctypes.POINTER(Opts)]
    lib.kvops_import_multi.argtypes = sig
    lib.kvops_import_multi_noalloc.argtypes = sig
    lib.kvops_alloc_status.argtypes = [ctypes.c_int, ctypes.POINTER(u64)]
    lib.kvops_poll_status.argtypes = [u64, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64)]
    rc = lib.kvops_init(0, b"", b"")
    assert rc in (0, 2), lib.kvops_last_error()  # 2: already initialised by earlier tests
    return lib


def _batch(torch, seed, R, K, ctx, dbs, nodes):
    g = torch.Generator(device="cuda").manual_seed(seed)
    topk = torch.argsort(torch.rand((R, ctx), generator=g, device="cuda"), dim=1)[:, :K].to(torch.int32).contiguous()
    miss = (torch.rand((R, K), generator=g, device="cuda") < 0.3).to(torch.int8)
    slots = torch.argsort(torch.rand((R, dbs), generator=g, device="cuda"), dim=1)[:, :K].to(torch.int32).contiguous()
    return topk, miss, slots


def test_noalloc_gather_matches_regular_two_calls():
    import torch
    lib = _lib()
    u64, u32 = ctypes.c_uint64, ctypes.c_uint32
    R, K, ctx, dbs, N, L = 8, 256, 2048, 512, 3, 2
    layer_rows = R * ctx
    plsr = (layer_rows + N - 1) // N
    segs = [torch.randint(0, 256, (L * plsr * RB,), dtype=torch.uint8, device="cuda") for _ in range(N)]
    seg_arr = (u64 * N)(*[s.data_ptr() for s in segs])
    pool = torch.arange(R, dtype=torch.int64, device="cuda")
    base = pool * ctx
    num_real = torch.tensor([R], dtype=torch.int32, device="cuda")
    status = u64()
    assert lib.kvops_alloc_status(8 * N, ctypes.byref(status)) == 0
    opts = Opts(dbs, 0, 0)
    for call, layer in enumerate((1, 0)):  # two calls in a row share the static scratch
        topk, miss, slots = _batch(torch, 10 + call, R, K, ctx, dbs, N)
        outs, words = [], []
        for fn, page in ((lib.kvops_import_multi, 0), (lib.kvops_import_multi_noalloc, N)):
            hot = torch.zeros(R * dbs * RB, dtype=torch.uint8, device="cuda")
            st = status.value + page * 64
            rc = fn(N, seg_arr, layer * plsr, plsr, RB, topk.data_ptr(), pool.data_ptr(), base.data_ptr(),
                    slots.data_ptr(), miss.data_ptr(), num_real.data_ptr(), hot.data_ptr(), K, R, 1, st, 0, 4,
                    ctypes.byref(opts))
            assert rc == 0, lib.kvops_last_error()
            w = []
            for s in range(N):
                for b in range(4):
                    out = ctypes.c_int64()
                    assert lib.kvops_poll_status(st + s * 64 + b * 8, 10_000_000, ctypes.byref(out)) == 0
                    w.append(out.value)
            torch.cuda.synchronize()
            outs.append(hot.cpu().numpy())
            words.append(w)
        assert words[0] == words[1] == [0] * (4 * N)
        np.testing.assert_array_equal(outs[1], outs[0])
        assert int(miss.sum()) > 0 and outs[0].any()


def test_noalloc_rejects_bad_arguments():
    lib = _lib()
    u64 = ctypes.c_uint64
    seg = (u64 * 1)(8)
    opts = Opts(0, 0, 0)
    rc = lib.kvops_import_multi_noalloc(1, seg, 0, 1, RB, 8, 8, 8, 8, 8, 8, 8, 1, 1, 1, 0, 0, 9, ctypes.byref(opts))
    assert rc == 3 and b"<= 8" in lib.kvops_last_error()
