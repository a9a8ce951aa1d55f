"""The no-allocation gather entry point, kvops_import_multi_noalloc, through the C ABI.

It exists for callers that cannot allocate device memory: an inference engine whose HBM
is owned by its own allocator or fixed budget, or a decode loop that cannot pay for
cudaMalloc/cudaFree. Its scratch is a static device array shared by all calls, so the
test checks two calls in a row against the regular kvops_import_multi, byte for byte, on
the hot buffer and on every status word, and both against the C restatement of the gather.
A second test runs it first thing in a fresh process (before any other entry point has set
the device up) and checks that the device's free memory does not move. This file is
collected last on purpose."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

RB = 1152


class Opts(ctypes.Structure):
    """KvopsRowOpts (include/kvops_b200.h)."""
    _fields_ = [("hot_req_stride_rows", ctypes.c_uint64), ("injective", ctypes.c_uint32),
                ("step_path", ctypes.c_uint32), ("err_word", ctypes.c_uint64), ("copy_wait_polls", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32)]


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
    opts = Opts(dbs, 0, 0, 0, 0, 0)
    segs_h = [s.cpu().numpy() for s in segs]
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
        exp = np.zeros(R * dbs * RB, np.uint8)
        n = oracle.gather_all(segs_h, layer * plsr, RB, topk.cpu().numpy(), pool.cpu().numpy(), base.cpu().numpy(),
                              slots.cpu().numpy(), miss.cpu().numpy(), R, exp, K, R, 1, hot_req_stride_rows=dbs)
        assert n == int(miss.sum())
        np.testing.assert_array_equal(outs[1], exp)


def test_noalloc_rejects_bad_arguments():
    lib = _lib()
    u64 = ctypes.c_uint64
    seg = (u64 * 1)(8)
    opts = Opts(0, 0, 0, 0, 0, 0)
    rc = lib.kvops_import_multi_noalloc(1, seg, 0, 1, RB, 8, 8, 8, 8, 8, 8, 8, 1, 1, 1, 0, 0, 9, ctypes.byref(opts))
    assert rc == 3 and b"<= 8" in lib.kvops_last_error()


_FRESH = r"""
import ctypes, sys
import numpy as np
from cuda.bindings import runtime as rt
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
import kv_offload_proto_b200 as kp
import oracle
from test_zz_no_alloc import Opts, RB


def ck(ret):
    assert ret[0] == rt.cudaError_t.cudaSuccess, ret
    return ret[1] if len(ret) == 2 else ret[1:]


lib = kp.load_library()  # registers the library's kernels; loaded into the context at creation
u64, u32 = ctypes.c_uint64, ctypes.c_uint32
sig = [u32, ctypes.POINTER(u64), u32, u32, u32] + [u64] * 7 + [u32, u32, u32, u64, u64, u32, ctypes.POINTER(Opts)]
lib.kvops_import_multi_noalloc.argtypes = sig
lib.kvops_poll_status.argtypes = [u64, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64)]
R, K, ctx, dbs = 4, 128, 1024, 256
rng = np.random.default_rng(3)
seg_h = rng.integers(0, 256, R * ctx * RB, dtype=np.uint8)
topk = np.stack([rng.choice(ctx, K, replace=False) for _ in range(R)]).astype(np.int32)
miss = (rng.random((R, K)) < 0.5).astype(np.int8)
slots = np.stack([rng.permutation(dbs)[:K] for _ in range(R)]).astype(np.int32)
pool, base = np.arange(R, dtype=np.int64), np.arange(R, dtype=np.int64) * ctx
ck(rt.cudaSetDevice(0))
ck(rt.cudaFree(0))


def d(a):  # device copy of a host array (inputs are the caller's, allocated before the measurement)
    a = np.ascontiguousarray(a)
    p = ck(rt.cudaMalloc(max(a.nbytes, 8)))
    ck(rt.cudaMemcpy(p, a.ctypes.data, a.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice))
    return p


seg, t_topk, t_miss, t_slots, t_pool, t_base = d(seg_h), d(topk), d(miss), d(slots), d(pool), d(base)
t_nr = d(np.array([R], np.int32))
hot = d(np.zeros(R * dbs * RB, np.uint8))
status = d(np.zeros(64, np.int64))  # device-memory status words
seg_arr = (u64 * 1)(seg)
opts = Opts(dbs, 0, 0, 0, 0, 0)
args = (1, seg_arr, 0, R * ctx, RB, t_topk, t_pool, t_base, t_slots, t_miss, t_nr, hot, K, R, 1, status, 0, 1,
        ctypes.byref(opts))
assert lib.kvops_import_multi_noalloc(*args) == 1, "must require kvops_init"
assert b"not inited" in lib.kvops_last_error()
assert lib.kvops_init(0, b"", b"") == 0, lib.kvops_last_error()
ck(rt.cudaDeviceSynchronize())
free0 = ck(rt.cudaMemGetInfo())[0]
for call in range(2):
    assert lib.kvops_import_multi_noalloc(*args) == 0, lib.kvops_last_error()
    out = ctypes.c_int64()
    assert lib.kvops_poll_status(status, 10_000_000, ctypes.byref(out)) == 0 and out.value == 0
ck(rt.cudaDeviceSynchronize())
free1 = ck(rt.cudaMemGetInfo())[0]
assert free1 == free0, ("device memory moved", free0, free1)
got = np.zeros(R * dbs * RB, np.uint8)
ck(rt.cudaMemcpy(got.ctypes.data, hot, got.nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost))
exp = np.zeros(R * dbs * RB, np.uint8)
oracle.gather_all([seg_h], 0, RB, topk, pool, base, slots, miss, R, exp, K, R, 1, hot_req_stride_rows=dbs)
np.testing.assert_array_equal(got, exp)
print("fresh-process no-alloc ok", free0 - free1)
"""


def test_noalloc_first_call_in_fresh_process_allocates_nothing():
    """Run in a child process (no torch there) so that this entry point is the first to touch
    the device after kvops_init (no ticket ring or scratch set up by earlier tests). Modules
    load eagerly there, so the library's code and static array are resident before the
    measurement starts and any allocation the call made would show in cudaMemGetInfo."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    r = subprocess.run([sys.executable, "-c", _FRESH, root], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fresh-process no-alloc ok 0" in r.stdout
