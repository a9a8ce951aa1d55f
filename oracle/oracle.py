"""ctypes front end of the C restatement in ``kvoracle.c`` (TEST INFRASTRUCTURE ONLY).

Layouts match the reference's state tensors (xds/xds_offload.py:43-53):
tokens int32[L, pool, padded], visited uint8[L, pool, vis_stride],
ht uint16[L, pool, ht_size], hand int32[L, pool, 16].
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libkvoracle.so")
_REF_PATH = os.path.join(_HERE, "_ref", "libkv_layout_ref.so")
_lib = None

__all__ = [
    "lib", "ht_size", "align", "hash32", "node_of", "seg_row_of", "seg_row_injective", "per_layer_seg_rows",
    "per_layer_seg_rows_injective", "seg_offset", "SieveState", "sieve_update", "gather_rows", "gather_all",
    "export_alllayer", "scatter_rows", "ref_layout_lib", "build",
]


def build(ref=False):
    """Compile the checker (and, with ref=True, the reference's layout header)."""
    cmd = ["make", "-s", "-C", _HERE, "all"] + (["ref"] if ref else [])
    subprocess.check_call(cmd)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
                os.path.join(_HERE, "kvoracle.c")):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i32, u32, i64, u64 = ctypes.c_int32, ctypes.c_uint32, ctypes.c_int64, ctypes.c_uint64
        L.ko_hash.argtypes = [i32]
        L.ko_hash.restype = u32
        L.ko_ht_size.argtypes = [i64, i64]
        L.ko_ht_size.restype = i64
        L.ko_sieve_update.argtypes = [P] * 10 + [i32] * 9
        L.ko_sieve_update.restype = ctypes.c_int
        L.ko_sieve_ht_init.argtypes = [P, P] + [i32] * 8
        L.ko_sieve_ht_init.restype = ctypes.c_int
        for f in (L.ko_node_of, L.ko_seg_row, L.ko_seg_row_injective):
            f.argtypes = [u32, u32, u32]
            f.restype = u32
        L.ko_gather_rows.argtypes = [P, u32, u32, P, P, P, P, P, i32, P, u32, u32, u32, u32, u32, i64,
                                     ctypes.c_int]
        L.ko_gather_rows.restype = i64
        L.ko_gather_all.argtypes = [P, u32, u32, P, P, P, P, P, i32, P, u32, u32, u32, u32, i64, ctypes.c_int,
                                    i32]
        L.ko_gather_all.restype = i64
        L.ko_scatter_rows.argtypes = [P, u32, u32, P, P, P, P, P, i32, P, u32, u32, u32, u32, u32, i64,
                                      ctypes.c_int]
        L.ko_scatter_rows.restype = i64
        L.ko_export_alllayer.argtypes = [P, u32, u32, u32, u32, u32, P, u64, u32, u32, u32, ctypes.c_int]
        L.ko_export_alllayer.restype = i64
        _lib = L
    return _lib


def ref_layout_lib():
    """The reference's common/kv_layout.h compiled into oracle/_ref (None if not built)."""
    if not os.path.exists(_REF_PATH):
        return None
    L = ctypes.CDLL(_REF_PATH)
    u32, u64 = ctypes.c_uint32, ctypes.c_uint64
    L.ref_per_layer_seg_rows.argtypes = [u32, u32]
    L.ref_per_layer_seg_rows.restype = u32
    for f in (L.ref_node_of, L.ref_seg_row_of):
        f.argtypes = [u32, u32, u32]
        f.restype = u32
    L.ref_seg_offset.argtypes = [u32, u32, u32, u32, u32, u32]
    L.ref_seg_offset.restype = u64
    L.ref_validate.argtypes = [u32] * 6
    L.ref_validate.restype = ctypes.c_int
    return L


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def ht_size(padded, top_k):
    return int(lib().ko_ht_size(padded, top_k))


def align(v, a):
    return (v + a - 1) // a * a


def hash32(token):
    return int(lib().ko_hash(int(token)))


# Stripe map (kvc_common.h:81-89; test/kv_layout_ref.py:7-24) restated in Python.
def per_layer_seg_rows(layer_rows, node_num):
    return (layer_rows + node_num - 1) // node_num


def per_layer_seg_rows_injective(layer_rows, stripe, node_num):
    stripes = (layer_rows + stripe - 1) // stripe
    return (stripes + node_num - 1) // node_num * stripe


def node_of(row, stripe, node_num):
    return 0 if stripe == 0 else (row // stripe) % node_num


def seg_row_of(row, stripe, node_num):
    return row if stripe == 0 else (row // stripe) // node_num


def seg_row_injective(row, stripe, node_num):
    return row if stripe == 0 else ((row // stripe) // node_num) * stripe + row % stripe


def seg_offset(layer, row, stripe, node_num, plsr, row_bytes):
    return (layer * plsr + seg_row_of(row, stripe, node_num)) * row_bytes


class SieveState:
    """Per-layer SIEVE state with the reference's tensor layout, on the host."""

    def __init__(self, layer_num, pool_size, dbs, top_k):
        self.layer_num, self.pool_size, self.dbs, self.top_k = layer_num, pool_size, dbs, top_k
        self.padded = align(dbs, 16)
        self.vis_stride = align((self.padded + 7) // 8, 64)
        self.ht_size = ht_size(self.padded, top_k)
        L, p = layer_num, pool_size
        self.tokens = np.full((L, p, self.padded), -1, dtype=np.int32)
        self.visited = np.zeros((L, p, self.vis_stride), dtype=np.uint8)
        self.ht = np.zeros((L, p, self.ht_size), dtype=np.uint16)
        self.hand = np.zeros((L, p, 16), dtype=np.int32)
        self.prefill_lens = np.zeros(p, dtype=np.int32)

    def admit(self, req_pool_idx, prefill_len):
        """Identity admission (xds/xds_offload.py:56-77): slot s holds token s."""
        n = min(prefill_len, self.dbs)
        self.tokens[:, req_pool_idx, :n] = np.arange(n, dtype=np.int32)
        self.visited[:, req_pool_idx, :] = 0
        self.hand[:, req_pool_idx, :] = 0
        self.prefill_lens[req_pool_idx] = prefill_len
        self.ht_init(req_pool_idx, 1, self.layer_num)

    def ht_init(self, req_start, num_reqs, nblocks):
        rc = lib().ko_sieve_ht_init(_p(self.tokens), _p(self.ht), req_start, num_reqs, self.layer_num,
                                    self.pool_size, self.dbs, self.padded, self.ht_size, nblocks)
        assert rc == 0

    def update(self, layer, topk, req_pool, seq_lens, num_real=None, nthreads=1):
        """One sieve_update on `layer`; returns (slots int32, is_miss int8) [max_num_reqs, top_k]."""
        topk = np.ascontiguousarray(topk, dtype=np.int32)
        m = topk.shape[0]
        req_pool = np.ascontiguousarray(req_pool, dtype=np.int64)
        seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
        num_real = m if num_real is None else num_real
        slots = np.empty((m, self.top_k), dtype=np.int32)
        miss = np.empty((m, self.top_k), dtype=np.int8)
        tok, vis, ht, hand = self.tokens[layer], self.visited[layer], self.ht[layer], self.hand[layer]
        rc = lib().ko_sieve_update(_p(topk), _p(req_pool), _p(seq_lens), _p(self.prefill_lens), _p(tok),
                                   _p(vis), _p(ht), _p(hand), _p(slots), _p(miss), num_real, self.top_k,
                                   self.dbs, self.padded, self.vis_stride, m, self.pool_size, self.ht_size,
                                   nthreads)
        assert rc == 0
        return slots, miss

    def copy(self):
        c = SieveState.__new__(SieveState)
        c.__dict__.update(self.__dict__)
        for k in ("tokens", "visited", "ht", "hand", "prefill_lens"):
            setattr(c, k, getattr(self, k).copy())
        return c


def sieve_update(topk, req_pool, seq_lens, prefill_lens, tokens, visited, ht, hand, num_real, top_k, dbs,
                 padded, vis_stride, pool_size, ht_sz, nthreads=1):
    """Flat form on caller-owned layer slices (all numpy, modified in place)."""
    m = topk.shape[0]
    slots = np.empty((m, top_k), dtype=np.int32)
    miss = np.empty((m, top_k), dtype=np.int8)
    rc = lib().ko_sieve_update(_p(topk), _p(req_pool), _p(seq_lens), _p(prefill_lens), _p(tokens),
                               _p(visited), _p(ht), _p(hand), _p(slots), _p(miss), num_real, top_k, dbs, padded,
                               vis_stride, m, pool_size, ht_sz, nthreads)
    assert rc == 0
    return slots, miss


def gather_rows(seg, layer_offset_rows, row_bytes, topk, req_pool, host_base, slots, is_miss, num_real, hot,
                top_k, max_num_reqs, stripe, nodes, my_node, hot_req_stride_rows=0, injective=False):
    """One import_seg launch on host byte arrays `seg` and `hot` (hot modified in place)."""
    return int(lib().ko_gather_rows(_p(seg), layer_offset_rows, row_bytes, _p(topk), _p(req_pool),
                                    _p(host_base), _p(slots), _p(is_miss), num_real, _p(hot), top_k,
                                    max_num_reqs, stripe, nodes, my_node, hot_req_stride_rows, int(injective)))


def scatter_rows(seg, layer_offset_rows, row_bytes, topk, req_pool, host_base, slots, export_flags, num_real, hot,
                 top_k, max_num_reqs, stripe, nodes, my_node, hot_req_stride_rows=0, injective=False):
    """One export_seg (kvc_scatter_rows) launch on host byte arrays (seg modified in place)."""
    return int(lib().ko_scatter_rows(_p(seg), layer_offset_rows, row_bytes, _p(topk), _p(req_pool),
                                     _p(host_base), _p(slots), _p(export_flags), num_real, _p(hot), top_k,
                                     max_num_reqs, stripe, nodes, my_node, hot_req_stride_rows, int(injective)))


def gather_all(segs, layer_offset_rows, row_bytes, topk, req_pool, host_base, slots, is_miss, num_real, hot,
               top_k, max_num_reqs, stripe, hot_req_stride_rows=0, injective=False, nthreads=1):
    """All N segments in one threaded pass (the CPU baseline gather)."""
    arr = (ctypes.c_void_p * len(segs))(*[s.ctypes.data for s in segs])
    return int(lib().ko_gather_all(arr, layer_offset_rows, row_bytes, _p(topk), _p(req_pool), _p(host_base),
                                   _p(slots), _p(is_miss), num_real, _p(hot), top_k, max_num_reqs, stripe,
                                   len(segs), hot_req_stride_rows, int(injective), nthreads))


def export_alllayer(seg, plsr, row_bytes, row_lo, row_cnt, layer_num, src, src_layer_stride, stripe, nodes,
                    my_node, injective=False):
    """One export_seg_alllayer launch on host byte arrays (seg modified in place)."""
    return int(lib().ko_export_alllayer(_p(seg), plsr, row_bytes, row_lo, row_cnt, layer_num, _p(src),
                                        src_layer_stride, stripe, nodes, my_node, int(injective)))
