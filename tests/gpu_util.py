"""Helpers for the -m gpu parity tests: one `_kvops` init per process, numpy <-> device
copies, and a device mirror of an oracle.SieveState driven through the C ABI."""
import ctypes

import numpy as np

_inited = False


def kv():
    """The `_kvops` module, initialised once on cuda:0 (re-init raises by contract)."""
    global _inited
    import torch
    import kv_offload_proto_b200 as kp
    mod = kp.install_kvops_ext()
    if not _inited:
        torch.cuda.init()
        try:
            mod.init(0, "")
        except RuntimeError as e:
            if "already inited" not in str(e):
                raise
        _inited = True
    return mod


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def host_view(addr, nbytes):
    """uint8 numpy view of pinned host memory at a UVA address."""
    return np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(addr))


class DeviceSieve:
    """Device copy of an oracle.SieveState; update() runs the CUDA sieve on one layer."""

    def __init__(self, st):
        import torch
        self.st = st
        self.tokens = dev(st.tokens)
        self.visited = dev(st.visited)
        self.ht = dev(st.ht.view(np.int16))
        self.hand = dev(st.hand)
        self.prefill = dev(st.prefill_lens)
        self.torch = torch

    def update(self, layer, topk, req_pool, seq_lens, num_real=None, block_dim=8):
        torch = self.torch
        st = self.st
        m = topk.shape[0]
        topk_d = dev(np.ascontiguousarray(topk, np.int32))
        rp = dev(np.asarray(req_pool, np.int64))
        sl = dev(np.asarray(seq_lens, np.int32))
        nr = dev(np.array([m if num_real is None else num_real], np.int32))
        slots = torch.full((m, st.top_k), 7777, dtype=torch.int32, device="cuda")
        miss = torch.full((m, st.top_k), 9, dtype=torch.int8, device="cuda")
        kv().sieve_update(topk_d.data_ptr(), rp.data_ptr(), sl.data_ptr(), self.prefill.data_ptr(),
                          self.tokens[layer].data_ptr(), self.visited[layer].data_ptr(), self.ht[layer].data_ptr(),
                          self.hand[layer].data_ptr(), slots.data_ptr(), miss.data_ptr(), nr.data_ptr(), st.top_k,
                          st.dbs, st.padded, st.vis_stride, m, st.pool_size, 0, block_dim)
        torch.cuda.synchronize()
        return host(slots), host(miss)

    def assert_state_equal(self, layer=None):
        st = self.st
        sel = slice(None) if layer is None else layer
        np.testing.assert_array_equal(host(self.tokens)[sel], st.tokens[sel])
        np.testing.assert_array_equal(host(self.visited)[sel], st.visited[sel])
        np.testing.assert_array_equal(host(self.ht).view(np.uint16)[sel], st.ht[sel])
        np.testing.assert_array_equal(host(self.hand)[sel][..., 0], st.hand[sel][..., 0])


def config_topk(rng, st, layer, reqs, top_k, miss_ratio, ext=0, invalid=0.0, dup=0.0):
    """BASELINE-style draw on the host from an oracle state: unique positions, hits from the
    current residents of each request's token row, misses from non-resident prefill positions."""
    out = np.empty((len(reqs), top_k), np.int32)
    for b, r in enumerate(reqs):
        r = int(r)
        prefill = int(st.prefill_lens[r]) if 0 <= r < st.pool_size else 1000
        if 0 <= r < st.pool_size:
            tok = st.tokens[layer, r, :st.dbs]
            res = np.unique(tok[(tok >= 0) & (tok < prefill)])
        else:
            res = np.empty(0, np.int64)
        nonres = np.setdiff1d(np.arange(prefill), res)
        n_miss = min(int(round(top_k * miss_ratio)), len(nonres))
        n_hit = min(top_k - n_miss, len(res))
        row = list(rng.choice(nonres, n_miss, replace=False)) + list(rng.choice(res, n_hit, replace=False))
        while len(row) < top_k:
            row.append(int(rng.integers(0, prefill)))
        row = np.array(row, np.int64)
        if ext:
            sel = rng.random(top_k) < 0.05
            row[sel] = rng.integers(prefill, prefill + ext, size=int(sel.sum()))
        if invalid:
            sel = rng.random(top_k) < invalid
            row[sel] = rng.choice([-1, -3, prefill + ext, prefill + ext + 9], size=int(sel.sum()))
        if dup:
            for i in np.nonzero(rng.random(top_k) < dup)[0]:
                row[i] = row[int(rng.integers(0, top_k))]
        rng.shuffle(row)
        out[b] = row
    return out
