"""Call traces of the reference's callers (xds/xds_offload.py, xds/xds_ems_pool.py) and of this
repository's restatements of them, for comparison.

The reference's driver sequence for BASELINE config 1 (xds/xds_decode.py:150-240: pool
creation, row allocation, fingerprint fill, all-layer export, admission, then decode steps of
sieve_update + batch_read + wait with the reference sampler, seed 42) is run against a module
that records every `_kvops` data-path call. Addresses are recorded as (tensor name, byte offset):
the tensors are named by the driver, segment bases by node, status words by slot. At each call
the bytes of every tensor it names are hashed, so two implementations that make the same calls
on the same tensor contents give the same trace.
"""
import hashlib
import types

import numpy as np

RB = 1152
C1 = dict(R=8, L=2, prefill=256, K=64, dbs=64, layer_rows=2048, S=1, steps=10, block_dim=8, seed=42, miss=0.5,
          nodes=2)
DATA_PATH = ("sieve_ht_init", "sieve_update", "import_seg", "export_seg_alllayer", "poll_status")
# keyword-only options of this repository's module; a call that leaves them at these values is
# the reference's call
DEFAULT_KW = {"hot_req_stride_rows": 0, "injective": False, "err_word": 0, "copy_wait_polls": 0, "path": "auto"}


class Recorder(types.ModuleType):
    """Stand-in for `kvops_ext._kvops` that records data-path calls (optionally forwarding them
    to a real module, whose results it returns)."""

    _FAKE_BASE = 1 << 52  # fake allocations live far above any process address

    def __init__(self, forward=None):
        super().__init__("kvops_ext._kvops")
        self.forward = forward
        self.ranges = []  # (base, nbytes, name, tensor or None)
        self.calls = []
        self._next = self._FAKE_BASE
        self._nseg = 0

    def name_tensor(self, name, t):
        self.ranges.append((t.data_ptr(), t.numel() * t.element_size(), name, t))

    def _fake(self, nbytes, name):
        a = self._next
        self._next += (nbytes + 0xFFFF) & ~0xFFFF
        self.ranges.append((a, nbytes, name, None))
        return a

    def _map(self, v):
        if isinstance(v, bool) or not isinstance(v, int) or v < 4096:
            return v
        for base, n, name, _ in self.ranges:
            if base <= v < base + max(n, 1):
                return [name, v - base]
        return v

    def _digests(self, args):
        out = {}
        for v in args:
            m = self._map(v)
            if isinstance(m, list):
                for base, n, name, t in self.ranges:
                    if name == m[0] and t is not None and t.device.type == "cpu":
                        out[name] = hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()[:16]
        return out

    # set-up calls: allocations are named, nothing is compared
    def init(self, *a, **k):
        return self.forward.init(*a, **k) if self.forward else None

    def close(self):
        return self.forward.close() if self.forward else None

    def alloc_status(self, count):
        if self.forward:
            a = self.forward.alloc_status(count)
            self.ranges.append((a, count * 128, "status", None))
            return a
        return self._fake(count * 128, "status")

    def segment_alloc(self, device, nbytes):
        name = "seg{}".format(self._nseg)
        self._nseg += 1
        if self.forward:
            a = self.forward.segment_alloc(device, nbytes)
            self.ranges.append((a, nbytes, name, None))
            return a
        return self._fake(nbytes, name)

    def segment_free(self, addr):
        return self.forward.segment_free(addr) if self.forward else None

    def enable_peer_access(self, *a):
        return self.forward.enable_peer_access(*a) if self.forward else None

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)

        def call(*args, **kw):
            if name in DATA_PATH:
                args_n = [self._map(v) for v in args]
                if name in ("import_seg", "export_seg_alllayer"):
                    args_n[0] = "channel"  # an opaque handle the B200 library ignores
                extra = {k: v for k, v in kw.items() if DEFAULT_KW.get(k, object()) != v}
                self.calls.append({"fn": name, "args": args_n, "kw": extra, "tensors": self._digests(args)})
            if self.forward is not None:
                return getattr(self.forward, name)(*args, **kw)
            return 0 if name == "poll_status" else None

        return call


def drive(make_pool, make_coord, rec, torch, device="cpu", cfg=C1):
    """The reference driver's config-1 sequence (xds_decode.py:150-240) on the given pool and
    coordinator implementations; returns (coord, hbm, per-step (topk, slots, is_miss))."""
    from kv_offload_proto_b200.workload import fingerprint_rows, ref_topk_batch
    R, L, prefill, K, dbs = cfg["R"], cfg["L"], cfg["prefill"], cfg["K"], cfg["dbs"]
    layer_rows, bd = cfg["layer_rows"], cfg["block_dim"]
    hbm = torch.zeros((L, layer_rows, RB // 4), dtype=torch.int32, device=device)
    rec.name_tensor("hbm", hbm)
    pool = make_pool(hbm)
    coord = make_coord()
    for name in ("device_buffer_tokens", "device_buffer_visited", "device_buffer_ht", "sieve_hand", "prefill_lens",
                 "req_host_base", "top_k_device_slots", "is_miss", "num_real"):
        rec.name_tensor(name, getattr(coord, name))
    alloc = pool.make_allocator()
    bases = []
    fill = np.zeros((L, layer_rows, RB // 4), np.uint32)
    for r in range(R):
        rows = alloc.alloc(prefill)
        assert rows == list(range(rows[0], rows[0] + prefill))
        bases.append(rows[0])
        for layer in range(L):
            fill[layer, rows[0]:rows[0] + prefill] = fingerprint_rows(np.arange(prefill) + rows[0], layer, RB // 4)
    hbm.copy_(torch.from_numpy(fill.view(np.int32)).to(device))
    st = pool.batch_write_alllayers(0, R * prefill, hbm[0, 0], layer_rows * RB)
    pool.wait(st)
    for r in range(R):
        coord.admit_request(r, r, prefill, bases[r])
    hbm.zero_()
    seq = torch.full((R,), prefill, dtype=torch.int32, device=device)
    pool_idx = torch.arange(R, dtype=torch.int64, device=device)
    rec.name_tensor("seq_lens", seq)
    rec.name_tensor("req_pool_indices", pool_idx)
    coord.set_batch(pool_idx, seq)
    rng = np.random.default_rng(cfg["seed"])
    topk_buf = torch.zeros((R, K), dtype=torch.int32, device=device)
    rec.name_tensor("topk", topk_buf)
    out = []
    for step in range(cfg["steps"]):
        batch = ref_topk_batch(rng, R, K, prefill, dbs, cfg["miss"])
        topk_buf.copy_(torch.from_numpy(batch).to(device))
        layer = step % L
        coord.sieve_update(layer, topk_buf, block_dim=bd)
        st = pool.batch_read(layer, topk_buf, pool_idx, coord.req_host_base, coord.top_k_device_slots,
                             coord.is_miss, coord.num_real, hbm[layer, 0:], R, K, block_dim=bd)
        pool.wait(st, block_dim=bd)
        out.append((batch, coord.top_k_device_slots.cpu().numpy().copy(), coord.is_miss.cpu().numpy().copy()))
    return coord, hbm, out, bases


def restatement_trace(torch, rec, device="cpu"):
    """This repository's callers (offload.XdsOffloadCoordinator, pool.DevicePool with one
    import_seg launch per segment, as EmsPool.batch_read issues them) under `rec`."""
    from kv_offload_proto_b200 import offload, pool as pool_mod

    class Coord(offload.XdsOffloadCoordinator):
        _require_cuda = device != "cpu"

    class Pool(pool_mod.DevicePool):
        def batch_read(self, *a, **k):
            return super().batch_read(*a, fused=False, **k)

    c = C1
    saved = (offload._kvops_module, pool_mod._kvops_module)
    offload._kvops_module = pool_mod._kvops_module = lambda: rec
    try:
        return drive(lambda hbm: Pool(0, c["L"], c["layer_rows"], RB, c["S"], segment_devices=(0,) * c["nodes"]),
                     lambda: Coord(device, c["L"], c["R"], c["dbs"], c["K"], c["R"], c["prefill"]), rec, torch,
                     device)
    finally:
        offload._kvops_module, pool_mod._kvops_module = saved


def reference_trace(torch, rec, ref_root):
    """The reference's own XdsOffloadCoordinator and EmsPool, imported unchanged from
    `ref_root`, under `rec`, with this repository's EMS control-plane shim standing in for the
    emsd master and the HCOMM client (the shim allocates the segments through `rec`)."""
    import importlib
    import sys

    from kv_offload_proto_b200 import ems_shim
    pkg = types.ModuleType("kvops_ext")
    pkg.__path__ = []
    pkg._kvops = rec
    saved = {k: sys.modules.get(k) for k in ("kvops_ext", "kvops_ext._kvops", "xds", "xds.xds_ems_pool",
                                             "xds.xds_offload")}
    saved_kv = ems_shim._kvops
    sys.modules["kvops_ext"], sys.modules["kvops_ext._kvops"] = pkg, rec
    for k in ("xds", "xds.xds_ems_pool", "xds.xds_offload"):
        sys.modules.pop(k, None)
    ems_shim.install((0,) * C1["nodes"])
    ems_shim._kvops = lambda: rec
    sys.path.insert(0, ref_root)
    port = 7411
    ems_shim.serve("127.0.0.1", port)
    try:
        xo = importlib.import_module("xds.xds_offload")
        xp = importlib.import_module("xds.xds_ems_pool")
        c = C1

        def make_pool(hbm):
            p = xp.EmsPool("127.0.0.1", port, 0, c["L"], c["layer_rows"], RB, c["S"])
            p.create_pool(hbm.data_ptr(), hbm.numel() * 4, "")
            return p

        return drive(make_pool, lambda: xo.XdsOffloadCoordinator("cpu", c["L"], c["R"], c["dbs"], c["K"], c["R"],
                                                                 c["prefill"]), rec, torch)
    finally:
        ems_shim.stop("127.0.0.1", port)
        ems_shim._kvops = saved_kv
        sys.path.remove(ref_root)
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
