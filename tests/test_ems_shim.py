"""The EMS control-plane shim (kv_offload_proto_b200.ems_shim) on the CPU: its client and `_cli`
API against the reference's, its host logic, and the reference's unchanged `EmsPool`
(xds/xds_ems_pool.py) driven through it with a recording stand-in for the GPU module. The
row copies themselves are covered on the GPU (tests/test_gpu_ems_shim.py)."""
import importlib.util
import inspect
import os
import struct
import sys
import types

import pytest

from kv_offload_proto_b200 import ems_shim

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_POOL = os.path.join(os.path.dirname(REPO), "reference", "xds", "xds_ems_pool.py")

# EmsClient methods used by EmsPool (ems/ems_client/client.py:16-79): name -> parameters
REFERENCE_CLIENT = {
    "__init__": ["self", "master_ip", "master_port", "timeout_sec"],
    "connect": ["self"], "close": ["self"], "ping": ["self"],
    "pool_create": ["self", "size_bytes", "layer_num", "layer_rows", "row_bytes", "stripe_rows"],
    "pool_destroy": ["self", "pool_id"],
    "link_exchange": ["self", "seg", "endpoint_desc", "mem_desc", "sock"],
}
# _cli functions (ems/ems_client/hcomm_cli_ext.cpp:273-282): name -> parameters
REFERENCE_CLI = {
    "init": ["device_id", "rootinfo", "acl_lib", "hcomm_lib"], "local_desc": [], "mem_reg": ["addr", "size", "tag"],
    "mem_desc": [], "mem_import": ["mem_desc"],
    "link_channel": ["peer_desc", "hcomm_port", "channel_tag", "ready_timeout_sec"],
    "channel_destroy": ["channel"], "close": [],
}
SEGMENT_FIELDS = ["node_id", "seg_base", "seg_size", "ctrl_ip", "ctrl_port", "hcomm_listen_port", "channel_tag",
                  "mem_desc", "ep_desc"]  # kv_proto.py:62-72


class FakeKvops(types.ModuleType):
    """Records the calls EmsPool and the shim make on `kvops_ext._kvops`; no GPU."""

    def __init__(self):
        super().__init__("kvops_ext._kvops")
        self.calls, self.live, self.next = [], set(), 0x7000_0000_0000

    def _addr(self, n):
        a = self.next
        self.next += (n + 0xFFFF) & ~0xFFFF
        return a

    def init(self, device_id, fatbin_path, rt_lib="libascendcl.so"):
        self.calls.append(("init", device_id))

    def close(self):
        self.calls.append(("close",))

    def alloc_status(self, count):
        return self._addr(count * 128)

    def segment_alloc(self, device, nbytes):
        a = self._addr(nbytes)
        self.live.add(a)
        self.calls.append(("segment_alloc", device, nbytes))
        return a

    def segment_free(self, addr):
        self.live.remove(addr)

    def enable_peer_access(self, device, peer):
        self.calls.append(("peer", device, peer))

    def import_seg(self, *a):
        self.calls.append(("import_seg",) + a)

    def export_seg_alllayer(self, *a):
        self.calls.append(("export",) + a)

    def poll_status(self, addr, timeout_us=-1):
        return 0


def test_client_and_cli_signatures_match_the_reference():
    for name, params in REFERENCE_CLIENT.items():
        assert list(inspect.signature(getattr(ems_shim.EmsClient, name)).parameters) == params, name
    for name, params in REFERENCE_CLI.items():
        assert list(inspect.signature(getattr(ems_shim.cli, name)).parameters) == params, name
    assert list(ems_shim.SegmentInfo.__dataclass_fields__) == SEGMENT_FIELDS
    assert list(ems_shim.PoolInfo.__dataclass_fields__) == ["pool_id", "node_num", "segments"]


def test_install_registers_the_reference_module_names():
    ems_shim.install((0,))
    import ems_client
    import ems_client._cli as cli
    assert ems_client.EmsClient is ems_shim.EmsClient and cli.mem_import == ems_shim.cli.mem_import


def test_client_without_master_refuses_and_cli_requires_init():
    c = ems_shim.EmsClient("127.0.0.1", 1)
    with pytest.raises(ConnectionRefusedError):
        c.connect()
    with pytest.raises(ems_shim.EmsError):
        c.ping()
    with pytest.raises(RuntimeError, match="not inited"):
        ems_shim.cli.local_desc()


def test_cli_descriptors_and_channels():
    cli = ems_shim.cli
    cli.init(3)
    try:
        with pytest.raises(RuntimeError, match="already inited"):
            cli.init(3)
        cli.mem_reg(0x1000, 4096, "kv_hbm")
        assert struct.unpack("<IiQQ", cli.mem_desc())[1:] == (3, 0x1000, 4096)
        desc = struct.pack("<IiQQ", 0x42323030, -1, 0xABC000, 1 << 20)  # a pinned host segment
        assert cli.mem_import(desc) == (0xABC000, 1 << 20, -1)
        with pytest.raises(RuntimeError):
            cli.mem_import(b"\x00" * 24)
        h1, st1 = cli.link_channel(b"x", 0, "t1")
        h2, _ = cli.link_channel(b"y", 0, "t2")
        assert st1 == 0 and h1 != h2 and h1 != 0
        cli.channel_destroy(h1)
    finally:
        cli.close()


def _load_reference_pool(monkeypatch, fake):
    ems_shim.install((0, 1, -1))
    pkg = types.ModuleType("kvops_ext")
    pkg.__path__ = []
    pkg._kvops = fake
    monkeypatch.setitem(sys.modules, "kvops_ext", pkg)
    monkeypatch.setitem(sys.modules, "kvops_ext._kvops", fake)
    monkeypatch.setattr(ems_shim, "_kvops", lambda: fake)
    spec = importlib.util.spec_from_file_location("ref_xds_ems_pool", REF_POOL)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.skipif(not os.path.exists(REF_POOL), reason="reference sources not present")
def test_reference_ems_pool_runs_unchanged_through_the_shim(monkeypatch):
    fake = FakeKvops()
    ref = _load_reference_pool(monkeypatch, fake)
    ems_shim.serve("127.0.0.1", 7301)
    try:
        L, rows, rb, S = 2, 1000, 1152, 1
        pool = ref.EmsPool("127.0.0.1", 7301, 0, L, rows, rb, S)
        pool.create_pool(0x5000_0000, 1 << 24, "")
        assert pool.node_num == 3 and len(pool.channels) == 3 and len(set(pool.channels)) == 3
        plsr = (rows + 2) // 3
        assert pool.per_layer_seg_rows == plsr
        allocs = [c for c in fake.calls if c[0] == "segment_alloc"]
        assert [c[1] for c in allocs] == [0, 1, -1] and all(c[2] == L * plsr * rb for c in allocs)
        assert ("peer", 0, 1) in fake.calls  # node 1 is a peer GPU
        st = pool.batch_read(1, 11, 12, 13, 14, 15, 16, 17, 4, 64)
        reads = [c for c in fake.calls if c[0] == "import_seg"]
        assert len(reads) == 3
        for s, c in enumerate(reads):
            seg = pool.pool.segments[s]
            # channel, seg_base, layer_offset, plsr, row_bytes, ..., node_num, my_node, status
            assert c[1:6] == (pool.channels[s], seg.seg_base, plsr, plsr, rb)
            assert c[-5:-2] == (3, s, st)
        pool.wait(st)
        pool.batch_write_alllayers(0, 100, 21, 1000 * rb)
        assert len([c for c in fake.calls if c[0] == "export"]) == 3
        pool.destroy()
        assert not fake.live  # every segment freed
        assert ("close",) in fake.calls
        with pytest.raises(RuntimeError, match="not inited"):
            ems_shim.cli.local_desc()
    finally:
        ems_shim.stop("127.0.0.1", 7301)
