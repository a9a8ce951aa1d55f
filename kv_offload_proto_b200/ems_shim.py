"""In-process stand-in for the reference's EMS control plane: the `ems_client` package
(ems/ems_client/client.py:16-79, kv_proto.py:62-79) and its native `_cli` extension
(ems/ems_client/hcomm_cli_ext.cpp:271-283), so that the reference's unchanged `EmsPool`
(xds/xds_ems_pool.py:108-241) creates, uses and destroys a striped pool on B200s.

There is no emsd daemon, TCP master or HCOMM channel here. A "master" is an in-process pool
manager registered under (ip, port) with `serve()`; `pool_create` allocates one segment per
configured device (own HBM, a peer GPU's HBM, or pinned host memory with device -1), each
`layer_num * ceil(layer_rows / N) * row_bytes` bytes as `EmsPool` lays them out (:161), and
reports them as SegmentInfo records whose `seg_base` is the address the kernels dereference.
`_cli.mem_import` hands that address back, `link_channel` returns a channel id that the B200
kernels ignore (segment addresses are UVA). Segments live in this process (the reference's
single-process UVA model); for pools owned by other processes use DevicePool with IPC handles.

    import kv_offload_proto_b200 as kp
    kp.install_kvops_ext()
    kp.ems_shim.install(segment_devices=(1, 2, 3))    # ems_client + ems_client._cli
    kp.ems_shim.serve("127.0.0.1", 9000)
    from xds.xds_ems_pool import EmsPool                # the reference's file, unchanged
"""
import struct
import sys
import threading
import types
from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Tuple

__all__ = ["EmsClient", "EmsError", "PoolInfo", "SegmentInfo", "serve", "stop", "install", "cli",
           "KV_OK", "KV_ERR_PROTO", "KV_ERR_PARAM", "KV_ERR_NO_RESOURCE", "KV_ERR_NOT_FOUND", "KV_ERR_STATE"]

# status values of common/kv_proto.h (ems/ems_client/kv_proto.py:19-26)
KV_OK = 0
KV_ERR_PROTO = -1
KV_ERR_PARAM = -2
KV_ERR_NO_RESOURCE = -3
KV_ERR_NOT_FOUND = -5
KV_ERR_STATE = -6

_MEM_MAGIC = 0x42323030  # descriptor tag of this shim
_MEM_FMT = "<IiQQ"        # magic, device, address, size


class EmsError(Exception):
    """Same shape as the reference client's error (client.py:10-13)."""

    def __init__(self, status: int, msg: str):
        super().__init__("status={} {}".format(status, msg))
        self.status = status


@dataclass
class SegmentInfo:
    """Field names of kv_proto.SegmentInfo (kv_proto.py:62-72)."""
    node_id: int = 0
    seg_base: int = 0
    seg_size: int = 0
    ctrl_ip: str = ""
    ctrl_port: int = 0
    hcomm_listen_port: int = 0
    channel_tag: str = ""
    mem_desc: bytes = b""
    ep_desc: bytes = b""


@dataclass
class PoolInfo:
    pool_id: int = 0
    node_num: int = 0
    segments: list = field(default_factory=list)


def _kvops():
    from . import kvops
    return kvops()


class _Master:
    """The in-process pool manager behind one (ip, port)."""

    def __init__(self, ip: str, port: int, segment_devices: Sequence[int]):
        if not 1 <= len(segment_devices) <= 64:
            raise ValueError("segment_devices: 1..64 entries")
        self.ip, self.port = ip, port
        self.devices = list(segment_devices)
        self.pools: Dict[int, PoolInfo] = {}
        self.next_id = 1
        self.lock = threading.Lock()

    def create(self, size_bytes, layer_num, layer_rows, row_bytes, stripe_rows) -> PoolInfo:
        if layer_num < 1 or layer_rows < 1 or row_bytes <= 0 or stripe_rows < 0:
            raise EmsError(KV_ERR_PARAM, "pool_create: bad dims L={} rows={} rowBytes={} S={}".format(
                layer_num, layer_rows, row_bytes, stripe_rows))
        n = len(self.devices)
        seg_bytes = layer_num * ((layer_rows + n - 1) // n) * row_bytes
        if size_bytes < layer_num * layer_rows * row_bytes:
            raise EmsError(KV_ERR_PARAM, "pool_create: size {} below the pool's {} bytes".format(
                size_bytes, layer_num * layer_rows * row_bytes))
        k = _kvops()
        with self.lock:
            pool_id = self.next_id
            self.next_id += 1
            segs = []
            try:
                for node, dev in enumerate(self.devices):
                    addr = k.segment_alloc(dev, seg_bytes)
                    segs.append(SegmentInfo(
                        node_id=node, seg_base=addr, seg_size=seg_bytes, ctrl_ip=self.ip, ctrl_port=self.port,
                        hcomm_listen_port=0, channel_tag="kv_pool_{}_{}".format(pool_id, node),
                        mem_desc=struct.pack(_MEM_FMT, _MEM_MAGIC, dev, addr, seg_bytes),
                        ep_desc=struct.pack("<Ii", _MEM_MAGIC, dev)))
            except RuntimeError as e:
                for s in segs:
                    k.segment_free(s.seg_base)
                raise EmsError(KV_ERR_NO_RESOURCE, "pool_create: {}".format(e)) from e
            pool = PoolInfo(pool_id=pool_id, node_num=n, segments=segs)
            self.pools[pool_id] = pool
            return pool

    def destroy(self, pool_id):
        with self.lock:
            pool = self.pools.pop(pool_id, None)
        if pool is None:
            raise EmsError(KV_ERR_NOT_FOUND, "pool_destroy failed, poolId={}".format(pool_id))
        k = _kvops()
        for s in pool.segments:
            k.segment_free(s.seg_base)

    def owns(self, seg: SegmentInfo) -> bool:
        with self.lock:
            return any(seg in p.segments for p in self.pools.values())


_MASTERS: Dict[Tuple[str, int], _Master] = {}
_MASTERS_LOCK = threading.Lock()


def serve(master_ip: str, master_port: int, segment_devices: Sequence[int] = None) -> None:
    """Starts the in-process master at (ip, port); segments go to `segment_devices` (default:
    the devices given to install(), else device 0)."""
    devs = list(segment_devices) if segment_devices is not None else list(_DEFAULTS["segment_devices"])
    with _MASTERS_LOCK:
        if (master_ip, master_port) in _MASTERS:
            raise EmsError(KV_ERR_STATE, "master {}:{} already serving".format(master_ip, master_port))
        _MASTERS[(master_ip, master_port)] = _Master(master_ip, master_port, devs)


def stop(master_ip: str, master_port: int) -> None:
    """Stops a master; pools it still holds are freed."""
    with _MASTERS_LOCK:
        m = _MASTERS.pop((master_ip, master_port), None)
    if m is not None:
        for pid in list(m.pools):
            m.destroy(pid)


class EmsClient:
    """The reference client's API (client.py:16-79) over the in-process master."""

    def __init__(self, master_ip: str, master_port: int, timeout_sec: float = 120.0):
        self.master = (master_ip, master_port)
        self.timeout = timeout_sec
        self._m = None

    def connect(self) -> None:
        with _MASTERS_LOCK:
            m = _MASTERS.get(self.master)
        if m is None:
            raise ConnectionRefusedError("no EMS master serving at {}:{}".format(*self.master))
        self._m = m

    def close(self) -> None:
        self._m = None

    def _master(self) -> _Master:
        if self._m is None:
            raise EmsError(KV_ERR_STATE, "not connected")
        return self._m

    def ping(self) -> None:
        self._master()

    def pool_create(self, size_bytes: int, layer_num: int, layer_rows: int, row_bytes: int,
                    stripe_rows: int = 1) -> PoolInfo:
        return self._master().create(size_bytes, layer_num, layer_rows, row_bytes, stripe_rows)

    def pool_destroy(self, pool_id: int) -> None:
        self._master().destroy(pool_id)

    def link_exchange(self, seg: SegmentInfo, endpoint_desc: bytes, mem_desc: bytes, sock=None) -> int:
        """KV_OK when the segment belongs to a live pool and both descriptors are present."""
        if not endpoint_desc or not mem_desc:
            return KV_ERR_PARAM
        with _MASTERS_LOCK:
            m = _MASTERS.get((seg.ctrl_ip, seg.ctrl_port))
        return KV_OK if m is not None and m.owns(seg) else KV_ERR_NOT_FOUND


class _Cli:
    """The `_cli` extension's functions (hcomm_cli_ext.cpp:271-283)."""

    def __init__(self):
        self.lock = threading.Lock()
        self.device = None
        self.regs: List[Tuple[int, int, str]] = []
        self.channels: Dict[int, str] = {}
        self.next_channel = 1

    def init(self, device_id, rootinfo="/etc/hccl_rootinfo.json", acl_lib="libascendcl.so",
             hcomm_lib="libhcomm.so"):
        with self.lock:
            if self.device is not None:
                raise RuntimeError("_cli already inited")
            self.device = int(device_id)

    def _need_init(self):
        if self.device is None:
            raise RuntimeError("_cli not inited")

    def local_desc(self) -> bytes:
        self._need_init()
        return struct.pack("<Ii", _MEM_MAGIC, self.device)

    def mem_reg(self, addr, size, tag="kv_hbm") -> None:
        self._need_init()
        if addr == 0 or size <= 0:
            raise RuntimeError("mem_reg: bad range")
        with self.lock:
            self.regs.append((int(addr), int(size), tag))

    def mem_desc(self) -> bytes:
        self._need_init()
        if not self.regs:
            raise RuntimeError("mem_desc: no registered memory")
        addr, size, _ = self.regs[-1]
        return struct.pack(_MEM_FMT, _MEM_MAGIC, self.device, addr, size)

    def mem_import(self, mem_desc) -> Tuple[int, int, int]:
        """(address, size, device) of a segment descriptor; the address is the segment's UVA base."""
        self._need_init()
        desc = bytes(mem_desc)
        if len(desc) != struct.calcsize(_MEM_FMT):
            raise RuntimeError("mem_import: descriptor of {} bytes".format(len(desc)))
        magic, dev, addr, size = struct.unpack(_MEM_FMT, desc)
        if magic != _MEM_MAGIC:
            raise RuntimeError("mem_import: not a descriptor of this pool")
        if dev >= 0 and dev != self.device:
            _kvops().enable_peer_access(self.device, dev)  # rows are read in-kernel over NVLink
        return addr, size, dev

    def link_channel(self, peer_desc, hcomm_port, channel_tag, ready_timeout_sec=60) -> Tuple[int, int]:
        self._need_init()
        if not bytes(peer_desc):
            raise RuntimeError("link_channel: empty peer descriptor")
        with self.lock:
            h = self.next_channel
            self.next_channel += 1
            self.channels[h] = str(channel_tag)
        return h, 0

    def channel_destroy(self, channel) -> None:
        with self.lock:
            self.channels.pop(int(channel), None)

    def close(self) -> None:
        with self.lock:
            self.device = None
            self.regs.clear()
            self.channels.clear()


cli = _Cli()
_DEFAULTS = {"segment_devices": (0,)}


def install(segment_devices: Sequence[int] = (0,)):
    """Registers this shim as the modules `ems_client` and `ems_client._cli` (what
    xds/xds_ems_pool.py:11-22 imports); `segment_devices` is the default placement of serve()."""
    _DEFAULTS["segment_devices"] = tuple(segment_devices)
    pkg = types.ModuleType("ems_client")
    pkg.EmsClient, pkg.EmsError, pkg.PoolInfo, pkg.SegmentInfo = EmsClient, EmsError, PoolInfo, SegmentInfo
    pkg.__path__ = []  # a package, so `import ems_client._cli` resolves
    cli_mod = types.ModuleType("ems_client._cli")
    for name in ("init", "local_desc", "mem_reg", "mem_desc", "mem_import", "link_channel", "channel_destroy",
                 "close"):
        setattr(cli_mod, name, getattr(cli, name))
    pkg._cli = cli_mod
    sys.modules["ems_client"] = pkg
    sys.modules["ems_client._cli"] = cli_mod
    return pkg
