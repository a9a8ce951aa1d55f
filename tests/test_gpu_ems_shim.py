"""The EMS control-plane shim on a B200: the call sequence of the reference's
EmsPool.create_pool / batch_read / wait / destroy (xds/xds_ems_pool.py:141-241) against
real segments (two in HBM, one in pinned host memory), with every gathered byte checked
against the C restatement. Runs in a fresh process: the sequence calls `_kvops.init`."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r'''
import numpy as np, torch
import kv_offload_proto_b200 as kp
from kv_offload_proto_b200 import ems_shim
from kv_offload_proto_b200.pool import device_view
import oracle
kv = kp.install_kvops_ext()
ems_shim.install((0, 0, -1))
ems_shim.serve("127.0.0.1", 7401)
from ems_client import EmsClient
import ems_client._cli as cli

L, rows, RB, S, layer = 2, 6 * 1024, 1152, 1, 1
R, K, ctx, dbs = 6, 128, 1024, 512
hot = torch.zeros(R * dbs * RB, dtype=torch.uint8, device="cuda")
# EmsPool.create_pool (:141-180)
ems = EmsClient("127.0.0.1", 7401, 120.0)
ems.connect()
ems.ping()
pool = ems.pool_create(L * rows * RB, L, rows, RB, S)
N = pool.node_num
plsr = (rows + N - 1) // N
cli.init(0, "/etc/hccl_rootinfo.json", "libascendcl.so", "libhcomm.so")
cli.mem_reg(hot.data_ptr(), hot.numel(), "kv_hbm")
local_desc, mem_desc = cli.local_desc(), cli.mem_desc()
channels = []
for seg in pool.segments:
    assert ems.link_exchange(seg, local_desc, mem_desc) == 0
    addr, _size, _t = cli.mem_import(seg.mem_desc)
    assert addr == seg.seg_base and seg.ep_desc
    h, _st = cli.link_channel(seg.ep_desc, seg.hcomm_listen_port, seg.channel_tag, 60)
    channels.append(h)
kv.init(0, "")
status = kv.alloc_status(8 * N)
# fill the segments
rng = np.random.default_rng(2)
segs_h = []
for s, seg in enumerate(pool.segments):
    h = rng.integers(0, 256, seg.seg_size, dtype=np.uint8)
    segs_h.append(h)
    if ems_shim._MASTERS[("127.0.0.1", 7401)].devices[s] < 0:
        np.ctypeslib.as_array((__import__("ctypes").c_uint8 * seg.seg_size).from_address(seg.seg_base))[:] = h
    else:
        device_view(seg.seg_base, seg.seg_size, "cuda:0").copy_(torch.from_numpy(h).cuda())
torch.cuda.synchronize()
topk = np.stack([rng.choice(ctx, K, replace=False) for _ in range(R)]).astype(np.int32)
miss = (rng.random((R, K)) < 0.3).astype(np.int8)
slots = np.stack([rng.permutation(dbs)[:K] for _ in range(R)]).astype(np.int32)
req_pool = np.arange(R, dtype=np.int64)
base = np.arange(R, dtype=np.int64) * ctx
t = [torch.from_numpy(a).cuda() for a in (topk, req_pool, base, slots, miss, np.array([R], np.int32))]
# EmsPool.batch_read (:204-217) with the per-request hot rows option
for s, seg in enumerate(pool.segments):
    kv.import_seg(channels[s], seg.seg_base, layer * plsr, plsr, RB, *[x.data_ptr() for x in t], hot.data_ptr(), K, R,
                  S, N, s, status, 0, 1, hot_req_stride_rows=dbs)
# EmsPool.wait (:233-241)
for s in range(N):
    assert kv.poll_status(status + s * 64, 10_000_000) == 0
torch.cuda.synchronize()
exp = np.zeros(R * dbs * RB, np.uint8)
n = 0
for s in range(N):
    n += oracle.gather_rows(segs_h[s], layer * plsr, RB, topk, req_pool, base, slots, miss, R, exp, K, R, S, N, s, dbs)
np.testing.assert_array_equal(hot.cpu().numpy(), exp)
assert n == int(miss.sum()) > 0
# EmsPool.destroy (:186-197)
for h in channels:
    cli.channel_destroy(h)
cli.close()
kv.close()
ems.pool_destroy(pool.pool_id)
ems.close()
print("ems shim ok", n)
'''


def test_ems_pool_call_sequence_through_the_shim():
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([REPO, os.path.join(REPO, "tests"), env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", SCRIPT], cwd=REPO, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "ems shim ok" in r.stdout
