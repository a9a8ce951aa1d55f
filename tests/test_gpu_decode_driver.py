"""The B200 decode driver (python -m kv_offload_proto_b200.decode, the reference's
xds/xds_decode.py on CUDA): the reference's acceptance lines (README.md:82-89) with every step
checked against the CPU SIEVE model, in a fresh process each."""
import os
import re
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_driver(tmp_path, *extra):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([REPO, env.get("PYTHONPATH", "")])
    cmd = [sys.executable, "-m", "kv_offload_proto_b200.decode", "--run-dir", str(tmp_path), *extra]
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    return r.returncode, r.stdout + r.stderr


@pytest.mark.parametrize("extra", [
    ("--layer-rows", "2048", "--oracle"),
    ("--layer-rows", "4096", "--oracle", "--segment-devices", "0,0,-1", "--stripe-rows", "2", "--injective",
     "--one-call"),
    ("--layer-rows", "512", "--req-num", "1", "--oracle", "--shared-hot", "--steps", "6"),
])
def test_decode_driver_acceptance_lines(tmp_path, extra):
    rc, out = run_driver(tmp_path, *extra)
    assert rc == 0, out[-3000:]
    assert "[xds][ERROR]" not in out
    assert re.search(r"\[xds\] pool ready: nodes=\d+ perLayerSegRows=\d+ channels=\d+", out)
    assert re.search(r"\[xds\] prefill export: \d+ rows x \d+ layers = \d+ B in [\d.]+ us", out)
    steps = re.findall(r"\[xds\] step \d+: layer=\d+ miss=(\d+) rows in [\d.]+ us \(checked=(\d+)\)", out)
    assert len(steps) >= 6 and all(int(m) > 0 and int(c) > 0 for m, c in steps)
    assert re.search(r"\[xds\] summary: imported \d+ miss rows, avg [\d.]+ us/row, aggregate [\d.]+ GB/s", out)
    assert "[xds] all done" in out
    assert os.path.exists(os.path.join(str(tmp_path), "xds_decode.log"))
