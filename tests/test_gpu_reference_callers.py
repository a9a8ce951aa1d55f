"""The reference's caller sequence on a B200: this repository's restatements of
xds/xds_offload.py and xds/xds_ems_pool.py, driven through BASELINE config 1 as
xds/xds_decode.py:150-240 drives them, make on the real `_kvops` exactly the calls the
reference's unchanged files make (the committed trace tests/golden/reference_callers_trace.json;
test_reference_callers.py pins that equivalence, tensor bytes included, on the CPU), and the
results are the reference's: slots and miss flags equal its Python oracle's (the c1 fixture),
and every gathered row holds its fingerprint (xds_decode.py:60-63,256-275)."""
import json
import os

import numpy as np
import pytest

from callers_trace import RB, Recorder, restatement_trace
from conftest import GOLDEN
from gpu_util import kv

pytestmark = pytest.mark.gpu


def test_reference_call_sequence_on_the_gpu():
    import torch
    from kv_offload_proto_b200.workload import fingerprint_rows
    rec = Recorder(forward=kv())
    coord, hbm, steps, bases = restatement_trace(torch, rec, device="cuda")
    with open(os.path.join(GOLDEN, "reference_callers_trace.json")) as f:
        exp = json.load(f)["calls"]
    got = json.loads(json.dumps(rec.calls))
    assert [c["fn"] for c in got] == [c["fn"] for c in exp]
    for g, e in zip(got, exp):
        assert g["args"] == e["args"] and g["kw"] == e["kw"], (g, e)
    fx = dict(np.load(os.path.join(GOLDEN, "sieve_c1_ref_sampler.npz")))
    hbm_h = hbm.cpu().numpy().view(np.uint32)
    checked = 0
    for s, (topk, slots, miss) in enumerate(steps):
        np.testing.assert_array_equal(topk, fx["topk"][s])
        np.testing.assert_array_equal(slots, fx["slots"][s])
        np.testing.assert_array_equal(miss, fx["is_miss"][s])
    # The last step of each layer left its miss rows in hbm[layer]. The reference's hot rows are
    # shared by all requests (hot_row_base + slot), so a slot several positions name ends up
    # holding, in each 16-byte chunk, that chunk of one of their rows (the copies of one launch
    # run concurrently, chunk by chunk, as the reference's per-position copies would race).
    for s in (len(steps) - 2, len(steps) - 1):
        topk, slots, miss = steps[s]
        layer = s % 2
        cands = {}
        for r, k in zip(*np.nonzero(miss)):
            cands.setdefault(int(slots[r, k]), []).append(bases[r] + int(topk[r, k]))
        for slot, rows in cands.items():
            fps = fingerprint_rows(rows, layer, RB // 4).reshape(len(rows), -1, 4)
            got = hbm_h[layer, slot].reshape(-1, 4)
            assert ((got[None] == fps).all(axis=2).any(axis=0)).all(), (s, slot)  # every chunk is some candidate's
            checked += 1
    assert checked >= 32
