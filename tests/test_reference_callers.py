"""The reference's callers, xds/xds_offload.py and xds/xds_ems_pool.py, against this
repository's restatements of them (offload.py, pool.py): driven through BASELINE config 1 as
xds/xds_decode.py:150-240 drives them, both must make the same `_kvops` data-path calls, in the
same order, with the same arguments (tensors by name and offset) on the same tensor bytes. The
reference's trace is the committed fixture tests/golden/reference_callers_trace.json, made from
the unchanged reference files (tests/golden/make_callers_trace.py); where the reference tree is
present, it is re-made and compared too. No GPU: a recording stand-in takes the calls."""
import json
import os

import pytest

from callers_trace import Recorder, reference_trace, restatement_trace
from conftest import GOLDEN, ROOT

REF_ROOT = os.environ.get("KVOPS_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")


def _fixture():
    with open(os.path.join(GOLDEN, "reference_callers_trace.json")) as f:
        return json.load(f)


def _compare(got, exp):
    assert len(got) == len(exp), (len(got), len(exp))
    for i, (g, e) in enumerate(zip(got, exp)):
        assert g["fn"] == e["fn"], (i, g["fn"], e["fn"])
        assert g["args"] == e["args"], (i, g["fn"], g["args"], e["args"])
        assert g["kw"] == e["kw"], (i, g["fn"], g["kw"])
        assert g["tensors"] == e["tensors"], (i, g["fn"], g["tensors"], e["tensors"])


def test_restatement_makes_the_reference_callers_calls():
    import torch
    rec = Recorder()
    restatement_trace(torch, rec)
    fx = _fixture()
    _compare(json.loads(json.dumps(rec.calls)), fx["calls"])
    fns = [c["fn"] for c in fx["calls"]]
    assert fns.count("sieve_update") == 10 and fns.count("import_seg") == 20 and fns.count("sieve_ht_init") == 8


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF_ROOT, "xds")), reason="reference tree not present")
def test_fixture_is_what_the_reference_files_do():
    import torch
    rec = Recorder()
    reference_trace(torch, rec, REF_ROOT)
    _compare(json.loads(json.dumps(rec.calls)), _fixture()["calls"])
