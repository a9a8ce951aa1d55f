"""Call-trace fixture of the reference's own callers: xds/xds_offload.py (XdsOffloadCoordinator)
and xds/xds_ems_pool.py (EmsPool), imported unchanged from the reference tree and driven through
BASELINE config 1 as xds/xds_decode.py:150-240 drives them, against a recording `_kvops`
(tests/callers_trace.py). The GPU box has no reference tree, so tests compare this repository's
restatements (offload.py, pool.py) with this fixture call for call, and replay them on the GPU.

  python tests/golden/make_callers_trace.py [--ref <reference tree>]
"""
import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from callers_trace import C1, Recorder, reference_trace  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("KVOPS_REFERENCE_DIR") or
                    os.path.join(os.path.dirname(ROOT), "reference"))
    a = ap.parse_args()
    import torch
    rec = Recorder()
    reference_trace(torch, rec, a.ref)
    out = {"config": C1, "source": "xds/xds_offload.py + xds/xds_ems_pool.py (unchanged), driven as "
                                   "xds/xds_decode.py:150-240 drives them", "calls": rec.calls}
    path = os.path.join(HERE, "reference_callers_trace.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=0)
    print("written", path, len(rec.calls), "calls")


if __name__ == "__main__":
    main()
