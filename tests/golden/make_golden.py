"""Generate the golden fixtures under tests/golden/ from the reference's own Python code.

Run where the reference tree is mounted (its root is given with --ref):

    python tests/golden/make_golden.py [--ref <reference root>]

It imports, read-only and unmodified:
  * xds.xds_decode._CpuSieveOracle   (xds/xds_decode.py:66-118)  — the SIEVE oracle
  * xds.xds_decode.row_word          (xds/xds_decode.py:60-63)   — the row fingerprint
  * test/kv_layout_ref.py            (whole file)                — the stripe map
  * xds.xds_ems_pool.compute_ht_size / align (xds/xds_ems_pool.py:42-51)

and records their outputs on seeded inputs as small .json/.npz files. The tests and
the GPU parity checks read only these files; the reference tree is never read at
test time. Decode-extension slots are normalised from the oracle's -2-off marker
to the kernel's padded+off encoding (hisp_sieve_update.cpp:123-128 vs
xds_decode.py:95-97).

The reference driver keeps one oracle per request across layers
(xds_decode.py:194,243) although the kernel state is per layer; the fixtures use one
oracle instance per (layer, request), which is what the kernel computes.
"""
import argparse
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_ref(ref):
    sys.path.insert(0, ref)
    from xds.xds_decode import _CpuSieveOracle, row_word  # noqa: E402
    from xds.xds_ems_pool import align, compute_ht_size  # noqa: E402
    spec = importlib.util.spec_from_file_location("kv_layout_ref", os.path.join(ref, "test", "kv_layout_ref.py"))
    lay = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(lay)
    return _CpuSieveOracle, row_word, align, compute_ht_size, lay


def padded_of(dbs):
    return (dbs + 15) // 16 * 16


def norm_slots(slots, padded):
    out = []
    for s in slots:
        out.append(padded + (-s - 2) if s <= -2 else s)
    return out


def kat_cases(Oracle):
    """The SIEVE known-answer cases of test/test_sieve_oracle.py:24-83, replayed through the
    reference oracle; each case is a list of (pool_idx, topk_row, seq_len) updates."""
    cases = [
        ("identity_hit", 1, 100, 8, [(0, [0, 3, 7], 100)]),
        ("miss_and_eviction", 1, 100, 8, [(0, [8, 9], 100), (0, [0], 100)]),
        ("second_chance", 1, 100, 4, [(0, [0, 1], 100), (0, [10], 100), (0, [11], 100), (0, [12], 100)]),
        ("ht_churn", 1, 1000, 16, [(0, [1000 - 1 - i], 1000) for i in range(200)]),
        ("decode_extend_and_invalid", 1, 10, 4, [(0, [12, -1, 3], 20)]),
        ("duplicate_first_hit", 1, 100, 8, [(0, [8, 8], 100)]),
        ("multi_req_independent", 2, 100, 4, [(0, [50, 51, 52, 53], 100), (1, [0, 1], 100)]),
    ]
    out = []
    for name, nreq, prefill, dbs, updates in cases:
        o = Oracle([(prefill, r) for r in range(nreq)])
        for r in range(nreq):
            o.reset(r, prefill, dbs)
        steps = []
        for pool_idx, row, seq_len in updates:
            s, m = o.update(pool_idx, list(row), seq_len)
            steps.append({"pool_idx": pool_idx, "topk": list(row), "seq_len": seq_len,
                          "slots": norm_slots(s, padded_of(dbs)), "is_miss": list(m)})
        final = [{"hand": o.state[r]["hand"], "t2s": sorted(o.state[r]["t2s"].items())} for r in range(nreq)]
        out.append({"name": name, "num_reqs": nreq, "prefill": prefill, "dbs": dbs, "steps": steps,
                    "final": final})
    return out


def ref_sampler_batches(rng, req_num, topk, prefill, dbs, miss_ratio):
    """The driver's topK draw, xds_decode.py:213-223, restated: hits with replacement from
    [0, min(prefill,dbs)), misses without replacement from [dbs, prefill), then an in-place
    shuffle of the flattened batch (which mixes positions across requests)."""
    hit_span = min(prefill, dbs)
    miss_span = max(prefill - dbs, 0)
    n_miss = int(topk * miss_ratio) if miss_span > 0 else 0
    n_hit = topk - n_miss
    batch = np.empty((req_num, topk), dtype=np.int32)
    for r in range(req_num):
        hits = rng.integers(0, hit_span, size=n_hit) if n_hit > 0 else np.empty(0, dtype=np.int64)
        misses = (rng.choice(miss_span, size=n_miss, replace=False) + dbs) if n_miss > 0 else np.empty(
            0, dtype=np.int64)
        batch[r] = np.concatenate([hits, misses]).astype(np.int32)
    rng.shuffle(batch.ravel())
    return batch


def c1_fixture(Oracle):
    """8 req, prefill 256, topK 64, dbs 64, 2 layers, 10 steps, seed 42,
    miss ratio 0.5, one layer per step (layer = step % layers, xds_decode.py:225)."""
    req, prefill, K, dbs, layers, steps, seed = 8, 256, 64, 64, 2, 10, 42
    rng = np.random.default_rng(seed)
    oracles = []
    for _ in range(layers):
        o = Oracle([(prefill, r) for r in range(req)])
        for r in range(req):
            o.reset(r, prefill, dbs)
        oracles.append(o)
    topk = np.zeros((steps, req, K), np.int32)
    slots = np.zeros((steps, req, K), np.int32)
    miss = np.zeros((steps, req, K), np.int8)
    for st in range(steps):
        b = ref_sampler_batches(rng, req, K, prefill, dbs, 0.5)
        topk[st] = b
        o = oracles[st % layers]
        for r in range(req):
            s, m = o.update(r, b[r], prefill)
            slots[st, r] = norm_slots(s, padded_of(dbs))
            miss[st, r] = m
    return dict(req=req, prefill=prefill, top_k=K, dbs=dbs, layers=layers, steps=steps, seed=seed,
                topk=topk, slots=slots, is_miss=miss)


def random_fixture(Oracle, name, seed, req, prefill, dbs, K, steps, layers, miss_ratio, ext=0, invalid=0.0,
                   dup=0.0):
    """Seeded mixed workload: resident hits drawn from the oracle's current residents, misses
    from non-resident prefill positions, plus optional decode-extension positions
    (seq_len = prefill + ext), invalid entries and within-row duplicates."""
    rng = np.random.default_rng(seed)
    oracles = []
    for _ in range(layers):
        o = Oracle([(prefill, r) for r in range(req)])
        for r in range(req):
            o.reset(r, prefill, dbs)
        oracles.append(o)
    seq_len = prefill + ext
    topk = np.zeros((steps, layers, req, K), np.int32)
    slots = np.zeros((steps, layers, req, K), np.int32)
    miss = np.zeros((steps, layers, req, K), np.int8)
    for st in range(steps):
        for l in range(layers):
            o = oracles[l]
            for r in range(req):
                res = np.array(sorted(o.state[r]["t2s"].keys()), dtype=np.int64)
                nonres = np.setdiff1d(np.arange(prefill), res)
                n_miss = min(int(round(K * miss_ratio)), len(nonres))
                n_hit = min(K - n_miss, len(res))
                row = list(rng.choice(nonres, n_miss, replace=False)) + list(rng.choice(res, n_hit, replace=False))
                while len(row) < K:
                    row.append(int(rng.integers(0, prefill)))
                row = np.array(row, dtype=np.int64)
                if ext:
                    sel = rng.random(K) < 0.1
                    row[sel] = rng.integers(prefill, seq_len, size=int(sel.sum()))
                if invalid:
                    sel = rng.random(K) < invalid
                    row[sel] = rng.choice([-1, -7, seq_len, seq_len + 3], size=int(sel.sum()))
                if dup:
                    sel = np.nonzero(rng.random(K) < dup)[0]
                    for i in sel:
                        row[i] = row[int(rng.integers(0, K))]
                rng.shuffle(row)
                topk[st, l, r] = row.astype(np.int32)
                s, m = o.update(r, list(int(x) for x in row), seq_len)
                slots[st, l, r] = norm_slots(s, padded_of(dbs))
                miss[st, l, r] = m
    return dict(name=name, seed=seed, req=req, prefill=prefill, dbs=dbs, top_k=K, steps=steps, layers=layers,
                seq_len=seq_len, topk=topk, slots=slots, is_miss=miss)


RANDOM_CASES = [
    # name, seed, req, prefill, dbs, K, steps, layers, miss, ext, invalid, dup
    ("mixed_small", 11, 4, 300, 40, 24, 30, 2, 0.3, 20, 0.05, 0.05),
    ("mid", 12, 3, 2000, 1000, 256, 8, 1, 0.3, 0, 0.0, 0.0),
    ("wrap_heavy", 13, 2, 500, 16, 64, 20, 1, 0.8, 0, 0.0, 0.02),
    ("dbs_unaligned", 14, 3, 400, 50, 40, 25, 1, 0.5, 8, 0.02, 0.02),
    ("c2_like", 15, 2, 8192, 4096, 2048, 4, 1, 0.2, 0, 0.0, 0.0),
]


def layout_fixture(lay, align, compute_ht_size, row_word):
    grid = []
    for S in (1, 2, 16, 64):
        for N in (1, 2, 3, 7, 8):
            rows = list(range(0, 700)) + [4095, 4096, 65535, 131071, 2 ** 31 - 1]
            grid.append({"S": S, "N": N, "rows": rows, "node": [lay.node_of(r, S, N) for r in rows],
                         "seg_row": [lay.seg_row_of(r, S, N) for r in rows]})
    plsr = [[lr, n, lay.per_layer_seg_rows(lr, n)] for lr in (0, 1, 99, 100, 101, 1024, 131072) for n in
            (1, 2, 3, 8)]
    offs = []
    rng = np.random.default_rng(5)
    for _ in range(200):
        S = int(rng.choice([1, 16, 64]))
        N = int(rng.integers(1, 9))
        layer = int(rng.integers(0, 61))
        row = int(rng.integers(0, 131072))
        p = lay.per_layer_seg_rows(131072, N)
        offs.append([layer, row, S, N, p, 1152, lay.seg_offset(layer, row, S, N, p, 1152),
                     lay.seg_addr(0x10000, layer, row, S, N, p, 1152)])
    val = []
    for args in ((2, 1024, 1152, 1, 2), (2, 1024, 1151, 1, 2), (0, 1024, 1152, 1, 2), (2, 1024, 1152, 0, 2),
                 (2, 1024, 1152, 1, 65), (2, 0, 1152, 1, 2), (61, 131072, 1152, 64, 8)):
        try:
            lay.validate(*args)
            ok = True
        except ValueError:
            ok = False
        val.append([list(args), ok])
    ht = [[p, k, compute_ht_size(p, k)] for p, k in ((16, 8), (4112, 2048), (1024, 1024), (64, 64), (4096, 2048),
                                                     (8192, 2048), (65520, 2048), (65504, 2048))]
    al = [[v, a, align(v, a)] for v, a in ((1, 64), (64, 64), (65, 64), (514, 64), (4096, 16), (65518, 16))]
    rw = [[r, l, k, row_word(r, l, k)] for r, l, k in ((0, 0, 0), (1, 0, 0), (5, 1, 3), (2047, 1, 287),
                                                       (123456, 60, 100), (2 ** 20, 7, 287))]
    return {"grid": grid, "plsr": plsr, "seg_offset": offs, "validate": val, "ht_size": ht, "align": al,
            "row_word": rw}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("KVOPS_REFERENCE_DIR") or
                    os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), "reference"),
                    help="the reference tree (default: $KVOPS_REFERENCE_DIR, else ../reference beside the repo)")
    a = ap.parse_args()
    Oracle, row_word, align, compute_ht_size, lay = _load_ref(a.ref)
    with open(os.path.join(HERE, "sieve_kat.json"), "w") as f:
        json.dump(kat_cases(Oracle), f)
    np.savez_compressed(os.path.join(HERE, "sieve_c1_ref_sampler.npz"), **c1_fixture(Oracle))
    for case in RANDOM_CASES:
        fx = random_fixture(Oracle, *case)
        np.savez_compressed(os.path.join(HERE, "sieve_{}.npz".format(case[0])), **fx)
    with open(os.path.join(HERE, "layout.json"), "w") as f:
        json.dump(layout_fixture(lay, align, compute_ht_size, row_word), f)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
