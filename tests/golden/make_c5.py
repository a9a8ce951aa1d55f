"""Checksum fixture of the SIEVE stress config from the C restatement of the
reference kernel (oracle/kvoracle.c, itself pinned to the reference's Python oracle by
make_golden.py's fixtures).

  python tests/golden/make_c5.py [--threads N] [--steps 50] [--reqs 1024]

1024 requests, hot buffer 65518 slots (padded 65520, table 262144 cells), topK 2048, context
131072 (prefill = context, identity admission), one layer, 50 steps, two draws:
  * uniform: per step and request, round(0.9 * 2048) positions drawn from the non-resident
    positions and the rest from the resident ones (workload.stress_topk_uniform, seed 123);
  * zipf: 2048 distinct positions per request from a finite Zipf(0.8) popularity over the
    context (workload.stress_topk_zipf, permutation seed 123, draw seed 124).
The draws are numpy-only, so bench.py --config c5 redraws the same positions from the state
it reads back from the GPU and compares its outputs with these digests step by step. The full
outputs (0.5 GB per draw) are not kept; per step the file holds the miss count and the SHA-256
of the slots (int32) and miss flags (int8), and at the end the digests of the state tensors.
"""
import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from kv_offload_proto_b200.workload import stress_topk_uniform, stress_topk_zipf, zipf_cdf  # noqa: E402

C5 = dict(reqs=1024, dbs=65518, top_k=2048, ctx=131072, steps=50, seed=123, miss_ratio=0.9, zipf=0.8)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def draws(dist, cfg):
    """The draw function of `dist`: f(rng, tokens_rows) -> [R, top_k] int32, and its seed."""
    if dist == "uniform":
        return (lambda rng, tok: stress_topk_uniform(rng, tok, cfg["dbs"], cfg["ctx"], cfg["top_k"],
                                                     cfg["miss_ratio"])), cfg["seed"]
    cdf, perm = zipf_cdf(cfg["ctx"], cfg["zipf"], cfg["seed"])
    return (lambda rng, tok: stress_topk_zipf(rng, tok.shape[0], cfg["ctx"], cfg["top_k"], cdf, perm)), \
        cfg["seed"] + 1


def run(dist, cfg, threads, log=print):
    R, dbs, K, ctx = cfg["reqs"], cfg["dbs"], cfg["top_k"], cfg["ctx"]
    st = oracle.SieveState(1, R, dbs, K)
    for r in range(R):
        st.admit(r, ctx)
    draw, seed = draws(dist, cfg)
    rng = np.random.default_rng(seed)
    pool, seq = np.arange(R, dtype=np.int64), np.full(R, ctx, np.int32)
    steps = []
    for step in range(cfg["steps"]):
        t0 = time.time()
        topk = draw(rng, st.tokens[0])
        slots, miss = st.update(0, topk, pool, seq, nthreads=threads)
        steps.append({"misses": int(miss.sum()), "slots": sha(slots), "is_miss": sha(miss), "topk": sha(topk)})
        log("{} step {} misses {} ({:.1f} s)".format(dist, step, steps[-1]["misses"], time.time() - t0))
    final = {"tokens": sha(st.tokens[0]), "visited": sha(st.visited[0]), "ht": sha(st.ht[0]),
             "hand": sha(st.hand[0][:, 0].copy())}
    return {"steps": steps, "final": final}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--steps", type=int, default=C5["steps"])
    ap.add_argument("--reqs", type=int, default=C5["reqs"])
    ap.add_argument("--out", default=os.path.join(HERE, "c5_checksums.json"))
    a = ap.parse_args()
    cfg = dict(C5, steps=a.steps, reqs=a.reqs)
    out = {"config": cfg, "draws": {}}
    for dist in ("uniform", "zipf"):
        out["draws"][dist] = run(dist, cfg, a.threads, log=lambda m: print(m, flush=True))
        with open(a.out, "w") as f:
            json.dump(out, f, indent=1)
    print("written", a.out)


if __name__ == "__main__":
    main()
