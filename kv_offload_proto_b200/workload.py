"""Synthetic decode workloads for the hot path (input generation only; not on the hot path).

* ``ref_topk_batch``: the reference driver's topK draw (xds/xds_decode.py:213-223), so a run
  sees exactly what the reference driver would feed for a given seed.
* ``sample_topk_device``: the BASELINE configs' draw on the GPU — unique positions per request,
  hits drawn from the tokens currently resident in the hot buffer (read from the device SIEVE
  state), misses from non-resident prefill positions, optionally weighted by a finite Zipf pmf.
* ``stress_topk_uniform`` / ``stress_topk_zipf``: the SIEVE stress config's host draws
  numpy only, so the same seed and state give the same positions wherever
  they are drawn (the checksum fixture of the CPU model and the GPU run).
* ``row_word`` / ``fill_fingerprint``: the reference's row fingerprint (xds/xds_decode.py:18,60-63).
"""
import numpy as np

P1, P2, M1, M2 = 0x9E3779B1, 0x85EBCA77, 0x27220A95, 0x165667B1

__all__ = ["ref_topk_batch", "sample_topk_device", "zipf_pmf", "stress_topk_uniform", "stress_topk_zipf",
           "row_word", "fingerprint_rows", "P1", "P2", "M1", "M2"]


def ref_topk_batch(rng, req_num, top_k, prefill, dbs, miss_ratio):
    """One decode step's [req_num, top_k] int32 positions drawn like xds_decode.py:213-223:
    hits with replacement from [0, min(prefill, dbs)), misses without replacement from
    [dbs, prefill), then an in-place shuffle of the flattened batch."""
    hit_span = min(prefill, dbs)
    miss_span = max(prefill - dbs, 0)
    n_miss = int(top_k * miss_ratio) if miss_span > 0 else 0
    n_hit = top_k - n_miss
    out = np.empty((req_num, top_k), dtype=np.int32)
    for r in range(req_num):
        h = rng.integers(0, hit_span, size=n_hit) if n_hit > 0 else np.empty(0, dtype=np.int64)
        m = rng.choice(miss_span, size=n_miss, replace=False) + dbs if n_miss > 0 else np.empty(0, dtype=np.int64)
        out[r] = np.concatenate([h, m]).astype(np.int32)
    rng.shuffle(out.ravel())
    return out


def zipf_pmf(n, s, perm_seed):
    """Finite Zipf(s) pmf over positions [0, n): p[perm[i]] ∝ (i+1)^-s for a seeded permutation."""
    w = np.arange(1, n + 1, dtype=np.float64) ** (-float(s))
    w /= w.sum()
    perm = np.random.default_rng(perm_seed).permutation(n)
    p = np.empty(n, dtype=np.float64)
    p[perm] = w
    return p


def stress_topk_uniform(rng, tokens_rows, dbs, ctx, top_k, miss_ratio):
    """[R, top_k] int32: per request, round(miss_ratio * top_k) distinct positions drawn
    uniformly from the positions of [0, ctx) that are not resident in its token row
    (tokens_rows[r, :dbs]) and the rest from the resident ones, in shuffled order. One uniform
    key per position; the smallest keys of each group win (buffers are reused across rows)."""
    R = tokens_rows.shape[0]
    out = np.empty((R, top_k), np.int32)
    n_miss = int(round(miss_ratio * top_k))
    n_hit = top_k - n_miss
    keys, grp = np.empty(ctx), np.empty(ctx)
    res = np.zeros(ctx, bool)
    for r in range(R):
        tok = tokens_rows[r, :dbs]
        res[:] = False
        res[tok[(tok >= 0) & (tok < ctx)]] = True
        nres = int(np.count_nonzero(res))
        if nres < n_hit or ctx - nres < n_miss:
            raise ValueError("stress_topk_uniform: too few resident or non-resident positions")
        rng.random(out=keys)
        np.copyto(grp, keys)
        grp[res] = np.inf
        m = np.sort(np.argpartition(grp, n_miss - 1)[:n_miss]) if n_miss else np.empty(0, np.int64)
        np.copyto(grp, keys)
        grp[~res] = np.inf
        h = np.sort(np.argpartition(grp, n_hit - 1)[:n_hit]) if n_hit else np.empty(0, np.int64)
        row = np.concatenate([m, h])
        out[r] = row[rng.permutation(top_k)]
    return out


def stress_topk_zipf(rng, R, ctx, top_k, cdf, perm):
    """[R, top_k] int32: per request, the first top_k distinct positions of a stream of draws
    from the finite Zipf pmf whose cumulative sums are `cdf` (cdf[-1] == 1) over the ranks,
    mapped to positions by the permutation `perm` (zipf_pmf's construction). The popularity
    does not depend on the state, so the miss ratio follows from the SIEVE itself."""
    out = np.empty((R, top_k), np.int32)
    for r in range(R):
        chosen = np.empty(0, np.int64)
        seen = np.zeros(ctx, bool)
        while chosen.size < top_k:
            pos = perm[np.searchsorted(cdf, rng.random(2 * top_k), side="right")]
            _, first = np.unique(pos, return_index=True)
            pos = pos[np.sort(first)]
            pos = pos[~seen[pos]]
            seen[pos] = True
            chosen = np.concatenate([chosen, pos[:top_k - chosen.size]])
        out[r] = chosen
    return out


def zipf_cdf(n, s, perm_seed):
    """(cdf over ranks with cdf[-1] == 1, rank -> position permutation) of zipf_pmf(n, s)."""
    w = np.arange(1, n + 1, dtype=np.float64) ** (-float(s))
    cdf = np.cumsum(w / w.sum())
    cdf[-1] = 1.0
    return cdf, np.random.default_rng(perm_seed).permutation(n)


def sample_topk_device(tokens_layer, prefill, dbs, top_k, miss_ratio, generator, log_pmf=None):
    """[R, top_k] int32 unique positions per request on the tokens' device.

    tokens_layer: int32 [R, padded] — one layer's token rows (slot -> token, -1 empty) of the
    requests in batch order; prefill: int; log_pmf: optional float32 [prefill] log-weights
    (Gumbel-top-k gives weighted sampling without replacement). The split is
    round(miss_ratio*top_k) misses and the rest hits, capped by availability."""
    import torch
    dev = tokens_layer.device
    R = tokens_layer.shape[0]
    n_miss = int(round(miss_ratio * top_k))
    n_hit = top_k - n_miss
    resident = torch.zeros((R, prefill), dtype=torch.bool, device=dev)
    tok = tokens_layer[:, :dbs].long()
    valid = (tok >= 0) & (tok < prefill)
    rows = torch.arange(R, device=dev)[:, None].expand_as(tok)
    resident[rows[valid], tok[valid]] = True

    def gumbel():
        u = torch.rand((R, prefill), generator=generator, device=dev).clamp_(1e-12, 1.0)
        g = -torch.log(-torch.log(u))
        return g + log_pmf[None, :] if log_pmf is not None else g

    # Hits: weighted sample without replacement among residents (Gumbel-top-k).
    neg = torch.full((R, prefill), float("-inf"), device=dev)
    hv, hi = torch.topk(torch.where(resident, gumbel(), neg), n_hit, dim=1)
    chosen = torch.zeros((R, prefill), dtype=torch.bool, device=dev)
    chosen.scatter_(1, hi, hv > float("-inf"))
    # Then the rest of the row: chosen hits first, then non-residents, and only if a row runs
    # short of non-residents, leftover residents. topk keeps every position distinct.
    g = gumbel()
    score = torch.where(chosen, torch.full_like(g, float("inf")), torch.where(resident, g - 1.0e6, g))
    pos = torch.topk(score, top_k, dim=1).indices
    perm = torch.argsort(torch.rand((R, top_k), generator=generator, device=dev), dim=1)
    return torch.gather(pos, 1, perm).to(torch.int32).contiguous()


def row_word(row, layer, k):
    """Fingerprint word k of (row, layer) (xds/xds_decode.py:60-63)."""
    v = (row * P1 + layer * P2) * M1 ^ M2
    return (v + k * M1) & 0xFFFFFFFF


def fingerprint_rows(rows, layer, words):
    """uint32 [len(rows), words] fingerprint block, vectorised (xds_decode.py:177-181)."""
    rows = np.asarray(rows, dtype=np.uint64)
    v = (rows * np.uint64(P1) + np.uint64(layer * P2)) * np.uint64(M1) ^ np.uint64(M2)
    ramp = np.arange(words, dtype=np.uint64) * np.uint64(M1)
    return ((v[:, None] + ramp[None, :]) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
