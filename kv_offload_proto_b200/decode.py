"""B200 version of the reference's decode driver (xds/xds_decode.py): pool creation, prefill
(fingerprint fill, all-layer export, admission), the decode loop (top-K sampling ->
sieve_update -> batch_read -> wait -> fingerprint check) and the summary line, with the same
options and log lines, on CUDA.

    python -m kv_offload_proto_b200.decode [--layers 2 --req-num 8 --prefill 256 --topk 64 ...]

Differences from the reference, each on purpose:
  * the pool is a DevicePool on --segment-devices (GPU ids, -1 = pinned host memory) instead of
    an EMS pool; --ems-master, --rootinfo and --fatbin are accepted and ignored;
  * hot rows are per request by default (dst = hot + (request*dbs + slot)*rowBytes), so every
    gathered row is checkable; --shared-hot gives the reference's shared layout, in which
    requests overwrite each other's slots (and the check can fail for more than one request);
  * --oracle compares against a restatement of the reference's CPU model, with its
    decode-extension slots (-2-off) mapped to the kernel's padded+off before comparing, and
    one model state per (layer, request): the reference keeps one per request, which matches
    the kernels' per-layer state only when --layers is 1 (the loop alternates layers).
The top-K sampler is the reference's numpy sequence (workload.ref_topk_batch), so a seed
feeds the same positions the reference driver would.
"""
import argparse
import os
import sys
import time

import numpy as np

from .workload import M1, M2, P1, P2, ref_topk_batch, row_word


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="decode pipeline driver (kv offload hot path on B200)")
    p.add_argument("--ems-master", default="", help="accepted for compatibility; the pool is --segment-devices")
    p.add_argument("--device", type=int, default=0)
    p.add_argument("--rootinfo", default="", help="accepted for compatibility (no EID discovery here)")
    p.add_argument("--fatbin", default="", help="accepted for compatibility (kernels are linked in)")
    p.add_argument("--segment-devices", default="0", help="comma-separated segment placement (-1 = pinned host)")
    p.add_argument("--layers", type=int, default=2)
    p.add_argument("--layer-rows", type=int, default=1024)
    p.add_argument("--kv-lora-rank", type=int, default=512)
    p.add_argument("--qk-rope", type=int, default=64)
    p.add_argument("--stripe-rows", type=int, default=1)
    p.add_argument("--req-num", type=int, default=8)
    p.add_argument("--prefill", type=int, default=256)
    p.add_argument("--topk", type=int, default=64)
    p.add_argument("--device-buffer-size", type=int, default=64)
    p.add_argument("--miss-ratio", type=float, default=0.5)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--block-dim", type=int, default=8)
    p.add_argument("--oracle", action="store_true", help="compare every step with the CPU SIEVE model")
    p.add_argument("--shared-hot", action="store_true", help="the reference's shared hot rows (no per-request stride)")
    p.add_argument("--one-call", action="store_true", help="sieve_and_read (one launch) instead of the call pair")
    p.add_argument("--injective", action="store_true",
                   help="collision-free stripe map (with the reference map and --stripe-rows > 1 the rows of a "
                        "stripe share one segment row, so checks fail)")
    p.add_argument("--run-dir", default="./log")
    return p.parse_args(argv)


class _Logger:
    def __init__(self, run_dir):
        os.makedirs(run_dir, exist_ok=True)
        self.path = os.path.join(run_dir, "xds_decode.log")
        self._f = open(self.path, "w", encoding="utf-8")

    def __call__(self, msg):
        print(msg, flush=True)
        self._f.write(msg + "\n")
        self._f.flush()

    def close(self):
        self._f.close()


class SieveChecker:
    """The reference driver's CPU model of one SIEVE step per request (xds_decode.py:66-118):
    slot -> token map, visited set, hand; a token found in the map is a hit, any other prefill
    token a miss that evicts the first slot from the hand whose visited mark is clear. States
    are kept per key (here (layer, request), like the kernels' state tensors)."""

    def __init__(self):
        self.st = {}

    def reset(self, key, prefill, dbs):
        n = min(prefill, dbs)
        self.st[key] = {"prefill": prefill, "dbs": dbs, "hand": 0, "visited": set(),
                        "slot_tok": {s: s for s in range(n)}, "tok_slot": {s: s for s in range(n)}}

    def update(self, key, topk_row, seq_len, padded):
        """(slots, is_miss) for one request; decode-extension positions -> padded + offset."""
        s = self.st[key]
        slots, miss = [], []
        for t in (int(x) for x in topk_row):
            if t < 0 or t >= seq_len:
                slots.append(-1)
                miss.append(0)
            elif t >= s["prefill"]:
                slots.append(padded + (t - s["prefill"]))
                miss.append(0)
            elif t in s["tok_slot"]:
                h = s["tok_slot"][t]
                s["visited"].add(h)
                slots.append(h)
                miss.append(0)
            else:
                h = s["hand"]
                while h in s["visited"]:
                    s["visited"].discard(h)
                    h = (h + 1) % s["dbs"]
                old = s["slot_tok"].get(h)
                if old is not None:
                    del s["tok_slot"][old]
                s["slot_tok"][h] = t
                s["tok_slot"][t] = h
                s["visited"].add(h)
                s["hand"] = (h + 1) % s["dbs"]
                slots.append(h)
                miss.append(1)
        return slots, miss


def _fill_fingerprints(torch, hbm, layer, rows, row_words32):
    """hbm[layer, rows] = fingerprint words (xds_decode.py:177-181) computed on the GPU (the
    uint64 arithmetic of the reference in int64, whose low 32 bits are the same)."""
    r = torch.as_tensor(rows, dtype=torch.int64, device=hbm.device)
    v = ((r * P1 + layer * P2) * M1) ^ M2
    k = torch.arange(row_words32, dtype=torch.int64, device=hbm.device) * M1
    w = (v[:, None] + k[None, :]) & 0xFFFFFFFF
    hbm[layer, r] = torch.where(w >= 1 << 31, w - (1 << 32), w).to(torch.int32)  # same 32 bits


def main(argv=None):
    args = parse_args(argv)
    log = _Logger(args.run_dir)
    rng = np.random.default_rng(args.seed)
    row_words = args.kv_lora_rank + args.qk_rope
    row_bytes = (row_words * 2 + 127) // 128 * 128
    words32 = row_bytes // 4
    dbs = args.device_buffer_size
    if dbs >= args.prefill:
        log("[xds][WARN] device-buffer-size >= prefill: no misses, --miss-ratio has no effect")
    import torch

    import kv_offload_proto_b200 as kp
    from .offload import XdsOffloadCoordinator
    from .pool import DevicePool

    dev = torch.device("cuda", args.device)
    torch.cuda.set_device(dev)
    mod = kp.install_kvops_ext()
    mod.init(args.device, "")
    log("[xds] config: layers={} layerRows={} rowWords={} rowBytes={} stripe={} reqs={} prefill={} topK={} "
        "dbs={} missRatio={}".format(args.layers, args.layer_rows, row_words, row_bytes, args.stripe_rows,
                                     args.req_num, args.prefill, args.topk, dbs, args.miss_ratio))
    strided = not args.shared_hot
    if strided and args.req_num * dbs > args.layer_rows:
        log("[xds][ERROR] per-request hot rows need req-num*device-buffer-size <= layer-rows (or --shared-hot)")
        return 1
    hbm = torch.zeros((args.layers, args.layer_rows, words32), dtype=torch.int32, device=dev)
    devices = [int(x) for x in args.segment_devices.split(",") if x.strip() != ""]
    pool = DevicePool(args.device, args.layers, args.layer_rows, row_bytes, args.stripe_rows, segment_devices=devices,
                      injective=args.injective)
    log("[xds] pool ready: nodes={} perLayerSegRows={} channels={} fatbin={}".format(
        pool.node_num, pool.per_layer_seg_rows, len(pool.channels), "(linked in)"))
    coord = XdsOffloadCoordinator(dev, args.layers, args.req_num, dbs, args.topk, args.req_num, args.prefill)
    log("[xds] coordinator: padded={} visitedStrideB={} htSize={}".format(
        coord.padded_buffer_size, coord.visited_stride_b, coord.ht_size))

    # prefill: row allocation (contiguous runs), fingerprint fill, all-layer export, admission
    allocator = pool.make_allocator()
    host_bases = []
    t0 = time.perf_counter()
    for _ in range(args.req_num):
        rows = allocator.alloc(args.prefill)
        assert rows == list(range(rows[0], rows[0] + args.prefill)), "row contiguity contract broken"
        host_bases.append(rows[0])
        for layer in range(args.layers):
            _fill_fingerprints(torch, hbm, layer, rows, words32)
    st = pool.batch_write_alllayers(0, args.req_num * args.prefill, hbm[0, 0], args.layer_rows * row_bytes)
    pool.wait(st)
    t_export = time.perf_counter() - t0
    log("[xds] prefill export: {} rows x {} layers = {} B in {:.1f} us".format(
        args.req_num * args.prefill, args.layers, args.layers * args.req_num * args.prefill * row_bytes,
        t_export * 1e6))
    checker = SieveChecker() if args.oracle else None
    for r in range(args.req_num):
        coord.admit_request(r, r, args.prefill, host_bases[r])
        if checker is not None:
            for layer in range(args.layers):
                checker.reset((layer, r), args.prefill, dbs)
    hbm.zero_()  # the decode loop must bring every checked row back from the pool

    seq_lens = torch.full((args.req_num,), args.prefill, dtype=torch.int32, device=dev)
    req_pool_indices = torch.arange(args.req_num, dtype=torch.int64, device=dev)
    coord.set_batch(req_pool_indices, seq_lens)
    stride = dbs if strided else 0
    total_miss, t_read_total = 0, 0.0
    stream = torch.cuda.current_stream(dev).cuda_stream
    for step in range(args.steps):
        batch = ref_topk_batch(rng, args.req_num, args.topk, args.prefill, dbs, args.miss_ratio)
        topk = torch.from_numpy(batch).to(dev)
        layer = step % args.layers
        hot = hbm[layer]
        t0 = time.perf_counter()
        if args.one_call:
            st = pool.sieve_and_read(coord, layer, topk, hot, stream, args.block_dim, hot_req_stride_rows=stride)
        else:
            coord.sieve_update(layer, topk, block_dim=args.block_dim)
            st = pool.batch_read(layer, topk, req_pool_indices, coord.req_host_base, coord.top_k_device_slots,
                                 coord.is_miss, coord.num_real, hot, args.req_num, args.topk, stream, args.block_dim,
                                 hot_req_stride_rows=stride)
        pool.wait(st, block_dim=args.block_dim)
        dt = time.perf_counter() - t0
        t_read_total += dt
        miss_cnt = int(coord.miss_count().item())
        total_miss += miss_cnt
        slots_h = coord.top_k_device_slots[:args.req_num].cpu().numpy()
        miss_h = coord.is_miss[:args.req_num].cpu().numpy()
        if checker is not None:
            for r in range(args.req_num):
                exp_slots, exp_miss = checker.update((layer, r), batch[r], args.prefill, coord.padded_buffer_size)
                if not np.array_equal(miss_h[r], np.array(exp_miss, np.int8)):
                    log("[xds][ERROR] oracle is_miss mismatch step={} req={}".format(step, r))
                    return 1
                if not np.array_equal(slots_h[r], np.array(exp_slots, np.int32)):
                    log("[xds][ERROR] oracle slots mismatch step={} req={}".format(step, r))
                    return 1
        # spot check: the first miss row of every request holds its fingerprint
        hot_h = hot.cpu().numpy().view(np.uint32)
        checked = 0
        for r in range(args.req_num):
            pos = np.nonzero(miss_h[r])[0]
            if pos.size == 0:
                continue
            k = int(pos[0])
            slot = int(slots_h[r, k])
            if slot < 0 or slot >= dbs:
                continue
            row = host_bases[r] + int(batch[r][k])
            got = int(hot_h[r * stride + slot, 0])
            if got != row_word(row, layer, 0):
                log("[xds][ERROR] verify failed step={} layer={} req={} token={} row={} slot={} expect={} got={}".format(
                    step, layer, r, int(batch[r][k]), row, slot, row_word(row, layer, 0), got))
                return 1
            checked += 1
        log("[xds] step {}: layer={} miss={} rows in {:.1f} us (checked={})".format(step, layer, miss_cnt, dt * 1e6,
                                                                                  checked))
    if total_miss > 0:
        log("[xds] summary: imported {} miss rows, avg {:.1f} us/row, aggregate {:.2f} GB/s".format(
            total_miss, t_read_total * 1e6 / total_miss, total_miss * row_bytes / t_read_total / 1e9))
    else:
        log("[xds] summary: no miss rows imported")
    pool.destroy()
    log("[xds] all done, log: {}".format(log.path))
    log.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
