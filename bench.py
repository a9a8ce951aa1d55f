"""Benchmark of the decode-time KV hot path: SIEVE miss detection + miss-row gather per
layer-step, BASELINE config 2 (DSA/MLA decode: 64 requests x 8192-token context, 61 layers,
topK 2048, hot buffer 4096 slots, miss ratio 0.2, 1152-byte fp16 rows N(0,1), seed 1).

A step is one decode step: every layer runs sieve_update then the gather of its miss rows
(the reference driver's per-layer sequence, xds/xds_decode.py:225-233). The metric is the
reference's own: miss rows x 1152 B / (sieve + gather) time (xds_decode.py:226-233,280), in
GB/s; p50/p99 microseconds per layer-step are reported beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

At N=1 the pool is one segment in the GPU's own HBM. Under torchrun with N>1 ranks, every
rank runs its own 64 requests (weak scaling) and its pool is striped S=1 over the other N-1
GPUs' HBM (segments mapped through CUDA IPC, read in-kernel over NVLink/NVSwitch); there is no
collective on the data path. `--impl reference` times the reference's CPU path (the C
restatement of its sieve plus a host memcpy gather following its stripe map) on rank 0.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

ROW_BYTES = 1152
CFG = dict(name="c2_dsa_decode", requests=64, ctx=8192, layers=61, top_k=2048, dbs=4096, miss_ratio=0.2,
           stripe_rows=1, seed=1)
METRIC = "miss-row import GB/s (sieve+gather, per layer-step)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--layers", type=int, default=CFG["layers"], help="layers per decode step (61 = config 2)")
    ap.add_argument("--path", choices=["auto", "coop", "fused", "split"], default="auto",
                    help="layer-step path of sieve_and_read (auto: cooperative when it fits)")
    ap.add_argument("--no-graph", action="store_true",
                    help="time the per-call loop only (default: `value` from decode steps replayed as CUDA graphs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clock and clock-event reasons sampled over the timed region (read-only): NVML every
    5 ms from a thread, else nvidia-smi every 200 ms. The GPU is found by its UUID, so the
    sample is of the device this process runs on whatever CUDA_VISIBLE_DEVICES says."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, torch, local):
        self.uuid = None
        try:
            u = str(torch.cuda.get_device_properties(local).uuid)
            self.uuid = u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            pass
        self.local = local
        self.samples, self.max_mhz, self.reasons = [], None, set()
        self.thread = self.proc = None
        self.stop_flag = False

    def _nvml_loop(self, nv, h):
        while not self.stop_flag:
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                for bit, name in self.REASONS.items():
                    if bits & bit:
                        self.reasons.add(name)
            except Exception:
                return
            time.sleep(0.005)

    def start(self):
        try:
            import threading

            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByUUID(self.uuid) if self.uuid else nv.nvmlDeviceGetHandleByIndex(self.local)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h), daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.out = open(os.path.join("/tmp", "kvb_clocks_{}.csv".format(os.getpid())), "w+")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.uuid or str(self.local),
                                          "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                                          "clocks_event_reasons.hw_thermal_slowdown,"
                                          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(5)
            src = "nvml 5 ms"
        elif self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.out.seek(0)
            names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
            for line in self.out.read().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 6:
                    continue
                try:
                    self.samples.append(float(f[0]))
                    self.max_mhz = float(f[1])
                except ValueError:
                    continue
                for name, v in zip(names, f[2:6]):
                    if v.lower().startswith("active"):
                        self.reasons.add(name)
            self.out.close()
            src = "nvidia-smi 200 ms"
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"]}
        sm = self.samples
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "samples": len(sm),
                "min_sm_mhz": min(sm) if sm else None, "source": src, "reasons": sorted(self.reasons)}


def pct(xs, q):
    xs = sorted(xs)
    if not xs:
        return None
    i = min(len(xs) - 1, max(0, int(round(q / 100.0 * (len(xs) - 1)))))
    return xs[i]


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def state_bytes(padded, vis, ht_size):
    """Bytes of one request's SIEVE state: token row, bitmap, table, hand word."""
    return padded * 4 + vis + ht_size * 2 + 4


def build_pool(mod, torch, dist, rank, world, local, L, layer_rows, seed):
    """Segments of this rank's pool (kv_offload_proto_b200.cluster): every rank allocates and
    fills the segments it hosts and maps its own pool's segments through CUDA IPC handles."""
    from kv_offload_proto_b200.cluster import exchange_handles, hosted_segments, pool_nodes
    from kv_offload_proto_b200.pool import device_view, per_layer_seg_rows
    nodes = pool_nodes(rank, world)
    seg_bytes = L * per_layer_seg_rows(layer_rows, len(nodes)) * ROW_BYTES
    hosted = {}
    for owner, idx in hosted_segments(rank, world):
        addr = mod.segment_alloc(local, seg_bytes)
        view = device_view(addr, seg_bytes, "cuda:{}".format(local)).view(torch.float16)
        gen = torch.Generator(device="cuda:{}".format(local)).manual_seed(seed * 7919 + owner * 131 + idx)
        chunk = 1 << 29
        for o in range(0, view.numel(), chunk):
            view[o:o + chunk].normal_(generator=gen)
        hosted[(owner, idx)] = addr
    if world == 1:
        return [hosted[(rank, 0)]], nodes, list(hosted.values()), []
    handles = exchange_handles(dist, rank, world, {k: mod.ipc_get_handle(a) for k, a in hosted.items()})
    mine = [mod.ipc_open_handle(local, h) for h in handles]
    return mine, nodes, list(hosted.values()), list(mine)


def run_b200(args):
    import datetime

    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    import kv_offload_proto_b200 as kp
    from kv_offload_proto_b200.offload import XdsOffloadCoordinator
    from kv_offload_proto_b200.pool import DevicePool
    from kv_offload_proto_b200.workload import sample_topk_device

    mod = kp.install_kvops_ext()
    mod.init(local, "")
    dev = torch.device("cuda", local)
    R, ctx, K, dbs, miss = CFG["requests"], CFG["ctx"], CFG["top_k"], CFG["dbs"], CFG["miss_ratio"]
    L = args.layers
    layer_rows = R * ctx
    W, S = args.warmup, args.steps
    T = W + S

    def barrier():
        if world > 1:
            dist.barrier()

    seg_addrs, nodes, hosted, opened = build_pool(mod, torch, dist, rank, world, local, L, layer_rows, CFG["seed"])
    pool = DevicePool(local, L, layer_rows, ROW_BYTES, CFG["stripe_rows"], segment_devices=nodes,
                      segment_addrs=seg_addrs)
    co = XdsOffloadCoordinator(dev, L, R, dbs, K, R, ctx)
    hot = torch.empty((L, R * dbs * ROW_BYTES), dtype=torch.uint8, device=dev)
    pre, base = [ctx] * R, [r * ctx for r in range(R)]
    co.admit_all(pre, base)
    co.set_batch(torch.arange(R, dtype=torch.int64, device=dev), torch.full((R,), ctx, dtype=torch.int32, device=dev))

    # Inputs: BASELINE config 2 draws (unique positions; hits from the current residents), made
    # once by running the device SIEVE ahead; the replay below starts from the same admitted
    # state, so every layer-step sees exactly the state its draw was made against.
    gen = torch.Generator(device=dev).manual_seed(CFG["seed"] * 1000 + rank)
    topk = torch.empty((T, L, R, K), dtype=torch.int32, device=dev)
    misses = torch.zeros((T, L), dtype=torch.int64, device=dev)
    for s in range(T):
        for l in range(L):
            topk[s, l] = sample_topk_device(co.device_buffer_tokens[l, :R], ctx, dbs, K, miss, gen)
            co.sieve_update(l, topk[s, l])
            misses[s, l] = co.is_miss.sum()
    misses_h = misses.cpu().numpy()
    co.admit_all(pre, base)

    stream = torch.cuda.current_stream(dev).cuda_stream
    # The public one-call layer-step (DevicePool.sieve_and_read, path "auto"): one cooperative
    # launch whose non-SIEVE CTAs copy each request's miss rows as soon as its hand sweep is
    # done (or, where that does not fit, the SIEVE kernel and the gather as its programmatic
    # dependent).
    def layer_step(s, l):
        pool.sieve_and_read(co, l, topk[s, l], hot[l], stream, 1, hot_req_stride_rows=dbs, path=args.path)

    def timed_pass(graphs):
        """W untimed then S timed steps from the admitted state; device time of the S steps,
        per-layer-step times, clock record. graphs: replay one captured graph per step, else
        one call per layer with CUDA events around each call."""
        co.admit_all(pre, base)
        for s in range(W):
            if graphs:
                graphs[s].replay()
            else:
                for l in range(L):
                    layer_step(s, l)
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(S * (1 if graphs else L))]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks = ClockSampler(torch, local)
        clocks.start()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.nvtx.range_push("timed" if graphs or args.no_graph else "per_call")  # profiler selection
        t0.record()
        for s in range(W, T):
            if graphs:
                e = evs[s - W]
                e[0].record()
                graphs[s].replay()
                e[1].record()
                continue
            for l in range(L):
                e = evs[(s - W) * L + l]
                e[0].record()
                layer_step(s, l)
                e[1].record()
        t1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        barrier()
        clk = clocks.stop()
        assert int(co.is_miss.sum().item()) == int(misses_h[T - 1, L - 1]), "replay diverged from the input pass"
        return (t0.elapsed_time(t1) * 1e-3, [e[0].elapsed_time(e[1]) * 1e3 / (L if graphs else 1) for e in evs], clk)

    # Per call: the public one-call API per layer, status words published (what a caller of
    # sieve_and_read gets without graphs).
    elapsed_pc, step_us_pc, clk_pc = timed_pass(None)
    path = mod.last_step_path()
    fused = path in ("coop", "fused")  # one kernel per layer-step
    graphs = None
    if not args.no_graph:  # one CUDA graph per decode step (its layers' calls), replayed in order
        from kv_offload_proto_b200.graph import StepGraph
        graphs = [StepGraph(pool, co, hot, L, path=args.path, hot_req_stride_rows=dbs, topk=topk[s]) for s in range(T)]
        elapsed, step_us, clk = timed_pass(graphs)
    else:
        elapsed, step_us, clk = elapsed_pc, step_us_pc, clk_pc
    last = int(co.is_miss.sum().item())
    miss_rows = int(misses_h[W:].sum())
    per_call = {"value": miss_rows * ROW_BYTES / elapsed_pc / 1e9, "unit": "GB/s",
                "ms_per_step": elapsed_pc * 1e3 / S, "step_us": step_us_pc, "clocks": clk_pc}

    # Kernel durations for the roofline: the same steps replayed from the admitted state with
    # an event around each kernel (an event between the two kernels also stops the gather from
    # launching early, so this pass is not the timed one).
    co.admit_all(pre, base)
    kev = []
    for s in range(T):
        for l in range(L):
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record()
            if fused:
                layer_step(s, l)
                e[1].record()
            else:
                co.sieve_update(l, topk[s, l], stream=stream)
                e[1].record()
                pool.batch_read(l, topk[s, l], co._req_pool_indices, co.req_host_base, co.top_k_device_slots,
                                co.is_miss, co.num_real, hot[l], R, K, stream, 1, fused=True, hot_req_stride_rows=dbs)
            e[2].record()
            if s >= W:
                kev.append(e)
    torch.cuda.synchronize()
    assert int(co.is_miss.sum().item()) == last, "kernel pass diverged"
    if fused:
        kernels = {"sieve_fast_kernel<{}>".format(2 if path == "coop" else 1):
                   [e[0].elapsed_time(e[1]) * 1e3 for e in kev]}
    else:
        kernels = {"sieve_fast_kernel": [e[0].elapsed_time(e[1]) * 1e3 for e in kev],
                   "gather_kernel": [e[1].elapsed_time(e[2]) * 1e3 for e in kev]}

    e2e = None
    if not args.no_e2e:
        e2e_pc = run_e2e(torch, co, pool, hot, topk, misses_h, pre, base, L, W, S, R, K, dbs, dev, args.path)
        if args.no_graph:
            e2e = dict(e2e_pc, api="sieve_and_read per layer, host polls the status words")
        else:
            e2e = run_e2e_graph(torch, co, pool, hot, topk, misses_h, pre, base, L, W, S, R, K, dbs, dev,
                                args.path)
            e2e["per_call"] = {k: e2e_pc[k] for k in ("value", "unit", "ms_per_step")}
            e2e["per_call"]["api"] = "sieve_and_read per layer, host polls the status words after each"

    res = dict(elapsed=elapsed, miss_rows=miss_rows, kernels=kernels, step_us=step_us, e2e=e2e, clocks=clk,
               nodes=len(nodes), fused=fused, path=path, graph=bool(graphs), per_call=per_call,
               launches=len(kev))
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, res)
    else:
        gathered = [res]
    for a in opened:
        mod.ipc_close_handle(a)
    barrier()
    for a in hosted:
        mod.segment_free(a)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        report_b200(args, world, gathered, co)


def run_e2e(torch, co, pool, hot, topk, misses_h, pre, base, L, W, S, R, K, dbs, dev, path):
    """The same decode steps through the public API with host inputs: each step copies its
    topK tensors from pinned host memory, runs every layer's sieve_and_read (the reference
    driver's sieve_update + batch_read pair, xds_decode.py:226-236, in one call) and waits on
    the status slots, then reads the per-layer miss counts back to the host. Host wall clock
    around the K timed steps."""
    T = W + S
    topk_host = topk.cpu().pin_memory()
    buf = torch.empty((L, R, K), dtype=torch.int32, device=dev)
    counts = torch.zeros(L, dtype=torch.int64, device=dev)
    counts_h = torch.zeros(L, dtype=torch.int64).pin_memory()
    co.admit_all(pre, base)
    stream = torch.cuda.current_stream(dev)

    def step(s):
        buf.copy_(topk_host[s], non_blocking=True)
        for l in range(L):
            st = pool.sieve_and_read(co, l, buf[l], hot[l], stream.cuda_stream, 1, hot_req_stride_rows=dbs,
                                     path=path)
            pool.wait(st)
            counts[l] = co.is_miss.sum()
        counts_h.copy_(counts, non_blocking=True)
        stream.synchronize()

    for s in range(W):
        step(s)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for s in range(W, T):
        step(s)
    dt = time.perf_counter() - t0
    assert np.array_equal(counts_h.numpy(), misses_h[T - 1]), "e2e replay diverged"
    rows = int(misses_h[W:].sum())
    return {"value": rows * ROW_BYTES / dt / 1e9, "unit": "GB/s", "ms_per_step": dt * 1e3 / S,
            "h2d_bytes_per_step": L * R * K * 4, "d2h_bytes_per_step": L * 8, "rows": rows, "seconds": dt}


def run_e2e_graph(torch, co, pool, hot, topk, misses_h, pre, base, L, W, S, R, K, dbs, dev, path):
    """The same decode steps through the public graph API (StepGraph, one replay per decode
    step) with host inputs, as a serving loop runs them: step s's top-K tensors are copied from
    pinned host memory on a copy stream while step s-1 replays (two input buffers, two captured
    graphs); the step's result, its last layer's miss count, is reduced inside the graph, read
    back to pinned host memory and checked on the host once the step is done. (A reduction after
    every layer would put a small kernel between each pair of cooperative launches, ~15 us per
    layer of launch gaps, which a decode step does not need.) Host wall clock from the first
    timed step's input copy to the last timed step's result."""
    from kv_offload_proto_b200.graph import StepGraph
    T = W + S
    topk_host = topk.cpu().pin_memory()
    bufs = [torch.empty((L, R, K), dtype=torch.int32, device=dev) for _ in range(2)]
    counts = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(2)]
    counts_h = torch.zeros((T, 1), dtype=torch.int64).pin_memory()

    def last_layer_count(c):
        return lambda l: torch.sum(co.is_miss.view(-1), 0, dtype=torch.int64, out=c[0]) if l == L - 1 else None

    graphs = [StepGraph(pool, co, hot, L, path=path, hot_req_stride_rows=dbs, topk=bufs[i],
                        after_layer=last_layer_count(counts[i])) for i in range(2)]
    co.admit_all(pre, base)
    main = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(device=dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    buf_free = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(T)]

    def stage(s):  # step s's inputs into buffer s % 2, once step s - 2 has stopped reading it
        i = s % 2
        if s >= 2:
            copy.wait_event(buf_free[i])
        with torch.cuda.stream(copy):
            bufs[i].copy_(topk_host[s], non_blocking=True)
        in_ready[i].record(copy)

    def run(s):
        i = s % 2
        main.wait_event(in_ready[i])
        graphs[i].replay()
        buf_free[i].record(main)
        counts_h[s].copy_(counts[i], non_blocking=True)
        done[s].record(main)

    def check(s):
        done[s].synchronize()
        assert int(counts_h[s, 0]) == int(misses_h[s, L - 1]), "e2e replay diverged at step %d" % s

    def steps(lo, hi):
        stage(lo)
        for s in range(lo, hi):
            run(s)
            if s + 1 < hi:
                stage(s + 1)
            if s > lo:
                check(s - 1)
        check(hi - 1)

    steps(0, W)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    steps(W, T)
    dt = time.perf_counter() - t0
    rows = int(misses_h[W:].sum())
    return {"value": rows * ROW_BYTES / dt / 1e9, "unit": "GB/s", "ms_per_step": dt * 1e3 / S,
            "h2d_bytes_per_step": L * R * K * 4, "d2h_bytes_per_step": 8, "rows": rows, "seconds": dt,
            "api": "StepGraph.replay per decode step; inputs copied from pinned host memory on a copy stream "
                   "during the previous step; the step's last-layer miss count read back and checked every step"}


def traffic_per_unit():
    """DRAM bytes per unit measured by ncu (profiles/traffic.json), if captured."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return {}
    with open(path) as f:
        return json.load(f)


def report_b200(args, world, gathered, co):
    hbm_peak, peak_kind = peaks()
    R, K = CFG["requests"], CFG["top_k"]
    L = args.layers
    elapsed = max(g["elapsed"] for g in gathered)
    miss_rows = sum(g["miss_rows"] for g in gathered)
    value = miss_rows * ROW_BYTES / elapsed / 1e9
    g0 = gathered[0]
    kern = {k: sum(v) / len(v) for k, v in g0["kernels"].items()}
    rows_per_launch = g0["miss_rows"] / g0["launches"]
    remote = world > 1
    tr = traffic_per_unit()
    sb = state_bytes(co.padded_buffer_size, co.visited_stride_b, co.ht_size)
    s_bytes = R * (2 * sb + 9 * K)  # SIEVE state read + written, topK read, slots + flags written
    # Gather: payload read + write (local pool), plus 9 B of metadata per position and 16 B per
    # request; from peer pools the bound is the NVLink ingress of the payload.
    meta = R * K * 9 + R * 16
    hbm_gather = rows_per_launch * 2 * ROW_BYTES + meta

    def roof(kernel, bound, nbytes, avg_us, peak, peak_source, traffic):
        return {"kernel": kernel, "bound": bound, "achieved": nbytes / (avg_us * 1e-6) / 1e9, "peak": peak,
                "unit": "GB/s", "frac": nbytes / (avg_us * 1e-6) / 1e9 / peak, "peak_source": peak_source,
                "traffic": traffic, "algorithmic_bytes": nbytes, "avg_us": avg_us}

    if g0["fused"]:
        (name, t), = kern.items()
        if g0["graph"]:  # one kernel per layer-step: the timed region's device time per launch
            t = max(g["elapsed"] for g in gathered) * 1e6 / (L * args.steps)
        hbm_bytes = s_bytes + hbm_gather
        if remote:  # rows cross NVLink; this GPU's HBM holds the state and the hot rows
            dominant = roof(name, "nvlink", rows_per_launch * ROW_BYTES, t, 770.0,
                            "peer copy 770 GB/s per direction (measured on this pool)", None)
            other = roof(name + ", HBM side", "hbm", s_bytes + rows_per_launch * ROW_BYTES + meta, t, hbm_peak,
                         peak_kind, None)
        else:
            traffic = None
            if "coop_per_launch" in tr:  # measured at 33,477 rows per launch; scaled by rows
                traffic = tr["coop_per_launch"] * rows_per_launch / 33477.0
            dominant = roof(name, "hbm", hbm_bytes, t, hbm_peak, peak_kind, traffic)
            other = None
    else:
        rs = roof("sieve_fast_kernel", "hbm", s_bytes, kern["sieve_fast_kernel"], hbm_peak, peak_kind,
                  tr["sieve_per_request"] * R if "sieve_per_request" in tr else None)
        rg = roof("gather_kernel", "hbm", hbm_gather, kern["gather_kernel"], hbm_peak, peak_kind,
                  tr["gather_per_row"] * rows_per_launch if "gather_per_row" in tr else None)
        dominant, other = (rs, rg) if rs["avg_us"] >= rg["avg_us"] else (rg, rs)
    steps_all = [x for g in gathered for x in g["step_us"]]
    out = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic",
        "config": {"workload": CFG["name"], "requests_per_gpu": R, "ctx": CFG["ctx"], "layers": L, "top_k": K,
                   "hot_slots": CFG["dbs"], "miss_ratio": CFG["miss_ratio"], "row_bytes": ROW_BYTES,
                   "stripe_rows": CFG["stripe_rows"],
                   "pool": "local HBM segment" if not remote else "striped over the other {} GPUs' HBM".format(
                       world - 1),
                   "l2": "inputs larger than L2 (SIEVE state {:.0f} MB, pool {:.1f} GB per GPU)".format(
                       L * R * sb / 1e6, L * R * CFG["ctx"] * ROW_BYTES / 1e9),
                   "step": "one decode step = {} layers x sieve_and_read, path {} ({}){}".format(
                       L, g0["path"], {"coop": "one cooperative kernel: SIEVE CTAs + row-copy CTAs",
                                       "fused": "one kernel: SIEVE + bulk-copy warp",
                                       "split": "SIEVE kernel + gather as programmatic dependent"}[g0["path"]],
                       ", each step replayed as one CUDA graph (no status words; completion on the stream)"
                       if g0["graph"] else "")},
        "p50_us_per_layer_step": pct(steps_all, 50), "p99_us_per_layer_step": pct(steps_all, 99),
        "graph": g0["graph"],
        "per_layer_step_timing": "decode-step graph time / layers" if g0["graph"] else "CUDA events around each call",
        "per_call": {"value": sum(g["miss_rows"] for g in gathered) * ROW_BYTES /
                              max(g["per_call"]["ms_per_step"] for g in gathered) / args.steps / 1e6,
                     "unit": "GB/s", "ms_per_step": max(g["per_call"]["ms_per_step"] for g in gathered),
                     "p50_us_per_layer_step": pct([x for g in gathered for x in g["per_call"]["step_us"]], 50),
                     "p99_us_per_layer_step": pct([x for g in gathered for x in g["per_call"]["step_us"]], 99),
                     "note": "one sieve_and_read call per layer with status words, CUDA events around each call"},
        "kernel_avg_us": kern,
        "kernel_timing": "kernel_avg_us: separate replay of the same steps with CUDA events around each kernel "
                         "(includes each launch's gap); roofline avg_us: " + (
                             "timed-region device time / launches (one kernel per layer-step)"
                             if g0["fused"] and g0["graph"] else "kernel_avg_us"),
        "miss_rows_per_layer_step": rows_per_launch,
        "roofline": dominant, "roofline_other": other,
        "gpu_launches": (1 if g0["fused"] else 2) * L * args.steps,
        "clocks": g0["clocks"],
    }
    if g0["e2e"] is not None:
        e = dict(g0["e2e"])
        if world > 1:  # all ranks' rows over the slowest rank's wall time
            dt = max(g["e2e"]["seconds"] for g in gathered)
            e["value"] = sum(g["e2e"]["rows"] for g in gathered) * ROW_BYTES / dt / 1e9
            e["ms_per_step"] = dt * 1e3 / args.steps
        out["e2e"] = e
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = run_cpu(layer_steps=8, warm=1)
    print(json.dumps(out), flush=True)


# ---- CPU legs: the reference's path on the host cores ------------------------------------

def host_topk(rng, st, layer, R, K, ctx, miss_ratio):
    """Config 2 draw from the checker's state: unique positions, hits from the residents."""
    out = np.empty((R, K), np.int32)
    n_miss = int(round(K * miss_ratio))
    for r in range(R):
        tok = st.tokens[layer, r, :st.dbs]
        res = tok[(tok >= 0) & (tok < ctx)]
        mask = np.ones(ctx, bool)
        mask[res] = False
        nonres = np.flatnonzero(mask)
        row = np.concatenate([rng.choice(nonres, n_miss, replace=False), rng.choice(res, K - n_miss, replace=False)])
        rng.shuffle(row)
        out[r] = row
    return out


class CpuPath:
    """The reference's CPU path on a bounded sample of config 2: each layer-step runs the
    checker's sieve (kvoracle.c, threaded over requests) then a host memcpy gather following
    the stripe map (threaded over positions), over `layers` layer states of 64 requests."""

    def __init__(self, threads=None, layers=4):
        import oracle
        self.oracle = oracle
        self.threads = threads or os.cpu_count() or 1
        self.layers = layers
        R, ctx, K, dbs = CFG["requests"], CFG["ctx"], CFG["top_k"], CFG["dbs"]
        self.rng = np.random.default_rng(CFG["seed"])
        self.st = oracle.SieveState(layers, R, dbs, K)
        for r in range(R):
            self.st.admit(r, ctx)
        self.seg = np.frombuffer(self.rng.bytes(R * ctx * ROW_BYTES), dtype=np.uint8).copy()
        self.hot = np.zeros(R * dbs * ROW_BYTES, np.uint8)
        self.pool_idx, self.seq = np.arange(R, dtype=np.int64), np.full(R, ctx, np.int32)
        self.base = np.arange(R, dtype=np.int64) * ctx
        self.i = 0

    def run(self, layer_steps):
        """Returns (seconds, miss rows) of `layer_steps` timed layer-steps."""
        R, ctx, K, dbs, miss = CFG["requests"], CFG["ctx"], CFG["top_k"], CFG["dbs"], CFG["miss_ratio"]
        total, rows = 0.0, 0
        for _ in range(layer_steps):
            l = self.i % self.layers
            self.i += 1
            topk = host_topk(self.rng, self.st, l, R, K, ctx, miss)
            t0 = time.perf_counter()
            slots, is_miss = self.st.update(l, topk, self.pool_idx, self.seq, nthreads=self.threads)
            n = self.oracle.gather_all([self.seg], 0, ROW_BYTES, topk, self.pool_idx, self.base, slots, is_miss, R,
                                       self.hot, K, R, 1, hot_req_stride_rows=dbs, nthreads=self.threads)
            total += time.perf_counter() - t0
            rows += n
        return total, rows

    def describe(self, layer_steps):
        return ("{} layer-steps of config 2 (64 req x 2048 topK, 20% miss) over {} layer states; sieve "
                "(kvoracle.c) + memcpy gather, {} host threads".format(layer_steps, self.layers, self.threads))


def run_cpu(layer_steps, warm=1):
    cp = CpuPath()
    cp.run(warm)
    secs, rows = cp.run(layer_steps)
    return {"value": rows * ROW_BYTES / secs / 1e9, "unit": "GB/s", "cores": cp.threads, "kind": "port",
            "sample": cp.describe(layer_steps), "us_per_layer_step": secs * 1e6 / layer_steps}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    L = 8
    cp = CpuPath()
    for _ in range(args.warmup):
        cp.run(L)
    secs, rows = 0.0, 0
    for _ in range(args.steps):
        s, r = cp.run(L)
        secs += s
        rows += r
    value = rows * ROW_BYTES / secs / 1e9
    cb = {"value": value, "unit": "GB/s", "cores": cp.threads, "kind": "port",
          "sample": "per step: " + cp.describe(L), "us_per_layer_step": secs * 1e6 / (L * args.steps)}
    out = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": secs * 1e3 / args.steps, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic",
           "config": {"workload": CFG["name"], "requests_per_gpu": CFG["requests"], "ctx": CFG["ctx"],
                      "top_k": CFG["top_k"], "hot_slots": CFG["dbs"], "miss_ratio": CFG["miss_ratio"],
                      "row_bytes": ROW_BYTES, "step": "{} layer-steps (bounded CPU sample)".format(L)},
           "impl": "reference", "cpu_baseline": cb,
           "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
