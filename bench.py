"""Benchmark of the decode-time KV hot path on B200.

Default (the headline, BASELINE config 2, DSA/MLA decode): 64 requests x 8192-token context,
61 layers, topK 2048, hot buffer 4096 slots, miss ratio 0.2, 1152-byte fp16 rows N(0,1),
seed 1. A step is one decode step: every layer runs sieve_update then the gather of its miss
rows (the reference driver's per-layer sequence, xds/xds_decode.py:225-233). The metric is the
reference's own: miss rows x 1152 B / (sieve + gather) time (xds_decode.py:226-233,280), in
GB/s; p50/p99 microseconds per layer-step are reported beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--config c2|c3|c4|link] [--pool hbm|host] [--no-verify] ...

Configs:
  c2    the headline above. At N=1 the pool is one segment in the GPU's own HBM; under torchrun
        with N>1 ranks every rank runs its own 64 requests (weak scaling) and its pool is
        striped S=1 over the other N-1 GPUs' HBM (segments mapped through CUDA IPC, read
        in-kernel over NVLink/NVSwitch).
  c3    large-batch decode: 256 requests in total (256/N per rank, strong scaling) x 32768
        context, 8 layers, dbs 8192, miss ratio 0.5, Zipf(1.1) token popularity, pool striped
        S=16 over all N GPUs (own included), injective segment rows.
  c4    prefill export: 16 requests x 8192 tokens x 61 layers of 1152-B rows per rank, exported
        HBM -> pool segments striped S=64 over all N GPUs (or pinned host memory with
        --pool host), one kvops_export_seg_alllayer launch per segment.
  link  single process over every visible GPU: the host-link and NVLink bandwidth the row
        kernels reach (contiguous and random rows, one peer and all peers at once), and the
        copy engines' peer and host copies, as roofline denominators.
--pool host places the decode pool's segments in pinned host memory (the host-link gather).
There is no collective on any data path. `--verify` (default on) checks, after the timed
region, the bytes of sampled gathered (or exported) rows against the pool's source rows, each
read by the rank that hosts it; `--impl reference` times the reference's CPU path (the C
restatement of its sieve plus a host memcpy gather following its stripe map) on rank 0.
"""
import argparse
import ctypes
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
CONFIGS = {
    "c2": dict(name="c2_dsa_decode", requests=64, ctx=8192, layers=61, top_k=2048, dbs=4096, miss_ratio=0.2,
               stripe_rows=1, seed=1, placement="others", zipf=None, injective=False, per_rank_requests=True),
    "c3": dict(name="c3_large_batch", requests=256, ctx=32768, layers=8, top_k=2048, dbs=8192, miss_ratio=0.5,
               stripe_rows=16, seed=7, placement="all", zipf=1.1, injective=True, per_rank_requests=False),
    "c4": dict(name="c4_prefill_export", requests=16, ctx=8192, layers=61, stripe_rows=64, seed=4,
               placement="all", injective=True),
    "c5": dict(name="c5_sieve_stress", requests=1024, ctx=131072, top_k=2048, dbs=65518, steps=50, seed=123,
               miss_ratio=0.9, zipf=0.8),
}
CFG = CONFIGS["c2"]
METRIC = "miss-row import GB/s (sieve+gather, per layer-step)"
EXPORT_METRIC = "prefill export GB/s (kvops_export_seg_alllayer, all layers)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=["c2", "c3", "c4", "c5", "link"], default="c2")
    ap.add_argument("--dist", choices=["uniform", "zipf", "both"], default="both", help="c5: the stress draws")
    ap.add_argument("--requests", type=int, default=None,
                    help="requests per GPU (default: the config's; smaller only for profiling captures)")
    ap.add_argument("--layers", type=int, default=None, help="layers per decode step (default: the config's)")
    ap.add_argument("--path", choices=["auto", "coop", "fused", "split"], default="auto",
                    help="layer-step path of sieve_and_read (auto: cooperative when it fits)")
    ap.add_argument("--pool", choices=["hbm", "host", "peer"], default="hbm",
                    help="pool segments in GPU HBM (placement of the config), in pinned host memory, or (one "
                         "process only) in the next GPU's HBM through peer access")
    ap.add_argument("--reference-map", action="store_true",
                    help="c3/c4: the reference's segment rows (S>1 stripes share one row) instead of injective rows")
    ap.add_argument("--no-graph", action="store_true",
                    help="time the per-call loop only (default: `value` from decode steps replayed as CUDA graphs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-verify", action="store_true")
    ap.add_argument("--verify-rows", type=int, default=4096, help="gathered rows byte-checked per rank")
    ap.add_argument("--link-span-gb", type=int, default=2,
                    help="link: also draw the all-GPU random reads from segments of this many GB (> 2)")
    return ap.parse_args()


def peaks():
    """HBM peak from the driver-measured MEASURED_PEAKS.json (burst copy), else the fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback"


def link_peaks():
    """NVLink and host-link denominators (GB/s per direction per GPU) with their sources.
    profiles/links.json holds this repository's own measurement (`--config link`): for NVLink
    the faster of the copy engines and the row kernel on contiguous peer rows, for the host link
    the faster of the copy engine and the row kernel reading (or writing) contiguous pinned rows.
    Without it: 770 GB/s, this pool's measured peer-copy reference, and 64 GB/s, the PCIe Gen5
    x16 nominal."""
    out = {"nvlink": (770.0, "pool reference peer copy 770 GB/s per direction"),
           "host_read": (64.0, "PCIe Gen5 x16 nominal 64 GB/s per direction"),
           "host_write": (64.0, "PCIe Gen5 x16 nominal 64 GB/s per direction")}
    path = os.path.join(ROOT, "profiles", "links.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        for key, field in (("nvlink", "nvlink_gbs"), ("host_read", "host_link_gbs"),
                           ("host_write", "host_link_write_gbs")):
            if d.get(field):
                out[key] = (float(d[field]), "measured {} (profiles/links.json)".format(field))
    return out


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


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


class Cluster:
    """This rank's view of the N-GPU job: process group (gloo, host plumbing only), barrier and
    object exchange. Every rank takes the same exchange steps in the same order."""

    def __init__(self, torch):
        import datetime

        import torch.distributed as dist
        self.rank, self.world, self.local = dist_env()
        self.seg_dev = self.local  # device whose memory holds the segments this rank hosts (-1: pinned host)
        torch.cuda.set_device(self.local)
        self.dist = dist
        if self.world > 1:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def all_gather(self, obj):
        if self.world == 1:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def set_pool_kind(torch, mod, cl, kind):
    """Where the segments this rank hosts live: its own HBM, its pinned host memory, or (one
    process only) the next GPU's HBM, mapped through peer access."""
    if kind == "host":
        cl.seg_dev = -1
    elif kind == "peer":
        if cl.world != 1 or torch.cuda.device_count() < 2:
            raise SystemExit("--pool peer needs one process and two visible GPUs")
        cl.seg_dev = (cl.local + 1) % torch.cuda.device_count()
        mod.enable_peer_access(cl.local, cl.seg_dev)
    else:
        cl.seg_dev = cl.local


def build_pool(mod, torch, cl, L, plsr, n_nodes, seed, placement, fill=True):
    """Segments of this rank's pool (kv_offload_proto_b200.cluster): every rank allocates and
    fills the segments it hosts and maps its own pool's segments through CUDA IPC handles.
    cl.seg_dev < 0: every segment of the rank's pool in its own pinned host memory instead;
    cl.seg_dev another GPU (one process): the pool's one segment there, read through peer access.
    Returns (segment addresses in node order, node devices, {(owner, node): hosted address},
    opened IPC mappings)."""
    from kv_offload_proto_b200.cluster import hosted_segments, pool_nodes
    from kv_offload_proto_b200.pool import device_view
    seg_bytes = L * plsr * ROW_BYTES
    dev = "cuda:{}".format(cl.local if cl.seg_dev < 0 else cl.seg_dev)

    def filled(owner, idx):
        addr = mod.segment_alloc(cl.seg_dev, seg_bytes)
        if fill:
            gen = torch.Generator(device=dev).manual_seed(seed * 7919 + owner * 131 + idx)
            chunk = 1 << 28
            if cl.seg_dev >= 0:  # drawn by the GPU that holds the segment, in its own memory
                view = device_view(addr, seg_bytes, dev).view(torch.float16)
                for o in range(0, view.numel(), chunk):
                    view[o:o + chunk].normal_(generator=gen)
            else:  # pinned host: drawn on the GPU, copied over by the copy engine
                host = torch.from_numpy(np.ctypeslib.as_array(
                    (ctypes.c_uint8 * seg_bytes).from_address(addr))).view(torch.float16)
                for o in range(0, host.numel(), chunk):
                    n = min(chunk, host.numel() - o)
                    host[o:o + n].copy_(torch.empty(n, dtype=torch.float16, device=dev).normal_(generator=gen))
        return addr

    if cl.seg_dev != cl.local:  # pinned host segments, or the peer GPU's: this rank's own, no exchange
        hosted = {(cl.rank, i): filled(cl.rank, i) for i in range(n_nodes)}
        return [hosted[(cl.rank, i)] for i in range(n_nodes)], [cl.seg_dev] * n_nodes, hosted, []
    nodes = pool_nodes(cl.rank, cl.world, placement)
    assert len(nodes) == n_nodes
    hosted = {(owner, idx): filled(owner, idx) for owner, idx in hosted_segments(cl.rank, cl.world, placement)}
    if cl.world == 1:
        return [hosted[(cl.rank, 0)]], nodes, hosted, []
    handles = {k: mod.ipc_get_handle(a) for k, a in hosted.items()}
    gathered = cl.all_gather(handles)
    mine = [None] * n_nodes
    for hd in gathered:
        for (owner, idx), h in hd.items():
            if owner == cl.rank:
                mine[idx] = h
    addrs = []
    for idx, h in enumerate(mine):
        addrs.append(hosted[(cl.rank, idx)] if nodes[idx] == cl.local else mod.ipc_open_handle(cl.local, h))
    opened = [a for idx, a in enumerate(addrs) if nodes[idx] != cl.local]
    return addrs, nodes, hosted, opened


def read_hosted_rows(torch, cl, hosted, asks, seg_bytes):
    """Answers every rank's byte requests for rows of the segments this rank hosts, reading
    only this rank's own memory. asks: list over ranks of {(owner, node): row-offset list}.
    Returns {(asker, owner, node): uint8 [n, ROW_BYTES]}."""
    from kv_offload_proto_b200.pool import device_view
    out = {}
    for asker, ask in enumerate(asks):
        for key, offs in ask.items():
            if key not in hosted or not len(offs):
                continue
            addr = hosted[key]
            idx = np.asarray(offs, np.int64)
            if (idx < 0).any() or ((idx + 1) * ROW_BYTES > seg_bytes).any():
                raise RuntimeError("verify: row offset outside the segment")
            if cl.seg_dev < 0:
                base = np.ctypeslib.as_array((ctypes.c_uint8 * seg_bytes).from_address(addr))
                out[(asker,) + key] = base.reshape(-1, ROW_BYTES)[idx].copy()
            else:  # read by the GPU whose memory it is
                view = device_view(addr, seg_bytes, "cuda:{}".format(cl.seg_dev)).view(-1, ROW_BYTES)
                out[(asker,) + key] = view[torch.as_tensor(idx, device=view.device)].cpu().numpy()
    return out


def exchange_rows(torch, cl, hosted, ask, seg_bytes):
    """Byte contents of the rows in `ask` ({(owner, node): row offsets}), each read by the rank
    that hosts its segment and sent back over the process group (host plumbing; no GPU reads
    another GPU's memory here)."""
    asks = cl.all_gather(ask)
    answers = read_hosted_rows(torch, cl, hosted, asks, seg_bytes)
    mine = {}
    for part in cl.all_gather(answers):
        for (asker, owner, node), rows in part.items():
            if asker == cl.rank:
                mine[(owner, node)] = rows
    return mine


# ---- decode configs (c2, c3) --------------------------------------------------------------

def run_decode(args, cfg):
    import torch
    cl = Cluster(torch)
    rank, world, local = cl.rank, cl.world, cl.local
    import kv_offload_proto_b200 as kp
    from kv_offload_proto_b200.offload import XdsOffloadCoordinator
    from kv_offload_proto_b200.pool import DevicePool, per_layer_seg_rows, per_layer_seg_rows_injective
    from kv_offload_proto_b200.workload import sample_topk_device, zipf_pmf

    mod = kp.install_kvops_ext()
    mod.init(local, "")
    set_pool_kind(torch, mod, cl, args.pool)
    dev = torch.device("cuda", local)
    R = args.requests or (cfg["requests"] if cfg["per_rank_requests"] else cfg["requests"] // world)
    ctx, K, dbs, miss = cfg["ctx"], cfg["top_k"], cfg["dbs"], cfg["miss_ratio"]
    L = args.layers or cfg["layers"]
    S = cfg["stripe_rows"]
    injective = cfg["injective"] and not args.reference_map
    layer_rows = R * ctx
    n_nodes = (max(world - 1, 1) if cfg["placement"] == "others" else world)
    plsr = per_layer_seg_rows_injective(layer_rows, S, n_nodes) if injective and S else \
        per_layer_seg_rows(layer_rows, n_nodes)
    W, Sn = args.warmup, args.steps
    T = W + Sn

    seg_addrs, nodes, hosted, opened = build_pool(mod, torch, cl, L, plsr, n_nodes, cfg["seed"], cfg["placement"])
    pool = DevicePool(local, L, layer_rows, ROW_BYTES, S, segment_devices=nodes, segment_addrs=seg_addrs,
                      injective=injective)
    assert pool.per_layer_seg_rows == plsr
    co = XdsOffloadCoordinator(dev, L, R, dbs, K, R, ctx)
    hot = torch.empty((L, R * dbs * ROW_BYTES), dtype=torch.uint8, device=dev)
    pre, base = [ctx] * R, [r * ctx for r in range(R)]
    co.admit_all(pre, base)
    co.set_batch(torch.arange(R, dtype=torch.int64, device=dev), torch.full((R,), ctx, dtype=torch.int32, device=dev))

    # Inputs: the config's draws (unique positions; hits from the current residents, misses from
    # the others, both weighted by the Zipf pmf where the config has one), made once by running
    # the device SIEVE ahead; every pass below starts from the same admitted state, so each
    # layer-step sees exactly the state its draw was made against.
    log_pmf = None
    if cfg["zipf"]:
        log_pmf = torch.as_tensor(np.log(zipf_pmf(ctx, cfg["zipf"], cfg["seed"])), dtype=torch.float32, device=dev)
    gen = torch.Generator(device=dev).manual_seed(cfg["seed"] * 1000 + rank)
    topk = torch.empty((T, L, R, K), dtype=torch.int32, device=dev)
    misses = torch.zeros((T, L), dtype=torch.int64, device=dev)
    for s in range(T):
        for l in range(L):
            topk[s, l] = sample_topk_device(co.device_buffer_tokens[l, :R], ctx, dbs, K, miss, gen, log_pmf)
            co.sieve_update(l, topk[s, l])
            misses[s, l] = co.is_miss.sum()
    misses_h = misses.cpu().numpy()
    co.admit_all(pre, base)

    stream = torch.cuda.current_stream(dev).cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    # The public one-call layer-step (DevicePool.sieve_and_read, path "auto"): one cooperative
    # launch whose non-SIEVE CTAs copy each request's miss rows as its hand sweep makes them
    # final (or, where that does not fit, the SIEVE kernel and the gather as its programmatic
    # dependent).
    def layer_step(s, l):
        pool.sieve_and_read(co, l, topk[s, l], hot[l], stream, 1, hot_req_stride_rows=dbs, path=args.path,
                            err_word=err)

    def timed_pass(graphs):
        """W untimed then Sn timed steps from the admitted state; device time of the timed
        steps, per-layer-step (or per-step) times, clock record. graphs: replay one captured
        graph per step, else one call per layer with CUDA events around each call."""
        co.admit_all(pre, base)
        for s in range(W):
            if graphs:
                graphs[s].replay()
            else:
                for l in range(L):
                    layer_step(s, l)
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(Sn * (1 if graphs else L))]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks = ClockSampler(torch, local)
        clocks.start()
        torch.cuda.synchronize()
        cl.barrier()
        torch.cuda.nvtx.range_push("timed" if graphs or args.no_graph else "per_call")  # profiler selection
        t0.record()
        h0 = time.perf_counter()
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
        host_issue_s = time.perf_counter() - h0
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        cl.barrier()
        clk = clocks.stop()
        clk["host_issue_us_per_call"] = host_issue_s * 1e6 / (Sn * (1 if graphs else L))
        assert int(co.is_miss.sum().item()) == int(misses_h[T - 1, L - 1]), "replay diverged from the input pass"
        return t0.elapsed_time(t1) * 1e-3, [e[0].elapsed_time(e[1]) * 1e3 for e in evs], clk

    # Per call: the public one-call API per layer, status words published (what a caller of
    # sieve_and_read gets without graphs); CUDA events around every call.
    elapsed_pc, call_us, clk_pc = timed_pass(None)
    path = mod.last_step_path()
    fused = path in ("coop", "fused")  # one kernel per layer-step
    graphs = None
    if not args.no_graph:  # one CUDA graph per decode step (its layers' calls), replayed in order
        from kv_offload_proto_b200.graph import StepGraph
        graphs = [StepGraph(pool, co, hot, L, path=args.path, hot_req_stride_rows=dbs, topk=topk[s]) for s in range(T)]
        elapsed, step_us, clk = timed_pass(graphs)
        graph_err = max(g.error() for g in graphs)
    else:
        elapsed, step_us, clk = elapsed_pc, call_us, clk_pc
        graph_err = 0
    last = int(co.is_miss.sum().item())
    miss_rows = int(misses_h[W:].sum())

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
        e2e_pc = run_e2e(torch, co, pool, hot, topk, misses_h, pre, base, L, W, Sn, R, K, dbs, dev, args.path)
        if args.no_graph:
            e2e = dict(e2e_pc, api="sieve_and_read per layer, host polls the status words")
        else:
            e2e = run_e2e_graph(torch, co, pool, hot, topk, misses_h, pre, base, L, W, Sn, R, K, dbs, dev, args.path)
            e2e["per_call"] = {k: e2e_pc[k] for k in ("value", "unit", "ms_per_step")}
            e2e["per_call"]["api"] = "sieve_and_read per layer, host polls the status words after each"
    device_err = int(err.item())

    verify = None
    if not args.no_verify:  # the state now is that of the last layer-step of step T-1 (every pass replays it)
        verify = verify_gather(torch, cl, co, pool, hot[L - 1], topk[T - 1, L - 1], L - 1, hosted, R, dbs, K,
                               args.verify_rows, cfg["seed"])

    res = dict(elapsed=elapsed, miss_rows=miss_rows, kernels=kernels, step_us=step_us, call_us=call_us, e2e=e2e,
               clocks=clk, nodes=len(nodes), fused=fused, path=path, graph=bool(graphs), launches=len(kev),
               per_call={"ms_per_step": elapsed_pc * 1e3 / Sn, "clocks": clk_pc}, rank=rank, R=R,
               errors={"device_err_word": device_err, "graph_err_word": graph_err}, verify=verify,
               remote_rows=remote_fraction(nodes, local))
    gathered = cl.all_gather(res)
    graphs = None
    for a in opened:
        mod.ipc_close_handle(a)
    torch.cuda.synchronize()
    cl.barrier()
    for a in hosted.values():
        mod.segment_free(a)
    cl.close()
    if rank == 0:
        report_decode(args, cfg, world, gathered, co, L, n_nodes, injective)


def remote_fraction(nodes, local):
    """Share of the pool's rows that are not in this GPU's HBM (rows are striped evenly over the
    nodes; a node on device -1 is pinned host memory)."""
    return sum(1 for d in nodes if d != local) / float(len(nodes))


def verify_gather(torch, cl, co, pool, hot_layer, topk_last, layer, hosted, R, dbs, K, nsample, seed):
    """Byte check of sampled miss rows of the last layer-step: the hot row the step wrote must
    equal the pool row its position names under the stripe map (kvc_gather_rows.cpp:54-84).
    The pool row is read by the rank that hosts its segment. Positions whose slot another miss
    of the same request also names (a wrapped sweep, see DESIGN F15) are left out."""
    from kv_offload_proto_b200.pool import node_of, seg_row_of
    slots = co.top_k_device_slots[:R].cpu().numpy()
    miss = co.is_miss[:R].cpu().numpy()
    tk = topk_last.cpu().numpy()
    base = co.req_host_base[:R].cpu().numpy()
    r_idx, k_idx = np.nonzero(miss)
    sl = slots[r_idx, k_idx]
    key = r_idx.astype(np.int64) * (1 << 20) + sl
    uniq, cnt = np.unique(key, return_counts=True)
    once = np.isin(key, uniq[cnt == 1])
    r_idx, k_idx, sl = r_idx[once], k_idx[once], sl[once]
    rng = np.random.default_rng(seed * 31 + cl.rank)
    pick = np.sort(rng.choice(len(r_idx), min(nsample, len(r_idx)), replace=False)) if len(r_idx) else \
        np.empty(0, np.int64)
    r_idx, k_idx, sl = r_idx[pick], k_idx[pick], sl[pick]
    rows = (base[r_idx] + tk[r_idx, k_idx]).astype(np.int64)
    ask, where = {}, []
    for i, row in enumerate(rows):
        node = node_of(int(row), pool.stripe_rows, pool.node_num)
        off = layer * pool.per_layer_seg_rows + seg_row_of(int(row), pool.stripe_rows, pool.node_num, pool.injective)
        ask.setdefault((cl.rank, node), []).append(off)
        where.append((node, len(ask[(cl.rank, node)]) - 1))
    src = exchange_rows(torch, cl, hosted, ask, pool.segment_bytes)
    hot_idx = torch.as_tensor(r_idx.astype(np.int64) * dbs + sl, device=hot_layer.device)
    got = hot_layer.view(-1, ROW_BYTES)[hot_idx].cpu().numpy() if len(r_idx) else np.empty((0, ROW_BYTES), np.uint8)
    bad = 0
    for i, (node, j) in enumerate(where):
        if not np.array_equal(got[i], src[(cl.rank, node)][j]):
            bad += 1
    return {"rows_checked": int(len(rows)), "mismatches": int(bad), "nodes": sorted({n for n, _ in where}),
            "method": "sampled miss rows of the last layer-step: hot row bytes == pool row bytes read by the "
                      "hosting rank from its own memory (stripe map of pool.py)"}


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
    graphs); the step's result, its last layer's miss count and the graph's error word, is read
    back to pinned host memory and checked on the host once the step is done. (A reduction after
    every layer would put a small kernel between each pair of cooperative launches, ~15 us per
    layer of launch gaps, which a decode step does not need.) Host wall clock from the first
    timed step's input copy to the last timed step's result."""
    from kv_offload_proto_b200.graph import StepGraph
    T = W + S
    topk_host = topk.cpu().pin_memory()
    bufs = [torch.empty((L, R, K), dtype=torch.int32, device=dev) for _ in range(2)]
    counts = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(2)]
    counts_h = torch.zeros((T, 2), dtype=torch.int64).pin_memory()

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
        counts_h[s, 0:1].copy_(counts[i], non_blocking=True)
        counts_h[s, 1:2].copy_(graphs[i].err, non_blocking=True)
        done[s].record(main)

    def check(s):
        done[s].synchronize()
        assert int(counts_h[s, 0]) == int(misses_h[s, L - 1]), "e2e replay diverged at step %d" % s
        assert int(counts_h[s, 1]) == 0, "device errCode 0x%x at step %d" % (int(counts_h[s, 1]), s)

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
            "h2d_bytes_per_step": L * R * K * 4, "d2h_bytes_per_step": 8 + 4, "rows": rows, "seconds": dt,
            "api": "StepGraph.replay per decode step; inputs copied from pinned host memory on a copy stream "
                   "during the previous step; the step's last-layer miss count and error word read back and "
                   "checked every step"}


def traffic_per_unit():
    """DRAM bytes per unit measured by ncu (profiles/traffic.json), if captured."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return {}
    with open(path) as f:
        return json.load(f)


def roofline(kernel, avg_us, hbm_bytes, link_bytes, link_peak, link_src, link_kind, traffic=None):
    """Roofline of one launch: the target time is the slower of its HBM bytes at the measured
    HBM peak and its link bytes (NVLink or host link) at that link's peak; `achieved` is the
    bound's bytes over the measured duration, `frac` the fraction of that bound's peak."""
    hbm_peak, hbm_src = peaks()
    t_hbm = hbm_bytes / (hbm_peak * 1e9)
    t_link = link_bytes / (link_peak * 1e9) if link_bytes else 0.0
    link_bound = t_link > t_hbm
    nbytes, peak, src = (link_bytes, link_peak, link_src) if link_bound else (hbm_bytes, hbm_peak, hbm_src)
    achieved = nbytes / (avg_us * 1e-6) / 1e9
    return {"kernel": kernel, "bound": link_kind if link_bound else "hbm", "achieved": achieved, "peak": peak,
            "unit": "GB/s", "frac": achieved / peak, "peak_source": src, "traffic": traffic,
            "algorithmic_bytes": nbytes, "hbm_bytes": hbm_bytes, "link_bytes": link_bytes, "avg_us": avg_us,
            "target_us": max(t_hbm, t_link) * 1e6}


def report_decode(args, cfg, world, gathered, co, L, n_nodes, injective):
    lp = link_peaks()
    K = cfg["top_k"]
    elapsed = max(g["elapsed"] for g in gathered)
    miss_rows = sum(g["miss_rows"] for g in gathered)
    value = miss_rows * ROW_BYTES / elapsed / 1e9
    g0 = gathered[0]
    R = g0["R"]
    kern = {k: sum(v) / len(v) for k, v in g0["kernels"].items()}
    rows_per_launch = g0["miss_rows"] / g0["launches"]
    tr = traffic_per_unit()
    sb = state_bytes(co.padded_buffer_size, co.visited_stride_b, co.ht_size)
    # Algorithmic bytes of one layer-step (counted once): SIEVE state read + written, the
    # positions read and the slots / miss flags written (9 B per position), 16 B of request
    # metadata; each miss row is read from its segment and written to the hot buffer.
    sieve_bytes = R * (2 * sb + 9 * K + 16)
    remote = g0["remote_rows"]
    link_kind = "host_link" if args.pool == "host" else "nvlink"
    link_peak, link_src = lp["host_read"] if args.pool == "host" else lp["nvlink"]
    rows_remote = rows_per_launch * remote
    rows_local = rows_per_launch - rows_remote
    payload_hbm = rows_local * 2 * ROW_BYTES + rows_remote * ROW_BYTES  # local: read + write; remote: write
    if g0["fused"]:
        (name, t), = kern.items()
        if g0["graph"]:  # one kernel per layer-step: the timed region's device time per launch
            t = elapsed * 1e6 / (L * args.steps)
        traffic = None
        if args.config == "c2" and world == 1 and args.pool == "hbm" and "coop_per_launch" in tr:
            traffic = tr["coop_per_launch"] * rows_per_launch / tr.get("coop_rows_per_launch", 33477.0)
        dominant = roofline(name, t, sieve_bytes + payload_hbm, rows_remote * ROW_BYTES, link_peak, link_src,
                            link_kind, traffic)
        other = None
    else:
        rs = roofline("sieve_fast_kernel", kern["sieve_fast_kernel"], sieve_bytes, 0, link_peak, link_src, link_kind,
                      tr["sieve_per_request"] * R if "sieve_per_request" in tr else None)
        rg = roofline("gather_kernel", kern["gather_kernel"], payload_hbm + R * (9 * K + 16), rows_remote * ROW_BYTES,
                      link_peak, link_src, link_kind,
                      tr["gather_per_row"] * rows_per_launch if "gather_per_row" in tr and not remote else None)
        dominant, other = (rs, rg) if rs["avg_us"] >= rg["avg_us"] else (rg, rs)
    call_all = [x for g in gathered for x in g["call_us"]]
    step_all = [x / L for g in gathered for x in g["step_us"]] if g0["graph"] else call_all
    pool_desc = ("pinned host memory, {} segment(s)".format(n_nodes) if args.pool == "host" else
                 "one segment in the next GPU's HBM, read through peer access (one process)"
                 if args.pool == "peer" else
                 "local HBM segment" if world == 1 else
                 "striped over the other {} GPUs' HBM".format(world - 1) if cfg["placement"] == "others" else
                 "striped over all {} GPUs' HBM (own included)".format(world))
    out = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak" if cfg["per_rank_requests"] else "strong", "vs_baseline": None, "dtype": "int32",
        "data": "synthetic",
        "config": {"workload": cfg["name"], "requests_per_gpu": R, "requests_total": R * world, "ctx": cfg["ctx"],
                   "layers": L, "top_k": K, "hot_slots": cfg["dbs"], "miss_ratio": cfg["miss_ratio"],
                   "zipf": cfg["zipf"], "row_bytes": ROW_BYTES, "stripe_rows": cfg["stripe_rows"],
                   "segment_rows": "injective" if injective else "reference map", "pool": pool_desc,
                   "l2": "inputs larger than L2 (SIEVE state {:.0f} MB, pool {:.1f} GB per GPU)".format(
                       L * R * sb / 1e6, L * R * cfg["ctx"] * ROW_BYTES / 1e9),
                   "step": "one decode step = {} layers x sieve_and_read, path {} ({}){}".format(
                       L, g0["path"], {"coop": "one cooperative kernel: SIEVE CTAs + row-copy CTAs",
                                       "fused": "one kernel: SIEVE + bulk-copy warp",
                                       "split": "SIEVE kernel + gather as programmatic dependent"}[g0["path"]],
                       ", each step replayed as one CUDA graph (no status words; completion on the stream)"
                       if g0["graph"] else "")},
        "p50_us_per_layer_step": pct(call_all, 50), "p99_us_per_layer_step": pct(call_all, 99),
        "latency_note": "p50/p99 over every layer-step call of every rank, CUDA events around each "
                        "sieve_and_read call (status words published); graph_us_per_layer_step: decode-step "
                        "graph replay time / layers",
        "graph_us_per_layer_step": {"p50": pct(step_all, 50), "p99": pct(step_all, 99)} if g0["graph"] else None,
        "graph": g0["graph"],
        "per_call": {"value": miss_rows * ROW_BYTES / max(g["per_call"]["ms_per_step"] for g in gathered) /
                     args.steps / 1e6, "unit": "GB/s",
                     "ms_per_step": max(g["per_call"]["ms_per_step"] for g in gathered),
                     "host_issue_us_per_call": g0["per_call"]["clocks"].get("host_issue_us_per_call"),
                     "note": "one sieve_and_read call per layer with status words, CUDA events around each call"},
        "per_rank": [{"rank": g["rank"], "ms_per_step": g["elapsed"] * 1e3 / args.steps,
                      "us_per_layer_step": g["elapsed"] * 1e6 / (args.steps * L), "miss_rows": g["miss_rows"],
                      "call_p50_us": pct(g["call_us"], 50), "call_p99_us": pct(g["call_us"], 99),
                      "e2e_seconds": (g["e2e"] or {}).get("seconds")} for g in gathered],
        "kernel_avg_us": kern,
        "kernel_timing": "kernel_avg_us: separate replay of the same steps with CUDA events around each kernel "
                         "(includes each launch's gap); roofline avg_us: " + (
                             "timed-region device time / launches (one kernel per layer-step)"
                             if g0["fused"] and g0["graph"] else "kernel_avg_us"),
        "miss_rows_per_layer_step": rows_per_launch,
        "roofline": dominant, "roofline_other": other,
        "gpu_launches": (1 if g0["fused"] else 2) * L * args.steps,
        "clocks": g0["clocks"],
        "device_errors": [g["errors"] for g in gathered],
    }
    if g0["verify"] is not None:
        vs = [g["verify"] for g in gathered]
        out["verify"] = {"rows_checked": sum(v["rows_checked"] for v in vs),
                         "mismatches": sum(v["mismatches"] for v in vs),
                         "per_rank": [[v["rows_checked"], v["mismatches"]] for v in vs], "method": vs[0]["method"]}
    if g0["e2e"] is not None:
        e = dict(g0["e2e"])
        if world > 1:  # all ranks' rows over the slowest rank's wall time
            dt = max(g["e2e"]["seconds"] for g in gathered)
            e["value"] = sum(g["e2e"]["rows"] for g in gathered) * ROW_BYTES / dt / 1e9
            e["ms_per_step"] = dt * 1e3 / args.steps
            e["seconds"] = dt
        out["e2e"] = e
    if world == 1 and not args.no_cpu_baseline and args.config == "c2":
        out["cpu_baseline"] = run_cpu(layer_steps=8, warm=1)
    print(json.dumps(out), flush=True)


# ---- prefill export (c4) ----------------------------------------------------------------

def run_export(args):
    import torch
    cfg = CONFIGS["c4"]
    cl = Cluster(torch)
    rank, world, local = cl.rank, cl.world, cl.local
    import kv_offload_proto_b200 as kp
    from kv_offload_proto_b200.pool import DevicePool, per_layer_seg_rows, per_layer_seg_rows_injective
    mod = kp.install_kvops_ext()
    mod.init(local, "")
    set_pool_kind(torch, mod, cl, args.pool)
    pinned = cl.seg_dev < 0
    dev = torch.device("cuda", local)
    L = args.layers or cfg["layers"]
    rows = cfg["requests"] * cfg["ctx"]
    S = cfg["stripe_rows"]
    injective = cfg["injective"] and not args.reference_map
    N = world
    plsr = per_layer_seg_rows_injective(rows, S, N) if injective else per_layer_seg_rows(rows, N)
    seg_addrs, nodes, hosted, opened = build_pool(mod, torch, cl, L, plsr, N, cfg["seed"], "all", fill=False)
    pool = DevicePool(local, L, rows, ROW_BYTES, S, segment_devices=nodes, segment_addrs=seg_addrs,
                      injective=injective)
    src = torch.empty((L, rows * ROW_BYTES // 2), dtype=torch.float16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(cfg["seed"] * 101 + rank)
    for l in range(L):
        src[l].normal_(generator=gen)
    stride = rows * ROW_BYTES
    # Destination rows written per segment: every row (injective), or one per stripe (the
    # reference's map, where the last row of each stripe wins).
    units = rows * L if injective else ((rows + S - 1) // S) * L
    local_units = sum(1 for d in nodes if d == local) * units / N
    W, Sn = args.warmup, args.steps

    def step():
        st = pool.batch_write_alllayers(0, rows, src.data_ptr(), stride, torch.cuda.current_stream(dev).cuda_stream)
        return st

    for _ in range(W):
        pool.wait(step())
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(Sn)]
    clocks = ClockSampler(torch, local)
    clocks.start()
    cl.barrier()
    t0 = time.perf_counter()
    for e in evs:
        e[0].record()
        st = step()
        e[1].record()
        pool.wait(st)
    wall = time.perf_counter() - t0
    torch.cuda.synchronize()
    cl.barrier()
    clk = clocks.stop()
    dev_s = sum(e[0].elapsed_time(e[1]) for e in evs) * 1e-3
    verify = None if args.no_verify else verify_export(torch, cl, pool, src, hosted, rows, L, S, injective,
                                                       args.verify_rows, cfg["seed"])
    res = dict(rank=rank, dev_s=dev_s, wall=wall, units=units, local_units=local_units, clocks=clk, verify=verify)
    gathered = cl.all_gather(res)
    for a in opened:
        mod.ipc_close_handle(a)
    torch.cuda.synchronize()
    cl.barrier()
    for a in hosted.values():
        mod.segment_free(a)
    cl.close()
    if rank != 0:
        return
    lp = link_peaks()
    tmax = max(g["dev_s"] for g in gathered)
    total_bytes = sum(g["units"] for g in gathered) * ROW_BYTES * Sn
    value = total_bytes / tmax / 1e9
    g0 = gathered[0]
    per_launch_s = g0["dev_s"] / Sn  # N launches per step (one per segment)
    remote_units = g0["units"] - g0["local_units"]
    hbm_bytes = (g0["units"] + g0["local_units"]) * ROW_BYTES  # every row read; local rows also written here
    link_kind = "host_link" if pinned else "nvlink"
    link_peak, link_src = lp["host_write"] if pinned else lp["nvlink"]
    roof = roofline("export_kernel", per_launch_s * 1e6, hbm_bytes, remote_units * ROW_BYTES, link_peak, link_src,
                    link_kind)
    roof["note"] = "per decode-step-equivalent: the N segment launches of one batch_write_alllayers together"
    wall_max = max(g["wall"] for g in gathered)
    out = {"metric": EXPORT_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": Sn, "warmup": W,
           "ms_per_step": tmax * 1e3 / Sn, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "u8", "data": "synthetic",
           "config": {"workload": cfg["name"], "rows_per_layer": rows, "layers": L, "row_bytes": ROW_BYTES,
                      "stripe_rows": S, "segment_rows": "injective" if injective else "reference map",
                      "nodes": N, "pool": "pinned host memory" if pinned else
                      "the next GPU's HBM (peer access)" if args.pool == "peer" else "HBM of all {} GPUs".format(world),
                      "l2": "inputs larger than L2 ({:.2f} GB source per GPU)".format(L * stride / 1e9),
                      "step": "one EmsPool.batch_write_alllayers: {} kvops_export_seg_alllayer launches".format(N)},
           "bytes_per_step_per_rank": g0["units"] * ROW_BYTES,
           "per_rank": [{"rank": g["rank"], "ms_per_step": g["dev_s"] * 1e3 / Sn} for g in gathered],
           "roofline": roof, "gpu_launches": N * Sn, "clocks": g0["clocks"],
           "e2e": {"value": total_bytes / wall_max / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0, "seconds": wall_max,
                   "api": "DevicePool.batch_write_alllayers + wait (host polls the status words) per step"}}
    if g0["verify"] is not None:
        vs = [g["verify"] for g in gathered]
        out["verify"] = {"rows_checked": sum(v["rows_checked"] for v in vs),
                         "mismatches": sum(v["mismatches"] for v in vs), "method": vs[0]["method"]}
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = run_cpu_export(injective)
    print(json.dumps(out), flush=True)


def verify_export(torch, cl, pool, src, hosted, rows, L, S, injective, nsample, seed):
    """Byte check of sampled destination rows: segment row segRow of layer l must hold the
    source row the export wrote there (kvc_scatter_rows_alllayer.cpp:34-53); with the reference
    map that is the last row of the stripe (the reference's ascending writes leave it)."""
    from kv_offload_proto_b200.pool import node_of, seg_row_of
    rng = np.random.default_rng(seed * 17 + cl.rank)
    n = min(nsample, rows * L)
    ls = rng.integers(0, L, n)
    rs = rng.integers(0, rows, n)
    if not injective:  # the row that ends up in the stripe's segment row
        rs = np.minimum((rs // S + 1) * S - 1, rows - 1)
    ask, where = {}, []
    for l, r in zip(ls, rs):
        node = node_of(int(r), S, pool.node_num)
        off = int(l) * pool.per_layer_seg_rows + seg_row_of(int(r), S, pool.node_num, injective)
        ask.setdefault((cl.rank, node), []).append(off)
        where.append((node, len(ask[(cl.rank, node)]) - 1))
    got = exchange_rows(torch, cl, hosted, ask, pool.segment_bytes)
    srows = src.view(torch.uint8).view(L, rows, ROW_BYTES)
    exp = srows[torch.as_tensor(ls, device=src.device), torch.as_tensor(rs, device=src.device)].cpu().numpy()
    bad = sum(0 if np.array_equal(exp[i], got[(cl.rank, node)][j]) else 1 for i, (node, j) in enumerate(where))
    return {"rows_checked": int(n), "mismatches": int(bad),
            "method": "sampled (layer, row): destination segment row (read by its hosting rank) == source row"}


def run_cpu_export(injective):
    """The reference's export loop on the host (the C restatement of kvc_scatter_rows_alllayer,
    one thread, ascending rows) over one layer of config 4 into one segment."""
    import oracle
    cfg = CONFIGS["c4"]
    rows, S = cfg["requests"] * cfg["ctx"], cfg["stripe_rows"]
    rng = np.random.default_rng(0)
    src = rng.integers(0, 256, rows * ROW_BYTES, dtype=np.uint8)
    plsr = oracle.per_layer_seg_rows_injective(rows, S, 1) if injective else oracle.per_layer_seg_rows(rows, 1)
    seg = np.zeros(plsr * ROW_BYTES, np.uint8)
    oracle.export_alllayer(seg, plsr, ROW_BYTES, 0, rows, 1, src, rows * ROW_BYTES, S, 1, 0, injective)
    t0 = time.perf_counter()
    n = oracle.export_alllayer(seg, plsr, ROW_BYTES, 0, rows, 1, src, rows * ROW_BYTES, S, 1, 0, injective)
    dt = time.perf_counter() - t0
    return {"value": n * ROW_BYTES / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": "one layer of config 4 ({} rows, S={}) into one host segment, the restated serial loop".format(
                rows, S), "cpu_model": cpu_model()}


# ---- SIEVE stress (c5) ------------------------------------------------------------------

def run_stress(args):
    """BASELINE config 5 on one GPU: 1024 requests, hot buffer 65518 slots, topK 2048, context
    131072, 50 steps of each stress draw (workload.stress_topk_uniform / stress_topk_zipf, numpy,
    drawn on the host from the state read back after every step). Every step's slots and miss
    flags are hashed and compared with the checksum fixture tests/golden/c5_checksums.json,
    which the C restatement of the reference kernel produced from the same draws
    (tests/golden/make_c5.py); the final state too. Device time of each sieve_update launch."""
    import hashlib

    import torch
    rank, world, local = dist_env()
    if rank != 0:
        return
    import kv_offload_proto_b200 as kp
    from kv_offload_proto_b200.offload import XdsOffloadCoordinator
    from kv_offload_proto_b200.workload import stress_topk_uniform, stress_topk_zipf, zipf_cdf
    cfg = CONFIGS["c5"]
    torch.cuda.set_device(local)
    mod = kp.install_kvops_ext()
    mod.init(local, "")
    dev = torch.device("cuda", local)
    R = args.requests or cfg["requests"]
    ctx, K, dbs = cfg["ctx"], cfg["top_k"], cfg["dbs"]
    steps = cfg["steps"] if args.steps == parse_defaults()["steps"] else args.steps
    fx = None
    fx_path = os.path.join(ROOT, "tests", "golden", "c5_checksums.json")
    if os.path.exists(fx_path):
        with open(fx_path) as f:
            fx = json.load(f)
        if fx["config"]["reqs"] != R or fx["config"]["steps"] < steps:
            fx = None

    def sha(a):
        return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()

    results = {}
    for dist in (("uniform", "zipf") if args.dist == "both" else (args.dist,)):
        co = XdsOffloadCoordinator(dev, 1, R, dbs, K, R, ctx)
        co.admit_all([ctx] * R, [r * ctx for r in range(R)])
        co.set_batch(torch.arange(R, dtype=torch.int64, device=dev), torch.full((R,), ctx, dtype=torch.int32,
                                                                                 device=dev))
        if dist == "uniform":
            rng = np.random.default_rng(cfg["seed"])
        else:
            cdf, perm = zipf_cdf(ctx, cfg["zipf"], cfg["seed"])
            rng = np.random.default_rng(cfg["seed"] + 1)
        ref = fx["draws"].get(dist) if fx else None
        us, matches, misses, tiers = [], 0, 0, set()
        clocks = ClockSampler(torch, local)
        clocks.start()
        for step in range(steps):
            if dist == "uniform":
                topk = stress_topk_uniform(rng, co.device_buffer_tokens[0].cpu().numpy(), dbs, ctx, K,
                                           cfg["miss_ratio"])
            else:
                topk = stress_topk_zipf(rng, R, ctx, K, cdf, perm)
            t = torch.from_numpy(topk).to(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            co.sieve_update(0, t)
            e1.record()
            torch.cuda.synchronize()
            tiers.add(mod.last_sieve_tier())
            us.append(e0.elapsed_time(e1) * 1e3)
            slots, miss = co.top_k_device_slots.cpu().numpy(), co.is_miss.cpu().numpy()
            misses += int(miss.sum())
            if ref is not None:
                r = ref["steps"][step]
                matches += int(r["slots"] == sha(slots) and r["is_miss"] == sha(miss) and r["topk"] == sha(topk))
        clk = clocks.stop()
        final = None
        if ref is not None and steps == len(ref["steps"]):
            got = {"tokens": sha(co.device_buffer_tokens[0].cpu().numpy()),
                   "visited": sha(co.device_buffer_visited[0].cpu().numpy()),
                   "ht": sha(co.device_buffer_ht[0].cpu().numpy().view(np.uint16)),
                   "hand": sha(co.sieve_hand[0, :, 0].cpu().numpy().copy())}
            final = got == ref["final"]
        results[dist] = {"steps": steps, "us_per_step_p50": pct(us, 50), "us_per_step_p99": pct(us, 99),
                         "us_per_step_mean": sum(us) / len(us), "us_first_step": us[0],
                         "us_per_request_step": sum(us) / len(us) / R, "miss_ratio": misses / (steps * R * K),
                         "tiers": sorted(tiers), "checksum_steps_matched": matches if ref is not None else None,
                         "final_state_matched": final, "clocks": clk}
        del co
        torch.cuda.empty_cache()
    out = {"metric": "SIEVE stress: sieve_update us per step (1024 requests) and bit-exactness vs the CPU model",
           "value": results[next(iter(results))]["us_per_step_mean"], "unit": "us/step", "n_gpus": 1,
           "steps": steps, "warmup": 0, "higher_is_better": False, "dtype": "int32", "data": "synthetic",
           "config": {"workload": cfg["name"], "requests": R, "hot_slots": dbs, "top_k": K, "ctx": ctx,
                      "ht_cells": 262144, "draws": list(results)},
           "fixture": os.path.relpath(fx_path, ROOT) if fx is not None else None, "draws": results,
           "gpu_launches": steps * len(results)}
    print(json.dumps(out), flush=True)


def parse_defaults():
    """argparse defaults (so a config can tell an explicit --steps from the default)."""
    return {"steps": 5}


# ---- link probe -------------------------------------------------------------------------

def run_link(args):
    """Bandwidth the row kernels reach over the host link and NVLink, in one process over every
    visible GPU (no torchrun): rows are moved by kvops_import_multi, contiguous (a plain stream)
    and random (the gather's pattern), and by the copy engines (cudaMemcpyPeerAsync / pinned
    cudaMemcpyAsync), each timed with CUDA events over several repetitions."""
    import torch
    import kv_offload_proto_b200 as kp
    from cuda.bindings import runtime as cudart
    mod = kp.install_kvops_ext()
    ngpu = torch.cuda.device_count()
    mod.init(0, "")
    nbytes = 1 << 31
    nrows = nbytes // ROW_BYTES
    reps = max(3, args.steps)
    def ok(ret):
        if ret[0] != cudart.cudaError_t.cudaSuccess:
            raise RuntimeError("cuda runtime call failed: {}".format(ret[0]))

    out = {"metric": "row-kernel link bandwidth GB/s", "n_gpus": ngpu, "unit": "GB/s", "rows": nrows,
           "row_bytes": ROW_BYTES, "reps": reps}

    def gather_rate(dst_dev, seg_addr, random_rows, K=4096):
        """import_multi on dst_dev copying nrows rows of seg_addr (one node, stripe 0)."""
        with torch.cuda.device(dst_dev):
            R = (nrows + K - 1) // K
            g = torch.Generator(device="cuda").manual_seed(1)
            perm = torch.randperm(nrows, generator=g, device="cuda") if random_rows else \
                torch.arange(nrows, device="cuda")
            topk = torch.full((R * K,), -1, dtype=torch.int32, device="cuda")
            topk[:nrows] = perm.to(torch.int32)
            topk = topk.view(R, K)
            slots = torch.arange(R * K, dtype=torch.int32, device="cuda").view(R, K) % K
            miss = (topk >= 0).to(torch.int8)
            pool_idx = torch.arange(R, dtype=torch.int64, device="cuda")
            base = torch.zeros(R, dtype=torch.int64, device="cuda")
            nr = torch.tensor([R], dtype=torch.int32, device="cuda")
            hot = torch.empty(R * K * ROW_BYTES, dtype=torch.uint8, device="cuda")
            args_ = ([seg_addr], 0, nrows, ROW_BYTES, topk.data_ptr(), pool_idx.data_ptr(), base.data_ptr(),
                     slots.data_ptr(), miss.data_ptr(), nr.data_ptr(), hot.data_ptr(), K, R, 0, 0,
                     torch.cuda.current_stream().cuda_stream, 1)
            mod.import_multi(*args_, hot_req_stride_rows=K)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                mod.import_multi(*args_, hot_req_stride_rows=K)
            e1.record()
            torch.cuda.synchronize()
            return nrows * ROW_BYTES * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9

    # host link: rows read from pinned host memory
    hseg = mod.segment_alloc(-1, nbytes)
    out["host_read_contiguous"] = gather_rate(0, hseg, False)
    out["host_read_random"] = gather_rate(0, hseg, True)
    with torch.cuda.device(0):
        d = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            ok(cudart.cudaMemcpyAsync(d.data_ptr(), hseg, nbytes, cudart.cudaMemcpyKind.cudaMemcpyHostToDevice, s))
        e1.record()
        torch.cuda.synchronize()
        out["host_copy_engine_h2d"] = nbytes * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9
        del d
    with torch.cuda.device(0):  # host write: export_seg_alllayer of nrows contiguous rows into pinned memory
        src = torch.empty(nrows * ROW_BYTES, dtype=torch.uint8, device="cuda")
        st0 = torch.cuda.current_stream().cuda_stream
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        mod.export_seg_alllayer(0, hseg, nrows, ROW_BYTES, 0, nrows, 1, src.data_ptr(), 0, 0, 1, 0, 0, st0, 1)
        e0.record()
        for _ in range(reps):
            mod.export_seg_alllayer(0, hseg, nrows, ROW_BYTES, 0, nrows, 1, src.data_ptr(), 0, 0, 1, 0, 0, st0, 1)
        e1.record()
        torch.cuda.synchronize()
        out["host_write_contiguous"] = nrows * ROW_BYTES * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9
        del src
    mod.segment_free(hseg)
    out["host_link_gbs"] = max(out["host_read_contiguous"], out["host_copy_engine_h2d"])
    out["host_link_write_gbs"] = out["host_write_contiguous"]
    if ngpu >= 2:
        for a in range(ngpu):
            for b in range(ngpu):
                if a != b:
                    mod.enable_peer_access(a, b)
        segs = [mod.segment_alloc(g, nbytes) for g in range(ngpu)]
        out["peer_read_contiguous"] = gather_rate(0, segs[1], False)
        out["peer_read_random"] = gather_rate(0, segs[1], True)
        with torch.cuda.device(0):
            d = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
            s = torch.cuda.current_stream().cuda_stream
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                ok(cudart.cudaMemcpyPeerAsync(d.data_ptr(), 0, segs[1], 1, nbytes, s))
            e1.record()
            torch.cuda.synchronize()
            out["peer_copy_engine"] = nbytes * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9
            del d
        out["nvlink_gbs"] = max(out["peer_read_contiguous"], out["peer_copy_engine"])
        # every GPU at once reads random rows: from all other GPUs, and from one other GPU each
        out["all_peers_random_per_gpu"] = all_to_all(torch, mod, segs, ngpu, nrows, reps)
        out["one_peer_random_per_gpu"] = all_to_all(torch, mod, segs, ngpu, nrows, reps, one_peer=True)
        for a in segs:
            mod.segment_free(a)
        if args.link_span_gb > 2:  # the same reads drawn from segments of the decode pool's size
            span = args.link_span_gb << 30
            segs = [mod.segment_alloc(g, span) for g in range(ngpu)]
            out["span_gb"] = args.link_span_gb
            out["all_peers_random_per_gpu_span"] = all_to_all(torch, mod, segs, ngpu, nrows, reps,
                                                              seg_rows=span // ROW_BYTES)
            out["one_peer_random_per_gpu_span"] = all_to_all(torch, mod, segs, ngpu, nrows, reps, one_peer=True,
                                                             seg_rows=span // ROW_BYTES)
            out["own_random_span"] = all_to_all(torch, mod, segs, 1, nrows, reps, own=True,
                                                seg_rows=span // ROW_BYTES)
            for a in segs:
                mod.segment_free(a)
    print(json.dumps(out), flush=True)


def all_to_all(torch, mod, segs, ngpu, nrows, reps, one_peer=False, K=4096, seg_rows=None, own=False):
    """Every GPU at once gathers nrows random rows from other GPUs' segments: from all of them
    (striped, the pool layout of config 2) or, with one_peer, only from GPU (g + 1) % N; with own,
    from its own segment. Rows are drawn from the first seg_rows rows of each segment (default
    nrows / segments). One launch per GPU per repetition; returns per-GPU GB/s."""
    per = []
    setup = []
    for g in range(ngpu):
        with torch.cuda.device(g):
            others = [segs[g]] if own else [segs[(g + 1) % len(segs)]] if one_peer else \
                [segs[h] for h in range(len(segs)) if h != g]
            n = len(others)
            R = (nrows + K - 1) // K
            span = seg_rows if seg_rows else nrows // n
            gen = torch.Generator(device="cuda").manual_seed(g + 11)
            rows = torch.randint(0, span * n, (R * K,), generator=gen, device="cuda", dtype=torch.int64)
            topk = rows.to(torch.int32).view(R, K)
            slots = (torch.arange(R * K, dtype=torch.int32, device="cuda") % K).view(R, K)
            miss = torch.ones((R, K), dtype=torch.int8, device="cuda")
            pool_idx = torch.arange(R, dtype=torch.int64, device="cuda")
            base = torch.zeros(R, dtype=torch.int64, device="cuda")
            nr = torch.tensor([R], dtype=torch.int32, device="cuda")
            hot = torch.empty(R * K * ROW_BYTES, dtype=torch.uint8, device="cuda")
            st = torch.cuda.Stream()
            setup.append((others, topk, slots, miss, pool_idx, base, nr, hot, st, R, span))
    evs = []
    for g in range(ngpu):
        with torch.cuda.device(g):
            evs.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
    for phase in range(2):  # warm-up, then timed
        for g in range(ngpu):
            others, topk, slots, miss, pool_idx, base, nr, hot, st, R, span = setup[g]
            with torch.cuda.device(g):
                with torch.cuda.stream(st):
                    if phase:
                        evs[g][0].record(st)
                    for _ in range(reps if phase else 1):
                        mod.import_multi(others, 0, span, ROW_BYTES, topk.data_ptr(),
                                         pool_idx.data_ptr(), base.data_ptr(), slots.data_ptr(), miss.data_ptr(),
                                         nr.data_ptr(), hot.data_ptr(), K, R, 1, 0, st.cuda_stream, 1,
                                         hot_req_stride_rows=K)
                    if phase:
                        evs[g][1].record(st)
        for g in range(ngpu):
            torch.cuda.synchronize(g)
    for g in range(ngpu):
        R = setup[g][9]
        per.append(R * K * ROW_BYTES * reps / (evs[g][0].elapsed_time(evs[g][1]) * 1e-3) / 1e9)
    return per


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
            "sample": cp.describe(layer_steps), "us_per_layer_step": secs * 1e6 / layer_steps,
            "cpu_model": cpu_model(), "nproc": os.cpu_count()}


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
          "sample": "per step: " + cp.describe(L), "us_per_layer_step": secs * 1e6 / (L * args.steps),
          "cpu_model": cpu_model(), "nproc": os.cpu_count()}
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
    elif args.config == "link":
        run_link(args)
    elif args.config == "c4":
        run_export(args)
    elif args.config == "c5":
        run_stress(args)
    else:
        run_decode(args, CONFIGS[args.config])


if __name__ == "__main__":
    main()
