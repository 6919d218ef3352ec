"""Benchmark of the paged KV-cache transfer path on B200.

One step = store every chunk of the workload's token sequence from the paged
KV cache into its LMCache object (multi_layer_kv_transfer, direction=True)
and retrieve every chunk back (direction=False): the data-parallel hot path
of LMCache's GPU connector (VLLMPagedMemGPUConnectorV2.from_gpu / to_gpu),
one call per chunk and direction. Stores run on one stream and each chunk's
retrieve on a second stream after its store, the way a serving engine
overlaps offload and reload (the one-stream figures are reported too).

  value  KV payload GB/s (both directions; skipped slots excluded) with the
         LMCache objects in HBM, inputs resident before the timed region; the
         step's calls are captured once as a CUDA graph and replayed.
  e2e    the same step with the LMCache objects in pinned host memory (the
         deployment case: zero-copy PCIe writes on store, staged DMA reads on
         retrieve), called through c_ops from Python per chunk, with each
         chunk's slot mapping copied from pinned host memory inside the timed
         region.

Default workload c2 (Llama-3-8B: 32 layers, 8 x 128 heads, block_size 16,
8192 blocks per layer, 8192 tokens in 32 chunks of 256). Multi-GPU: one
process per GPU (torchrun); each rank moves its own KV shard with its own
seed; no collective is on the data path (gloo only for the start barrier and
the max-over-ranks timing).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2]
  python bench.py --impl reference      # CPU path of the reference semantics
  python bench.py --component cachegen  # CacheGen codec kernels
  python bench.py --component layerwise  # single_layer_kv_transfer, per chunk vs batched
  python bench.py --component rotary     # fused K re-rotation
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "lmcache-ascend_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "KV store/retrieve GB/s (HBM & pinned-host MemoryObj)"
# In the two-stream step, chunk i is retrieved once the store of chunk
# i + RETRIEVE_LAG has finished. The lag keeps a retrieve from reading object
# rows its own store has just left in L2, so the HBM figure is DRAM traffic.
RETRIEVE_LAG = 4
# The pinned-host step's lag: its objects live in host memory, so L2 reuse is
# moot, and every chunk the retrieve stream waits at the start (and the store
# stream idles at the end) is PCIe time with one direction idle: a step of n
# chunks takes about n + lag + 1 chunk times, so 32 chunks keep both
# directions busy for 32 / 37 of the step with a lag of 4 and 32 / 33 with
# none (each chunk's retrieve follows its own store).
HOST_RETRIEVE_LAG = 0
UNIT = "GB/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c2")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--component", default="transfer",
                    choices=["transfer", "cachegen", "layerwise", "rotary"],
                    help="cachegen: time the CacheGen CDF / encode / decode kernels instead; "
                         "layerwise: time the per-layer single_layer_kv_transfer path; "
                         "rotary: time the fused K re-rotation")
    ap.add_argument("--e2e-steps", type=int, default=None,
                    help="timed steps of the pinned-host leg (default: --steps)")
    ap.add_argument("--cpu-budget", type=float, default=15.0,
                    help="seconds of CPU work for the CPU baseline sample")
    ap.add_argument("--cpu-max-blocks", type=int, default=0,
                    help="paged blocks per layer of the host-resident CPU baseline buffers "
                         "(0: the workload's own count when host RAM allows)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c5-leg", action="store_true",
                    help="skip the pinned-host c5 (TP-8 shard) sub-measurement")
    ap.add_argument("--skip-e2e", action="store_true",
                    help="HBM leg only (kernel tuning runs; the line then has no e2e)")
    ap.add_argument("--blocks", type=int, default=None,
                    help="override paged blocks per layer (small profiling cases only)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# process group / clocks
# ---------------------------------------------------------------------------


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "source": "fallback"}


def measure_pcie(dev, stream, nbytes: int = 256 << 20, reps: int = 5) -> dict:
    """Copy-engine bandwidth between pinned host and HBM (cudaMemcpyAsync of
    `nbytes`, best of `reps`): the practical PCIe ceiling the pinned-host
    legs are compared with."""
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    devbuf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = {}
    for name, (dst, src) in (("h2d", (devbuf, host)), ("d2h", (host, devbuf))):
        best = 0.0
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dst.copy_(src, non_blocking=True)
            b.record(stream)
            torch.cuda.synchronize()
            best = max(best, nbytes / (a.elapsed_time(b) / 1e3) / 1e9)
        out[name] = round(best, 2)
    return out


def measure_pcie_duplex(dev, world: int, chunk: int = 32 << 20, n: int = 32) -> float:
    """Whole-job copy-engine bandwidth with both directions at once: on every
    rank an H2D stream and a D2H stream each copy `n` chunks of `chunk` bytes
    (bytes of all ranks and both directions over the slowest rank's time).
    The ceiling of the two-stream pinned-host step."""
    h_src = torch.empty(chunk * 4, dtype=torch.uint8).pin_memory()
    h_dst = torch.empty(chunk * 4, dtype=torch.uint8).pin_memory()
    d_src = torch.empty(chunk * 4, dtype=torch.uint8, device=dev)
    d_dst = torch.empty(chunk * 4, dtype=torch.uint8, device=dev)
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    best = 0.0
    for _ in range(3):
        torch.cuda.synchronize()
        barrier(world)
        cur = torch.cuda.current_stream()
        a = torch.cuda.Event(enable_timing=True)
        a.record(cur)
        up.wait_event(a)
        down.wait_event(a)
        for i in range(n):
            j = (i % 4) * chunk
            with torch.cuda.stream(up):
                d_dst[j:j + chunk].copy_(h_src[j:j + chunk], non_blocking=True)
            with torch.cuda.stream(down):
                h_dst[j:j + chunk].copy_(d_src[j:j + chunk], non_blocking=True)
        cur.wait_stream(up)
        cur.wait_stream(down)
        b = torch.cuda.Event(enable_timing=True)
        b.record(cur)
        torch.cuda.synchronize()
        ms = max_over_ranks(a.elapsed_time(b), world)
        best = max(best, world * 2 * n * chunk / (ms / 1e3) / 1e9)
    return round(best, 2)


def measure_pcie_concurrent(dev, stream, world: int, nbytes: int = 256 << 20,
                            reps: int = 3) -> dict:
    """Whole-job copy-engine bandwidth with every rank copying at once (host
    barrier, then each rank copies `nbytes` per rep; bytes of all ranks over
    the slowest rank's time): the host-side ceiling shared by all GPUs."""
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    devbuf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = {}
    for name, (dst, src) in (("h2d", (devbuf, host)), ("d2h", (host, devbuf))):
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            dst.copy_(src, non_blocking=True)
        b.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(a.elapsed_time(b), world)
        out[name] = round(world * reps * nbytes / (ms / 1e3) / 1e9, 2)
    return out


def workload_config(spec, world: int) -> dict:
    """The workload as both arms name it (identical keys and values)."""
    return {
        "workload": f"{spec.name}: {spec.description}",
        "num_layers": spec.num_layers,
        "kv_heads": spec.num_heads,
        "head_dim": spec.head_size,
        "block_size": spec.block_size,
        "blocks_per_layer": spec.num_blocks,
        "tokens": spec.num_tokens,
        "chunk_tokens": spec.chunk_size,
        "use_mla": spec.use_mla,
        "l2": "inputs larger than L2 (each step touches 2x payload of distinct paged rows and "
              "LMCache objects, >126 MB)",
        "parallelism": f"{world} independent ranks (per-rank KV shard), no collective",
    }


def committed_traffic(kernel: str, workload: str):
    """dram read+write bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------


def pinned_host_leg(spec, dev, world, rank, steps, warmup):
    """The two-stream pinned-host step (stores on one stream, chunk i's
    retrieve on a second stream after the store of chunk i + HOST_RETRIEVE_LAG)
    on every rank at once, each with its own seeded workload; returns the
    whole-job GB/s (payload of all ranks over the slowest rank's time)."""
    from lmcache_b200 import c_ops
    from lmcache_b200 import workloads as wl
    from lmcache_b200.v1.memory_management import PinMemoryAllocator

    caches = wl.make_kv_caches(spec, dev, seed=rank)
    ptrs = wl.pointer_tensor(caches, dev)
    slots = wl.make_slot_mapping(spec, seed=rank)
    host_chunks = [c.contiguous().pin_memory() for c in wl.chunks(slots, spec.chunk_size)]
    dev_bufs = [torch.empty_like(c, device=dev) for c in host_chunks]
    n = len(host_chunks)
    obj_bytes = sum(torch.Size(spec.memobj_shape(len(c))).numel() * 2 for c in host_chunks)
    arena = PinMemoryAllocator(obj_bytes + 256 * n + (1 << 20))
    objs = [arena.allocate(spec.memobj_shape(len(c)), torch.bfloat16).tensor for c in host_chunks]
    pbs = spec.page_buffer_size
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream(device=dev)
    lag = min(HOST_RETRIEVE_LAG, n - 1)

    def step():
        for i in range(n + lag):
            if i < n:
                dev_bufs[i].copy_(host_chunks[i], non_blocking=True)
                c_ops.multi_layer_kv_transfer(objs[i], ptrs, dev_bufs[i], dev, pbs, True,
                                              spec.use_mla)
            j = i - lag
            if j >= 0:
                side.wait_stream(stream)
                with torch.cuda.stream(side):
                    c_ops.multi_layer_kv_transfer(objs[j], ptrs, dev_bufs[j], dev, pbs, False,
                                                  spec.use_mla)
        stream.wait_stream(side)

    for _ in range(max(1, min(warmup, 3))):
        step()
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b), world)
    payload = 2 * wl.payload_bytes(spec, slots)
    value = sum_over_ranks(payload * steps, world) / (ms / 1e3) / 1e9
    arena.close()
    del caches, objs
    torch.cuda.empty_cache()
    return value


def run_ours(args):
    rank, world, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    from lmcache_b200 import c_ops
    from lmcache_b200 import workloads as wl
    from lmcache_b200.v1.gpu_connector import VLLMPagedMemGPUConnectorV2
    from lmcache_b200.v1.memory_management import MemoryFormat, PinMemoryAllocator

    spec = wl.SPECS[args.workload]
    if args.blocks:
        import dataclasses

        spec = dataclasses.replace(spec, num_blocks=args.blocks)
    seed = rank
    caches = wl.make_kv_caches(spec, dev, seed=seed)
    ptrs = wl.pointer_tensor(caches, dev)
    slots = wl.make_slot_mapping(spec, seed=seed)
    host_chunks = [c.contiguous().pin_memory() for c in wl.chunks(slots, spec.chunk_size)]
    dev_chunks = [c.to(dev) for c in host_chunks]
    n_chunks = len(dev_chunks)
    # The connector passes num_blocks * block_size for MLA caches too
    # (npu_connector.py:34-37); the kernels then bound-check MLA slots as well.
    pbs = spec.page_buffer_size
    payload = wl.payload_bytes(spec, slots)  # one direction, whole sequence
    step_payload = 2 * payload
    hbm_objs = [torch.empty(spec.memobj_shape(len(c)), dtype=torch.bfloat16, device=dev)
                for c in dev_chunks]
    stream = torch.cuda.current_stream()

    def run_dir(direction: bool):
        for i in range(n_chunks):
            c_ops.multi_layer_kv_transfer(hbm_objs[i], ptrs, dev_chunks[i], dev, pbs, direction,
                                          spec.use_mla)

    def step_hbm():
        run_dir(True)
        run_dir(False)

    # ---- value: HBM-resident objects, chunk loops replayed as CUDA graphs --
    # Each direction's chunk loop (the same c_ops calls, one kernel launch per
    # chunk) is captured once; replaying it removes the per-call host
    # overhead so the timed region measures the kernels back to back.
    for _ in range(args.warmup):
        step_hbm()
    torch.cuda.synchronize()
    graphs = {}
    for direction in (True, False):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            run_dir(direction)
        graphs[direction] = g
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        graphs[True].replay()
        graphs[False].replay()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    for k in range(args.steps):
        ev[k][0].record(stream)
        graphs[True].replay()
        ev[k][1].record(stream)
        graphs[False].replay()
        ev[k][2].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    t_ms = max_over_ranks(start.elapsed_time(end), world)
    total_payload = sum_over_ranks(step_payload * args.steps, world)
    value = total_payload / (t_ms / 1e3) / 1e9
    store_ms = sum(ev[k][0].elapsed_time(ev[k][1]) for k in range(args.steps))
    retr_ms = sum(ev[k][1].elapsed_time(ev[k][2]) for k in range(args.steps))
    n_launch = args.steps * n_chunks  # per direction
    n_valid = [int((c >= 0).sum()) for c in host_chunks]
    launch_payload = [n * spec.num_layers * spec.kv * spec.hidden * 2 for n in n_valid]
    # Algorithmic HBM bytes per launch: payload read + written, slot ids, layer pointers.
    alg = [2 * p + len(c) * 8 + spec.num_layers * 8 for p, c in zip(launch_payload, host_chunks)]
    alg_total = sum(alg) * 2 * args.steps
    # Kernel time per launch = graph replay time / launches (gaps included).
    achieved = alg_total / ((store_ms + retr_ms) / 1e3) / 1e9
    peaks = measured_peaks()
    avg_launch_ms = (store_ms + retr_ms) / (2 * n_launch)
    avg_alg = sum(alg) / len(alg)
    for g in graphs.values():
        g.reset()

    # Same step issued eagerly (one c_ops call per chunk from Python).
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0 = time.perf_counter()
    e0.record(stream)
    for _ in range(args.steps):
        step_hbm()
    e1.record(stream)
    host_s = time.perf_counter() - h0
    torch.cuda.synchronize()
    eager_ms = max_over_ranks(e0.elapsed_time(e1), world)
    value_eager = sum_over_ranks(step_payload * args.steps, world) / (eager_ms / 1e3) / 1e9
    host_us_per_call = host_s / (args.steps * 2 * n_chunks) * 1e6

    # Same calls captured as one graph with two chains: stores on the
    # capture stream, each chunk's retrieve on a second stream once the store
    # LAG chunks later has finished, so the launches of the two chains overlap
    # and a retrieve never reads an object still resident in L2 from its own
    # store (LAG x 64 MB of traffic passes in between, more than the 126 MB L2).
    lag = min(RETRIEVE_LAG, n_chunks - 1)
    side_hbm = torch.cuda.Stream(device=dev)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, capture_error_mode="thread_local"):
        cap = torch.cuda.current_stream()
        side_hbm.wait_stream(cap)
        # Issued in the order an engine would issue them: store chunk i, then
        # the retrieve that chunk i's store releases (chunk i - lag).
        for i in range(n_chunks + lag):
            if i < n_chunks:
                c_ops.multi_layer_kv_transfer(hbm_objs[i], ptrs, dev_chunks[i], dev, pbs, True,
                                              spec.use_mla)
            j = i - lag
            if j >= 0:
                # chunk j waits for the stores issued so far: through chunk
                # min(j + lag, last)
                side_hbm.wait_stream(cap)
                with torch.cuda.stream(side_hbm):
                    c_ops.multi_layer_kv_transfer(hbm_objs[j], ptrs, dev_chunks[j], dev, pbs,
                                                  False, spec.use_mla)
        cap.wait_stream(side_hbm)
    for _ in range(args.warmup):
        g2.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        g0.record(stream)
        for _ in range(args.steps):
            g2.replay()
        g1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    duplex_hbm_ms = max_over_ranks(g0.elapsed_time(g1), world)
    clock_summary = clocks.summary()
    value_duplex = sum_over_ranks(step_payload * args.steps, world) / (duplex_hbm_ms / 1e3) / 1e9
    duplex_frac = (sum(alg) * 2 * args.steps / (duplex_hbm_ms / 1e3) / 1e9) / measured_peaks()["hbm_gbs"]
    g2.reset()
    # Headline: the two-chain step. The single-stream figures above stay in
    # the line for comparison (value_single_stream, per-direction launch times).
    value_single = value
    frac_single = achieved / peaks["hbm_gbs"]
    value = value_duplex
    t_ms = duplex_hbm_ms
    achieved = alg_total / (duplex_hbm_ms / 1e3) / 1e9
    avg_launch_ms = duplex_hbm_ms / (2 * n_launch)

    # Same step with all chunks of each direction in one launch
    # (c_ops.multi_layer_kv_transfer_batched, what the connector's
    # batched_from_gpu / batched_to_gpu issue).
    slots_dev = slots.to(dev)
    bounds = [0]
    for c in host_chunks:
        bounds.append(bounds[-1] + len(c))

    def step_batched():
        for direction in (True, False):
            c_ops.multi_layer_kv_transfer_batched(hbm_objs, ptrs, slots_dev, bounds[:-1],
                                                  bounds[1:], dev, pbs, direction, spec.use_mla)

    for _ in range(args.warmup):
        step_batched()
    torch.cuda.synchronize()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(stream)
    for _ in range(args.steps):
        step_batched()
    b1.record(stream)
    torch.cuda.synchronize()
    batched_ms = max_over_ranks(b0.elapsed_time(b1), world)
    value_batched = sum_over_ranks(step_payload * args.steps, world) / (batched_ms / 1e3) / 1e9
    batched_frac = (sum(alg) * 2 * args.steps / (batched_ms / 1e3) / 1e9) / measured_peaks()["hbm_gbs"]

    # ---- e2e: pinned-host objects through c_ops ------------------------
    if args.skip_e2e:
        if rank == 0:
            print(json.dumps({"value": round(value, 2), "ms_per_step": round(t_ms / args.steps, 4),
                              "value_eager": round(value_eager, 2),
                              "value_batched": round(value_batched, 2),
                              "batched_frac": round(batched_frac, 4),
                              "value_single_stream": round(value_single, 2),
                              "single_stream_frac": round(frac_single, 4),
                              "host_us_per_call": round(host_us_per_call, 2),
                              "achieved": round(achieved, 1),
                              "frac": round(achieved / peaks["hbm_gbs"], 4),
                              "store_avg_us": round(store_ms / n_launch * 1e3, 2),
                              "retrieve_avg_us": round(retr_ms / n_launch * 1e3, 2),
                              "clocks": clock_summary}), flush=True)
        return
    obj_bytes = sum(torch.Size(spec.memobj_shape(len(c))).numel() * 2 for c in dev_chunks)
    arena = PinMemoryAllocator(obj_bytes + 256 * n_chunks + (1 << 20))
    obj_fmt = MemoryFormat.KV_MLA_FMT if spec.use_mla else MemoryFormat.KV_2LTD
    host_mobjs = [arena.allocate(spec.memobj_shape(len(c)), torch.bfloat16, obj_fmt)
                  for c in dev_chunks]
    host_objs = [m.tensor for m in host_mobjs]
    slot_dev_bufs = [torch.empty_like(c) for c in dev_chunks]

    def step_e2e():
        for i in range(n_chunks):
            slot_dev_bufs[i].copy_(host_chunks[i], non_blocking=True)
            c_ops.multi_layer_kv_transfer(host_objs[i], ptrs, slot_dev_bufs[i], dev, pbs, True,
                                          spec.use_mla)
        for i in range(n_chunks):
            c_ops.multi_layer_kv_transfer(host_objs[i], ptrs, slot_dev_bufs[i], dev, pbs, False,
                                          spec.use_mla)

    side = torch.cuda.Stream(device=dev)

    def step_e2e_duplex():
        """The same calls with the retrieves on a second stream, each chunk's
        retrieve ordered after its store: PCIe carries the stores' writes
        and the retrieves' reads at the same time (full duplex)."""
        lag = min(HOST_RETRIEVE_LAG, n_chunks - 1)
        # Issued in engine order: store chunk i, then the retrieve of chunk
        # i - lag, which waits for the stores issued so far.
        for i in range(n_chunks + lag):
            if i < n_chunks:
                slot_dev_bufs[i].copy_(host_chunks[i], non_blocking=True)
                c_ops.multi_layer_kv_transfer(host_objs[i], ptrs, slot_dev_bufs[i], dev, pbs,
                                              True, spec.use_mla)
            j = i - lag
            if j >= 0:
                side.wait_stream(stream)
                with torch.cuda.stream(side):
                    c_ops.multi_layer_kv_transfer(host_objs[j], ptrs, slot_dev_bufs[j], dev, pbs,
                                                  False, spec.use_mla)
        stream.wait_stream(side)

    e2e_steps = args.e2e_steps or args.steps
    for _ in range(max(1, min(args.warmup, 3))):
        step_e2e_duplex()
    torch.cuda.synchronize()
    barrier(world)
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    for _ in range(e2e_steps):
        step_e2e_duplex()
    d1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    duplex_ms = max_over_ranks(d0.elapsed_time(d1), world)
    e2e_duplex = sum_over_ranks(step_payload * e2e_steps, world) / (duplex_ms / 1e3) / 1e9

    e2e = {}
    for mode in ("zerocopy", "dma"):
        os.environ["LMCB_HOST_RETRIEVE"] = mode
        for _ in range(max(1, min(args.warmup, 3))):
            step_e2e()
        torch.cuda.synchronize()
        barrier(world)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(e2e_steps):
            step_e2e()
        s1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(s0.elapsed_time(s1), world)
        e2e[mode] = sum_over_ranks(step_payload * e2e_steps, world) / (ms / 1e3) / 1e9
    os.environ.pop("LMCB_HOST_RETRIEVE", None)
    # Separate store / retrieve pinned-host rates (zero-copy store; both retrieve paths).
    dir_rates = {}
    for label, direction, mode in (("store_zerocopy", True, "zerocopy"),
                                   ("store_dma", True, "dma"),
                                   ("retrieve_zerocopy", False, "zerocopy"),
                                   ("retrieve_dma", False, "dma")):
        os.environ["LMCB_HOST_RETRIEVE"] = mode
        os.environ["LMCB_HOST_STORE"] = mode
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(2):
            for i in range(n_chunks):
                c_ops.multi_layer_kv_transfer(host_objs[i], ptrs, dev_chunks[i], dev, pbs,
                                              direction, spec.use_mla)
        s1.record(stream)
        torch.cuda.synchronize()
        dir_rates[label] = round(2 * payload / (s0.elapsed_time(s1) / 1e3) / 1e9, 2)
    os.environ.pop("LMCB_HOST_RETRIEVE", None)
    os.environ.pop("LMCB_HOST_STORE", None)
    best_mode = max(e2e, key=e2e.get)

    # The connector LMCache's engine drives (pinned-host objects, device slot
    # mapping): per chunk (from_gpu / to_gpu, each returning once its host
    # object holds the data, as the engine expects) and batched
    # (batched_from_gpu / batched_to_gpu, one launch per direction).
    conn = VLLMPagedMemGPUConnectorV2(spec.hidden, spec.num_layers, use_mla=spec.use_mla)
    starts_c = [0]
    for c in host_chunks:
        starts_c.append(starts_c[-1] + len(c))
    conn_rates = {}
    for label in ("per_chunk", "batched"):
        def conn_step():
            if label == "per_chunk":
                for i, m in enumerate(host_mobjs):
                    conn.from_gpu(m, starts_c[i], starts_c[i + 1], kvcaches=caches,
                                  slot_mapping=slots_dev)
                for i, m in enumerate(host_mobjs):
                    conn.to_gpu(m, starts_c[i], starts_c[i + 1], kvcaches=caches,
                                slot_mapping=slots_dev)
            else:
                conn.batched_from_gpu(host_mobjs, starts_c[:-1], starts_c[1:], kvcaches=caches,
                                      slot_mapping=slots_dev)
                conn.batched_to_gpu(host_mobjs, starts_c[:-1], starts_c[1:], kvcaches=caches,
                                    slot_mapping=slots_dev)
        for _ in range(max(1, min(args.warmup, 3))):
            conn_step()
        torch.cuda.synchronize()
        barrier(world)
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(e2e_steps):
            conn_step()
        c1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(c0.elapsed_time(c1), world)
        conn_rates[label] = round(sum_over_ranks(step_payload * e2e_steps, world)
                                  / (ms / 1e3) / 1e9, 2)
    conn_rates["pointer_uploads"] = conn.pointer_uploads
    pcie = measure_pcie(dev, stream)
    pcie_all = measure_pcie_concurrent(dev, stream, world)
    pcie_duplex = measure_pcie_duplex(dev, world)
    # The TP-8 deployment case (Llama-3-70B shard, 256-byte rows, pinned-host
    # objects) on every rank at once, next to the main workload.
    c5 = None
    if spec.name != "c5" and not args.no_c5_leg:
        c5_spec = wl.SPECS["c5"]
        c5_value = pinned_host_leg(c5_spec, dev, world, rank, e2e_steps, args.warmup)
        c5 = {"workload": f"c5: {c5_spec.description}",
              "value": round(c5_value, 2), "unit": UNIT,
              "step": "store + retrieve of every chunk, pinned-host objects, two streams "
                      "(as e2e), all ranks at once, each with its own seeded shard",
              "frac_of_duplex_copy_engines": round(c5_value / pcie_duplex, 4)}

    # ---- CPU baseline (rank 0, N = 1) -----------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.cpu_baseline import CpuTransfer

        ct = CpuTransfer(spec, max_blocks=args.cpu_max_blocks, seed=0)
        m = ct.measure(args.cpu_budget)
        cpu = {
            "value": round(m["gbps"], 3),
            "unit": UNIT,
            "cores": m["threads"],
            "kind": "port",
            "sample": (f"torch index_select/index_copy_ store+retrieve of {m['chunks_per_step']} "
                       f"of {n_chunks} chunks x {m['steps']} steps ({m['seconds']:.1f} s), "
                       f"{spec.name} per-chunk shapes, "
                       + blocks_note(m["blocks_per_layer"], m["full_blocks_per_layer"])),
        }
        del ct

    if rank == 0:
        traffic = committed_traffic("transfer_rows_bulk_kernel", spec.name)
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(t_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 KV, seeded random block slot mappings)",
            "config": workload_config(spec, world),
            "step": "store all chunks then retrieve all chunks (one multi_layer_kv_transfer "
                    "per chunk and direction), captured once as a CUDA graph with two chains: "
                    "stores on one stream, chunk i's retrieve on a second stream after the "
                    f"store of chunk i+{RETRIEVE_LAG} (no L2 reuse between a store and its "
                    "retrieve)",
            "detail": {
                "value_single_stream": round(value_single, 2),
                "single_stream_roofline_frac": round(frac_single, 4),
                "value_eager": round(value_eager, 2),
                "host_us_per_call": round(host_us_per_call, 2),
                "value_batched": round(value_batched, 2),
                "batched_roofline_frac": round(batched_frac, 4),
                "payload_bytes_per_step_per_gpu": step_payload,
            },
            "e2e": {
                "value": round(e2e_duplex, 2),
                "unit": UNIT,
                "h2d_bytes_per_step": payload + sum(c.numel() * 8 for c in host_chunks),
                "d2h_bytes_per_step": payload,
                "path": "pinned-host MemoryObjs through c_ops, called per chunk from Python; "
                        "stores on one stream, chunk i's retrieve on a second stream after the "
                        f"store of chunk i+{HOST_RETRIEVE_LAG} (its own store when 0), so PCIe "
                        "carries both directions at once; objects of 8 MiB "
                        "and more go through a device staging buffer and one DMA per object, "
                        "smaller ones through zero-copy kernel accesses",
                "single_stream": round(e2e[best_mode], 2),
                "single_stream_by_retrieve_path": {k: round(v, 2) for k, v in e2e.items()},
                "per_direction_gbs": dir_rates,
                "connector": {
                    "path": "VLLMPagedMemGPUConnectorV2 with pinned-host KV_2LTD objects and "
                            "the slot mapping in HBM: per_chunk = from_gpu then to_gpu per "
                            "chunk (each call returns once its host object holds the data); "
                            "batched = batched_from_gpu + batched_to_gpu (one launch each)",
                    **conn_rates},
                "pcie_copy_engine_gbs": pcie,
                "pcie_copy_engine_all_ranks_gbs": pcie_all,
                # both directions run at once: the ceiling is the copy engines
                # running H2D and D2H together on every rank
                "pcie_copy_engine_duplex_all_ranks_gbs": pcie_duplex,
                "frac_of_duplex_copy_engines": round(e2e_duplex / pcie_duplex, 4),
                "c5_tp8_shard": c5,
            },
            "roofline": {
                "bound": "hbm",
                "kernel": "transfer_rows_bulk_kernel",
                "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"],
                "peak_source": peaks["source"],
                "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": traffic,
                "algorithmic_bytes_per_launch": round(avg_alg),
                "avg_launch_us": round(avg_launch_ms * 1e3, 2),
                "single_stream_store_avg_us": round(store_ms / n_launch * 1e3, 2),
                "single_stream_retrieve_avg_us": round(retr_ms / n_launch * 1e3, 2),
                "timing": "CUDA events around replays of the two-chain CUDA graph (the timed "
                          "region); per-launch time = replay time / launches. The single-stream "
                          "per-direction times come from replays of one-direction graphs.",
            },
            "cpu_baseline": cpu,
            "gpu_launches": args.steps * 2 * n_chunks * world,
            "clocks": clock_summary,
        }
        print(json.dumps(line), flush=True)
    arena.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# reference arm: the reference-semantics CPU path on the host cores
# ---------------------------------------------------------------------------


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    # Nothing of the lmcache_b200 package is imported here: the workload
    # definitions are loaded from their file, and the line reports which of
    # the package's native libraries ended up mapped (none).
    from oracle.cpu_baseline import CpuTransfer, load_workloads, mapped_product_libraries

    wl = load_workloads()
    spec = wl.SPECS[args.workload]
    ct = CpuTransfer(spec, max_blocks=args.cpu_max_blocks, seed=0)
    # Size one step to about 2 s of CPU work (at most the whole sequence).
    _, dt = ct.run_step(1)
    n = max(1, min(len(ct.chunks), int(2.0 / max(dt, 1e-6))))
    for _ in range(args.warmup):
        ct.run_step(n)
    total_b, total_t = 0, 0.0
    for _ in range(args.steps):
        b, t = ct.run_step(n)
        total_b += b
        total_t += t
    value = total_b / total_t / 1e9
    sample = (f"torch index_select/index_copy_ store+retrieve of {n} of {len(ct.chunks)} chunks "
              f"per step, {spec.name} per-chunk shapes, "
              + blocks_note(ct.spec.num_blocks, spec.num_blocks))
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_t / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded bf16 KV, seeded random block slot mappings)",
        "config": workload_config(spec, 1),
        "step": "store then retrieve a bounded sample of chunks on host cores (rank 0 only, "
                "all host threads)",
        "product_libraries_loaded": mapped_product_libraries(),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": ct.threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def blocks_note(blocks: int, full: int) -> str:
    if blocks == full:
        return f"full paged buffers ({full} blocks/layer, same slots as the GPU arm) in host RAM"
    return f"paged buffers reduced to {blocks} of {full} blocks/layer in host RAM"


def run_cachegen(args):
    """CacheGen codec on one c2-shaped chunk of quantised symbols
    ([32 layers, 256 tokens, 1024 channels], 32 bins, a skewed distribution
    per channel): GB/s of symbols through calculate_cdf, encode and decode,
    and the C oracle's single-thread rate on the same input."""
    import numpy as np

    from lmcache_b200 import c_ops
    from oracle import cachegen as cg

    dev = torch.device("cuda", 0)
    L, T, C, mb = 32, 256, 1024, 32
    rng = np.random.default_rng(0)
    p = np.exp(-np.arange(mb) / 4.0)
    p /= p.sum()
    sym = rng.choice(mb, size=(L, T, C), p=p).astype(np.uint8)
    sym_dev = torch.from_numpy(sym.view(np.int8)).to(dev)
    cap = 2 * T + 16
    out = torch.zeros((L, C, cap), dtype=torch.uint8, device=dev)
    lengths = torch.zeros((L, C), dtype=torch.int32, device=dev)
    dec = torch.empty_like(sym_dev)
    cdf = c_ops.calculate_cdf(sym_dev, mb)
    c_ops.encode_fast_new(cdf, sym_dev, out, lengths)

    def timed(fn, reps):
        for _ in range(args.warmup):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps / 1e3

    nbytes = sym.size
    t_cdf = timed(lambda: c_ops.calculate_cdf(sym_dev, mb), args.steps)
    t_enc = timed(lambda: c_ops.encode_fast_new(cdf, sym_dev, out, lengths), args.steps)
    t_dec = timed(lambda: c_ops.decode_fast_new(cdf, out, lengths, dec), args.steps)
    assert torch.equal(dec, sym_dev)
    comp = float(lengths.sum()) / nbytes
    cdf_np = cdf.cpu().numpy()
    t0 = time.perf_counter()
    streams, ln = cg.encode(cdf_np, sym, cap)
    t_cpu_enc = time.perf_counter() - t0
    t0 = time.perf_counter()
    cg.decode(cdf_np, streams, ln, T)
    t_cpu_dec = time.perf_counter() - t0
    line = {
        "metric": "CacheGen codec GB/s of symbols (calculate_cdf / encode / decode)",
        "value": round(nbytes / t_enc / 1e9, 3),
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "dtype": "u8",
        "data": "synthetic (seeded geometric-like symbol distribution)",
        "config": {"workload": "one c2 chunk of symbols [32 layers, 256 tokens, 1024 channels], "
                               "32 bins", "compressed_fraction": round(comp, 4)},
        "cdf_gbs": round(nbytes / t_cdf / 1e9, 3),
        "encode_gbs": round(nbytes / t_enc / 1e9, 3),
        "decode_gbs": round(nbytes / t_dec / 1e9, 3),
        "us": {"cdf": round(t_cdf * 1e6, 1), "encode": round(t_enc * 1e6, 1),
               "decode": round(t_dec * 1e6, 1)},
        "cpu_baseline": {"encode_gbs": round(nbytes / t_cpu_enc / 1e9, 4),
                         "decode_gbs": round(nbytes / t_cpu_dec / 1e9, 4), "cores": 1,
                         "kind": "port", "sample": "the C oracle on the same chunk"},
    }
    print(json.dumps(line), flush=True)


def run_layerwise(args):
    """The layerwise connector's path (single_layer_kv_transfer) on the c2
    workload: every layer of every 256-token chunk stored into, then
    retrieved from, token-major [T, 2, H] objects in HBM. Two ways to issue
    it:
    * per chunk: one single_layer_kv_transfer per (layer, chunk), as the
      reference's layerwise connector issues them (npu_connector.py:227-252);
    * batched: one single_layer_kv_transfer_batched per layer over all chunks,
      as this connector issues them."""
    from lmcache_b200 import c_ops
    from lmcache_b200 import workloads as wl

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    spec = wl.SPECS[args.workload]
    if spec.use_mla:
        raise SystemExit("layerwise: an MLA cache has no separate K and V caches")
    caches = wl.make_kv_caches(spec, dev, seed=0)
    slots = wl.make_slot_mapping(spec, seed=0)
    chunks = [c.to(dev) for c in wl.chunks(slots, spec.chunk_size)]
    slots_dev = slots.to(dev)
    bounds = [0]
    for c in chunks:
        bounds.append(bounds[-1] + len(c))
    H = spec.hidden
    objs = [[torch.empty((len(c), spec.kv, H), dtype=torch.bfloat16, device=dev) for c in chunks]
            for _ in range(spec.num_layers)]
    kv_of = [(t[0], t[1]) for t in caches]

    def per_chunk(direction):
        for layer in range(spec.num_layers):
            k, v = kv_of[layer]
            for i, c in enumerate(chunks):
                c_ops.single_layer_kv_transfer(objs[layer][i], k, v, c, direction, True)

    def batched(direction):
        for layer in range(spec.num_layers):
            k, v = kv_of[layer]
            c_ops.single_layer_kv_transfer_batched(objs[layer], k, v, slots_dev, bounds[:-1],
                                                   bounds[1:], direction, True)

    payload = wl.payload_bytes(spec, slots)  # one direction
    n_valid = int((slots >= 0).sum())
    alg = 2 * (2 * payload + n_valid * 8 * spec.num_layers)  # both directions, HBM bytes
    peak = measured_peaks()["hbm_gbs"]
    stream = torch.cuda.current_stream()
    out = {}
    # Both ways are replayed from CUDA graphs, so the figures are GPU time
    # (from Python a call costs ~5 us of host time, per chunk or batched).
    # The batched calls carry their object table in the kernel parameters,
    # which is what lets them be captured. The batched calls issued eagerly
    # are timed too (batched_eager).
    for name, fn, launches, graphed in (
            ("per_chunk", per_chunk, spec.num_layers * len(chunks), True),
            ("batched", batched, spec.num_layers, True),
            ("batched_eager", batched, spec.num_layers, False)):
        for _ in range(args.warmup):
            fn(True)
            fn(False)
        torch.cuda.synchronize()
        graphs = []
        if graphed:
            for direction in (True, False):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, capture_error_mode="thread_local"):
                    fn(direction)
                graphs.append(g)
            for _ in range(args.warmup):
                for g in graphs:
                    g.replay()
            run_step = [g.replay for g in graphs]
        else:
            run_step = [lambda: fn(True), lambda: fn(False)]
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            for run in run_step:
                run()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        for g in graphs:
            g.reset()
        out[name] = {"gbs": round(2 * payload / (ms / 1e3) / 1e9, 2),
                     "roofline_frac": round(alg / (ms / 1e3) / 1e9 / peak, 4),
                     "ms_per_step": round(ms, 4), "launches_per_step": 2 * launches,
                     "us_per_launch": round(ms * 1e3 / (2 * launches), 2)}
    # The connector keeps a store stream and a load stream (the reference's
    # npu_connector.py:103-145,219-256), so an engine's layer stores and layer
    # retrieves can overlap. Captured as one graph: stores on the capture
    # stream, layer l's retrieve on a second stream once the store of layer
    # l + lag has finished. The lag puts at least 256 MB of traffic between a
    # layer's store and its retrieve, so the retrieve reads from DRAM, not L2.
    layer_traffic = alg / 2 / spec.num_layers
    lag = min(spec.num_layers - 1, max(RETRIEVE_LAG, -(-(256 << 20) // int(layer_traffic))))
    side = torch.cuda.Stream(device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        cap = torch.cuda.current_stream()
        side.wait_stream(cap)
        for i in range(spec.num_layers + lag):
            if i < spec.num_layers:
                k, v = kv_of[i]
                c_ops.single_layer_kv_transfer_batched(objs[i], k, v, slots_dev, bounds[:-1],
                                                       bounds[1:], True, True)
            j = i - lag
            if j >= 0:
                side.wait_stream(cap)
                with torch.cuda.stream(side):
                    k, v = kv_of[j]
                    c_ops.single_layer_kv_transfer_batched(objs[j], k, v, slots_dev, bounds[:-1],
                                                           bounds[1:], False, True)
        cap.wait_stream(side)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    g.reset()
    out["batched_two_streams"] = {
        "gbs": round(2 * payload / (ms / 1e3) / 1e9, 2),
        "roofline_frac": round(alg / (ms / 1e3) / 1e9 / peak, 4),
        "ms_per_step": round(ms, 4), "launches_per_step": 2 * spec.num_layers,
        "retrieve_lag_layers": lag,
        "step": "stores on one stream, layer l's retrieve on a second stream after the store of "
                f"layer l+{lag}, one CUDA graph"}
    line = {
        "metric": "Layerwise KV store/retrieve GB/s (single_layer_kv_transfer)",
        "value": out["batched"]["gbs"],
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 KV, seeded random block slot mappings)",
        "config": {"workload": f"{args.workload}: every layer of every {spec.chunk_size}-token "
                               f"chunk, token-major [T, 2, H] objects in HBM, store then "
                               f"retrieve", "peak_hbm_gbs": peak},
        "per_chunk": out["per_chunk"],
        "batched": out["batched"],
        "batched_eager": out["batched_eager"],
        "batched_two_streams": out["batched_two_streams"],
    }
    print(json.dumps(line), flush=True)


def run_rotary(args):
    """rotary_embedding_k_fused (CacheBlend's K re-rotation) over the cached K
    of a c2-shaped request: 32 layers x 8192 tokens x 8 heads x 128 bf16 (512
    MiB, one call over all rows, as the op is per token), moved from positions
    0..8191 to 4096..12287, neox layout, fp32 cos/sin cache of 32768
    positions. GB/s of algorithmic HBM bytes (K read and written, each
    distinct cos/sin row once, two positions per token) against the copy
    roofline."""
    from lmcache_b200 import c_ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, T, heads, hd, max_pos = 32, 8192, 8, 128, 32768
    g = torch.Generator(device=dev).manual_seed(0)
    key = torch.randn(L * T, heads, hd, generator=g, device=dev).to(torch.bfloat16)
    old = torch.arange(T, device=dev, dtype=torch.int64).repeat(L)
    new = old + 4096
    inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    freqs = torch.outer(torch.arange(max_pos, dtype=torch.float64), inv)
    cache = torch.cat([freqs.cos(), freqs.sin()], dim=-1).to(torch.float32).to(dev)
    n = L * T
    # K read and written, each distinct cos/sin row read once (positions repeat
    # across layers, so the per-token re-reads hit L2), both positions read.
    distinct_rows = int(torch.unique(torch.cat([old, new])).numel())
    alg = 2 * key.numel() * key.element_size() + distinct_rows * hd * 4 + n * 2 * 8
    for _ in range(args.warmup):
        c_ops.rotary_embedding_k_fused(old, new, key, hd, cache, True)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        c_ops.rotary_embedding_k_fused(old, new, key, hd, cache, True)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    peak = measured_peaks()["hbm_gbs"]
    gbs = alg / (ms / 1e3) / 1e9
    line = {
        "metric": "Fused K re-rotation GB/s (rotary_embedding_k_fused)",
        "value": round(gbs, 2),
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "dtype": "bf16 keys, fp32 math",
        "data": "synthetic (seeded N(0,1) bf16 K)",
        "config": {"workload": "c2-shaped K: 32 layers x 8192 tokens x 8 heads x 128, neox, "
                               "positions +4096, fp32 cos/sin cache of 32768 positions",
                   "algorithmic_bytes": alg},
        "us_per_call": round(ms * 1e3, 1),
        "roofline_frac": round(gbs / peak, 4),
        "peak_hbm_gbs": peak,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.component == "cachegen":
        run_cachegen(args)
    elif args.component == "layerwise":
        run_layerwise(args)
    elif args.component == "rotary":
        run_rotary(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
