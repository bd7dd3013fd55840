#!/usr/bin/env python3
"""Benchmark: Llama-70B-shaped int8 weight fetch (the sharded weight-fetch configuration).

One step = one model pass: 16 layers x {q, k, v, o, gate, up, down} int8
[out, in] matrices with per-row f32 scales (lognormal(-5, 0.5)), held in
pinned host memory, each moved to the GPU, dequantized, narrowed to f16 (RNE)
and transposed to [in, out] by the fused sm_100a kernel. With N GPUs (default
`--multi peer`) rank k copies the contiguous int8 source rows of its shard of
every matrix (sized by each GPU's measured concurrent host-to-device
bandwidth, `--balance 1`) into its own HBM, and every rank's kernels read all
shards -- its peers' over NVLink through CUDA IPC mappings -- writing the full
f16 layer locally: NVLink carries int8, not f16. `--multi allgather`: every
rank produces its 1/N window of result rows and an in-place NCCL all-gather
assembles the layer.

Metric: layers/s of the whole job (every layer assembled on every GPU), with
relocated GB/s and its fraction of the measured pinned-memcpy H2D ceiling
alongside.

  value           : host-to-device + transform (the metric's own work): int8
                    in pinned host memory when the timed region starts, every
                    layer crosses PCIe inside it; CUDA events on the caller
                    stream, max over ranks.
  e2e             : the same job through the public API a user calls (N = 1:
                    pyreloc.execute_dispatch, the drop-in C-ABI call, once per
                    matrix; N > 1: workloads.PeerShardedFetch), plus a
                    device-to-host read of the step's result; host wall clock
                    between synchronization points, max over ranks.
  device_resident : the transform kernels alone with the int8 already in HBM
                    (peer reads over NVLink for N > 1), for the kernel
                    roofline; not the metric.

After the timed regions the last assembled layer is hashed (SHA-256 per
matrix): every rank's digests must agree, rank 0 compares them with the
single-GPU path on the same synthetic layer (N > 1), and at N = 1 the
CPU-baseline leg compares them with the reference executor's output. A
mismatch exits 1.

Synthetic data (no checkpoints): int8 uniform[-127, 127]; scales
exp(N(-5, 0.5)); seed = layer index. Host memory holds `--distinct-layers`
(default 2) layers and the 16 layers of a step cycle over them -- every layer
still crosses PCIe in full; layers are 855 MB >> L2 (126 MB) and >> the host
LLC, so no cache can serve a repeat.

`--impl reference`: the reference's own CPU executor (oracle/_ref, typed::
executeHost with a GatherPool of every host core) on a bounded sample of
the same workload (one layer per step), rank 0 only.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

METRIC = "relocated GB/s/GPU (H2D+transform) as % of pinned memcpy ceiling; layers/s"
LLAMA70B = [("q", 8192, 8192), ("k", 1024, 8192), ("v", 1024, 8192), ("o", 8192, 8192),
            ("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672)]  # (name, out, in)
LAYERS = 16
LLAMA7B = [("q", 4096, 4096), ("k", 4096, 4096), ("v", 4096, 4096), ("o", 4096, 4096),
           ("gate", 11008, 4096), ("up", 11008, 4096), ("down", 4096, 11008)]
# --config -> (matrix shapes, layers per step, workload name)
MODELS = {"c5": (LLAMA70B, LAYERS, "llama70b_int8_fetch"), "c4": (LLAMA7B, 32, "llama7b_int8_fetch")}
# DRAM bytes (read + write) per element of the gate launch, from one ncu
# capture of `bench.py --kernel-case` (k_tma_tall, dynamic tile order):
# 235.2 MB + 412.2 MB over 28672 x 8192 elements. Writes sit below the
# algorithmic 2 B/element because the last dirty lines are still in L2 when
# the kernel ends.
GATE_DRAM_BYTES_PER_ELEM = (235.18976e6 + 412.207872e6) / (28672 * 8192)


def int8_tile_kernel():
    """Name of the TMA kernel that moves int8 weight matrices whose source
    rows are whole 128-row tiles (the library's SYM_B200_TMA_TALL switch)."""
    return "k_tma_tile" if os.environ.get("SYM_B200_TMA_TALL", "1")[:1] == "0" else "k_tma_tall"


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def make_layer(seed, shapes=None):
    rng = np.random.default_rng(seed)
    mats = []
    for name, out_f, in_f in shapes or LLAMA70B:
        q = rng.integers(-127, 128, size=(out_f, in_f), dtype=np.int8)
        scale = np.exp(rng.normal(-5.0, 0.5, out_f)).astype(np.float32)
        mats.append((name, q, scale))
    return mats


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------

def run_reference(args):
    from helpers import encode, recipe_c4
    from oracle import ref

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if not ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "reference runtime (oracle/_ref) not built"}))
        return 0
    threads = len(os.sched_getaffinity(0))
    pool = ref.GatherPool(threads)
    shapes, _, workload = MODELS[args.config]
    blob = encode(recipe_c4())
    mats = make_layer(0, shapes)
    progs = []
    for name, q, scale in mats:
        out_f, in_f = q.shape
        p = ref.TypedProgram(blob, {"out_features": out_f, "in_features": in_f},
                             {"scale": ("float32", [out_f], scale.tobytes())})
        progs.append((p, q.reshape(-1).view(np.uint8), np.empty(out_f * in_f * 2, np.uint8)))

    def step():
        for p, src, dst in progs:
            p.execute_into(src, dst, pool=pool)

    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    layers_per_s = args.steps / total
    elems = sum(o * i for _, o, i in shapes)
    line = {
        "impl": "reference", "metric": METRIC, "value": layers_per_s, "unit": "layers/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8->f16", "data": "synthetic",
        "config": {"workload": workload, "layers": 1, "matrices": [m[0] for m in shapes],
                   "executor": "reference typed::executeHost host->host (TiledTranspose), GatherPool"},
        "gbs_source": elems / (total / args.steps) / 1e9,
        "cpu_baseline": {"value": layers_per_s, "unit": "layers/s", "cores": pool.threads, "kind": "reference",
                         "sample": f"one layer ({len(shapes)} matrices, {elems:,} int8 elements) per step"},
        "e2e": {"value": layers_per_s, "unit": "layers/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def gpu_selector(torch, device_index):
    """nvidia-smi's -i argument for this process's GPU: its UUID (robust to
    CUDA_VISIBLE_DEVICES), else the physical index."""
    try:
        uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        if uuid:
            return uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
        pass
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        return visible.split(",")[device_index].strip()
    return str(device_index)


class Clocks:
    """nvidia-smi samples of ONE GPU (read-only queries) during a timed
    region; the reported clock is the median of the samples taken under load
    (utilization above zero)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, selector):
        self.selector = selector
        self.path = Path(tempfile.mkstemp(prefix="clocks", suffix=".csv")[1])
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.selector, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                rows.append((float(f[0]), float(f[1]), float(f[3]), f[4:8]))
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        loaded = [r for r in rows if r[2] > 0] or rows
        reasons = sorted({n for r in loaded for n, v in zip(self.REASONS, r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded) if loaded else None,
                "sm_max_mhz": max(r[1] for r in rows) if rows else None, "reasons": reasons,
                "samples": len(rows), "samples_under_load": len([r for r in rows if r[2] > 0]),
                "gpu": self.selector}


def pinned_h2d_gbs(torch, device, nbytes=256 << 20, reps=10, d2h=False):
    """Best-of-``reps`` pinned cudaMemcpyAsync H2D (or D2H) GB/s of this GPU
    alone."""
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    gpu = torch.empty(nbytes, dtype=torch.uint8, device=device)
    src, dst = (gpu, host) if d2h else (host, gpu)
    s = torch.cuda.Stream(device)
    best = 0.0
    with torch.cuda.stream(s):
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            dst.copy_(src, non_blocking=True)
            b.record(s)
            b.synchronize()
            best = max(best, nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    return best


def sustained_h2d_gbs(torch, device, barrier, hosts, reps=2):
    """Sustained pinned H2D GB/s of this GPU while every rank copies at once:
    the workload's own pinned host buffers (one layer's matrices, so the same
    memory and NUMA placement as the timed copies) copied ``reps`` times back
    to back into one device scratch buffer, started together after a
    barrier. The job's host-to-device bound is the sum over ranks."""
    flat = [h.reshape(-1).view(torch.uint8) for h in hosts]
    gpu = torch.empty(max(f.numel() for f in flat), dtype=torch.uint8, device=device)
    s = torch.cuda.Stream(device)
    with torch.cuda.stream(s):
        gpu[:flat[0].numel()].copy_(flat[0], non_blocking=True)
    s.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        a.record(s)
        for _ in range(reps):
            for f in flat:
                gpu[:f.numel()].copy_(f, non_blocking=True)
        b.record(s)
    b.synchronize()
    rate = sum(f.numel() for f in flat) * reps / (a.elapsed_time(b) * 1e-3) / 1e9
    del gpu
    return rate


def device_map(mode, local, world, visible):
    """GPU index of local rank `local`: identity, or `halves` -- ranks
    alternate between the two halves of the visible GPUs (0, V/2, 1, V/2+1,
    ...), which sit behind different host bridges on the pool's 8-GPU boxes,
    so N < V ranks do not share one bridge's host-to-device bandwidth."""
    if mode == "identity" or world >= visible or visible < 2:
        return local
    half = visible // 2
    return (local % 2) * half + local // 2


def layer_digests(torch, outs):
    """SHA-256 of each matrix's result bytes (the output check)."""
    return [hashlib.sha256(o.contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest() for o in outs]


def run_ours(args):
    import torch
    import torch.distributed as dist

    from helpers import encode, recipe_c4
    from sym_b200 import pyreloc

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    gpu_index = device_map(args.gpu_map, local, world, torch.cuda.device_count())
    torch.cuda.set_device(gpu_index)
    dev = torch.device("cuda", gpu_index)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[gpu_index])

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather(obj):
        if world == 1:
            return [obj]
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    # A retained quota that holds the ring (4 x 16 MiB) and the parameters, so
    # blocking calls keep their scratch between matrices (the reference's
    # 64 MiB default would release and re-allocate it after every call).
    res = pyreloc.DispatchResources(max_retained_bytes=256 << 20)
    _, compute_s = res.streams(gpu_index)
    compute_stream = torch.cuda.ExternalStream(compute_s, device=dev)

    # host data and templates
    shapes, n_layers, workload = MODELS[args.config]
    blob = encode(recipe_c4())
    plan = pyreloc.load_typed_plan(blob)
    distinct = []
    for d in range(args.distinct_layers):
        mats = []
        for name, q, scale in make_layer(d, shapes):
            out_f, in_f = q.shape
            bound = pyreloc.bind_typed(plan, {"out_features": out_f, "in_features": in_f},
                                       {"scale": ("float32", [out_f], scale.tobytes())})
            tmpl = pyreloc.prepare_dispatch_template(bound, "h2d", "cuda", implementation="b200_fused_h2d@dma_ring")
            host = torch.from_numpy(q).pin_memory()
            mats.append({"name": name, "out": out_f, "in": in_f, "tmpl": tmpl, "host": host, "dev": host.to(dev),
                         "scale": scale,
                         "sv": pyreloc.BufferView(host.data_ptr(), host.numel(), 0, [out_f, in_f], [in_f, 1], 1,
                                                  "host", -1)})
        distinct.append(mats)
    outs = [[torch.empty((m["in"], m["out"]), dtype=torch.float16, device=dev) for m in distinct[0]]
            for _ in range(2)]
    from sym_b200.workloads import PeerShardedFetch, ShardedLayerFetch

    sample = torch.empty(32, dtype=torch.float16).pin_memory()
    # Host-to-device bandwidth: this GPU alone (best of 10 256 MiB copies) and
    # sustained while every rank copies one layer's host buffers twice at once
    # (the job's bound; taken again after the timed regions, the higher of the
    # two is the ceiling, since the box's host bandwidth is shared with other
    # jobs and drifts).
    alone = pinned_h2d_gbs(torch, dev)
    layer_hosts = [m["host"] for m in distinct[0]]
    concurrent = sustained_h2d_gbs(torch, dev, barrier, layer_hosts)
    rates = gather(concurrent)
    peer = args.multi == "peer" and (world > 1 or args.n1_path == "peer")
    weights = rates if (peer and args.balance) else None
    if peer:
        fetcher = PeerShardedFetch(res, gpu_index, world, rank, [(m["out"], m["in"]) for m in distinct[0]],
                                   weights=weights, buffers=len(distinct), copy_chunk_bytes=args.peer_copy_chunk)
        for d, mats in enumerate(distinct):
            fetcher.preload(d, [m["host"] for m in mats])
        torch.cuda.synchronize(dev)
        barrier()
    else:
        fetcher = ShardedLayerFetch(res, gpu_index, world, rank, chunk_bytes=args.chunk_bytes,
                                    ring_slots=args.ring_slots, route=args.route)

    def layer(l, host_source):
        mats = distinct[l % len(distinct)]
        if peer:
            hosts = [m["host"] for m in mats] if host_source else None
            return fetcher.fetch([m["tmpl"] for m in mats], outs[l % 2], l % len(distinct), hosts)
        return fetcher.fetch(mats, outs[l % 2], host_source)

    def step(host_source):
        handles = []
        for l in range(n_layers):
            handles += layer(l, host_source)
            if len(handles) > 7 * 2:  # bound outstanding collectives to two layers
                for h in handles[:-7]:
                    h.wait()
                handles = handles[-7:]
        for h in handles:
            h.wait()

    cur = torch.cuda.current_stream(dev)

    def public_step():
        """One step through the public API, with the result read back."""
        if world == 1:
            pending = []  # submitted layers, at most two in flight
            for l in range(n_layers):
                views = []
                for m, out in zip(distinct[l % len(distinct)], outs[l % 2]):
                    dv = pyreloc.BufferView(out.data_ptr(), out.numel() * 2, 0, [m["in"], m["out"]],
                                            [m["out"], 1], 2, "cuda", gpu_index)
                    views.append((m, dv))
                if args.e2e_api in ("submit", "group"):  # one transfer group per layer, one completion
                    group = pyreloc.prepare_dispatch_group([(m["tmpl"], m["sv"], dv, "h2d") for m, dv in views])
                    if args.e2e_api == "group":
                        pyreloc.execute_dispatch_group(group, resources=res, caller_stream=cur.cuda_stream,
                                                       chunk_size=args.chunk_bytes, n_buffers=args.ring_slots)
                        continue
                    if len(pending) == 2:
                        pending.pop(0).wait()
                    pending.append(pyreloc.submit_dispatch_group(group, resources=res, caller_stream=cur.cuda_stream,
                                                                 chunk_size=args.chunk_bytes,
                                                                 n_buffers=args.ring_slots))
                    continue
                for m, dv in views:  # one blocking dispatch per matrix
                    req = pyreloc.prepare_dispatch_from_template(m["tmpl"], m["sv"], dv)
                    pyreloc.execute_dispatch(req, resources=res, caller_stream=cur.cuda_stream,
                                             chunk_size=args.chunk_bytes, n_buffers=args.ring_slots)
            for c in pending:
                c.wait()
        else:
            step(True)
        sample.copy_(outs[(n_layers - 1) % 2][-1].view(-1)[:32], non_blocking=True)
        torch.cuda.synchronize(dev)

    def timed(host_source, steps):
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            step(host_source)
        b.record()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        return max_over_ranks(a.elapsed_time(b) * 1e-3)

    def timed_public(steps):
        torch.cuda.synchronize(dev)
        barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            public_step()
        dt = time.perf_counter() - t0
        barrier()
        return max_over_ranks(dt)

    for _ in range(args.warmup):
        step(True)
        step(False)
        public_step()
    torch.cuda.synchronize(dev)

    clocks = Clocks(gpu_selector(torch, gpu_index))
    clocks.start()
    l0 = pyreloc.kernel_launches()
    t_value = timed(True, args.steps)
    l1 = pyreloc.kernel_launches()
    t_e2e = timed_public(args.steps)
    t_dev = timed(False, args.steps)
    ck = clocks.stop()
    launches_value = l1 - l0
    clock_records = gather(ck)
    rates_pre = rates
    rates = [max(x, y) for x, y in zip(rates_pre, gather(sustained_h2d_gbs(torch, dev, barrier, layer_hosts)))]

    # Output check: the last layer the e2e region assembled, on every rank.
    last = (n_layers - 1) % len(distinct)
    digests = layer_digests(torch, outs[(n_layers - 1) % 2])
    all_digests = gather(digests)
    check = {"sha256_last_layer": digests, "layer_seed": last,
             "ranks_agree": all(d == digests for d in all_digests)}
    if world > 1 and rank == 0:
        # the single-GPU path on the same synthetic layer, into fresh buffers
        single = []
        for m in distinct[last]:
            o = torch.empty((m["in"], m["out"]), dtype=torch.float16, device=dev)
            pyreloc.execute_rows(m["tmpl"], m["host"].data_ptr(), o.data_ptr(), 0, m["in"], device=gpu_index,
                                 host_source=True, resources=res)
            single.append(o)
        check["vs_single_gpu"] = "match" if layer_digests(torch, single) == digests else "mismatch"
        del single

    # dominant kernel (k_tma_tile<1, ...>, every launch of the step): one launch on the
    # largest matrix (gate), device-resident source, timed on the compute stream it
    # runs on. Algorithmic bytes per launch: 1 B int8 read + 2 B f16 written per
    # element + 4 B per source-row scale.
    torch.cuda.synchronize(dev)
    gi = [m["name"] for m in distinct[0]].index("gate")
    gm, gout = distinct[0][gi], outs[0][gi]

    def gate_launch():
        pyreloc.execute_rows(gm["tmpl"], gm["dev"].data_ptr(), gout.data_ptr(), 0, gm["in"], device=gpu_index,
                             host_source=False, resources=res, async_completion=True)

    for _ in range(3):
        gate_launch()
    # 705 MB per launch: larger than L2, so launches do not hit each other's
    # lines. Each launch between its own pair of events; median and p95.
    reps = 20
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    marks[0].record(compute_stream)
    for i in range(reps):
        gate_launch()
        marks[i + 1].record(compute_stream)
    torch.cuda.synchronize(dev)
    launch_s = sorted(marks[i].elapsed_time(marks[i + 1]) * 1e-3 for i in range(reps))
    kernel_s = statistics.median(launch_s)
    kernel_p95_s = launch_s[int(0.95 * (reps - 1) + 0.5)]
    gate_elems = gm["out"] * gm["in"]
    kernel_bytes = gate_elems * 3 + gm["out"] * 4
    achieved_gbs = kernel_bytes / kernel_s / 1e9
    # the ncu capture is of the 70B gate launch; other shapes carry no traffic figure
    traffic = GATE_DRAM_BYTES_PER_ELEM * gate_elems if args.config == "c5" else None

    layer_src_bytes = sum(o * i for _, o, i in shapes)
    layers_value = args.steps * n_layers / t_value
    layers_e2e = args.steps * n_layers / t_e2e
    layers_dev = args.steps * n_layers / t_dev
    aggregate_ceiling = sum(rates)  # GB/s of the whole box while every rank copies
    bound_layers = aggregate_ceiling * 1e9 / layer_src_bytes
    gpus = gather(gpu_index)

    if peer:
        fetcher.close()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return 0
    peaks = _peaks()
    hbm = peaks.get("hbm_gbs")
    peak_note = "measured" if hbm else "fallback"
    hbm = hbm or 6650.0
    cpu = None
    from oracle import ref

    if world == 1 and ref.available():
        cpu = cpu_baseline(distinct[last], digests)
        check["vs_reference"] = cpu.pop("output_check")
    ok = check["ranks_agree"] and check.get("vs_single_gpu", "match") == "match" and \
        check.get("vs_reference", "match") == "match"
    check["status"] = "match" if ok else "mismatch"
    extras = run_extras() if (world == 1 and args.extras) else None
    gbs_job = layer_src_bytes * layers_value / 1e9
    if peer and world == 1:
        shard = "one shard per matrix: one DMA per matrix into HBM, then one tile launch (the N>1 fetch path)"
    elif peer:
        shard = ("int8 source rows per rank (weighted by sustained concurrent H2D bandwidth)" if args.balance
                 else "int8 source rows per rank, equal") + "; every rank's kernels read all shards (peers' over " \
                                                           "NVLink, CUDA IPC)"
    elif world > 1:
        shard = "result rows [k*in/N,(k+1)*in/N) + in-place NCCL all-gather"
    else:
        shard = "none"
    line = {
        "metric": METRIC, "value": layers_value, "unit": "layers/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_value / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8->f16", "data": "synthetic",
        "config": {"workload": workload, "layers_per_step": n_layers,
                   "matrices": {n: [o, i] for n, o, i in shapes}, "distinct_host_layers": args.distinct_layers,
                   "shard": shard, "shard_weights": weights, "gpu_map": args.gpu_map, "gpus": gpus,
                   "route": args.route, "ring_slots": args.ring_slots, "chunk_bytes": args.chunk_bytes,
                   "l2": "inputs larger than L2 (855 MB int8 per layer)",
                   "value_timing": "CUDA events on the caller stream around the steps, max over ranks"},
        "gbs_per_gpu": gbs_job / world, "gbs_job": gbs_job,
        "pinned_h2d_sustained_gbs_per_rank": rates, "pinned_h2d_sustained_gbs_per_rank_before": rates_pre,
        "pinned_h2d_aggregate_gbs": aggregate_ceiling,
        "pinned_h2d_alone_gbs": alone,
        "pct_of_pinned_memcpy": 100.0 * gbs_job / aggregate_ceiling,
        "h2d_bound_layers_per_s": bound_layers,
        "e2e": {"value": layers_e2e, "unit": "layers/s", "ms_per_step": 1e3 * t_e2e / args.steps,
                "h2d_bytes_per_step": int(layer_src_bytes / world * n_layers),
                "d2h_bytes_per_step": int(sample.numel() * 2),
                "api": ({"submit": "pyreloc.submit_dispatch_group per layer (sb_submit_dispatch_group, two layers "
                                   "in flight, each completion waited)",
                         "group": "pyreloc.execute_dispatch_group per layer (sb_execute_dispatch_group)",
                         "dispatch": "pyreloc.execute_dispatch per matrix (sb_execute_dispatch)"}[args.e2e_api])
                       if world == 1 else
                       "workloads.PeerShardedFetch.fetch" if peer else "workloads.ShardedLayerFetch.fetch",
                "timing": "host wall clock between synchronizations, max over ranks",
                "pct_of_pinned_memcpy": 100.0 * layer_src_bytes * layers_e2e / 1e9 / aggregate_ceiling},
        "device_resident": {"value": layers_dev, "unit": "layers/s", "ms_per_step": 1e3 * t_dev / args.steps,
                            "note": "int8 already in HBM; transform kernels only"
                                    + (" (peer shards read over NVLink)" if peer else "")},
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm, "unit": "GB/s",
                     "frac": achieved_gbs / hbm, "traffic": traffic, "peak_source": peak_note,
                     "kernel": f"{int8_tile_kernel()}<int8, CH_DQ_F16, per-column scale> on gate [{gm['out']}, {gm['in']}]",
                     "bytes_per_launch": kernel_bytes, "launch_ms": kernel_s * 1e3,
                     "launch_ms_p95": kernel_p95_s * 1e3, "launches_timed": reps,
                     "bytes_per_launch_note": "int8 read + f16 write per element + 4 B per source-row scale",
                     "traffic_note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the full gate launch "
                                     "(--kernel-case)"},
        "output_check": check,
        "gpu_launches": int(launches_value), "clocks": _merge_clocks(clock_records),
    }
    if cpu:
        line["cpu_baseline"] = cpu
    if extras:
        line["configs"] = extras
    print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0 if ok else 1


def _merge_clocks(records):
    """One clock record for the job: the lowest per-GPU median under load,
    the union of the reasons seen, every GPU's own record beside them."""
    meds = [r.get("sm_mhz") for r in records if r.get("sm_mhz") is not None]
    maxes = [r.get("sm_max_mhz") for r in records if r.get("sm_max_mhz") is not None]
    reasons = sorted({x for r in records for x in r.get("reasons", [])})
    return {"sm_mhz": min(meds) if meds else None, "sm_max_mhz": max(maxes) if maxes else None,
            "reasons": reasons, "per_gpu": records}


def host_info():
    """The host the CPU baseline ran on: logical CPUs, the CPUs this process
    may use, the CPU model and the NUMA nodes."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        nodes = sorted(n for n in os.listdir("/sys/devices/system/node") if n.startswith("node") and n[4:].isdigit())
    except OSError:
        nodes = []
    return {"nproc": os.cpu_count(), "affinity": len(os.sched_getaffinity(0)), "cpu_model": model,
            "numa_nodes": len(nodes) or None}


def cpu_baseline(mats, digests, seconds=10.0):
    """The reference CPU executor (typed::executeHost, GatherPool of every
    usable host thread) on the bench's last synthetic layer, whole: repeated
    for about ``seconds`` (at least once), then once with 8 threads (the
    reference's own qualified setting). Its result's digests are compared with
    the GPU's (the output check)."""
    from helpers import encode, recipe_c4
    from oracle import ref

    threads = len(os.sched_getaffinity(0))
    blob = encode(recipe_c4())
    progs = []
    for m in mats:
        p = ref.TypedProgram(blob, {"out_features": m["out"], "in_features": m["in"]},
                             {"scale": ("float32", [m["out"]], m["scale"].tobytes())})
        progs.append((p, m["host"].numpy().reshape(-1).view(np.uint8), np.empty(m["out"] * m["in"] * 2, np.uint8)))

    def layer(pool):
        for p, src, dst in progs:
            p.execute_into(src, dst, pool=pool)

    pool = ref.GatherPool(threads)
    t0 = time.perf_counter()
    layer(pool)
    busy = time.perf_counter() - t0
    ref_digests = [hashlib.sha256(dst.tobytes()).hexdigest() for _, _, dst in progs]
    runs = 1
    while busy < seconds and runs < 8:
        t = time.perf_counter()
        layer(pool)
        busy += time.perf_counter() - t
        runs += 1
    t = time.perf_counter()
    layer(ref.GatherPool(8))
    t8 = time.perf_counter() - t
    return {"value": runs / busy, "unit": "layers/s", "cores": pool.threads, "kind": "reference",
            "sample": f"the bench's last layer (7 matrices, {sum(m['out'] * m['in'] for m in mats):,} int8 "
                      f"elements) x{runs} via typed::executeHost",
            "value_8_threads": 1.0 / t8, "host": host_info(),
            "output_check": "match" if ref_digests == digests else "mismatch"}


def run_kernel_case(args):
    """Profiling case: the fused dequant->f16->transpose kernel alone on one
    Llama-70B gate matrix [28672, 8192] already in HBM (235 MB int8 in,
    470 MB f16 out: larger than L2), `--warmup` untimed launches then
    `--steps` launches. Prints the per-launch time and HBM GB/s."""
    import torch

    from helpers import encode, recipe_c4
    from sym_b200 import pyreloc

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    res = pyreloc.DispatchResources()
    _, compute_s = res.streams(0)
    stream = torch.cuda.ExternalStream(compute_s, device=dev)
    out_f, in_f = 28672, 8192
    rng = np.random.default_rng(0)
    q = torch.from_numpy(rng.integers(-127, 128, size=(out_f, in_f), dtype=np.int8)).to(dev)
    scale = np.exp(rng.normal(-5.0, 0.5, out_f)).astype(np.float32)
    bound = pyreloc.bind_typed(pyreloc.load_typed_plan(encode(recipe_c4())),
                               {"out_features": out_f, "in_features": in_f},
                               {"scale": ("float32", [out_f], scale.tobytes())})
    tmpl = pyreloc.prepare_dispatch_template(bound)
    out = torch.empty((in_f, out_f), dtype=torch.float16, device=dev)

    def launch():
        pyreloc.execute_rows(tmpl, q.data_ptr(), out.data_ptr(), 0, in_f, device=0, host_source=False,
                             resources=res, async_completion=True)

    for _ in range(args.warmup):
        launch()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        launch()
    b.record(stream)
    torch.cuda.synchronize()
    dt = a.elapsed_time(b) * 1e-3 / args.steps
    nbytes = out_f * in_f * 3 + out_f * 4
    print(json.dumps({"case": "gate[28672,8192] s8->f16 transpose", "ms_per_launch": dt * 1e3,
                      "hbm_gbs": nbytes / dt / 1e9, "bytes_per_launch": nbytes}))
    return 0


# ---------------------------------------------------------------------------
# the other configs (C1-C3): one tensor per step, one GPU
# ---------------------------------------------------------------------------

WIDTH = {"float32": 4, "int8": 1, "float16": 2, "bfloat16": 2}


def _dense(extents):
    strides, run = [], 1
    for e in reversed(extents):
        strides.append(run)
        run *= e
    return list(reversed(strides))


def _config_case(name, c2_batch=64):
    """The plan, symbols, parameters, synthetic source (seed 0) and accounting
    of one config. `kernel_bytes` is the algorithmic HBM traffic of one
    device-resident execution; `unit_per_step` the amount of the config's
    unit that one step moves. `c2_batch`: images of C2 (64 in the config;
    other batches measure how the launch's fixed cost weighs with size)."""
    from helpers import encode, recipe_c1, recipe_c2, recipe_c3, recipe_tc

    rng = np.random.default_rng(0)
    if name == "c1":
        n = 1 << 24
        src = rng.uniform(-1.0, 1.0, n).astype(np.float32)
        return {"blob": encode(recipe_c1()), "layout": True, "symbols": {"N": n}, "params": {}, "src": src,
                "dst_bytes": 4 * n, "kernel_bytes": 8 * n, "unit": "GB/s", "unit_per_step": 4 * n / 1e9,
                "workload": "c1_transpose_f32", "shape": {"N": n}, "dtype": "f32",
                "bytes_note": "4 B read + 4 B write per element"}
    if name == "c2":
        b = c2_batch
        src = rng.uniform(0.0, 1.0, (b, 3, 224, 224)).astype(np.float32)
        px = b * 224 * 224
        return {"blob": encode(recipe_c2(b)), "layout": False, "symbols": {}, "params": {}, "src": src,
                "dst_bytes": px * 8, "kernel_bytes": 20 * px, "unit": "images/s", "unit_per_step": b,
                "workload": "c2_nchw_to_nhwc_pad4_f16" + ("" if b == 64 else f"_batch{b}"),
                "shape": [b, 3, 224, 224], "dtype": "f32->f16", "bytes_note": "12 B read + 8 B write per pixel"}
    if name == "tc":  # the reference latency table's transpose + cast (rows of 1024 move intact)
        shape = (128, 128, 1024)
        n = 128 * 128 * 1024
        src = rng.uniform(-1.0, 1.0, shape).astype(np.float32)
        return {"blob": encode(recipe_tc(shape)), "layout": False, "symbols": {}, "params": {}, "src": src,
                "dst_bytes": 2 * n, "kernel_bytes": 6 * n, "unit": "GB/s", "unit_per_step": 4 * n / 1e9,
                "workload": "transpose_cast_128x128x1024_f32_f16", "shape": list(shape), "dtype": "f32->f16",
                "bytes_note": "4 B read + 2 B write per element"}
    if name == "c3q_d2h":  # KV-cache eviction: f32 on the GPU -> int8 in host memory
        case = _config_case("c3q")
        case.update(d2h=True, workload="c3q_d2h_quantize_evict")
        return case
    if name in ("c3q", "c3d"):
        s = 8192
        e = 8 * s * 4096
        x = rng.standard_normal(e, dtype=np.float32)
        if name == "c3q":
            src, sw, dw = x, 4, 1
        else:  # the quantized tensor: round-half-even of x * 20 (= 1 / 0.05f), clamped
            src, sw, dw = np.clip(np.rint(x * np.float32(20.0)), -128, 127).astype(np.int8), 1, 4
        return {"blob": encode(recipe_c3("quantize" if name == "c3q" else "dequantize")), "layout": False,
                "symbols": {"B": 8, "S": s}, "params": {}, "src": src, "dst_bytes": e * dw,
                "kernel_bytes": e * (sw + dw), "unit": "GB/s", "unit_per_step": e * sw / 1e9,
                "workload": f"{name}_{'quantize' if name == 'c3q' else 'dequantize'}", "shape": [8, s, 4096],
                "dtype": "f32->s8" if name == "c3q" else "s8->f32",
                "bytes_note": f"{sw} B read + {dw} B write per element"}
    raise ValueError(name)


def _cpu_config(case, threads, seconds=5.0):
    """The reference CPU executor on the config's whole input, host->host
    (each run finishes in well under a second); returns (rate, seconds, runs)."""
    from oracle import ref

    src = np.ascontiguousarray(case["src"]).reshape(-1).view(np.uint8)
    dst = np.empty(case["dst_bytes"], np.uint8)
    if case["layout"]:
        p = ref.LayoutPlan(case["blob"], case["symbols"])
        run = lambda: p.execute_into(src, dst, threads=threads)  # noqa: E731
    else:
        pool = ref.GatherPool(threads)
        p = ref.TypedProgram(case["blob"], case["symbols"], case["params"])
        run = lambda: p.execute_into(src, dst, pool=pool)  # noqa: E731
    run()
    t0, n = time.perf_counter(), 0
    while n < 3 or (time.perf_counter() - t0 < seconds and n < 20):
        run()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return case["unit_per_step"] / dt, dt, n


def measure_config(name, steps, warmup, cpu_seconds=5.0, cpu_8_threads=True, device=0, c2_batch=64):
    """One config (C1, C2, C3q, C3d, tc, c3q_d2h) on one GPU: `value` with
    the source resident in HBM (the kernels alone, L2 flushed before each
    timed launch), `e2e` through the public dispatch API from pinned host
    memory (the source crosses PCIe inside the timed region, plus a 4 KiB
    device->host read of the result per step), the kernel roofline, and the
    reference CPU executor on the same input. Returns the JSON-line dict."""
    import torch

    from oracle import ref
    from sym_b200 import pyreloc

    threads = len(os.sched_getaffinity(0))
    case = _config_case(name, c2_batch)
    dev = torch.device("cuda", device)
    torch.cuda.set_device(dev)
    res = pyreloc.DispatchResources()
    _, compute_s = res.streams(device)
    compute = torch.cuda.ExternalStream(compute_s, device=dev)
    if case["layout"]:
        bound = pyreloc.bind(pyreloc.load_plan(case["blob"]), case["symbols"])
        tmpl = pyreloc.prepare_transfer_template(bound)
    else:
        bound = pyreloc.bind_typed(pyreloc.load_typed_plan(case["blob"]), case["symbols"], case["params"])
        tmpl = pyreloc.prepare_dispatch_template(bound, "h2d", "cuda")
    d2h = bool(case.get("d2h"))
    tmpl_d2h = pyreloc.prepare_dispatch_template(bound, "d2h", "cuda") if d2h else None
    desc = tmpl.describe()
    rows = desc["padded_rows"]
    host = torch.from_numpy(np.ascontiguousarray(case["src"]).reshape(-1).view(np.uint8)).pin_memory()
    dsrc = host.to(dev)
    out = torch.empty(case["dst_bytes"], dtype=torch.uint8, device=dev)
    # L2 flush by READING 256 MB (> the 126 MB L2): a write flush would leave
    # ~126 MB of dirty lines whose write-back lands inside the timed launch
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)

    def kernel():
        pyreloc.execute_rows(tmpl, dsrc.data_ptr(), out.data_ptr(), 0, rows, device=device, host_source=False,
                             resources=res, async_completion=True)

    for _ in range(warmup):
        kernel()
    torch.cuda.synchronize(dev)
    clocks = Clocks(gpu_selector(torch, device))
    clocks.start()
    l0 = pyreloc.kernel_launches()
    times = []
    for _ in range(steps):
        flush.sum()
        compute.wait_stream(torch.cuda.default_stream(dev))  # the flush ends before the launch
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(compute)
        kernel()
        b.record(compute)
        torch.cuda.synchronize(dev)
        times.append(a.elapsed_time(b) * 1e-3)
    launches = pyreloc.kernel_launches() - l0
    t_kernel = statistics.median(times)
    t_p95 = sorted(times)[int(0.95 * (len(times) - 1) + 0.5)]
    # A plain device copy moving the same number of bytes (half read, half
    # written), timed the same way: the fixed cost of a launch of this size
    # (ramp-up, tail, events) that no transform kernel can beat.
    half = max(16, case["kernel_bytes"] // 2 // 16 * 16)
    cx = torch.empty(half, dtype=torch.uint8, device=dev).fill_(1)
    cy = torch.empty_like(cx)
    copy_times = []
    for i in range(3 + steps):
        flush.sum()
        compute.wait_stream(torch.cuda.default_stream(dev))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(compute):
            a.record(compute)
            cy.copy_(cx)
            b.record(compute)
        torch.cuda.synchronize(dev)
        if i >= 3:
            copy_times.append(a.elapsed_time(b) * 1e-3)
    t_copy = statistics.median(copy_times)
    del cx, cy

    # end to end through the public API: pinned host source -> device result
    # (d2h: device source -> pinned host result)
    sample = torch.empty(4096, dtype=torch.uint8).pin_memory()
    cur = torch.cuda.current_stream(dev)
    host_out = torch.empty(case["dst_bytes"], dtype=torch.uint8).pin_memory() if d2h else None
    if d2h:
        info = bound.describe()
        sw, dw = WIDTH[info["source_dtype"]], WIDTH[info["result_dtype"]]

        def request():
            sv = pyreloc.BufferView(dsrc.data_ptr(), dsrc.numel(), 0, info["source_extents"],
                                    _dense(info["source_extents"]), sw, "cuda", device)
            dv = pyreloc.BufferView(host_out.data_ptr(), host_out.numel(), 0, info["result_extents"],
                                    _dense(info["result_extents"]), dw, "host", -1)
            return pyreloc.prepare_dispatch_from_template(tmpl_d2h, sv, dv)
    elif case["layout"]:
        def request():
            sv = pyreloc.BufferView(host.data_ptr(), host.numel(), 0, [host.numel() // 4], [1], 4, "host", -1)
            dv = pyreloc.BufferView(out.data_ptr(), out.numel(), 0, [out.numel() // 4], [1], 4, "cuda", device)
            return pyreloc.make_transfer(bound, sv, dv)
    else:
        info = bound.describe()
        sw, dw = WIDTH[info["source_dtype"]], WIDTH[info["result_dtype"]]

        def request():
            sv = pyreloc.BufferView(host.data_ptr(), host.numel(), 0, info["source_extents"],
                                    _dense(info["source_extents"]), sw, "host", -1)
            dv = pyreloc.BufferView(out.data_ptr(), out.numel(), 0, info["result_extents"],
                                    _dense(info["result_extents"]), dw, "cuda", device)
            return pyreloc.prepare_dispatch_from_template(tmpl, sv, dv)

    def e2e_step():
        # one blocking call per step (returning asynchronously measured 1-2 %
        # better on C1 / C2 and 3-4 % worse on C3q / C3d)
        rep = pyreloc.execute_dispatch(request(), resources=res, caller_stream=cur.cuda_stream)
        if not d2h:
            sample.copy_(out[:4096], non_blocking=True)
        return rep

    for _ in range(3):
        rep = e2e_step()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(cur)
    for _ in range(steps):
        e2e_step()
    b.record(cur)
    torch.cuda.synchronize(dev)
    t_e2e = a.elapsed_time(b) * 1e-3 / steps
    ck = clocks.stop()
    ceiling = pinned_h2d_gbs(torch, dev, d2h=d2h)
    peaks = _peaks()
    hbm = peaks.get("hbm_gbs") or 6650.0
    achieved = case["kernel_bytes"] / t_kernel / 1e9
    cpu_rate, _, cpu_n = _cpu_config(case, threads, cpu_seconds) if ref.available() else (None, None, 0)
    h2d = 0 if d2h else host.numel()
    wire = case["dst_bytes"] if d2h else h2d  # bytes that cross PCIe per step
    line = {
        "metric": f"{case['workload']} {case['unit']}", "value": case["unit_per_step"] / t_kernel,
        "unit": case["unit"], "n_gpus": 1, "steps": steps, "warmup": warmup,
        "ms_per_step": t_kernel * 1e3, "ms_per_step_p95": t_p95 * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": case["dtype"], "data": "synthetic",
        "config": {"workload": case["workload"], "shape": case["shape"],
                   "l2": "flushed (256 MB read) before each timed kernel launch; the e2e source crosses PCIe "
                         "every step"},
        "e2e": {"value": case["unit_per_step"] / t_e2e, "unit": case["unit"], "ms_per_step": t_e2e * 1e3,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": case["dst_bytes"] if d2h else sample.numel(),
                "pct_of_pinned_memcpy": 100.0 * (wire / t_e2e / 1e9) / ceiling,
                "route": rep.get("route"), "implementation": rep.get("implementation")},
        ("pinned_d2h_ceiling_gbs" if d2h else "pinned_h2d_ceiling_gbs"): ceiling,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": None, "peak_source": "measured" if peaks.get("hbm_gbs") else "fallback",
                     "kernel": desc.get("device_kernel"), "bytes_per_launch": case["kernel_bytes"],
                     "launches_per_execution": launches / max(1, steps),
                     "bytes_per_launch_note": case["bytes_note"],
                     "copy_same_bytes": {"ms": t_copy * 1e3, "frac": 2 * half / t_copy / 1e9 / hbm,
                                         "note": "torch device copy of the same byte count (half read, half "
                                                 "written), L2 flushed and event-timed the same way"}},
        "gpu_launches": int(launches), "clocks": ck,
    }
    if cpu_rate is not None:
        line["cpu_baseline"] = {"value": cpu_rate, "unit": case["unit"], "cores": threads, "kind": "reference",
                                "sample": f"the whole input x{cpu_n}, reference executor host->host",
                                "host": host_info()}
        if cpu_8_threads:
            line["cpu_baseline"]["value_8_threads"] = _cpu_config(case, 8, cpu_seconds)[0]
    res.close()
    return line


def run_config(args):
    """One JSON line for config C1, C2, C3q, C3d, c3q_d2h or tc on one GPU
    (see measure_config); `--impl reference` times the reference CPU executor
    on the same input."""
    from oracle import ref

    if args.impl == "reference":
        threads = len(os.sched_getaffinity(0))
        case = _config_case(args.config, args.c2_batch)
        if not ref.available():
            print(json.dumps({"impl": "reference", "unavailable": "reference runtime (oracle/_ref) not built"}))
            return 0
        rate, dt, n = _cpu_config(case, threads)
        print(json.dumps({"impl": "reference", "metric": f"{case['workload']} {case['unit']}", "value": rate,
                          "unit": case["unit"], "n_gpus": args.gpus, "steps": n, "warmup": 1,
                          "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": case["dtype"], "data": "synthetic",
                          "config": {"workload": case["workload"], "shape": case["shape"]},
                          "cpu_baseline": {"value": rate, "unit": case["unit"], "cores": threads,
                                           "kind": "reference", "sample": "the whole config input per step"},
                          "e2e": {"value": rate, "unit": case["unit"], "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return 0
    print(json.dumps(measure_config(args.config, args.steps, args.warmup, c2_batch=args.c2_batch)))
    return 0


def measure_c4(steps=2, warmup=3, cpu_seconds=3.0):
    """Config 4 (Llama-7B int8 weight streaming, 32 layers, one GPU) in
    brief: host-pinned H2D+transform layers/s (CUDA events), the gate
    kernel's roofline with its source in HBM (L2 flushed before each launch),
    and the reference CPU executor on one layer."""
    import torch

    from helpers import encode, recipe_c4
    from oracle import ref
    from sym_b200 import pyreloc
    from sym_b200.workloads import ShardedLayerFetch

    dev = torch.device("cuda", 0)
    res = pyreloc.DispatchResources()
    _, compute_s = res.streams(0)
    compute = torch.cuda.ExternalStream(compute_s, device=dev)
    blob = encode(recipe_c4())
    plan = pyreloc.load_typed_plan(blob)
    layers = []
    for d in range(2):
        mats = []
        for name, q, scale in make_layer(d, LLAMA7B):
            out_f, in_f = q.shape
            bound = pyreloc.bind_typed(plan, {"out_features": out_f, "in_features": in_f},
                                       {"scale": ("float32", [out_f], scale.tobytes())})
            host = torch.from_numpy(q).pin_memory()
            mats.append({"name": name, "out": out_f, "in": in_f, "host": host, "dev": host.to(dev), "q": q,
                         "scale": scale, "tmpl": pyreloc.prepare_dispatch_template(
                             bound, "h2d", "cuda", implementation="b200_fused_h2d@dma_ring")})
        layers.append(mats)
    outs = [[torch.empty((m["in"], m["out"]), dtype=torch.float16, device=dev) for m in layers[0]] for _ in range(2)]
    fetch = ShardedLayerFetch(res, 0, 1, 0, chunk_bytes=16 << 20)

    def step():
        for l in range(32):
            fetch.fetch(layers[l % 2], outs[l % 2], True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize(dev)
    t = a.elapsed_time(b) * 1e-3
    gm, gout = layers[0][4], outs[0][4]
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    times = []
    for _ in range(10):
        flush.sum()
        compute.wait_stream(torch.cuda.default_stream(dev))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(compute)
        pyreloc.execute_rows(gm["tmpl"], gm["dev"].data_ptr(), gout.data_ptr(), 0, gm["in"], device=0,
                             host_source=False, resources=res, async_completion=True)
        e1.record(compute)
        torch.cuda.synchronize(dev)
        times.append(e0.elapsed_time(e1) * 1e-3)
    tk = statistics.median(times)
    kbytes = gm["out"] * gm["in"] * 3 + gm["out"] * 4
    hbm = _peaks().get("hbm_gbs") or 6650.0
    layer_bytes = sum(o * i for _, o, i in LLAMA7B)
    line = {"workload": "llama7b_int8_fetch", "value": 32 * steps / t, "unit": "layers/s",
            "gbs": layer_bytes * 32 * steps / t / 1e9,
            "roofline": {"kernel": f"{int8_tile_kernel()} on gate [11008, 4096]", "achieved": kbytes / tk / 1e9, "peak": hbm,
                         "frac": kbytes / tk / 1e9 / hbm, "launch_ms": tk * 1e3, "unit": "GB/s"}}
    if ref.available():
        threads = len(os.sched_getaffinity(0))
        pool = ref.GatherPool(threads)
        progs = []
        for m in layers[0]:
            p = ref.TypedProgram(blob, {"out_features": m["out"], "in_features": m["in"]},
                                 {"scale": ("float32", [m["out"]], m["scale"].tobytes())})
            progs.append((p, m["q"].reshape(-1).view(np.uint8), np.empty(m["out"] * m["in"] * 2, np.uint8)))
        t0, n = time.perf_counter(), 0
        while n < 1 or (time.perf_counter() - t0 < cpu_seconds and n < 10):
            for p, src, dst in progs:
                p.execute_into(src, dst, pool=pool)
            n += 1
        line["cpu_baseline"] = {"value": n / (time.perf_counter() - t0), "unit": "layers/s", "cores": pool.threads,
                                "kind": "reference", "sample": f"one Llama-7B layer x{n}"}
    res.close()
    return line


def run_extras():
    """Configs 1-4 in brief beside the headline line (one GPU, about a
    minute): each one's kernel roofline fraction, e2e rate and fraction of
    the pinned-memcpy ceiling, and the reference CPU rate."""
    out = {}
    for name in ("c1", "c2", "c3q", "c3d"):
        try:
            line = measure_config(name, steps=10, warmup=3, cpu_seconds=2.0, cpu_8_threads=False)
            out[name] = {"workload": line["config"]["workload"], "value": line["value"], "unit": line["unit"],
                         "kernel_frac": line["roofline"]["frac"], "kernel": line["roofline"]["kernel"],
                         "copy_frac_same_bytes": line["roofline"]["copy_same_bytes"]["frac"],
                         "e2e": line["e2e"]["value"],
                         "e2e_pct_of_pinned_memcpy": line["e2e"]["pct_of_pinned_memcpy"],
                         "cpu_baseline": (line.get("cpu_baseline") or {}).get("value"),
                         "clocks_sm_mhz": line["clocks"].get("sm_mhz")}
        except Exception as e:  # reported, not hidden: the headline line still stands
            out[name] = {"error": f"{type(e).__name__}: {e}"}
    try:
        out["c4"] = measure_c4()
    except Exception as e:
        out["c4"] = {"error": f"{type(e).__name__}: {e}"}
    return out


LATENCY_CASES = (  # the cases of the reference's typed H2D latency table (bench/results/typed-h2d-221)
    ("small_cast", (65539,), None),
    ("large_cast", (16777219,), None),
    ("transpose_cast", (128, 128, 1024), (1, 0, 2)),
)


def run_latency(args):
    """Warm completed latency (ms, p50 / p95 over --steps samples, at least
    100) of typed f32 -> f16 H2D transfers through the public Torch API
    (``reloc_torch.dispatch``), each call allocating its output, preparing,
    executing and completing; beside it the PyTorch controls of the same
    table on the same box: eager (CPU cast, then upload), retained pinned
    (CPU cast into a retained pinned buffer, then upload) and upload-then-
    convert (pinned f32 upload, cast on the GPU). One JSON line; `value` is
    the large cast's p50 through the pageable-source path."""
    import torch

    from sym_b200.reloc_torch import dispatch
    from sym_b200.reloc_torch.compiler import CompilerClient
    from sym_b200.reloc_torch.recipe import Cast, Recipe, TensorSpec, Transpose
    from sym_b200.reloc_torch.resources import TransferResources
    from sym_b200.reloc_torch.symbolic import Const, Symbol, dense_strides

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    samples = max(100, args.steps)
    warm = max(8, args.warmup)

    def spec(shape, dtype):
        shape = tuple(Symbol(e) if isinstance(e, str) else Const(e) for e in shape)
        return TensorSpec(shape, dense_strides(shape), Const(0), dtype)

    client = CompilerClient.from_environment()
    cast = client.compile(Recipe(spec(("n",), "float32"), (Cast("float16", "ieee_rne"),), spec(("n",), "float16"),
                                 "h2d"))
    trans = client.compile(Recipe(spec((128, 128, 1024), "float32"), (Transpose((1, 0, 2)), Cast("float16", "ieee_rne")),
                                  spec((128, 128, 1024), "float16"), "h2d"))

    def timeit(fn):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(dev)
        ts = []
        for _ in range(samples):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        ts.sort()
        return {"p50": 1e3 * ts[len(ts) // 2], "p95": 1e3 * ts[int(0.95 * (len(ts) - 1) + 0.5)]}

    table, launches, exact = {}, 0, True
    from sym_b200 import pyreloc

    with TransferResources(max_typed_retained_bytes=128 << 20) as owner:
        for name, shape, perm in LATENCY_CASES:
            gen = torch.Generator().manual_seed(0)
            x = torch.rand(shape, generator=gen) * 2 - 1
            xp = x.pin_memory()
            compiled = trans if perm else cast
            staged = torch.empty(shape if perm is None else tuple(shape[d] for d in perm), dtype=torch.float16,
                                 pin_memory=True)

            def ours(src):
                req = dispatch.prepare_typed_transfer(compiled, src, dev)
                return dispatch.execute_typed_transfer(req, resources=owner).tensor

            def eager():
                y = x.permute(*perm).contiguous().half() if perm else x.half()
                out = y.to(dev)
                torch.cuda.synchronize(dev)
                return out

            def pinned():
                staged.copy_(x.permute(*perm) if perm else x)
                out = staged.to(dev, non_blocking=True)
                torch.cuda.synchronize(dev)
                return out

            def gpu_cast():
                y = xp.to(dev, non_blocking=True)
                out = (y.permute(*perm).contiguous() if perm else y).half()
                torch.cuda.synchronize(dev)
                return out

            want = eager()
            exact &= bool(torch.equal(ours(x).view(torch.int16), want.view(torch.int16)))
            l0 = pyreloc.kernel_launches()
            row = {"sym_b200_pageable": timeit(lambda: ours(x))}
            launches += pyreloc.kernel_launches() - l0
            row["sym_b200_pinned"] = timeit(lambda: ours(xp))
            row["torch_eager"] = timeit(eager)
            row["torch_retained_pinned"] = timeit(pinned)
            row["torch_upload_then_gpu_cast"] = timeit(gpu_cast)
            row["source_bytes"] = x.numel() * 4
            table[name] = row
    value = table["large_cast"]["sym_b200_pageable"]["p50"]
    print(json.dumps({
        "metric": "typed H2D f32->f16 warm completed latency p50 (large cast, 64 MiB source)", "value": value,
        "unit": "ms", "n_gpus": 1, "steps": samples, "warmup": warm, "ms_per_step": value,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32->f16",
        "data": "synthetic", "bit_exact_vs_torch": exact,
        "config": {"workload": "typed_h2d_latency", "cases": {n: list(s) for n, s, _ in LATENCY_CASES},
                   "timing": "host wall clock per call, output allocation + prepare + execute + completion",
                   "l2": "every call moves its source over PCIe"},
        "latency_ms": table, "gpu_launches": launches,
        "reference_published_ms": {"large_cast": {"p50": 4.472, "p95": 4.719},
                                   "transpose_cast": {"p50": 5.309, "p95": 5.473},
                                   "small_cast": {"p50": 0.282, "p95": 0.293},
                                   "hardware": "EPYC 7351 + RTX 2080 Ti (PCIe Gen3)"},
    }))
    return 0


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--c2-batch", type=int, default=64,
                        help="images of --config c2 (64 in the config; other sizes show the launch's fixed cost)")
    parser.add_argument("--config", default="c5",
                        choices=["c1", "c2", "c3q", "c3d", "c3q_d2h", "c4", "c5", "tc", "latency"],
                        help="c5 (default): the headline Llama-70B fetch; c4: Llama-7B, 32 layers; "
                             "c1-c3d: the other configs on one GPU; tc: the transpose + cast of the reference's "
                             "latency table; latency: typed H2D call latency")
    parser.add_argument("--kernel-case", action="store_true",
                        help="profiling case: the hot kernel alone on one device-resident matrix")
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="ours", choices=["ours", "reference"])
    parser.add_argument("--distinct-layers", type=int, default=2)
    parser.add_argument("--chunk-bytes", type=int, default=16 << 20)
    parser.add_argument("--ring-slots", type=int, default=4)
    parser.add_argument("--route", default="dma_ring", choices=["dma_ring", "zero_copy"],
                        help="host-source route of the result-row fetch (N=1 and --multi allgather)")
    parser.add_argument("--multi", default="peer", choices=["peer", "allgather"],
                        help="N>1: peer (int8 shards read over NVLink by every rank's kernel) or allgather "
                             "(f16 result rows all-gathered by NCCL)")
    parser.add_argument("--peer-copy-chunk", type=int, default=0,
                        help="peer fetch: copy each shard in pieces of about this many bytes (0: one copy per shard)")
    parser.add_argument("--e2e-api", default="submit", choices=["submit", "group", "dispatch"],
                        help="N=1 e2e: one dispatch group per layer (7 matrices, one completion) submitted with two "
                             "layers in flight, or executed blocking, or one blocking dispatch per matrix")
    parser.add_argument("--n1-path", default="peer", choices=["peer", "dispatch"],
                        help="N=1 `value` path: peer (the same shard fetch as N>1, one shard per matrix: one DMA "
                             "per matrix, then one tile launch) or dispatch (the chunked HBM ring of "
                             "sb_execute_rows); `e2e` is the C-ABI dispatch call either way")
    parser.add_argument("--balance", type=int, default=1,
                        help="N>1 peer: size shards by each rank's sustained concurrent H2D bandwidth (1) or "
                             "equally (0)")
    parser.add_argument("--gpu-map", default="halves", choices=["identity", "halves"],
                        help="rank -> GPU: alternate between the two halves of the visible GPUs (default; on the "
                             "pool's 8-GPU boxes GPUs 0-3 and 4-7 sit behind different host bridges: N=4 measured "
                             "224 layers/s against 134 with identity), or identity")
    parser.add_argument("--extras", type=int, default=1,
                        help="N=1 headline run: also measure configs 1-4 in brief (about a minute)")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.kernel_case:
        return run_kernel_case(args)
    if args.config not in MODELS:
        if int(os.environ.get("RANK", "0")) != 0:
            return 0  # one-GPU configs: the other ranks have nothing to do
        if args.config == "latency":
            if args.impl == "reference":
                print(json.dumps({"impl": "reference", "unavailable": "the reference's latency table is its "
                                  "GPU pipeline; its CPU executor alone is timed by the other configs"}))
                return 0
            return run_latency(args)
        return run_config(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
