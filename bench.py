"""Benchmark of the B200 KV block store on the Qwen3-32B-shaped workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one step): an 8192-token prompt of a Qwen3-32B-shaped paged KV cache -- 64 layers,
8 KV heads, head_dim 128, bf16, 64-token blocks (16 MiB of KV per block, 128 blocks = 2 GiB) --
is put (gathered from a 4096-block paged pool into the store, write-through to the pinned host
tier included) and then restored by get into 128 fresh pool blocks with a 100% device-tier hit
rate. Values are seeded N(0,1) bf16; block tables are random permutations of the pool; keys are
64-bit chained prefix-block hashes, fresh for every step. The metric is payload GB/s of put + get
(2 x 2 GiB per step).

N > 1 (torchrun, one rank per GPU): one store hash-sharded over all GPUs (kvcache_manager.sharded).
Every rank gets back the 128 blocks it put in the previous step and puts a fresh prompt; blocks
owned by other GPUs cross NVLink as P2P stores issued by the copy kernels (weak scaling: the
per-rank work is fixed). Time is the max over ranks and `value` is the bytes all ranks moved
divided by it. --parallelism independent gives each GPU its own store instead; --transport nccl
moves packed values with NCCL send/recv.

--mix (torchrun, N > 1): the hash-sharded 70/30 get/put mix of 256-block batches with the config-1
KV shape and `--resident` blocks per GPU, timed with both transports on the same store.

--impl reference times the reference's host-DRAM path restated in C (the oracle: run planner,
memcpy gather/scatter, directory, host write-through) on the host cores with all threads.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tt-infinity_b200"))

METRIC = "KV put/get GB/s (device-timed) at 1/2/4/8 B200; p50/p99 get latency per block"
UNIT = "GB/s"
GB = 1e9

# Qwen3-32B-shaped KV on one B200
LAYERS, HEADS, HEAD_DIM, BLOCK_TOKENS = 64, 8, 128, 64
POOL_BLOCKS, BATCH_BLOCKS = 4096, 128
SEG_BYTES = HEADS * BLOCK_TOKENS * HEAD_DIM * 2  # 128 KiB per (layer, K|V, block)
BLOCK_PAYLOAD = 2 * LAYERS * SEG_BYTES  # 16 MiB
UNIT_BYTES = 4288
WORKLOAD = "qwen3-32b-kv-8192tok-put-get"


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="N=1: skip the config-3 multi-turn and connector-restore runs that follow the main step")
    ap.add_argument("--latency-samples", type=int, default=200)
    ap.add_argument("--sweep", action="store_true",
                    help="fp8 + per-block-scale layout, batches of 1..4096 blocks (prints a sweep table)")
    ap.add_argument("--multiturn", action="store_true",
                    help="32 sessions x 5 turns of prefix reuse with a slab of 25%% of the working set")
    ap.add_argument("--small", action="store_true",
                    help="profiling case: 16 layers, 512-block pool, 64 blocks per step (same kernels)")
    ap.add_argument("--parallelism", choices=["sharded", "independent"], default="sharded",
                    help="N > 1: one hash-sharded store over all GPUs (default) or an independent store per GPU")
    ap.add_argument("--placement", choices=["d2h", "uniform"], default="d2h",
                    help="N > 1: place keys in proportion to each GPU's device->host rate measured while all "
                         "copy at once (the write-through bound; default) or uniformly (fnv1a32 mod N)")
    ap.add_argument("--transport", choices=["p2p", "nccl"], default="p2p",
                    help="sharded store: P2P stores over NVLink (default) or NCCL send/recv of packed values")
    ap.add_argument("--mix", action="store_true",
                    help="hash-sharded 70/30 get/put mix of 256-block batches, config-1 KV shape, both transports")
    ap.add_argument("--latency", action="store_true",
                    help="single-block get latency on the Qwen3-32B-shaped block from a small pool")
    ap.add_argument("--restore", action="store_true",
                    help="the connector's batched restore of a Qwen3-32B-shaped 8192-token prompt (64 layers)")
    ap.add_argument("--fill", action="store_true",
                    help="token-granular paged fill: 8192 tokens of 4 requests into 64 layers' caches")
    ap.add_argument("--ref-blocks", type=int, default=0,
                    help="--impl reference: blocks put and got per step (default: the GPU step's 128); the CPU "
                         "tests use a few to check the line's contract quickly")
    ap.add_argument("--resident", type=int, default=0,
                    help="--mix: resident blocks per GPU (default: 1M / N, capped so that the pinned host "
                         "tier, which mirrors every resident block, stays within 35%% of the host's available memory)")
    args = ap.parse_args()
    if args.small:
        global LAYERS, POOL_BLOCKS, BATCH_BLOCKS, BLOCK_PAYLOAD, WORKLOAD
        LAYERS, POOL_BLOCKS, BATCH_BLOCKS = 16, 512, 64
        BLOCK_PAYLOAD = 2 * LAYERS * SEG_BYTES
        WORKLOAD = "qwen3-32b-shaped-16-layer-profiling-case"
    return args


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.proc = None
        self.gpus = gpu_indices
        # KVS_CLOCKS_DIR keeps the raw samples; by default they go to the temporary directory
        self.path = Path(os.environ.get("KVS_CLOCKS_DIR", tempfile.gettempdir())) / f"clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(str(g) for g in self.gpus)], stdout=self.f, stderr=subprocess.DEVNULL)
            t0 = time.time()  # the timed region starts once the first sample is in
            while time.time() - t0 < 5 and self.path.stat().st_size == 0:
                time.sleep(0.05)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        under = sorted(sm)
        med = statistics.median(under[len(under) // 2:]) if under else None  # busy half of samples
        return {"sm_mhz": med, "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ measured peaks / profiles


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic_per_launch(kernel: str):
    """dram bytes (read + write) per launch from the committed ncu summary, if present."""
    prof = ROOT / "profiles" / f"{kernel}.md"
    if not prof.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", prof.read_text())
    return float(m.group(1)) if m else None


# ------------------------------------------------------------------ the GPU workload


def build_pool(torch, device, rank=0):
    """128 member tensors (K, V per layer) of (4096, 8, 64, 128) bf16 filled with seeded N(0,1)."""
    kv = []
    g = torch.Generator(device=device)
    g.manual_seed(20261201 + rank)
    for _ in range(LAYERS):
        pair = []
        for _ in range(2):
            t = torch.empty((POOL_BLOCKS, HEADS, BLOCK_TOKENS, HEAD_DIM), dtype=torch.bfloat16, device=device)
            t.normal_(generator=g)
            pair.append(t)
        kv.append(tuple(pair))
    return kv


def _bits(t):
    """The tensor's bytes as integers (float compares would treat -0 / +0 as equal and NaN as unequal)."""
    import torch

    return t.contiguous().view(torch.uint8)


def byte_gate(torch, members, src, dst, device, snapshot=None):
    """Bit-exact check that block dst[i] of every member holds what block src[i] held (the current
    source blocks, or `snapshot[m]` taken before the sources could change). Raises on a mismatch."""
    di = torch.as_tensor(np.asarray(dst), device=device)
    si = None if snapshot is not None else torch.as_tensor(np.asarray(src), device=device)
    checked = 0
    for m, t in enumerate(members):
        want = snapshot[m] if snapshot is not None else t.index_select(0, si)
        got = t.index_select(0, di)
        if not torch.equal(_bits(got), _bits(want)):
            raise RuntimeError(f"member {m}: restored blocks differ from the source blocks")
        checked += got.numel() * got.element_size()
    return {"check": "byte compare of every restored block with its source, every member tensor",
            "members": len(members), "blocks": int(di.numel()), "bytes": int(checked)}


def pcie_peaks(torch, device, stream, nbytes=1 << 30):
    """(device->host, host->device) GB/s of a pinned 1 GiB copy, best of 3, CUDA events."""
    pin = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    out = []
    for to_host in (True, False):
        best = 0.0
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if to_host:
                pin.copy_(dev, non_blocking=True)
            else:
                dev.copy_(pin, non_blocking=True)
            e1.record(stream)
            torch.cuda.synchronize()
            best = max(best, nbytes / (e0.elapsed_time(e1) / 1e3) / GB)
        out.append(best)
    del pin, dev
    return out[0], out[1]


def write_through_summary(wt, expected_bytes, d2h_peak):
    """The write-through's own device time (CUDA events on the shard's write-through stream)."""
    ms = wt["total_ms"]
    achieved = wt["bytes"] / max(ms / 1e3, 1e-12) / GB
    return {"bytes": int(wt["bytes"]), "expected_bytes": int(expected_bytes), "batches": int(wt["launches"]),
            "device_ms": round(ms, 3), "achieved_GBps": round(achieved, 2), "pcie_d2h_peak_GBps": round(d2h_peak, 2),
            "frac": round(achieved / d2h_peak, 4) if d2h_peak else None,
            "how": "CUDA events on the write-through stream around each put's device->host copies",
            "note": "every put is written through to the pinned host tier and the next get waits for it "
                    "(the reference's commit barrier)"}


def step_split(elapsed_ms, steps, gather, scatter, wt):
    """Per step: the copy kernels' and the write-through's own device time, and the rest."""
    kern = (gather["total_ms"] + scatter["total_ms"]) / steps
    wt_ms = wt["total_ms"] / steps
    step = elapsed_ms / steps
    return {"step": round(step, 3), "copy_kernels": round(kern, 3), "write_through": round(wt_ms, 3),
            "rest": round(step - kern - wt_ms, 3),
            "note": "rest = lookups, replica updates, host catalog work and the ordering between them"}


def _native_lib():
    from kvcache_manager import _native

    return _native.load()


def one_block_get_latency(torch, client, layout, keys, dst, samples):
    """p50 / p99 in ms of Client.get_blocks of one committed device-resident block, from the call
    to its return (the block has landed: get_blocks synchronises its own work), 5 untimed calls
    first; keys[j] is restored into dst[j]."""
    n = len(keys)
    for j in range(5):  # untimed: the first calls size the staging areas
        client.get_blocks(layout, keys[j:j + 1], dst[j:j + 1])
    lat = []
    for i in range(samples):
        j = i % n
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        ok = client.get_blocks(layout, keys[j:j + 1], dst[j:j + 1])
        lat.append((time.perf_counter() - t1) * 1e3)
        torch.cuda.synchronize()
        assert ok.all()
    lat.sort()
    return lat[len(lat) // 2], lat[min(len(lat) - 1, math.ceil(0.99 * len(lat)) - 1)]


def run_ours(args, rank, local_rank, world):
    import torch
    import torch.distributed as dist

    from kvcache_manager import Client, PagedLayout, Server, codec
    from kvcache_manager import _native

    device = local_rank
    torch.cuda.set_device(device)
    kv = build_pool(torch, device)
    layout = PagedLayout.from_kv_caches(kv)
    vlen = layout.value_bytes()
    units = -(-vlen // UNIT_BYTES)
    block_units = 1 << (units - 1).bit_length()
    slab_values = 3 * BATCH_BLOCKS  # room for three prompts before LRU eviction starts
    max_keys = 4 * BATCH_BLOCKS  # catalog of four prompts: older keys are replaced
    server = Server(device, max_keys=max_keys, heap_bytes=slab_values * block_units * UNIT_BYTES,
                    host_pool_bytes=(max_keys + 8) * units * UNIT_BYTES, max_value_bytes=64 << 20)
    client = Client(device, server)
    rng = np.random.default_rng(1000 + rank)
    lib = _native.load()

    def step_inputs(step):
        perm = rng.permutation(POOL_BLOCKS)
        keys = np.array(codec.chained_block_hashes(step * 7919 + rank * 104729 + 1, BATCH_BLOCKS), dtype=np.uint64)
        return keys, perm[:BATCH_BLOCKS].astype(np.int64), perm[BATCH_BLOCKS:2 * BATCH_BLOCKS].astype(np.int64)

    def one_step(step):
        keys, src, dst = step_inputs(step)
        client.put_blocks(layout, keys, src)
        found = client.get_blocks(layout, keys, dst)
        if not found.all():
            raise RuntimeError(f"step {step}: device-tier get missed {int((~found).sum())} blocks")
        return keys, src, dst

    # correctness gate before timing: every restored block equals its source, byte for byte, in
    # every one of the 128 member tensors (64 layers x K, V)
    keys, src, dst = one_step(0)
    torch.cuda.synchronize()
    gate = byte_gate(torch, [t for pair in kv for t in pair], src, dst, device)
    for w in range(args.warmup):
        one_step(1 + w)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- timed region: K steps, device-timed with CUDA events on the caller stream
    sampler = ClockSampler([device]) if rank == 0 else None
    if sampler:
        sampler.start()
    client.kernel_timing()
    client.set_kernel_timing(True)
    server.write_through_timing()
    server.set_write_through_timing(True)
    launches0 = lib.kvs_kernel_launch_count()
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start.record(stream)
    for k in range(args.steps):
        one_step(1000 + k)
    client.flush()  # every put of the timed region is host-committed inside it
    end.record(stream)
    torch.cuda.synchronize()
    launches = lib.kvs_kernel_launch_count() - launches0
    elapsed_ms = start.elapsed_time(end)
    timing = client.kernel_timing()
    client.set_kernel_timing(False)
    wt = server.write_through_timing()
    server.set_write_through_timing(False)
    clocks = sampler.stop() if sampler else None
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    step_bytes = 2 * BATCH_BLOCKS * BLOCK_PAYLOAD  # put + get payload
    value = world * args.steps * step_bytes / (elapsed_ms / 1e3) / GB

    # ---- e2e: the public Python API with host key / block-table arrays, wall clock
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for k in range(args.steps):
        one_step(5000 + k)
    client.flush()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * args.steps * step_bytes / e2e_s / GB

    # ---- p50 / p99 get latency per block (committed, device-resident blocks): with the default
    # engine choice (one-wave engine for a one-block copy), then with the persistent bulk engine
    keys, src, dst = step_inputs(9999)
    client.put_blocks(layout, keys, src, sync_commit=True)
    p50, p99 = one_block_get_latency(torch, client, layout, keys, dst, args.latency_samples)
    lib = _native_lib()
    lib.kvs_set_small_copy_limit(0)
    p50_bulk, p99_bulk = one_block_get_latency(torch, client, layout, keys, dst, args.latency_samples)
    lib.kvs_set_small_copy_limit(-1)

    # ---- PCIe copy peaks (pinned, 1 GiB, best of 3): device->host bounds the write-through,
    # host->device the host-tier admissions
    best, h2d_best = pcie_peaks(torch, device, stream)

    # ---- roofline of the dominant kernel (gather or scatter, by device time)
    peak, peak_kind = measured_peaks()
    g, s = timing["gather"], timing["scatter"]
    dom_name, dom = ("chunk_copy_scatter_get", s) if s["total_ms"] >= g["total_ms"] else ("chunk_copy_gather_put", g)
    avg_ms = dom["total_ms"] / max(1, dom["launches"])
    bytes_per_launch = 2 * dom["bytes"] / max(1, dom["launches"])  # read + write of the payload
    achieved = bytes_per_launch / (avg_ms / 1e3) / GB
    traffic = ncu_traffic_per_launch("chunk_copy_qwen3_32b_128blk")
    stats = server.stats()
    client.close()
    server.close()
    if world > 1:
        dist.barrier()
    if rank != 0:
        return None
    h2d = 2 * BATCH_BLOCKS * 16  # keys + block ids for put and get
    d2h = BATCH_BLOCKS * 32 + BATCH_BLOCKS  # lookup records + found flags
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) bf16 KV, random block tables, 64-bit chained prefix-hash keys",
        "parity": gate,
        "config": {
            "workload": WORKLOAD,
            "layers": LAYERS, "kv_heads": HEADS, "head_dim": HEAD_DIM, "block_tokens": BLOCK_TOKENS,
            "pool_blocks": POOL_BLOCKS, "blocks_per_step": BATCH_BLOCKS, "bytes_per_block": BLOCK_PAYLOAD,
            "step": f"put {BATCH_BLOCKS} blocks (gather + host write-through) then get {BATCH_BLOCKS} blocks (100% device hit)",
            "l2": f"inputs larger than L2 ({BATCH_BLOCKS * BLOCK_PAYLOAD / 2**30:.2f} GiB moved per direction per step)",
            "parallelism": f"dp{world} (independent shard per GPU)",
            "slab_bytes": slab_values * block_units * UNIT_BYTES,
        },
        "e2e": {"value": round(e2e, 3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": int(launches),
        "roofline": {
            "kernel": dom_name,
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "peak_kind": peak_kind,
            "traffic": traffic,
            "algorithmic_bytes_per_launch": int(bytes_per_launch),
            "avg_launch_ms": round(avg_ms, 4),
        },
        "kernels": {
            "gather_put": {"launches": g["launches"], "avg_ms": round(g["total_ms"] / max(1, g["launches"]), 4),
                           "GBps_2x_payload": round(2 * g["bytes"] / max(1e-9, g["total_ms"] / 1e3) / GB, 1)},
            "scatter_get": {"launches": s["launches"], "avg_ms": round(s["total_ms"] / max(1, s["launches"]), 4),
                            "GBps_2x_payload": round(2 * s["bytes"] / max(1e-9, s["total_ms"] / 1e3) / GB, 1)},
        },
        "device_paths": device_path_rates(None, None, None, timing, 1),
        "write_through": write_through_summary(wt, BATCH_BLOCKS * BLOCK_PAYLOAD * args.steps, best),
        "step_split_ms": step_split(elapsed_ms, args.steps, g, s, wt),
        "pcie_peaks_GBps": {"d2h": round(best, 2), "h2d": round(h2d_best, 2),
                            "how": "torch copy of 1 GiB between device memory and pinned host memory, best of 3, "
                                   "CUDA events"},
        "get_latency_ms_per_block": {"p50": round(p50, 4), "p99": round(p99, 4), "block_bytes": BLOCK_PAYLOAD,
                                     "samples": args.latency_samples,
                                     "note": "one committed device-resident block per Client.get_blocks call, "
                                             "timed from the call to its return (the block has landed)",
                                     "engine": "one-wave copy (copies up to 512 MiB)",
                                     "bulk_engine": {"p50": round(p50_bulk, 4), "p99": round(p99_bulk, 4)}},
        "store": {k: stats[k] for k in ("writes_through", "victims_evicted", "catalog_replacements", "live_keys")},
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(seconds=12.0)
    return line


# ------------------------------------------------------------------ hash-sharded store over N GPUs

NVLINK_NOMINAL_GBS = 900.0  # NVLink 5 per direction per GPU (nominal)


def _peer_copy_rates(torch, dist, device, nbytes=1 << 30):
    """Measured NVLink rate per direction: every rank copies 1 GiB from its GPU into the next rank's
    GPU with cudaMemcpyAsync (the copy engines, not this library's kernels), all ranks at once,
    best of 3, CUDA events. Returns (this rank's GB/s, min over ranks)."""
    import ctypes as C

    from cuda.bindings import runtime as cudart

    from kvcache_manager import _native

    lib = _native.load()
    rank, world = dist.get_rank(), dist.get_world_size()
    buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
    src = torch.empty(nbytes, dtype=torch.uint8, device=device)
    h, off = _native.IpcHandle(), C.c_uint64()
    _native.check(lib.kvs_ipc_export(C.c_void_p(buf.data_ptr()), C.byref(h), C.byref(off)))
    handles = [None] * world
    dist.all_gather_object(handles, (bytes(h.bytes), off.value))
    peer = (rank + 1) % world
    ph = _native.IpcHandle()
    C.memmove(ph.bytes, handles[peer][0], 64)
    base = C.c_void_p()
    _native.check(lib.kvs_ipc_open(device, C.byref(ph), C.byref(base)))
    dst = base.value + handles[peer][1]
    stream = torch.cuda.current_stream(device)
    best = 0.0
    for _ in range(3):
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        err, = cudart.cudaMemcpyAsync(dst, src.data_ptr(), nbytes, cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice,
                                      stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        if err != cudart.cudaError_t.cudaSuccess:
            raise RuntimeError(f"peer copy: {err}")
        best = max(best, nbytes / (e0.elapsed_time(e1) / 1e3) / GB)
    dist.barrier()  # every copy into a peer's buffer has finished before any buffer goes away
    lib.kvs_ipc_close(device, base)
    dist.barrier()
    del buf, src
    return best, -_max_over_ranks(torch, dist, -best, device)


def device_path_rates(torch, dist, device, timing, world):
    """Payload GB/s of the copy kernels alone, over all ranks: the put (gather) and get (scatter)
    kernels' payload bytes per launch, summed over ranks, over the slowest rank's average launch
    time. The step's value also waits for the host write-through; these show what the device
    paths move (at N > 1 they include the P2P stores over NVLink)."""
    out = {}
    for name, t in (("put", timing["gather"]), ("get", timing["scatter"])):
        launches = max(1, t["launches"])
        per_launch, ms = t["bytes"] / launches, t["total_ms"] / launches
        if world > 1:
            per_launch = _sum_over_ranks(torch, dist, per_launch, device)
            ms = _max_over_ranks(torch, dist, ms, device)
        out[name + "_GBps"] = round(per_launch / max(ms / 1e3, 1e-12) / GB, 1)
    out["how"] = ("payload bytes per launch summed over ranks / the slowest rank's average launch time (CUDA "
                  "events); the step's value also waits for the write-through")
    return out


def _max_over_ranks(torch, dist, value, device):
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(torch, dist, value, device):
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t)
    return float(t.item())


def _host_write_rates(torch, dist, device, chunks=128, chunk=16 << 20):
    """Device->host copy rate of every rank while all ranks copy at once (barrier-aligned): the
    write-through ceiling of the box. 128 x 16 MiB copies into a 2 GiB pinned buffer per rank.
    Returns (this rank's GB/s, min over ranks, sum over ranks)."""
    pin = torch.empty(chunks * chunk, dtype=torch.uint8, pin_memory=True)
    src = torch.empty(chunk, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    best = 0.0
    for _ in range(2):
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(chunks):
            pin[i * chunk:(i + 1) * chunk].copy_(src, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        best = max(best, chunks * chunk / (e0.elapsed_time(e1) / 1e3) / GB)
    del pin, src
    t = torch.tensor([best, -best, best], device=device, dtype=torch.float64)
    lo = t[1:2].clone()
    dist.all_reduce(lo, op=dist.ReduceOp.MAX)
    tot = t[2:3].clone()
    dist.all_reduce(tot)
    return best, -float(lo.item()), float(tot.item())


def _placement_weights(torch, dist, device):
    """Every rank's device->host rate while all ranks copy at once, clipped to [0.5, 1.5] x the mean:
    the write-through each shard can absorb per second, used as its share of the keys."""
    mine, _, _ = _host_write_rates(torch, dist, device)
    t = torch.zeros(dist.get_world_size(), dtype=torch.float64, device=device)
    t[dist.get_rank()] = mine
    dist.all_reduce(t)
    rates = t.cpu().numpy()
    clipped = np.clip(rates, 0.5 * rates.mean(), 1.5 * rates.mean())
    return [round(float(x), 3) for x in rates], [round(float(x), 3) for x in clipped]


def _nvlink_roofline(torch, dist, device, timing, counters0, counters1, payload):
    """Per launch: the payload bytes that crossed NVLink / the launch's device time, for the client
    put kernel (P2P stores into the owners' slabs) and the owner get kernel (P2P stores into the
    requesters' pools); the dominant one by device time is the roofline kernel."""
    g, s = timing["gather"], timing["scatter"]
    out = {}
    for name, t, key in (("put_push", g, "puts_remote"), ("get_push", s, "served_remote")):
        remote = (counters1[key] - counters0[key]) * payload
        ms = t["total_ms"]
        launches = max(1, t["launches"])
        out[name] = {"launches": t["launches"], "avg_ms": round(ms / launches, 4),
                     "nvlink_bytes_per_launch": int(remote / launches),
                     "achieved_nvlink_GBps": round(remote / max(ms / 1e3, 1e-12) / GB, 1),
                     "hbm_GBps_2x_payload": round(2 * t["bytes"] / max(ms / 1e3, 1e-12) / GB, 1)}
    dom = "put_push" if g["total_ms"] >= s["total_ms"] else "get_push"
    # rank 0's view, max over ranks of launch time is what bounds the step
    achieved = _sum_over_ranks(torch, dist, out[dom]["achieved_nvlink_GBps"], device) / dist.get_world_size()
    return dom, out, achieved


def run_sharded(args, rank, local_rank, world):
    """The Qwen3-32B-shaped step through one store hash-sharded over all N GPUs: every rank gets
    back the 128 blocks it put in the previous step and puts a fresh 8192-token prompt; (N-1)/N of
    the blocks live on other GPUs and cross NVLink as P2P stores."""
    import torch
    import torch.distributed as dist

    from kvcache_manager import PagedLayout, _native, codec, sharded

    device = local_rank
    torch.cuda.set_device(device)
    kv = build_pool(torch, device, rank)
    layout = PagedLayout.from_kv_caches(kv)
    vlen = layout.value_bytes()
    units = -(-vlen // UNIT_BYTES)
    block_units = 1 << (units - 1).bit_length()
    slab_values = 3 * BATCH_BLOCKS
    max_keys = 4 * BATCH_BLOCKS
    rates, weights = _placement_weights(torch, dist, device) if args.placement == "d2h" else (None, None)
    # with weights within [0.5, 1.5] x their mean a shard takes at most 192 / 256 / 307 puts per step
    # at N = 2 / 4 / 8, which fit the 384 slab values and 512 catalog slots once the previous step's
    # blocks, served at the start of the step, make room
    store = sharded.create(layout, max_batch=BATCH_BLOCKS, transport=args.transport, max_keys=max_keys,
                           heap_bytes=slab_values * block_units * UNIT_BYTES,
                           host_pool_bytes=(max_keys + 8) * units * UNIT_BYTES, max_value_bytes=64 << 20,
                           weights=weights)
    eng = store.engine
    rng = np.random.default_rng(1000 + rank)
    lib = _native.load()
    prev = {"keys": np.zeros(0, np.uint64)}

    def one_step(step):
        perm = rng.permutation(POOL_BLOCKS)
        keys = np.array(codec.chained_block_hashes(step * 7919 + rank * 104729 + 1, BATCH_BLOCKS), np.uint64)
        src, dst = perm[:BATCH_BLOCKS].astype(np.int64), perm[BATCH_BLOCKS:2 * BATCH_BLOCKS].astype(np.int64)
        gk = prev["keys"]
        gd = dst[:gk.size]
        found = store.step(gk, gd, keys, src)
        if not found.all():
            raise RuntimeError(f"step {step}: device-tier get missed {int((~found).sum())} blocks")
        prev["keys"], prev["src"] = keys, src
        return gd

    # correctness gate: the blocks restored from the (mostly remote) shards equal their sources
    # byte for byte in every member tensor; the sources are snapshotted first (2 GiB), since the
    # next step's gets may land in them
    members = [t for pair in kv for t in pair]
    one_step(0)
    torch.cuda.synchronize()
    src_idx = torch.as_tensor(prev["src"], device=device)
    snap = [t.index_select(0, src_idx) for t in members]
    got_blocks = one_step(1)
    torch.cuda.synchronize()
    try:
        gate, bad = byte_gate(torch, members, None, got_blocks, device, snapshot=snap), 0.0
    except RuntimeError as exc:
        gate, bad = str(exc), 1.0
    del snap, src_idx
    if _max_over_ranks(torch, dist, bad, device) > 0:  # every rank stops together
        raise RuntimeError(f"rank {rank}: restored blocks differ from their sources somewhere: {gate}")
    gate["ranks"] = world
    for w in range(args.warmup):
        one_step(2 + w)
    torch.cuda.synchronize()
    dist.barrier()

    sampler = ClockSampler([device]) if rank == 0 else None
    if sampler:
        sampler.start()
    eng.client.kernel_timing()
    eng.client.set_kernel_timing(True)
    eng.server.write_through_timing()
    eng.server.set_write_through_timing(True)
    c0 = dict(store.counters)
    launches0 = lib.kvs_kernel_launch_count()
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    dist.barrier()
    start.record(stream)
    for k in range(args.steps):
        one_step(1000 + k)
    store.flush()  # this shard's puts of the timed region are host-committed inside it
    end.record(stream)
    torch.cuda.synchronize()
    launches = lib.kvs_kernel_launch_count() - launches0
    elapsed_ms = _max_over_ranks(torch, dist, start.elapsed_time(end), device)
    timing = eng.client.kernel_timing()
    eng.client.set_kernel_timing(False)
    wt = eng.server.write_through_timing()
    eng.server.set_write_through_timing(False)
    c1 = dict(store.counters)
    clocks = sampler.stop() if sampler else None
    step_bytes = 2 * BATCH_BLOCKS * BLOCK_PAYLOAD
    # this shard's write-through: its own device time; the slowest shard's bounds the step
    wt_ms_step = wt["total_ms"] / args.steps
    wt_gbps = wt["bytes"] / max(wt["total_ms"] / 1e3, 1e-12) / GB
    wt_ms_max = _max_over_ranks(torch, dist, wt_ms_step, device)
    wt_gbps_min = -_max_over_ranks(torch, dist, -wt_gbps, device)
    value = world * args.steps * step_bytes / (elapsed_ms / 1e3) / GB
    dom, kernels, nvlink_achieved = _nvlink_roofline(torch, dist, device, timing, c0, c1, BLOCK_PAYLOAD)
    paths = device_path_rates(torch, dist, device, timing, world)

    # e2e: the public sharded API with host key / block-table arrays, wall clock (max over ranks)
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    for k in range(args.steps):
        one_step(5000 + k)
    store.flush()
    torch.cuda.synchronize()
    e2e_s = _max_over_ranks(torch, dist, time.perf_counter() - t0, device)
    e2e = world * args.steps * step_bytes / e2e_s / GB

    # latency: one collective step in which every rank gets one committed block
    one_step(9000)
    store.flush()
    keys, dst = prev["keys"], np.arange(BATCH_BLOCKS, 2 * BATCH_BLOCKS, dtype=np.int64)
    lat = []
    for j in range(3):  # untimed, on every rank alike
        store.step(keys[j:j + 1], dst[j:j + 1])
    for i in range(args.latency_samples):
        j = i % BATCH_BLOCKS
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        ok = store.step(keys[j:j + 1], dst[j:j + 1])
        torch.cuda.synchronize()
        lat.append((time.perf_counter() - t1) * 1e3)
        assert ok.all()
    lat.sort()
    p50 = lat[len(lat) // 2]
    p99 = lat[min(len(lat) - 1, math.ceil(0.99 * len(lat)) - 1)]
    stats = store.stats()
    rounds = (c1["grant_rounds"] - c0["grant_rounds"]) / args.steps
    store.close()
    hw_mine, hw_min, hw_sum = _host_write_rates(torch, dist, device)
    peer_mine, peer_min = _peer_copy_rates(torch, dist, device)
    wt_per_gpu = BATCH_BLOCKS * BLOCK_PAYLOAD / (elapsed_ms / args.steps / 1e3) / GB
    if rank != 0:
        return None
    hbm_peak, peak_kind = measured_peaks()
    k = kernels[dom]
    return {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) bf16 KV, random block tables, 64-bit chained prefix-hash keys",
        "config": {
            "workload": WORKLOAD,
            "layers": LAYERS, "kv_heads": HEADS, "head_dim": HEAD_DIM, "block_tokens": BLOCK_TOKENS,
            "pool_blocks": POOL_BLOCKS, "blocks_per_step": BATCH_BLOCKS, "bytes_per_block": BLOCK_PAYLOAD,
            "step": (f"every rank: get the {BATCH_BLOCKS} blocks it put in the previous step (100% device hit) "
                     f"and put {BATCH_BLOCKS} fresh blocks, keys hash-sharded over {world} GPUs"),
            "l2": f"inputs larger than L2 ({BATCH_BLOCKS * BLOCK_PAYLOAD / 2**30:.2f} GiB per direction per rank per step)",
            "parallelism": f"hash-sharded store over {world} GPUs, transport {args.transport}",
            "slab_bytes": slab_values * block_units * UNIT_BYTES,
            "placement": ({"by": "each GPU's device->host rate while all copy at once (GB/s), clipped to "
                                 "[0.5, 1.5] x the mean; keys go to fnv1a32 slots in proportion",
                           "rates": rates, "weights": weights} if weights else {"by": "fnv1a32 mod N"}),
        },
        "e2e": {"value": round(e2e, 3), "unit": UNIT,
                "h2d_bytes_per_step": 2 * 8 * world * sharded.request_words(BATCH_BLOCKS),
                "d2h_bytes_per_step": 2 * 8 * world * sharded.reply_words(BATCH_BLOCKS)},
        "gpu_launches": int(launches),
        "parity": gate,
        "roofline": {
            "kernel": dom, "bound": "nvlink", "achieved": round(nvlink_achieved, 1), "peak": NVLINK_NOMINAL_GBS,
            "unit": "GB/s", "frac": round(nvlink_achieved / NVLINK_NOMINAL_GBS, 4),
            "peak_kind": "nominal NVLink 5 per direction per GPU",
            "measured_peer_copy_GBps": {"rank0": round(peer_mine, 1), "min": round(peer_min, 1),
                                        "how": "cudaMemcpyAsync of 1 GiB into the next rank's GPU, all ranks at "
                                               "once, best of 3, in this run"},
            "frac_of_measured_peer_copy": round(nvlink_achieved / peer_min, 4) if peer_min else None,
            "traffic": None,
            "algorithmic_bytes_per_launch": k["nvlink_bytes_per_launch"], "avg_launch_ms": k["avg_ms"],
            "hbm_peak": hbm_peak, "hbm_peak_kind": peak_kind,
        },
        "kernels": kernels,
        "device_paths": paths,
        "limiter": {
            "step_ms": round(elapsed_ms / args.steps, 3),
            "write_through_ms_slowest_shard": round(wt_ms_max, 3),
            "push_kernels_ms_rank0": round((timing["gather"]["total_ms"] + timing["scatter"]["total_ms"]) / args.steps, 3),
            "bound": ("host write-through (the next step's gets wait for it)" if wt_ms_max > 0.5 * elapsed_ms / args.steps
                      else "NVLink pushes and the per-step protocol"),
        },
        "write_through": {
            "bytes_per_step_per_gpu": BATCH_BLOCKS * BLOCK_PAYLOAD,
            "device_ms_per_step_slowest_shard": round(wt_ms_max, 3),
            "measured_GBps_rank0": round(wt_gbps, 2), "measured_GBps_min": round(wt_gbps_min, 2),
            "how": "CUDA events on each shard's write-through stream around its device->host copies",
            "achieved_GBps_per_gpu": round(wt_per_gpu, 2),
            "concurrent_d2h_GBps_per_gpu": {"rank0": round(hw_mine, 2), "min": round(hw_min, 2)},
            "concurrent_d2h_GBps_all_gpus": round(hw_sum, 1),
            "frac_of_slowest_gpu": round(wt_per_gpu / hw_min, 4),
            "frac_of_box_aggregate": round(world * wt_per_gpu / hw_sum, 4),
            "note": ("every put is written through to the owner's pinned host tier and the next step's gets wait "
                     "for it: with equal key shares the step is bound by the slowest GPU's device->host rate "
                     "while all GPUs copy at once; with shares by rate, by the box's aggregate rate"),
        },
        "get_latency_ms_per_block": {"p50": round(p50, 4), "p99": round(p99, 4), "block_bytes": BLOCK_PAYLOAD,
                                     "samples": args.latency_samples, "note": "one collective step, every rank gets one block"},
        "grant_rounds_per_step": rounds,
        "store": {k2: stats[k2] for k2 in ("writes_through", "victims_evicted", "catalog_replacements", "live_keys")},
        "clocks": clocks,
    }


# config-1 KV shape for the hash-sharded get/put mix
MIX_LAYERS, MIX_HEADS, MIX_DIM, MIX_BT, MIX_POOL = 2, 8, 128, 32, 1024
MIX_BATCH, MIX_GETS = 256, 179  # 70 / 30 get / put
MIX_PAYLOAD = 2 * MIX_LAYERS * MIX_HEADS * MIX_BT * MIX_DIM * 2  # 256 KiB


def _host_bytes_available() -> int:
    """MemAvailable of this host (0 if unknown)."""
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def _splitmix64(x: np.ndarray) -> np.ndarray:
    z = (x + np.uint64(0x9E3779B97F4A7C15)).astype(np.uint64)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def run_mix(args, rank, local_rank, world):
    """Hash-sharded store over N GPUs with `resident` blocks per GPU; every rank issues 256-block
    batches of 179 gets (uniform over every rank's resident keys) and 77 puts (overwrites of its
    own keys), targets uniform over shards; timed once with P2P stores and once with NCCL
    send/recv of packed values on the same store."""
    import torch
    import torch.distributed as dist

    from kvcache_manager import PagedLayout, sharded

    device = local_rank
    torch.cuda.set_device(device)
    g = torch.Generator(device=device)
    g.manual_seed(77 + rank)
    members = [torch.empty((MIX_POOL, MIX_HEADS, MIX_BT, MIX_DIM), dtype=torch.bfloat16, device=device).normal_(generator=g)
               for _ in range(2 * MIX_LAYERS)]
    layout = PagedLayout(members, members_per_layer=2)
    vlen = layout.value_bytes()
    units = -(-vlen // UNIT_BYTES)
    block_units = 1 << (units - 1).bit_length()
    # config 4 asks for 1 M resident blocks over the N GPUs; every resident block also lives in its
    # owner's pinned host tier, so the default takes 1 M / N per GPU up to a pinned budget of 35 % of
    # the host memory available (shared by the N processes of the box)
    want = (1 << 20) // world
    avail = _host_bytes_available()
    per_block_host = units * UNIT_BYTES
    cap = int(0.35 * avail / world / per_block_host) if avail else 16384
    R = args.resident or min(want, cap)
    residency = {"requested_per_gpu": want, "host_available_bytes": avail, "pinned_budget": "35% of available / N",
                 "pinned_bytes_per_gpu": R * per_block_host,
                 "limited_by": "--resident" if args.resident else ("host memory" if cap < want else "none")}
    max_keys = R + R // 8 + 1024
    store = sharded.create(layout, max_batch=MIX_BATCH, transport="p2p", max_keys=max_keys,
                           heap_bytes=max_keys * block_units * UNIT_BYTES,
                           host_pool_bytes=max_keys * units * UNIT_BYTES)
    eng = store.engine
    rng = np.random.default_rng(500 + rank)

    def key(r, i):
        return _splitmix64((np.uint64(r) << np.uint64(40)) | np.asarray(i, np.uint64))

    # populate: every rank puts its R keys (the blocks land on their owners over NVLink)
    t_pop = time.perf_counter()
    for b0 in range(0, R, MIX_BATCH):
        ids = np.arange(b0, min(R, b0 + MIX_BATCH))
        store.step((), (), key(rank, ids), (ids % MIX_POOL).astype(np.int64))
    store.flush()
    torch.cuda.synchronize()
    dist.barrier()
    t_pop = time.perf_counter() - t_pop

    def one_step():
        perm = rng.permutation(MIX_POOL)
        gr = rng.integers(0, world, MIX_GETS)
        gk = _splitmix64((gr.astype(np.uint64) << np.uint64(40)) | rng.integers(0, R, MIX_GETS).astype(np.uint64))
        pk = key(rank, rng.choice(R, MIX_BATCH - MIX_GETS, replace=False))
        found = store.step(gk, perm[:MIX_GETS].astype(np.int64), pk, perm[MIX_GETS:MIX_BATCH].astype(np.int64))
        if not found.all():
            raise RuntimeError(f"rank {rank}: {int((~found).sum())} resident blocks missed")

    results = {}
    for transport in ("p2p", "nccl"):
        store.transport = transport
        for _ in range(args.warmup):
            one_step()
        torch.cuda.synchronize()
        dist.barrier()
        eng.client.kernel_timing()
        eng.client.set_kernel_timing(True)
        c0 = dict(store.counters)
        stream = torch.cuda.current_stream(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler = ClockSampler([device]) if rank == 0 else None
        if sampler:
            sampler.start()
        torch.cuda.synchronize()
        dist.barrier()
        start.record(stream)
        for _ in range(args.steps):
            one_step()
        store.flush()
        end.record(stream)
        torch.cuda.synchronize()
        ms = _max_over_ranks(torch, dist, start.elapsed_time(end), device)
        timing = eng.client.kernel_timing()
        eng.client.set_kernel_timing(False)
        c1 = dict(store.counters)
        clocks = sampler.stop() if sampler else None
        moved = _sum_over_ranks(torch, dist, (c1["gets_found"] - c0["gets_found"] + c1["puts"] - c0["puts"]) * MIX_PAYLOAD,
                                device)
        dom, kernels, nvl = _nvlink_roofline(torch, dist, device, timing, c0, c1, MIX_PAYLOAD)
        entry = {"value": round(moved / (ms / 1e3) / GB, 3), "ms_per_step": round(ms / args.steps, 3),
                 "kernels": kernels, "clocks": clocks,
                 "grant_rounds_per_step": (c1["grant_rounds"] - c0["grant_rounds"]) / args.steps}
        if transport == "p2p":
            entry.update(roofline_kernel=dom, nvlink_achieved_GBps=round(nvl, 1),
                         nvlink_frac_of_nominal=round(nvl / NVLINK_NOMINAL_GBS, 4))
        else:
            # the copy kernels pack and unpack rows in this GPU's memory; NCCL moves them over NVLink
            for k in entry["kernels"].values():
                k.pop("nvlink_bytes_per_launch", None)
                k.pop("achieved_nvlink_GBps", None)
            entry["note"] = "kernels copy rows within this GPU; the bytes cross NVLink inside NCCL send/recv"
        results[transport] = entry
    stats = store.stats()
    store.close()
    hw_mine, hw_min, hw_sum = _host_write_rates(torch, dist, device)
    if rank != 0:
        return None
    p = results["p2p"]
    return {
        "metric": METRIC, "value": p["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": p["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) bf16 KV, 64-bit splitmix keys, uniform targets",
        "config": {"workload": "hash-sharded-config1-kv-70-30-get-put-256blk", "layers": MIX_LAYERS,
                   "kv_heads": MIX_HEADS, "head_dim": MIX_DIM, "block_tokens": MIX_BT, "pool_blocks": MIX_POOL,
                   "bytes_per_block": MIX_PAYLOAD, "batch": f"{MIX_GETS} gets + {MIX_BATCH - MIX_GETS} puts per rank",
                   "resident_blocks_per_gpu": R, "resident_blocks_total": R * world, "residency": residency,
                   "populate_s": round(t_pop, 2), "parallelism": f"hash-sharded store over {world} GPUs"},
        "transports": results,
        "concurrent_d2h_GBps_per_gpu": {"rank0": round(hw_mine, 2), "min": round(hw_min, 2),
                                        "all_gpus": round(hw_sum, 1)},
        "store": {k: stats[k] for k in ("live_keys", "device_resident_keys", "writes_through", "victims_evicted")},
    }


# ------------------------------------------------------------------ CPU baseline (the oracle)


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


_CPU_POOLS: dict = {}
_CPU_STORES: dict = {}
_CPU_STORE_RUNS: list = []


def _cpu_pool(pool_blocks: int) -> list:
    """Host-resident paged pool of every member (K and V of each layer), seeded bf16 bit patterns:
    one 16 MiB random pattern tiled over each member (the copies do not look at the values)."""
    if pool_blocks not in _CPU_POOLS:
        _CPU_POOLS.clear()
        rng = np.random.default_rng(7)
        pattern = rng.integers(0, 1 << 16, (16 << 20) // 2, dtype=np.uint16).view(np.uint8)
        members = []
        for m in range(2 * LAYERS):
            a = np.empty(pool_blocks * SEG_BYTES, np.uint8)
            reps = -(-a.size // pattern.size)
            a[:] = np.tile(np.roll(pattern, m * 4096), reps)[:a.size]
            members.append(a)
        _CPU_POOLS[pool_blocks] = members
    return _CPU_POOLS[pool_blocks]


def cpu_run(n_blocks_per_step: int, steps: int, threads: int, warmup: int = 1):
    """The reference host-DRAM path restated in C: put (gather + write-through) then get (scatter)
    of `n_blocks_per_step` Qwen3-32B-shaped blocks per step on a host-resident paged pool of
    2 x n + 32 blocks (every step puts n fresh keys from random blocks and gets them into n other
    random blocks)."""
    from oracle import kvs_oracle as O

    pool_blocks = 2 * n_blocks_per_step + 32
    members = _cpu_pool(pool_blocks)
    rng = np.random.default_rng(7 + len(_CPU_STORE_RUNS))
    if n_blocks_per_step not in _CPU_STORES:  # one store per process: its arenas are faulted in once
        _, _, vlen = O.block_format([SEG_BYTES] * (2 * LAYERS))
        units = -(-vlen // UNIT_BYTES)
        block_units = 1 << (units - 1).bit_length()
        _CPU_STORES[n_blocks_per_step] = O.Store(
            max_keys=4 * n_blocks_per_step, heap_bytes=3 * n_blocks_per_step * block_units * UNIT_BYTES,
            host_pool_bytes=(4 * n_blocks_per_step + 8) * units * UNIT_BYTES, max_value_bytes=64 << 20)
    store = _CPU_STORES[n_blocks_per_step]
    _CPU_STORE_RUNS.append(n_blocks_per_step)
    salt = 1000003 * len(_CPU_STORE_RUNS)  # fresh keys in every run on the same store
    from kvcache_manager import codec  # pure-python key derivation (no device code)

    def step(k):
        perm = rng.permutation(pool_blocks)
        keys = np.array(codec.chained_block_hashes(salt + k * 31 + 5, n_blocks_per_step), np.uint64)
        store.put_blocks(members, [SEG_BYTES] * (2 * LAYERS), keys, perm[:n_blocks_per_step], n_threads=threads)
        f = store.get_blocks(members, [SEG_BYTES] * (2 * LAYERS), keys, perm[n_blocks_per_step:2 * n_blocks_per_step],
                             n_threads=threads)
        assert f.all()

    for w in range(max(1, warmup)):
        step(w)
    store.flush()
    t0 = time.perf_counter()
    for k in range(steps):
        step(100 + k)
    store.flush()
    dt = time.perf_counter() - t0
    return steps * 2 * n_blocks_per_step * BLOCK_PAYLOAD / dt / GB, dt


def cpu_baseline(seconds: float) -> dict:
    """The CPU port on the GPU arm's own step (put then get of BATCH_BLOCKS blocks), all host
    threads and one, each for a bounded number of steps (about `seconds`, a quarter for one)."""
    threads = cpu_threads()
    n = BATCH_BLOCKS
    gbps, dt = cpu_run(n, 1, threads)
    steps = max(1, min(2000, int(seconds / max(dt, 1e-3))))  # about `seconds` of CPU work
    gbps, dt = cpu_run(n, steps, threads)
    out = {"value": round(gbps, 3), "unit": UNIT, "cores": threads, "kind": "port",
           "sample": f"{steps} steps x (put {n} + get {n}) Qwen3-32B-shaped 16 MiB blocks on a {2 * n + 32}-block "
                     f"host pool, {threads} threads, {dt:.1f} s"}
    if threads > 1:  # the same step on one core
        g1, d1 = cpu_run(n, 1, 1, warmup=0)
        s1 = max(1, min(2000, int(seconds / 4 / max(d1, 1e-3))))
        g1, d1 = cpu_run(n, s1, 1, warmup=0)
        out["single_thread"] = {"value": round(g1, 3), "cores": 1, "sample": f"{s1} steps, 1 thread, {d1:.1f} s"}
    return out


def run_reference(args, rank, world):
    if rank != 0:
        return None
    threads = cpu_threads()
    n = args.ref_blocks or BATCH_BLOCKS
    gbps, dt = cpu_run(n, args.steps, threads, warmup=args.warmup)
    return {
        "metric": METRIC, "value": round(gbps, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic: seeded random bf16 bit patterns, random block tables, chained prefix-hash keys",
        "config": {"workload": WORKLOAD, "blocks_per_step": n, "bytes_per_block": BLOCK_PAYLOAD,
                   "step": f"put {n} blocks (gather + host write-through) then get {n} blocks on the host path",
                   "pool_blocks": 2 * n + 32},
        "impl": "reference",
        "cpu_baseline": {"value": round(gbps, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps x (put {n} + get {n}) 16 MiB blocks on a {2 * n + 32}-block "
                                   f"host pool, {threads} threads"},
        "e2e": {"value": round(gbps, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------ fp8 batch sweep (latency vs bandwidth)

FP8_LAYERS, FP8_HEADS, FP8_DIM, FP8_BLOCK_TOKENS = 80, 8, 128, 16
FP8_POOL_BLOCKS = 65536  # 160 GiB of fp8 blocks; the slab beside it holds the largest batch (4096 values)


def fp8_layout(torch, device, pool_blocks):
    """Per layer: K and V fp8 e4m3 (pool_blocks, 8, 16, 128) and one fp32 scale per block."""
    from kvcache_manager import PagedLayout

    g = torch.Generator(device=device)
    g.manual_seed(5)
    members = []
    for _ in range(FP8_LAYERS):
        for _ in range(2):
            t = torch.empty((pool_blocks, FP8_HEADS, FP8_BLOCK_TOKENS, FP8_DIM), dtype=torch.uint8, device=device)
            t.random_(0, 256, generator=g)
            members.append(t.view(torch.float8_e4m3fn))
        members.append(torch.rand((pool_blocks,), generator=g, device=device))
    return PagedLayout(members, members_per_layer=3)


def run_sweep(args):
    """put (landed) and get (device hit) GB/s and per-call latency for batches of 1..4096 blocks."""
    import torch

    from kvcache_manager import Client, Server, codec

    torch.cuda.set_device(0)
    layout = fp8_layout(torch, 0, FP8_POOL_BLOCKS)
    vlen = layout.value_bytes()
    payload = sum(layout.member_block_bytes)
    units = -(-vlen // UNIT_BYTES)
    block_units = 1 << (units - 1).bit_length()
    server = Server(0, max_keys=2 * 4096 + 64, heap_bytes=(4096 + 4) * block_units * UNIT_BYTES,
                    host_pool_bytes=(4096 + 4) * units * UNIT_BYTES)
    client = Client(0, server)
    rng = np.random.default_rng(9)
    rows = []
    checked = 0
    client.set_kernel_timing(True)
    for batch in [1, 4, 16, 64, 256, 1024, 4096]:
        put_ms, get_ms = [], []
        client.kernel_timing()  # reset the totals
        reps = max(2, min(20, 2048 // batch))
        for r in range(reps + 1):
            perm = rng.permutation(FP8_POOL_BLOCKS)
            keys = np.array(codec.chained_block_hashes(batch * 1000 + r, batch), np.uint64)
            src, dst = perm[:batch], perm[batch:2 * batch]
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            client.put_blocks(layout, keys, src)
            torch.cuda.current_stream().synchronize()  # landed: the caller's stream, not the write-through
            t1 = time.perf_counter()
            client.flush()
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            found = client.get_blocks(layout, keys, dst)  # returns once the blocks have landed
            t3 = time.perf_counter()
            torch.cuda.synchronize()
            assert found.all()
            if r == 0:  # untimed: payload and scale bytes of every restored block equal their sources
                checked += byte_gate(torch, layout.members, src, dst, 0)["bytes"]
            for k in keys:  # keep the catalog bounded
                client.delete(int(k))
            if r:
                put_ms.append((t1 - t0) * 1e3)
                get_ms.append((t3 - t2) * 1e3)
        p50p, p50g = statistics.median(put_ms), statistics.median(get_ms)
        kt = client.kernel_timing()  # every repetition, the untimed first one included
        kg, ks = kt["gather"], kt["scatter"]
        kernel = {"gather_ms": round(kg["total_ms"] / max(1, reps + 1), 4),
                  "scatter_ms": round(ks["total_ms"] / max(1, reps + 1), 4),
                  "scatter_hbm_frac": round(2 * ks["bytes"] / max(1e-9, ks["total_ms"] / 1e3) / GB / measured_peaks()[0], 4)}
        rows.append({"blocks": batch, "bytes": batch * payload, "kernels_per_call": kernel,
                     "put_landed_ms_p50": round(p50p, 4), "put_landed_GBps": round(batch * payload / p50p / 1e6, 2),
                     "get_ms_p50": round(p50g, 4), "get_ms_p99": round(sorted(get_ms)[-1], 4),
                     "get_GBps": round(batch * payload / p50g / 1e6, 2), "reps": reps})
    client.close()
    server.close()
    return {"sweep": "fp8 e4m3 KV + fp32 per-block scales, 80 layers x 8 heads x 128 dim, 16-token blocks",
            "pool_blocks": FP8_POOL_BLOCKS, "bytes_per_block": payload, "value_bytes": vlen,
            "parity": {"check": "byte compare of every restored block (payload and scales) with its source, first "
                                "repetition of every batch size", "bytes": checked},
            "note": "put = landed (gather into the slab, then the caller's stream synchronised; the write-through is "
                    "flushed outside the put time); get = device-tier hit, wall clock around the Python API call, "
                    "which returns once the blocks have landed",
            "rows": rows}


# ------------------------------------------------------------------ multi-turn prefix reuse (config-1 shape)

def multiturn_plan(n_sessions, n_turns, seed=3, lo=512, hi=4096, block_tokens=32):
    """Per session and turn: the prompt's full-block count; each turn extends the prior conversation."""
    rng = np.random.default_rng(seed)
    plan = []
    for s in range(n_sessions):
        total, turns = 0, []
        for t in range(n_turns):
            total += int(rng.integers(lo, hi + 1))
            turns.append(total // block_tokens)
        plan.append(turns)
    return plan


def run_multiturn_workload(client, layout, plan, pool_blocks, seed=3, on_turn=None, phase_s=None):
    """Each turn: exists on the prompt's blocks, get the longest contiguous prefix of hits, put the
    rest. Block keys are chained prefix hashes per session, so turn t+1 shares turn t's prefix.
    phase_s (optional dict): host wall seconds spent in each call kind."""
    from kvcache_manager import codec

    rng = np.random.default_rng(seed + 1)
    stats = {"blocks": 0, "prefix_hits": 0, "puts": 0, "gets": 0}
    order = [(t, s) for t in range(len(plan[0])) for s in range(len(plan))]  # sessions interleave by turn
    clock = time.perf_counter
    for t, s in order:
        n = plan[s][t]
        keys = np.array(codec.chained_block_hashes(1_000_003 * (s + 1), n), np.uint64)
        t0 = clock()
        found = client.exists_batch(keys)
        t1 = clock()
        hit = int(np.argmin(found)) if not found.all() else n
        slots = rng.permutation(pool_blocks)[:n]
        if hit:
            got = client.get_blocks(layout, keys[:hit], slots[:hit])
            assert got.all(), "a prefix block reported by exists was not restored"
        t2 = clock()
        if hit < n:
            client.put_blocks(layout, keys[hit:], slots[hit:])
        t3 = clock()
        if phase_s is not None:
            for k, v in (("exists", t1 - t0), ("get", t2 - t1), ("put", t3 - t2)):
                phase_s[k] = phase_s.get(k, 0.0) + v
        stats["blocks"] += n
        stats["prefix_hits"] += hit
        stats["gets"] += hit
        stats["puts"] += n - hit
        if on_turn:
            on_turn(t, s, keys, hit, slots)
    return stats


def run_multiturn(args):
    import torch

    from kvcache_manager import Client, PagedLayout, Server

    torch.cuda.set_device(0)
    layers, heads, dim, bt, pool = 2, 8, 128, 32, 1024
    g = torch.Generator(device=0)
    g.manual_seed(7)
    kv = [tuple(torch.empty((pool, heads, bt, dim), dtype=torch.bfloat16, device=0).normal_(generator=g)
                for _ in range(2)) for _ in range(layers)]
    layout = PagedLayout.from_kv_caches(kv)
    plan = multiturn_plan(32, 5)
    working_set = sum(p[-1] for p in plan)  # distinct blocks the sessions produce
    vlen = layout.value_bytes()
    units = -(-vlen // UNIT_BYTES)
    block_bytes = (1 << (units - 1).bit_length()) * UNIT_BYTES
    slab = max(block_bytes, working_set * block_bytes // 4)  # 25 % of the working set
    server = Server(0, max_keys=2 * working_set, heap_bytes=slab, host_pool_bytes=(working_set + 64) * units * UNIT_BYTES)
    client = Client(0, server)
    stream = torch.cuda.current_stream(0)
    d2h_peak, h2d_peak = pcie_peaks(torch, 0, stream)
    torch.cuda.synchronize()
    client.set_kernel_timing(True)
    server.set_write_through_timing(True)
    phase = {}
    t0 = time.perf_counter()
    st = run_multiturn_workload(client, layout, plan, pool, phase_s=phase)
    client.flush()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    kt, ht, wt = client.kernel_timing(), client.host_tier_timing(), server.write_through_timing()
    sst = server.stats()
    client.close()
    server.close()
    payload = sum(layout.member_block_bytes)

    def rate(t, peak):
        gbps = t["bytes"] / max(t["total_ms"] / 1e3, 1e-12) / GB
        return {"launches": int(t["launches"]), "bytes": int(t["bytes"]), "device_ms": round(t["total_ms"], 3),
                "GBps": round(gbps, 2), "frac_of_peak": round(gbps / peak, 4) if peak else None}

    return {"multiturn": "32 sessions x 5 turns, U(512, 4096) tokens per turn, config-1 KV shape, slab = 25% of the working set",
            "working_set_blocks": working_set, "slab_bytes": slab, "wall_s": round(dt, 3),
            "blocks_restored": st["gets"], "blocks_put": st["puts"],
            "prefix_hit_rate": round(st["prefix_hits"] / max(1, st["blocks"]), 4),
            "host_tier_serves": sst["host_serves"], "admissions": sst["admissions"],
            "victims_evicted": sst["victims_evicted"],
            "moved_GBps": round((st["gets"] + st["puts"]) * payload / dt / GB, 3),
            "host_s_by_call": {k: round(v, 4) for k, v in phase.items()},
            "pcie_peaks_GBps": {"d2h": round(d2h_peak, 2), "h2d": round(h2d_peak, 2)},
            "device_timed": {
                "admissions_h2d": rate(ht["admissions"], h2d_peak),
                "host_tier_hit_scatters": rate(ht["serves"], 0),
                "write_through_d2h": rate(wt, d2h_peak),
                "device_hit_scatters": rate(kt["scatter"], 0),
                "put_gathers": rate(kt["gather"], 0),
                "how": "CUDA events around each copy launch on the client stream and around each write-through "
                       "batch on the shard's write-through stream; host-tier hit scatters read the slab blocks "
                       "their admissions just filled (device memory), or the pinned copy when no block was free"},
            "pcie_bytes": {"h2d_admissions": sst["admissions"] * vlen, "d2h_write_through": sst["writes_through"] * vlen}}


def run_fill(args):
    """moreh_paged_fill_cache_varlen on B200: per layer, 8192 packed tokens of 4 requests (chunked-
    prefill start positions) into a paged bf16 cache of 64-token blocks, 8 KV heads x 128; the 64
    layers use distinct inputs and caches (4 GiB of fill, more than L2). Kernel time from CUDA
    events around each launch; algorithmic bytes = read + write of every filled row."""
    import torch

    from kvcache_manager import ops

    torch.cuda.set_device(0)
    rng = np.random.default_rng(11)
    lens, starts, bs = [3072, 2048, 1024, 2048], [0, 512, 4096, 64], 64
    max_blocks = max((s0 + n + bs - 1) // bs for s0, n in zip(starts, lens))
    nb = 4 * max_blocks + 1
    pt = torch.from_numpy(rng.permutation(np.arange(1, nb))[: 4 * max_blocks].reshape(4, max_blocks).astype(np.int32)).cuda()
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device="cuda")
    sp = torch.tensor(starts, dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    layers = 8 if args.small else 64
    fills = [[torch.empty((1, HEADS, 8192, HEAD_DIM), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
              for _ in range(2)] for _ in range(layers)]
    caches = [[torch.zeros((nb, HEADS, bs, HEAD_DIM), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
              for _ in range(layers)]
    for _ in range(args.warmup):
        for (kf, vf), (ck, cv) in zip(fills, caches):
            ops.paged_fill_cache_varlen(kf, vf, cu, pt, sp, ck, cv)
    torch.cuda.synchronize()
    times = []
    stream = torch.cuda.current_stream()
    for _ in range(args.steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(layers)]
        # hold the stream while the host queues every layer, so each event pair brackets the
        # kernel alone and not the host's argument checks
        torch.cuda._sleep(50_000_000)
        for ((kf, vf), (ck, cv)), (e0, e1) in zip(zip(fills, caches), ev):
            e0.record(stream)
            ops.paged_fill_cache_varlen(kf, vf, cu, pt, sp, ck, cv)
            e1.record(stream)
        torch.cuda.synchronize()
        times += [e0.elapsed_time(e1) for e0, e1 in ev]
    def check_layer(i):  # one layer against a plain torch restatement of the fill
        kf, ck = fills[i][0], caches[i][0]
        tok = 0
        for r, (n, s0) in enumerate(zip(lens, starts)):
            pos = torch.arange(s0, s0 + n, device="cuda")
            blk = pt[r][pos // bs].long()
            want = kf[0, :, tok:tok + n].permute(1, 0, 2)
            if not torch.equal(ck[blk, :, pos % bs], want):
                raise RuntimeError(f"paged fill of layer {i} differs from the torch restatement")
            tok += n

    check_layer(7)
    # the same per-layer calls back to back, one event pair around all of them (a restore loop
    # over layers; consecutive fills may overlap launch and drain)
    seq_times = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(50_000_000)
        e0.record(stream)
        for (kf, vf), (ck, cv) in zip(fills, caches):
            ops.paged_fill_cache_varlen(kf, vf, cu, pt, sp, ck, cv)
        e1.record(stream)
        torch.cuda.synchronize()
        seq_times.append(e0.elapsed_time(e1) / layers)
    check_layer(layers - 2)
    # every layer in one launch (paged_fill_cache_varlen_layers), same inputs, caches zeroed first
    for ck, cv in caches:
        ck.zero_()
        cv.zero_()
    ks, vs = [f[0] for f in fills], [f[1] for f in fills]
    cks, cvs = [c[0] for c in caches], [c[1] for c in caches]
    for _ in range(args.warmup):
        ops.paged_fill_cache_varlen_layers(ks, vs, cu, pt, sp, cks, cvs)
    torch.cuda.synchronize()
    check_layer(0)
    check_layer(layers - 1)
    all_times = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000)  # the host's argument checks stay outside the event pair
        e0.record(stream)
        ops.paged_fill_cache_varlen_layers(ks, vs, cu, pt, sp, cks, cvs)
        e1.record(stream)
        torch.cuda.synchronize()
        all_times.append(e0.elapsed_time(e1))
    row = HEAD_DIM * 2
    bytes_per_launch = 2 * 2 * HEADS * sum(lens) * row  # K and V, read + write
    avg_ms = statistics.mean(times)
    achieved = bytes_per_launch / (avg_ms / 1e3) / GB
    peak, kind = measured_peaks()
    seq_ms = statistics.mean(seq_times)
    seq_achieved = bytes_per_launch / (seq_ms / 1e3) / GB
    all_ms = statistics.mean(all_times)
    all_achieved = layers * bytes_per_launch / (all_ms / 1e3) / GB
    return {"fill": "moreh_paged_fill_cache_varlen restated token-granular: 8192 tokens, 4 requests, 8 KV heads x 128 "
                    f"bf16, 64-token blocks, {layers} layers (distinct inputs)",
            "launches": len(times), "avg_launch_ms": round(avg_ms, 4), "algorithmic_bytes_per_launch": bytes_per_launch,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_kind": kind,
                         "frac": round(achieved / peak, 4), "unit": "GB/s"},
            "restore_64_layers_ms": round(avg_ms * layers, 3),
            "per_layer_calls_back_to_back": {"layers": layers, "steps": len(seq_times),
                                             "avg_per_layer_ms": round(seq_ms, 4),
                                             "roofline": {"bound": "hbm", "achieved": round(seq_achieved, 1),
                                                          "peak": peak, "frac": round(seq_achieved / peak, 4),
                                                          "unit": "GB/s"}},
            "all_layers_one_launch": {"launches": len(all_times), "avg_launch_ms": round(all_ms, 4),
                                      "roofline": {"bound": "hbm", "achieved": round(all_achieved, 1), "peak": peak,
                                                   "frac": round(all_achieved / peak, 4), "unit": "GB/s"}}}


def run_restore(args):
    """The connector's batched restore of a Qwen3-32B-shaped prompt: vLLM-layout caches of 64 layers
    ([2, 4096 blocks, 64 tokens, 8 KV heads, 128] bf16), an 8192-token request stored as 32 chunks of
    256 tokens (the raw-byte chunk blobs, 64 MiB each), its blocks cleared, then restored by
    GPUConnector.batched_to_gpu: one store call whose fill launch writes every chunk into all 64
    layers from the slab. Kernel time from the client's CUDA events; algorithmic bytes = read +
    write of every restored row (2 x payload); the whole call's wall time beside it."""
    import asyncio

    import torch

    from kvcache_manager import Client, Server
    from kvcache_manager.connector import GPUConnector, KVCacheClient, RemoteConnector, kv_caches_from_vllm, raw_codec_for

    class _Key:
        def __init__(self, s):
            self.s = s

        def to_string(self):
            return self.s

    torch.cuda.set_device(0)
    layers, nb, bs, tokens, chunk = (8, 512, BLOCK_TOKENS, 8192, 256) if args.small else (LAYERS, POOL_BLOCKS,
                                                                                         BLOCK_TOKENS, 8192, 256)
    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    vllm = [torch.empty((2, nb, bs, HEADS, HEAD_DIM), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
            for _ in range(layers)]
    caches = kv_caches_from_vllm(vllm)
    raw = raw_codec_for(caches, bs)
    rng = np.random.default_rng(21)
    first = int(rng.integers(0, nb - tokens // bs))  # the request's blocks: one contiguous run
    slots = torch.arange(first * bs, first * bs + tokens, device="cuda")
    n_chunks = tokens // chunk
    vlen = raw.device_shard_plan(caches, layers, slots[:chunk].tolist(), 0)["value_len"]
    units = -(-vlen // UNIT_BYTES)
    block_units = 1 << (units - 1).bit_length()
    server = Server(0, max_keys=4 * n_chunks, heap_bytes=(n_chunks + 2) * block_units * UNIT_BYTES,
                    host_pool_bytes=(n_chunks + 2) * units * UNIT_BYTES, max_value_bytes=vlen)
    client = Client(0, server)
    kc = KVCacheClient(client, raw)
    gpu = GPUConnector(kc, num_layers=layers, block_size=bs)
    remote = RemoteConnector(kc, allocate=lambda shape, dtype, fmt=None: object(), meta_shape=(1,), meta_dtype=None)
    starts = [i * chunk for i in range(n_chunks)]
    ends = [s0 + chunk for s0 in starts]
    keys = [_Key(f"prompt@{i}") for i in range(n_chunks)]
    mos = [object() for _ in keys]
    gpu.batched_from_gpu(mos, starts, ends, kvcaches=vllm, slot_mapping=slots)
    asyncio.run(remote.batched_put(keys, mos))
    client.flush()
    blocks = slice(first, first + tokens // bs)
    want = [t[:, blocks].clone() for t in vllm]
    times, walls = [], []
    for it in range(args.warmup + args.steps):
        for t in vllm:
            t[:, blocks].zero_()
        torch.cuda.synchronize()
        phs = asyncio.run(remote.batched_get(keys))
        client.kernel_timing()
        client.set_kernel_timing(True)
        t0 = time.perf_counter()
        gpu.batched_to_gpu(phs, starts, ends, kvcaches=vllm, slot_mapping=slots)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        kt = client.kernel_timing()["scatter"]
        client.set_kernel_timing(False)
        if it == 0:  # untimed: every restored byte equals what was stored
            for t, w in zip(vllm, want):
                if not torch.equal(t[:, blocks].view(torch.int16), w.view(torch.int16)):
                    raise RuntimeError("restored blocks differ from the stored chunks")
        if it >= args.warmup:
            times.append(kt["total_ms"])
            walls.append(wall * 1e3)
    client.close()
    server.close()
    payload = 2 * layers * tokens * HEADS * HEAD_DIM * 2
    ms = statistics.mean(times)
    achieved = 2 * payload / (ms / 1e3) / GB
    peak, kind = measured_peaks()
    wall_ms = statistics.median(walls)
    return {"restore": f"connector batched_to_gpu of {tokens} tokens in {n_chunks} chunks of {chunk}, {layers} layers "
                       f"of vLLM-layout bf16 caches (8 KV heads x 128, {bs}-token blocks): one store call, one fill "
                       "launch from the slab",
            "payload_bytes": payload, "steps": len(times), "fill_ms": round(ms, 4), "call_wall_ms_p50": round(wall_ms, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_kind": kind,
                         "frac": round(achieved / peak, 4), "unit": "GB/s",
                         "algorithmic_bytes_per_launch": 2 * payload},
            "call_GBps_payload": round(payload / (wall_ms / 1e3) / GB, 1),
            "parity": "byte compare of every restored block with the stored chunks (first call)"}


def run_latency(args):
    """Single-block get latency on the Qwen3-32B-shaped block (64 layers, 16 MiB values) from a small
    pool: p50 / p99 wall time of Client.get_blocks of one committed, device-resident block (the
    call returns once the block has landed) and the scatter kernel's own time from CUDA events,
    with the one-wave engine (the default for a one-block copy) and with the bulk engine; then the
    same call through the C ABI alone (ctypes with prepared addresses), the Python facade's share."""
    import torch

    from kvcache_manager import Client, PagedLayout, Server, codec
    from kvcache_manager import _facade

    torch.cuda.set_device(0)
    pool, n = 64, 16
    g = torch.Generator(device=0)
    g.manual_seed(1)
    kv = [tuple(torch.empty((pool, HEADS, BLOCK_TOKENS, HEAD_DIM), dtype=torch.bfloat16, device=0).normal_(generator=g)
                for _ in range(2)) for _ in range(LAYERS)]
    layout = PagedLayout.from_kv_caches(kv)
    vlen = layout.value_bytes()
    units = -(-vlen // UNIT_BYTES)
    block_units = 1 << (units - 1).bit_length()
    server = Server(0, max_keys=4 * n, heap_bytes=(n + 4) * block_units * UNIT_BYTES,
                    host_pool_bytes=(n + 4) * units * UNIT_BYTES)
    client = Client(0, server)
    keys = np.array(codec.chained_block_hashes(5, n), np.uint64)
    client.put_blocks(layout, keys, np.arange(n), sync_commit=True)
    dst = np.arange(n, 2 * n)
    lib = _native_lib()
    out = {"latency": "one committed device-resident 16 MiB block per Client.get_blocks call (64 layers x K, V "
                      "of 8 x 64 x 128 bf16), wall time from the call to its return",
           "samples": args.latency_samples}
    for name, limit in (("one_wave", -1), ("bulk", 0)):
        lib.kvs_set_small_copy_limit(limit)
        p50, p99 = one_block_get_latency(torch, client, layout, keys, dst, args.latency_samples)
        client.set_kernel_timing(True)
        for i in range(args.latency_samples):
            client.get_blocks(layout, keys[i % n:i % n + 1], dst[i % n:i % n + 1])
        sc = client.kernel_timing()["scatter"]
        client.set_kernel_timing(False)
        out[name] = {"p50_us": round(1e3 * p50, 2), "p99_us": round(1e3 * p99, 2),
                     "scatter_kernel_avg_us": round(1000 * sc["total_ms"] / max(1, sc["launches"]), 2)}
    lib.kvs_set_small_copy_limit(-1)
    # the C ABI call alone: addresses and the stream handle prepared once
    found = np.zeros(1, np.bool_)
    k_addr = [_facade._addr(keys[j:j + 1]) for j in range(n)]
    ids = dst.astype(np.int64)
    b_addr = [_facade._addr(ids[j:j + 1]) for j in range(n)]
    f_addr, h, ref = _facade._addr(found), client._handle(), layout.ref
    stream = _facade._stream_handle(0)
    lat = []
    for i in range(args.latency_samples + 5):
        j = i % n
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        rc = lib.kvs_get_blocks(h, ref, 1, k_addr[j], b_addr[j], f_addr, stream)
        if i >= 5:
            lat.append((time.perf_counter() - t0) * 1e6)
        assert rc == 0 and found[0]
    lat.sort()
    out["c_abi_call"] = {"p50_us": round(lat[len(lat) // 2], 2),
                         "note": "kvs_get_blocks through ctypes with prepared arguments, one-wave engine"}
    client.close()
    server.close()
    for t, blk in zip([t for p in kv for t in p][:4], range(4)):
        if not torch.equal(t[dst[blk]].view(torch.int16), t[blk].view(torch.int16)):
            raise RuntimeError("a restored block differs from its source")
    out["scatter_note"] = "CUDA events around the launch on the client stream (includes the launch's own " \
                          "device-side overhead)"
    return out


def main():
    args = parse()
    if args.sweep or args.multiturn or args.fill or args.restore or args.latency:
        run = (run_sweep if args.sweep else run_multiturn if args.multiturn else run_fill if args.fill
               else run_restore if args.restore else run_latency)
        print(json.dumps(run(args)))
        return
    rank, local_rank, world = dist_env()
    if args.mix and world == 1:
        print(json.dumps({"error": "--mix shards the store over N > 1 GPUs: run it under torchrun"}))
        sys.exit(2)
    if world != args.gpus and world == 1 and args.gpus > 1:
        print(json.dumps({"error": "run N>1 under torchrun (one rank per GPU)"}))
        sys.exit(2)
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        if world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
        if args.mix:
            line = run_mix(args, rank, local_rank, world)
        elif world > 1 and args.parallelism == "sharded":
            line = run_sharded(args, rank, local_rank, world)
        else:
            line = run_ours(args, rank, local_rank, world)
            if world == 1 and line is not None and not args.no_extras:
                import torch

                torch.cuda.empty_cache()
                line["multiturn_config3"] = run_multiturn(args)  # the host-tier path, on the same box
                torch.cuda.empty_cache()
                line["restore_connector"] = run_restore(args)  # the connector's batched restore
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
    if rank == 0 and line is not None:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
