"""Benchmark of the B200 KV block store on the Qwen3-32B-shaped workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one step): an 8192-token prompt of a Qwen3-32B-shaped paged KV cache -- 64 layers,
8 KV heads, head_dim 128, bf16, 64-token blocks (16 MiB of KV per block, 128 blocks = 2 GiB) --
is put (gathered from a 4096-block paged pool into the store, write-through to the pinned host
tier included) and then restored by get into 128 fresh pool blocks with a 100% device-tier hit
rate. Values are seeded N(0,1) bf16; block tables are random permutations of the pool; keys are
64-bit chained prefix-block hashes, fresh for every step. The metric is payload GB/s of put + get
(2 x 2 GiB per step).

N > 1 (torchrun, one rank per GPU): every rank runs the same workload against its own shard on its
own GPU (weak scaling, no data-path collective); time is the max over ranks and `value` is the
bytes all ranks moved divided by it.

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
    ap.add_argument("--latency-samples", type=int, default=40)
    ap.add_argument("--small", action="store_true",
                    help="profiling case: 16 layers, 512-block pool, 64 blocks per step (same kernels)")
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
        self.path = ROOT / "gpurun_out" / f"clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
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


def build_pool(torch, device):
    """128 member tensors (K, V per layer) of (4096, 8, 64, 128) bf16 filled with seeded N(0,1)."""
    kv = []
    g = torch.Generator(device=device)
    g.manual_seed(20261201)
    for _ in range(LAYERS):
        pair = []
        for _ in range(2):
            t = torch.empty((POOL_BLOCKS, HEADS, BLOCK_TOKENS, HEAD_DIM), dtype=torch.bfloat16, device=device)
            t.normal_(generator=g)
            pair.append(t)
        kv.append(tuple(pair))
    return kv


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

    # correctness gate before timing: restored blocks equal the sources (checksums)
    keys, src, dst = one_step(0)
    torch.cuda.synchronize()
    for layer in (0, LAYERS // 2, LAYERS - 1):
        for t in kv[layer]:
            a = t[torch.as_tensor(src, device=device)].view(torch.int16).to(torch.int64).sum()
            b = t[torch.as_tensor(dst, device=device)].view(torch.int16).to(torch.int64).sum()
            if int(a) != int(b):
                raise RuntimeError("restored blocks differ from the source blocks")
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

    # ---- p50 / p99 get latency per block (committed, device-resident blocks)
    lat = []
    keys, src, dst = step_inputs(9999)
    client.put_blocks(layout, keys, src, sync_commit=True)
    for i in range(args.latency_samples):
        j = i % BATCH_BLOCKS
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        ok = client.get_blocks(layout, keys[j:j + 1], dst[j:j + 1])
        torch.cuda.synchronize()
        lat.append((time.perf_counter() - t1) * 1e3)
        assert ok.all()
    lat.sort()
    p50 = lat[len(lat) // 2]
    p99 = lat[min(len(lat) - 1, math.ceil(0.99 * len(lat)) - 1)]

    # ---- PCIe device->host copy peak (pinned), the bound of the host write-through
    pin = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    src_buf = torch.empty(1 << 30, dtype=torch.uint8, device=device)
    best = 0.0
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        pin.copy_(src_buf, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        best = max(best, (1 << 30) / (e0.elapsed_time(e1) / 1e3) / GB)
    del pin, src_buf

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
        "write_through": {
            "bytes_per_step": BATCH_BLOCKS * BLOCK_PAYLOAD,
            "achieved_GBps": round(BATCH_BLOCKS * BLOCK_PAYLOAD / (elapsed_ms / args.steps / 1e3) / GB, 2),
            "pcie_d2h_peak_GBps": round(best, 2),
            "frac": round(BATCH_BLOCKS * BLOCK_PAYLOAD / (elapsed_ms / args.steps / 1e3) / GB / best, 4),
            "note": "every put is written through to the pinned host tier and get waits for it (commit barrier)",
        },
        "get_latency_ms_per_block": {"p50": round(p50, 4), "p99": round(p99, 4), "block_bytes": BLOCK_PAYLOAD,
                                     "samples": len(lat)},
        "store": {k: stats[k] for k in ("writes_through", "victims_evicted", "catalog_replacements", "live_keys")},
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(seconds=12.0)
    return line


# ------------------------------------------------------------------ CPU baseline (the oracle)


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_run(n_blocks_per_step: int, steps: int, threads: int, pool_blocks: int = 96, warmup: int = 1):
    """The reference host-DRAM path restated in C: put (gather + write-through) then get (scatter)
    of `n_blocks_per_step` Qwen3-32B-shaped blocks per step on a host-resident paged pool."""
    from oracle import kvs_oracle as O

    rng = np.random.default_rng(7)
    members = []
    for _ in range(2 * LAYERS):
        a = np.empty(pool_blocks * SEG_BYTES, np.uint8)
        a.view(np.uint16)[:] = rng.integers(0, 1 << 16, a.size // 2, dtype=np.uint16)
        members.append(a)
    _, _, vlen = O.block_format([SEG_BYTES] * (2 * LAYERS))
    units = -(-vlen // UNIT_BYTES)
    block_units = 1 << (units - 1).bit_length()
    store = O.Store(max_keys=4 * n_blocks_per_step, heap_bytes=3 * n_blocks_per_step * block_units * UNIT_BYTES,
                    host_pool_bytes=(4 * n_blocks_per_step + 8) * units * UNIT_BYTES, max_value_bytes=64 << 20)
    from kvcache_manager import codec  # pure-python key derivation (no device code)

    def step(k):
        perm = rng.permutation(pool_blocks)
        keys = np.array(codec.chained_block_hashes(k * 31 + 5, n_blocks_per_step), np.uint64)
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
    store.close()
    return steps * 2 * n_blocks_per_step * BLOCK_PAYLOAD / dt / GB, dt


def cpu_baseline(seconds: float) -> dict:
    threads = cpu_threads()
    n = 16
    gbps, dt = cpu_run(n, 1, threads)
    steps = max(1, min(20, int(seconds / max(dt, 1e-3))))
    gbps, dt = cpu_run(n, steps, threads)
    return {"value": round(gbps, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} steps x (put {n} + get {n}) Qwen3-32B-shaped 16 MiB blocks on a 96-block host pool, "
                      f"{threads} threads, {dt:.1f} s"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    threads = cpu_threads()
    n = 16
    gbps, dt = cpu_run(n, args.steps, threads, warmup=args.warmup)
    return {
        "metric": METRIC, "value": round(gbps, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic: seeded random bf16 bit patterns, random block tables, chained prefix-hash keys",
        "config": {"workload": WORKLOAD, "blocks_per_step": n, "bytes_per_block": BLOCK_PAYLOAD,
                   "step": "put then get of 16 blocks on the host path (bounded sample of the 128-block step)"},
        "impl": "reference",
        "cpu_baseline": {"value": round(gbps, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps x (put {n} + get {n}) 16 MiB blocks, {threads} threads"},
        "e2e": {"value": round(gbps, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    rank, local_rank, world = dist_env()
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
        line = run_ours(args, rank, local_rank, world)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
    if rank == 0 and line is not None:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
