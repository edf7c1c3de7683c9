"""Benchmark of the indexed sparse gated-FFN decode layer (one JSON line on rank 0).

Workload: batch-1 decode of one FFN layer, hidden 5120, intermediate 17408,
bf16 weights ~ N(0, 0.02^2) in neuron-major packed records, K/N = 0.25
(K = 4352), ids = sort(randperm(N, seed=1000+token)[:K]).  One step = one
token through the layer.  Algorithmic bytes per step =
K*3*H*2 + x + ids(int32) + y = 133,731,328 B.

* value       -- algorithmic GB/s over the timed steps (whole job), inputs
                 already in HBM, each step timed with CUDA events on the
                 launching stream, L2 flushed (256 MiB write) between steps
                 outside the events, max over ranks.
* e2e         -- the same bytes / wall time of the public API call with host
                 buffers: pinned x and ids copied in, y copied back, synced.
* roofline    -- the fused kernel's algorithmic GB/s against the measured HBM
                 copy bandwidth; traffic from the committed ncu summary.
* cpu_baseline-- the CPU restatement of the reference path (index_select +
                 F.linear + SiLU in bf16, runtime/ffn.py:20-39) on this host's
                 cores, a bounded sample of tokens.

N > 1 (torchrun, one process per GPU): the intermediate dimension is split
into N contiguous record ranges; every rank holds the same global ids, keeps
its range (qcc_build_union), computes an fp32 partial y and the partials are
summed with an NCCL all-reduce, then cast to bf16.  Total work per step is
fixed, so scaling is "strong".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import qcc_b200.workloads as workloads  # noqa: E402

METRIC = "indexed sparse-FFN µs/layer & achieved HBM GB/s (bs=1, K/N=0.25, bf16) at 1–8 GPUs"
HIDDEN, INTERMEDIATE, RETENTION = workloads.DECODE_HIDDEN, workloads.DECODE_INTERMEDIATE, 0.25
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--retention", type=float, default=RETENTION)
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="bound on the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-sweep", action="store_true")
    return p.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            pass
    return {}


def committed_traffic() -> dict | None:
    """DRAM bytes per launch of the decode kernel from the committed ncu summary."""
    path = ROOT / "profiles" / "decode_ffn_traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if self.proc is None or self.file is None:
            return None
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append({"sm": float(parts[1]), "max": float(parts[2]), "power": float(parts[3]),
                             "hw": parts[5], "hw_thermal": parts[6], "sw_thermal": parts[7], "power_cap": parts[8]})
            except ValueError:
                continue
        os.unlink(self.file.name)
        if not rows:
            return None
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                              ("sw_thermal", "sw_thermal_slowdown"), ("power_cap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in rows), "sm_max_mhz": max(r["max"] for r in rows),
                "power_w_max": max(r["power"] for r in rows), "samples": len(rows), "reasons": sorted(reasons)}


def step_bytes(k: int) -> int:
    return workloads.decode_bytes(k, HIDDEN, 2)


def cpu_reference_sample(layer_cpu, retention: float, seconds: float) -> dict:
    """Time the CPU restatement of the reference path (runtime/ffn.py:20-39) on this host."""
    from oracle import ffn as offn  # CPU baseline leg only

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gate, up, down = layer_cpu
    k = workloads.retention_k(INTERMEDIATE, retention)
    x = workloads.decode_x()
    times = []
    token = 0
    with torch.inference_mode():
        for _ in range(3):  # warm-up
            offn.dynamic_sparse_ffn(x, workloads.decode_ids(INTERMEDIATE, k, token).long(), gate, up, down)
            token += 1
        start_all = time.perf_counter()
        while (time.perf_counter() - start_all < seconds and len(times) < 200) or len(times) < 5:
            ids = workloads.decode_ids(INTERMEDIATE, k, token).long()
            t0 = time.perf_counter()
            offn.dynamic_sparse_ffn(x, ids, gate, up, down)
            times.append(time.perf_counter() - t0)
            token += 1
    med = statistics.median(times)
    return {"seconds_median": med, "seconds_p95": sorted(times)[int(0.95 * (len(times) - 1))], "tokens": len(times),
            "threads": threads, "gbs": step_bytes(k) / med / 1e9}


def host_description() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU path (restated), host cores only
# ---------------------------------------------------------------------------

def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    k = workloads.retention_k(INTERMEDIATE, args.retention)
    gen_device = "cuda" if torch.cuda.is_available() else "cpu"
    layer = workloads.decode_layer(device=gen_device)
    packed = layer.packed.cpu()
    del layer
    gate = packed[:, :HIDDEN].contiguous()
    up = packed[:, HIDDEN:2 * HIDDEN].contiguous()
    down = packed[:, 2 * HIDDEN:].t().contiguous()
    del packed
    from oracle import ffn as offn  # the reference arm executes the CPU restatement by design

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x = workloads.decode_x()
    times = []
    with torch.inference_mode():
        for step in range(args.warmup + args.steps):
            ids = workloads.decode_ids(INTERMEDIATE, k, step).long()
            t0 = time.perf_counter()
            offn.dynamic_sparse_ffn(x, ids, gate, up, down)
            dt = time.perf_counter() - t0
            if step >= args.warmup:
                times.append(dt)
    total = sum(times)
    bytes_ = step_bytes(k)
    value = bytes_ * len(times) / total / 1e9
    sample = f"{len(times)} decode tokens (K={k}) of the bf16 layer on {threads} host threads ({host_description()})"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / len(times), 4),
        "us_per_layer": round(1e6 * total / len(times), 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) x)",
        "config": {"workload": "decode layer H=5120 N=17408 K/N=0.25 batch 1", "hidden": HIDDEN,
                   "intermediate": INTERMEDIATE, "k": k, "batch": 1, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        group = dist.group.WORLD

    from qcc_b200.runtime.engine import IndexedSparseFFN
    from qcc_b200.runtime.packing import PackedFFNWeights
    from qcc_b200.runtime.sharded import ShardedIndexedFFN, shard_range

    k = workloads.retention_k(INTERMEDIATE, args.retention)
    begin, end = shard_range(INTERMEDIATE, world, rank)
    layer = workloads.decode_layer(device=device, record_range=(begin, end))
    weights = PackedFFNWeights(layer.packed, HIDDEN, end - begin, begin, INTERMEDIATE)
    if world == 1:
        engine = IndexedSparseFFN(weights)
        launches_per_step = 1
    else:
        engine = ShardedIndexedFFN(weights, group=group)
        launches_per_step = 3  # shard filter, fused FFN, cast (the all-reduce is NCCL's)

    x = workloads.decode_x().to(device)
    n_ids = args.warmup + args.steps
    ids_all = torch.stack([workloads.decode_ids(INTERMEDIATE, k, t) for t in range(n_ids)]).to(device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    # Warm-up (also builds workspaces / NCCL communicators).
    for t in range(args.warmup):
        engine(x, ids_all[t])
    torch.cuda.synchronize(device)
    barrier()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(device.index) as clocks:
        barrier()
        torch.cuda.synchronize(device)
        for i in range(args.steps):
            flush.fill_(i & 0xFF)  # evict the previous step's records from L2 (outside the events)
            starts[i].record(stream)
            engine(x, ids_all[args.warmup + i])
            ends[i].record(stream)
        torch.cuda.synchronize(device)
        barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = torch.tensor([sum(step_ms)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(total_ms, op=torch.distributed.ReduceOp.MAX)
    total_ms = float(total_ms.item())
    ms_per_step = total_ms / args.steps
    bytes_ = step_bytes(k)
    value = bytes_ / (ms_per_step * 1e-3) / 1e9

    # Kernel-only duration of the fused FFN launch (N=1: the whole step is one launch).
    kernel_ms = ms_per_step if world == 1 else None

    # End-to-end through the public API with host buffers.
    x_host = workloads.decode_x().pin_memory()
    ids_host = [workloads.decode_ids(INTERMEDIATE, k, t).pin_memory() for t in range(min(args.steps, 64))]
    y_host = torch.empty((1, HIDDEN), dtype=torch.bfloat16).pin_memory()
    for t in range(3):
        y = engine(x_host.to(device, non_blocking=True), ids_host[t].to(device, non_blocking=True))
        y_host.copy_(y, non_blocking=True)
    torch.cuda.synchronize(device)
    barrier()
    e2e_times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        xd = x_host.to(device, non_blocking=True)
        idd = ids_host[i % len(ids_host)].to(device, non_blocking=True)
        y = engine(xd, idd)
        y_host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        e2e_times.append(time.perf_counter() - t0)
    e2e_s = torch.tensor([sum(e2e_times) / len(e2e_times)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(e2e_s, op=torch.distributed.ReduceOp.MAX)
    e2e_step = float(e2e_s.item())

    sweep = None
    if not args.no_sweep and world == 1:
        sweep = {}
        for r in (0.5, 0.25, 0.1, 0.05):
            kk = workloads.retention_k(INTERMEDIATE, r)
            sids = [workloads.decode_ids(INTERMEDIATE, kk, 5000 + t).to(device) for t in range(20)]
            for t in range(3):
                engine(x, sids[t])
            times = []
            for t in range(20):
                flush.fill_(t & 0xFF)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                engine(x, sids[t])
                e.record(stream)
                e.synchronize()
                times.append(s.elapsed_time(e))
            us = 1e3 * statistics.median(times)
            sweep[str(r)] = {"k": kk, "us_per_layer": round(us, 2),
                             "gbs": round(step_bytes(kk) / (us * 1e-6) / 1e9, 1)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        packed = layer.packed.cpu()
        layer_cpu = (packed[:, :HIDDEN].contiguous(), packed[:, HIDDEN:2 * HIDDEN].contiguous(),
                     packed[:, 2 * HIDDEN:].t().contiguous())
        del packed
        cpu = cpu_reference_sample(layer_cpu, args.retention, args.cpu_seconds)
        del layer_cpu

    if world > 1:
        engine.close()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return

    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = float(peak or FALLBACK_HBM_GBS)
    traffic = committed_traffic()
    roofline = None
    if kernel_ms is not None:
        achieved = bytes_ / (kernel_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "peak_source": peak_src,
                    "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
                    "algorithmic_bytes": bytes_, "kernel": "indexed_ffn_decode_kernel"}
    clock_summary = clocks.summary()
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "us_per_layer": round(ms_per_step * 1e3, 3),
        "tokens_per_s": round(1e3 / ms_per_step, 1), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) x)",
        "config": {"workload": "decode layer H=5120 N=17408 K/N=0.25 batch 1", "hidden": HIDDEN,
                   "intermediate": INTERMEDIATE, "k": k, "batch": 1, "retention": args.retention,
                   "parallelism": f"intermediate-dim shard x{world}" if world > 1 else "single GPU",
                   "l2": "256 MiB flush write between timed steps (outside the events); per-step records 133.7 MB"},
        "gpu_launches": launches_per_step * args.steps,
        "e2e": {"value": round(bytes_ / e2e_step / 1e9, 3), "unit": "GB/s",
                "us_per_layer": round(e2e_step * 1e6, 2),
                "h2d_bytes_per_step": x_host.numel() * 2 + ids_host[0].numel() * 4,
                "d2h_bytes_per_step": y_host.numel() * 2},
        "roofline": roofline,
        "clocks": clock_summary,
    }
    if sweep is not None:
        line["sweep"] = sweep
    if cpu is not None:
        line["cpu_baseline"] = {"value": round(cpu["gbs"], 4), "unit": "GB/s", "cores": cpu["threads"],
                                "kind": "port", "us_per_layer": round(cpu["seconds_median"] * 1e6, 1),
                                "sample": f"{cpu['tokens']} decode tokens (K={k}) of the same bf16 layer, "
                                          f"median, {cpu['threads']} threads ({host_description()})"}
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
