"""Benchmark of the indexed sparse gated-FFN decode layer (one JSON line on rank 0).

Workload: batch-1 decode of one FFN layer, hidden 5120, intermediate 17408,
bf16 weights ~ N(0, 0.02^2) in neuron-major packed records, K/N = 0.25
(K = 4352), ids = sort(randperm(N, seed=1000+token)[:K]).  One step = one
token through the layer.  Algorithmic bytes per step =
K*3*H*2 + x + ids(int32) + y = 133,731,328 B.

* value       -- algorithmic GB/s over the timed steps (whole job), inputs
                 already in HBM.  The K timed steps run back to back in one
                 CUDA graph, timed with CUDA events on the launching stream
                 around the replay.  Step i runs layer i mod 4 of four
                 independently drawn layers with the ids of token i, as
                 consecutive layers of a decode pass would: each step reads a
                 133.7 MB record set (larger than the 126 MB L2) that the step
                 before did not touch.  Max over ranks.
* e2e         -- the same bytes / wall time of the public API call with host
                 buffers: pinned x and ids copied in, y copied back, synced.
* roofline    -- the fused kernel's algorithmic GB/s against the measured HBM
                 copy bandwidth; traffic from the committed ncu summary.
* cpu_baseline-- the CPU restatement of the reference path (index_select +
                 F.linear + SiLU in bf16, runtime/ffn.py:20-39) on this host's
                 cores, a bounded sample of tokens.

N > 1 (torchrun, one process per GPU): the intermediate dimension is split
into N contiguous record ranges; every rank holds the same global ascending
ids and runs the fused kernel on them with its range (the kernel finds the
run of ids inside the range and rebases them); the sum over ranks is fused
into that kernel's epilogue (column sums stored into every
rank's exchange buffer over NVLink, added in rank order), so y comes out in
bf16 on every rank with no NCCL call.  Total work per step is fixed, so
scaling is "strong".

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
FALLBACK_BF16_TFLOPS = 1590.0
LAYERS = 4  # independently drawn layers the steps cycle through


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
    p.add_argument("--no-selector", action="store_true", help="skip the selector + fused FFN measurement")
    p.add_argument("--no-offload", action="store_true", help="skip the 8-layer host-offload measurement")
    p.add_argument("--offload-tokens", type=int, default=12)
    p.add_argument("--no-prefill", action="store_true", help="skip the block-sparse prefill measurement")
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


def step_call(engine, x, ids, out, ids_ready=True):
    """One decode step through the engine (single GPU: the kernels write into `out`).

    ids_ready: the step's ids are inputs resident before the steps run (not
    produced by an earlier launch of this library on the stream), so each
    step may start its record copies while the step before finishes.
    """
    if hasattr(engine, "partial"):
        return engine(x, ids, ids_ready=ids_ready)
    return engine(x, ids, out=out, ids_ready=ids_ready)


def step_bytes(k: int) -> int:
    return workloads.decode_bytes(k, HIDDEN, 2)


def workload_config(k: int, retention: float) -> dict:
    """The workload both arms measure (identical dicts; how each arm runs it is reported beside)."""
    return {"workload": "decode layer H=5120 N=17408 K/N=0.25 batch 1", "hidden": HIDDEN,
            "intermediate": INTERMEDIATE, "k": k, "batch": 1, "retention": retention, "layers": LAYERS,
            "l2": "inputs larger than L2: each step reads a 133.7 MB record set of the next of 4 "
                  "independently drawn layers (ids of a different token)"}


def cross_rank_parity(engine, x, ids, group, device, rank: int, world: int, begin: int, end: int) -> dict:
    """One token through the fused exchange and through the NCCL path on every rank.

    y of the fused path must be bit-identical on every rank and both paths
    within the bf16 tolerance (rel-L2 1e-2) of a float64 torch evaluation of
    the whole layer (rank 0 draws the full layer of the same seed).  Every
    rank takes the same collective steps.
    """
    import torch.distributed as dist
    from qcc_b200.runtime.sharded import ShardedIndexedFFN

    y_fused = engine(x, ids)
    nccl = ShardedIndexedFFN(engine.weights, group=group, allreduce="nccl")
    y_nccl = nccl(x, ids)
    gathered = [torch.empty_like(y_fused) for _ in range(world)]
    dist.all_gather(gathered, y_fused, group=group)
    torch.cuda.synchronize(device)
    engine.check()
    identical = all(torch.equal(g, gathered[0]) for g in gathered)
    out = {"token": 0, "ranks_identical": identical, "tolerance_rel_l2": 1e-2}
    if rank == 0:
        full = workloads.decode_layer(device=device, seed=0).packed
        sel = full.index_select(0, ids.long())
        g, u, d = (sel[:, i * HIDDEN:(i + 1) * HIDDEN].double() for i in range(3))
        xd = x.double()
        gv, uv = xd @ g.t(), xd @ u.t()
        ref = (gv * torch.sigmoid(gv) * uv) @ d
        del full, sel, g, u, d

        def rel(y):
            return float(torch.linalg.vector_norm(y.double() - ref) / torch.linalg.vector_norm(ref))

        out["fused_vs_f64_rel_l2"] = rel(y_fused)
        out["nccl_vs_f64_rel_l2"] = rel(y_nccl)
        out["ok"] = identical and out["fused_vs_f64_rel_l2"] <= 1e-2 and out["nccl_vs_f64_rel_l2"] <= 1e-2
    del nccl
    torch.cuda.empty_cache()
    return out


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


def graph_time_us(fn, steps: int, stream: torch.cuda.Stream, side: torch.cuda.Stream) -> float:
    """Mean device time of fn(i) for i < steps, captured back to back in one CUDA graph."""
    with torch.cuda.stream(side):
        for i in range(min(3, steps)):
            fn(i)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(steps):
            fn(i)
    graph.replay()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    graph.replay()
    end.record(stream)
    end.synchronize()
    del graph
    return 1e3 * start.elapsed_time(end) / steps


def measure_selector(engine, x, device, stream, side) -> dict:
    """Selector workload: top-K (K/N = 0.2) over per-neuron fp32 scores, then the fused FFN.

    Batch 1 uses the selected ids directly; batch 8 merges the per-token id
    sets (qcc_build_union) and runs the fused kernel with per-record token bits.
    """
    from qcc_b200.runtime.selector import build_union, select_topk

    k = workloads.retention_k(INTERMEDIATE, 0.2)
    out = {"k": k, "scores": "Laplace(0,1) with a Zipf(1.1)-boosted hot 10% (seeded)"}
    steps = 20
    scores1 = workloads.selector_scores(steps, seed=21).to(device)
    ids1 = torch.empty((1, k), dtype=torch.int32, device=device)
    y1 = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=device)
    out["select_us_batch1"] = round(graph_time_us(lambda i: select_topk(scores1[i:i + 1], k, out=ids1), steps,
                                                  stream, side), 2)

    def step1(i):
        select_topk(scores1[i:i + 1], k, out=ids1)
        engine(x, ids1[0], out=y1)

    out["select_ffn_us_batch1"] = round(graph_time_us(step1, steps, stream, side), 2)
    # Batches of 2, 4 and 8 tokens with their own selections: selector, union of
    # the ids with per-token bits, one decode over the union (2-8 tokens: one
    # tensor-core launch and its reduce).  union_gbs: the union's record bytes
    # (+ x, ids, y) over the step time.
    for batch in (2, 4, 8):
        scores_b = [workloads.selector_scores(batch, seed=40 + i).to(device) for i in range(steps)]
        ids_b = torch.empty((batch, k), dtype=torch.int32, device=device)
        x_b = workloads.decode_x(batch=batch).to(device)
        y_b = torch.empty((batch, HIDDEN), dtype=torch.bfloat16, device=device)

        def step_b(i, scores_b=scores_b, ids_b=ids_b, x_b=x_b, y_b=y_b):
            select_topk(scores_b[i], k, out=ids_b)
            union, mask, count = build_union(ids_b, 0, INTERMEDIATE)
            engine(x_b, union, token_mask=mask, n_ids_dev=count, out=y_b)

        us = graph_time_us(step_b, steps, stream, side)
        records = float(torch.stack([build_union(select_topk(scores_b[i], k), 0, INTERMEDIATE)[2]
                                     for i in range(steps)]).float().mean().item())
        union_bytes = records * 3 * HIDDEN * 2 + batch * HIDDEN * 2 * 2 + records * 4
        out[f"select_union_ffn_us_batch{batch}"] = round(us, 2)
        out[f"union_records_batch{batch}"] = round(records, 1)
        out[f"union_gbs_batch{batch}"] = round(union_bytes / (us * 1e-6) / 1e9, 1)
    out["score_select"] = measure_score_select(engine, x, device, stream, side)
    return out


def selector_predictor(seed: int = 7) -> dict:
    """A residual latent predictor with the reference CudaSelector's shape (hidden 5120, latent 32)."""
    g = torch.Generator().manual_seed(seed)
    latent = 32
    return {"enc_w": torch.randn(latent, HIDDEN, generator=g) * 0.02, "enc_b": torch.randn(latent, generator=g) * 0.1,
            "fc1_w": torch.randn(latent, latent, generator=g) * 0.2, "fc1_b": torch.randn(latent, generator=g) * 0.1,
            "fc2_w": torch.randn(latent, latent, generator=g) * 0.2, "fc2_b": torch.randn(latent, generator=g) * 0.1,
            "ln_w": 1 + 0.1 * torch.randn(latent, generator=g), "ln_b": 0.1 * torch.randn(latent, generator=g),
            "out_w": torch.randn(INTERMEDIATE, latent, generator=g) * 0.2,
            "out_b": torch.randn(INTERMEDIATE, generator=g) * 0.1}


def measure_score_select(engine, x, device, stream, side) -> dict:
    """The fused score producer + top-K (the reference's runtime selector in one launch).

    Predictor: residual, hidden 5120, latent 32, 17408 neurons, bf16 weights
    (runtime/cuda_selector.py's shape); k = N // 2 (CudaSelector) and K/N = 0.2.
    Also selector + fused FFN from x, and the reference's path (predictor as
    torch ops + torch.topk) on the host cores.
    """
    from qcc_b200.runtime.cuda_selector import FusedScoreSelector

    params = selector_predictor()
    steps = 20
    xs = torch.randn(steps, 1, HIDDEN, generator=torch.Generator().manual_seed(8)).to(device, torch.bfloat16)
    out = {"predictor": "residual, hidden 5120, latent 32, N 17408, bf16 weights, fp32 arithmetic"}
    for name, k in (("k_half", INTERMEDIATE // 2), ("k_r0.2", workloads.retention_k(INTERMEDIATE, 0.2))):
        sel = FusedScoreSelector(params, kind=0, k=k, dtype=torch.bfloat16, device=device)
        out[f"us_batch1_{name}"] = round(graph_time_us(lambda i: sel.run(xs[i], want_scores=False), steps, stream,
                                                       side), 2)
        if name == "k_r0.2":
            y1 = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=device)
            out["select_ffn_us_batch1_r0.2"] = round(graph_time_us(
                lambda i: engine(xs[i], sel.run(xs[i], want_scores=False)[1][0], out=y1), steps, stream, side), 2)
        sel.check()
    return out


def score_select_cpu_sample(seconds: float) -> dict:
    """The reference's runtime selector on the host: predictor forward + torch.topk (fp32)."""
    from oracle import predictor as opred  # CPU baseline leg only

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    params = selector_predictor()
    x = torch.randn(1, HIDDEN, generator=torch.Generator().manual_seed(8))
    k = INTERMEDIATE // 2
    times = []
    start = time.perf_counter()
    with torch.inference_mode():
        for _ in range(3):
            opred.torch_runtime_selector(x, params, k)
        while time.perf_counter() - start < seconds or len(times) < 20:
            t0 = time.perf_counter()
            opred.torch_runtime_selector(x, params, k)
            times.append(time.perf_counter() - t0)
            if len(times) >= 2000:
                break
    return {"us_batch1_k_half": round(statistics.median(times) * 1e6, 2), "cores": threads, "kind": "port",
            "sample": f"{len(times)} calls, median, fp32 torch ops ({host_description()})"}


def measure_dense_and_oracle(device, stream, side, sparse_us: float) -> dict:
    """The dense layer the sparse path replaces, and the oracle-mode path, at full layer size (bf16).

    * dense: reference runtime/ffn.py:11-17 (DenseFFN) as torch ops --
      three cuBLAS GEMVs over the whole layer (267 MB) -- at batch 1;
      ``speedup_of_sparse_decode`` = dense time / the headline step time.
    * oracle_mode: ``OracleModeFFN`` (gate|up pass over every record, |a| *
      ||D|| top-K per token, down pass over the selected records) at 1 and 4
      tokens, K/N 0.25; bytes = gate|up of every record + the down parts of
      the tokens' union + x + y.  Beside it the reference's formulation of the
      same step as torch ops on this GPU (end_to_end/oracle_sparse_mlp.py:
      dense gate/up, |a| * norms, torch.topk, scatter into zeros, dense down).
    Steps alternate two independently drawn layers in one CUDA graph.
    """
    from qcc_b200.runtime.oracle_mode import OracleModeFFN, down_column_norms
    from qcc_b200.runtime.packing import PackedFFNWeights
    import torch.nn.functional as F

    layers = [workloads.decode_layer(device=device, seed=500 + s) for s in range(2)]
    views = [(l.gate(), l.up(), l.down()) for l in layers]
    steps = 20
    xs = torch.randn(steps, 4, HIDDEN, generator=torch.Generator().manual_seed(31)).to(device, torch.bfloat16)
    out = {}

    def dense_step(i, rows):
        g, u, d = views[i % 2]
        x = xs[i, :rows]
        return F.linear(F.silu(F.linear(x, g)) * F.linear(x, u), d)

    dense_us = graph_time_us(lambda i: dense_step(i, 1), steps, stream, side)
    dense_bytes = 3 * HIDDEN * INTERMEDIATE * 2
    out["dense"] = {"us_per_layer": round(dense_us, 2), "gbs": round(dense_bytes / (dense_us * 1e-6) / 1e9, 1),
                    "impl": "torch F.linear x3 (cuBLAS), batch 1",
                    "speedup_of_sparse_decode": round(dense_us / sparse_us, 2)}
    engines = [OracleModeFFN(PackedFFNWeights(l.packed, HIDDEN, INTERMEDIATE), 0.25) for l in layers]
    k = engines[0].k
    for rows in (1, 4):
        us = graph_time_us(lambda i: engines[i % 2](xs[i, :rows]), steps, stream, side)
        _, ids = engines[0](xs[0, :rows])
        union = int(torch.unique(ids).numel())
        nbytes = INTERMEDIATE * 2 * HIDDEN * 2 + union * HIDDEN * 2 + 2 * rows * HIDDEN * 2
        norms = [down_column_norms(e.weights) for e in engines]

        def torch_step(i, rows=rows):
            g, u, d = views[i % 2]
            x = xs[i, :rows]
            a = F.silu(F.linear(x, g)) * F.linear(x, u)
            scores = a.abs().float() * norms[i % 2]
            idx = torch.topk(scores, k, dim=-1, sorted=False).indices
            sparse = torch.zeros_like(a).scatter_(-1, idx, a.gather(-1, idx))
            return F.linear(sparse, d)

        torch_us = graph_time_us(torch_step, steps, stream, side)
        out[f"oracle_mode_tokens{rows}"] = {
            "us": round(us, 2), "algorithmic_bytes": nbytes, "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
            "union_records": union, "k": k,
            "launches": 4 * ((rows + engines[0].max_batch - 1) // engines[0].max_batch) + 1,
            "reference_formulation_torch_us": round(torch_us, 2)}
        for e in engines:
            e.check()
    del engines, layers, views
    torch.cuda.empty_cache()
    return out


def measure_prefill(device, stream, side, cpu_seconds: float) -> dict:
    """Block-sparse prefill: 512 tokens in four 128-token tiles, hidden 5120, N 17408, bf16.

    Records form 272 blocks of 64; a seeded 20 % of the blocks is on for every
    tile, every other block per tile with the probability that makes 30 % of
    the blocks on per tile.  Steps alternate between two independently drawn
    layers (1.07 GB of records) in one CUDA graph.  Roofline: tensor-core
    FLOPs (2 * 128 * 3 * H per selected record per tile) against the measured
    bf16 GEMM peak; the unique record bytes are reported beside it.
    """
    from qcc_b200.runtime.packing import PackedFFNWeights
    from qcc_b200.runtime.prefill import BlockSparsePrefill, tile_block_lists

    layers = [workloads.decode_layer(device=device, seed=300 + s) for s in range(2)]
    engines = [BlockSparsePrefill(PackedFFNWeights(l.packed, HIDDEN, INTERMEDIATE)) for l in layers]
    x = workloads.prefill_x(device=device)
    _, tiles = workloads.prefill_tile_blocks()
    flat, offsets = tile_block_lists(tiles, device)
    y = torch.empty_like(x)
    steps = 20
    us = graph_time_us(lambda i: engines[i % 2](x, (flat, offsets), out=y), steps, stream, side)
    flops = workloads.prefill_flops(tiles)
    unique = workloads.prefill_unique_bytes(tiles)
    peaks = measured_peaks()
    peak = peaks.get("bf16_tflops")
    peak_src = "measured" if peak else "fallback"
    peak = float(peak or FALLBACK_BF16_TFLOPS)
    achieved = flops / (us * 1e-6) / 1e12
    out = {"tokens": workloads.PREFILL_TOKENS, "tiles": len(tiles), "blocks_per_tile": [t.numel() for t in tiles],
           "block_records": workloads.PREFILL_BLOCK, "us": round(us, 2), "tflops": round(achieved, 1),
           "tokens_per_s": round(workloads.PREFILL_TOKENS / (us * 1e-6), 1),
           "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(achieved / peak, 4), "peak_source": peak_src, "flops": flops,
                        "unique_record_bytes": unique,
                        "hbm_gbs_of_unique_bytes": round(unique / (us * 1e-6) / 1e9, 1)},
           "gpu_launches_per_step": 2}
    del engines
    # The same call on fp32 records (kind::tf32: the products use the tf32 part
    # of each operand, sums in fp32); the tf32 dense rate is half the bf16 one.
    engines = [BlockSparsePrefill(PackedFFNWeights(l.packed.float(), HIDDEN, INTERMEDIATE)) for l in layers]
    del layers
    x32, y32 = x.float(), torch.empty(x.shape, dtype=torch.float32, device=device)
    us32 = graph_time_us(lambda i: engines[i % 2](x32, (flat, offsets), out=y32), steps, stream, side)
    achieved32 = flops / (us32 * 1e-6) / 1e12
    out["fp32_records"] = {"us": round(us32, 2), "tflops": round(achieved32, 1),
                           "frac_of_half_bf16_peak": round(achieved32 / (peak / 2), 4),
                           "record_bytes_unique": 2 * unique}
    del engines
    torch.cuda.empty_cache()
    if cpu_seconds > 0:
        out["cpu_baseline"] = prefill_cpu_sample(tiles, cpu_seconds)
    return out


def prefill_cpu_sample(tiles, seconds: float) -> dict:
    """The reference's per-tile path on the host: TorchDynamicSparseFFN on the expanded ids of a tile."""
    from oracle import ffn as offn  # CPU baseline leg only

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    layer = workloads.decode_layer(device="cpu", seed=300)
    gate, up = layer.gate().contiguous(), layer.up().contiguous()
    down = layer.down().contiguous()
    x = workloads.prefill_x()
    times = []
    start = time.perf_counter()
    with torch.inference_mode():
        for t, blocks in enumerate(tiles):
            ids = (blocks.long()[:, None] * workloads.PREFILL_BLOCK + torch.arange(workloads.PREFILL_BLOCK)).flatten()
            t0 = time.perf_counter()
            offn.dynamic_sparse_ffn(x[t * 128:(t + 1) * 128], ids, gate, up, down)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - start > seconds:
                break
    per_tile = statistics.median(times)
    return {"value": round(per_tile * len(tiles) * 1e6, 1), "unit": "us per 512-token prefill", "cores": threads,
            "kind": "port", "sample": f"{len(times)} of {len(tiles)} tiles (128 tokens each), median tile time x "
                                      f"{len(tiles)}, {threads} threads"}


def measure_offload(device, tokens: int) -> dict:
    """Eight layers with 25 % of their records in HBM and the rest in pinned host RAM.

    Per token every layer selects K = ceil(0.1 N) ids (80 % from the hot set,
    50 % reused from the previous token); misses stream from the host store
    into an LRU cache of 2048 slots per layer while the resident records run.
    """
    from qcc_b200.runtime.stager import HostOffloadLayer

    n_layers, capacity = 8, 2048
    k = workloads.retention_k(INTERMEDIATE, 0.1)
    layers, seqs = [], []
    for l in range(n_layers):
        packed = workloads.decode_layer(device=device, seed=100 + l).packed
        hot = workloads.offload_hot_set(INTERMEDIATE, seed=11 + l)
        layers.append(HostOffloadLayer(packed, HIDDEN, hot, capacity=capacity, max_k=k, device=device))
        del packed
        seqs.append([t.to(device) for t in workloads.offload_token_ids(INTERMEDIATE, k, hot, tokens, seed=12 + l)])
    torch.cuda.empty_cache()
    x = workloads.decode_x().to(device)
    stream = torch.cuda.current_stream(device)
    # One call per layer with no ids first: kernels loaded, workspaces and
    # events made, the cache left empty -- so that token 0 times the cold
    # cache, not first-call set-up.
    no_ids = torch.empty(0, dtype=torch.int32, device=device)
    for layer in layers:
        layer(x, no_ids)
    torch.cuda.synchronize(device)
    per_token_ms, misses = [], []
    for t in range(tokens):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        token_misses = 0
        for l, layer in enumerate(layers):
            layer(x, seqs[l][t])
        end.record(stream)
        end.synchronize()
        for layer in layers:
            token_misses += layer.stats()["misses"]
        per_token_ms.append(start.elapsed_time(end))
        misses.append(token_misses)
    record = layers[0].record_bytes
    steady = list(range(2, tokens))
    steady_ms = sum(per_token_ms[t] for t in steady)
    steady_bytes = sum(misses[t] for t in steady) * record
    # Pinned host -> device copy peak on this box (cudaMemcpyAsync, 256 MiB).
    host = torch.empty(256 << 20, dtype=torch.uint8).pin_memory()
    dev = torch.empty_like(host, device=device)
    best = 0.0
    for _ in range(3):
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        dev.copy_(host, non_blocking=True)
        e0.record(stream)
        e0.synchronize()
        best = max(best, host.numel() / (s0.elapsed_time(e0) * 1e-3) / 1e9)
    return {"layers": n_layers, "tokens": tokens, "k": k, "hot_fraction": 0.25, "cache_slots": capacity,
            "cold_start_us_per_layer": round(1e3 * per_token_ms[0] / n_layers, 1),
            "steady_us_per_layer": round(1e3 * steady_ms / (len(steady) * n_layers), 1),
            "steady_miss_records_per_layer": round(sum(misses[t] for t in steady) / (len(steady) * n_layers), 1),
            "steady_cold_gbs": round(steady_bytes / (steady_ms * 1e-3) / 1e9, 2),
            "pinned_h2d_peak_gbs": round(best, 2)}


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
        "config": workload_config(k, args.retention),
        "execution": f"reference CPU path (restated), {threads} host threads, steps one after another",
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
    from qcc_b200.runtime.sharded import PeerExchange, ShardedIndexedFFN, shard_range

    k = workloads.retention_k(INTERMEDIATE, args.retention)
    begin, end = shard_range(INTERMEDIATE, world, rank)
    # Consecutive steps run consecutive layers (independently drawn weights),
    # as a decode pass does: no step finds its records in L2 from the step
    # before (the same layer recurs only after ~400 MB of other records).
    layers = [workloads.decode_layer(device=device, record_range=(begin, end), seed=s) for s in range(LAYERS)]
    if world == 1:
        engines = [IndexedSparseFFN(PackedFFNWeights(l.packed, HIDDEN, end - begin, begin, INTERMEDIATE))
                   for l in layers]
        launches_per_step = 2  # record-streaming launch + reduce launch
    else:
        # One exchange buffer per rank serves every layer: the calls of one stream never overlap.
        exchange = PeerExchange(group, device, 1, HIDDEN, torch.bfloat16)
        engines = [ShardedIndexedFFN(PackedFFNWeights(l.packed, HIDDEN, end - begin, begin, INTERMEDIATE),
                                     group=group, allreduce="fused", exchange=exchange) for l in layers]
        launches_per_step = 2  # records of the shard's range, then the reduce with the cross-rank sum
    engine = engines[0]
    layer = layers[0]

    x = workloads.decode_x().to(device)
    n_ids = args.warmup + args.steps
    ids_all = torch.stack([workloads.decode_ids(INTERMEDIATE, k, t) for t in range(n_ids)]).to(device)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    # N > 1: driver-visible correctness of the sharded path before any timing.
    parity = cross_rank_parity(engines[0], x, ids_all[0], group, device, rank, world, begin, end) if world > 1 else None

    # Warm-up (builds the stream workspace / NCCL communicators) on the stream
    # the graph is captured on, so the capture finds everything ready.
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    out_buf = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=device)
    with torch.cuda.stream(side):
        for t in range(args.warmup):
            step_call(engines[t % LAYERS], x, ids_all[t], out_buf)
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)

    def run_steps(first: int, count: int) -> None:
        for i in range(first, first + count):
            step_call(engines[i % LAYERS], x, ids_all[i], out_buf)

    # Timed: the K steps back to back in one CUDA graph, CUDA events on the
    # launching stream around the replay.  With N > 1 every rank captures the
    # same sequence of fused launches (their exchange slots rotate in step);
    # the graph is released before the process group is destroyed.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        run_steps(args.warmup, args.steps)
    # One untimed replay first: the first launch of a graph also uploads it
    # (measured at ~4 us per step of a 20-step graph), which is set-up, not a step.
    graph.replay()
    torch.cuda.synchronize(device)
    barrier()
    start_ev, end_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clocks:
        barrier()
        torch.cuda.synchronize(device)
        start_ev.record(stream)
        graph.replay()
        end_ev.record(stream)
        torch.cuda.synchronize(device)
        barrier()
    total_ms = torch.tensor([start_ev.elapsed_time(end_ev)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(total_ms, op=torch.distributed.ReduceOp.MAX)
    total_ms = float(total_ms.item())
    ms_per_step = total_ms / args.steps
    bytes_ = step_bytes(k)
    value = bytes_ / (ms_per_step * 1e-3) / 1e9
    del graph

    # The same steps with the ids read only after the wait for the step before
    # (as when a selector launch on the stream produces them): reported beside
    # the headline, not part of it.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(args.warmup, args.warmup + args.steps):
            step_call(engines[i % LAYERS], x, ids_all[i], out_buf, ids_ready=False)
    torch.cuda.synchronize(device)
    barrier()
    graph.replay()
    torch.cuda.synchronize(device)
    barrier()
    s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s1.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(device)
    late_ms = torch.tensor([s1.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(late_ms, op=torch.distributed.ReduceOp.MAX)
    late_us = 1e3 * float(late_ms.item()) / args.steps
    del graph
    barrier()

    # Duration of one step's launches (the record-streaming launch and its
    # reduce; at N > 1 the reduce also does the cross-rank sum).
    kernel_ms = ms_per_step
    # Bytes this rank streams per step: its shard's records among the step's ids.
    timed_ids = ids_all[args.warmup:args.warmup + args.steps]
    local_k = float(((timed_ids >= begin) & (timed_ids < end)).sum().item()) / args.steps
    rank_bytes = local_k * 3 * HIDDEN * 2 + HIDDEN * 2 * 2 + k * 4

    # End-to-end through the public API with host buffers: per step one
    # host->device copy of that step's x and ids (packed in one pinned
    # buffer), the layer call, and a device->host copy of y, then a sync;
    # wall-clock time, steps cycling through the layers as above.
    x_bytes = HIDDEN * 2
    id_bytes = k * 4
    host_in = []
    for t in range(min(args.steps, 64)):
        buf = torch.empty(x_bytes + id_bytes, dtype=torch.uint8).pin_memory()
        buf[:x_bytes].copy_(workloads.decode_x().view(torch.uint8).reshape(-1))
        buf[x_bytes:].copy_(workloads.decode_ids(INTERMEDIATE, k, t).view(torch.uint8))
        host_in.append(buf)
    dev_in = torch.empty(x_bytes + id_bytes, dtype=torch.uint8, device=device)
    x_dev = dev_in[:x_bytes].view(torch.bfloat16).view(1, HIDDEN)
    ids_dev = dev_in[x_bytes:].view(torch.int32)
    y_host = torch.empty((1, HIDDEN), dtype=torch.bfloat16).pin_memory()
    y_dev = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=device)  # the caller's output buffer (out=)

    def e2e_step(i: int) -> None:
        dev_in.copy_(host_in[i % len(host_in)], non_blocking=True)
        y = engines[i % LAYERS](x_dev, ids_dev, out=y_dev)
        y_host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()

    for t in range(4):
        e2e_step(t)
    barrier()
    e2e_times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        e2e_step(i)
        e2e_times.append(time.perf_counter() - t0)
    e2e_s = torch.tensor([sum(e2e_times) / len(e2e_times)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(e2e_s, op=torch.distributed.ReduceOp.MAX)
    e2e_step_s = float(e2e_s.item())

    sweep = None
    if not args.no_sweep and world == 1:
        sweep = {}
        for r in (0.5, 0.25, 0.1, 0.05):
            kk = workloads.retention_k(INTERMEDIATE, r)
            sids = torch.stack([workloads.decode_ids(INTERMEDIATE, kk, 5000 + t) for t in range(40)]).to(device)
            with torch.cuda.stream(side):
                for t in range(4):
                    step_call(engines[t % LAYERS], x, sids[t], out_buf)
            torch.cuda.current_stream(device).wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                for t in range(40):
                    step_call(engines[t % LAYERS], x, sids[t], out_buf)
            g.replay()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            g.replay()
            e0.record(stream)
            e0.synchronize()
            del g
            us = 1e3 * s0.elapsed_time(e0) / 40
            sweep[str(r)] = {"k": kk, "us_per_layer": round(us, 2),
                             "gbs": round(step_bytes(kk) / (us * 1e-6) / 1e9, 1)}

    selector = None
    if not args.no_selector and world == 1:
        selector = measure_selector(engines[0], x, device, stream, side)
        if not args.no_cpu_baseline:
            selector["score_select"]["cpu_baseline"] = score_select_cpu_sample(3.0)
    offload = None
    if not args.no_offload and world == 1:
        offload = measure_offload(device, args.offload_tokens)
    dense_oracle = None
    if not args.no_selector and world == 1:
        dense_oracle = measure_dense_and_oracle(device, stream, side, ms_per_step * 1e3)
    prefill = None
    if not args.no_prefill and world == 1:
        prefill = measure_prefill(device, stream, side, 0.0 if args.no_cpu_baseline else 10.0)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        packed = layer.packed.cpu()
        layer_cpu = (packed[:, :HIDDEN].contiguous(), packed[:, HIDDEN:2 * HIDDEN].contiguous(),
                     packed[:, 2 * HIDDEN:].t().contiguous())
        del packed
        cpu = cpu_reference_sample(layer_cpu, args.retention, args.cpu_seconds)
        del layer_cpu

    if world > 1:
        for e in engines:
            e.close()
        exchange.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return

    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = float(peak or FALLBACK_HBM_GBS)
    traffic = committed_traffic()
    if world == 1:
        achieved = bytes_ / (kernel_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "peak_source": peak_src,
                    "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
                    "algorithmic_bytes": bytes_, "kernel": "indexed_ffn_decode_kernel (+ decode_reduce_kernel)"}
    else:
        achieved = rank_bytes / (kernel_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "scope": "per rank: rank 0's shard bytes over the max-over-ranks step time",
                    "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "peak_source": peak_src, "traffic": None, "algorithmic_bytes": int(rank_bytes),
                    "local_records_per_step": round(local_k, 1),
                    "kernel": "indexed_ffn_decode_kernel (+ decode_reduce_kernel with the cross-rank sum)"}
    clock_summary = clocks.summary()
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "us_per_layer": round(ms_per_step * 1e3, 3),
        "tokens_per_s": round(1e3 / ms_per_step, 1), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) x)",
        "config": workload_config(k, args.retention),
        "execution": (f"intermediate-dim shard x{world}, cross-rank sum fused into the reduce launch" if world > 1
                      else "single GPU") + "; steps back to back in one CUDA graph; ids are inputs resident before "
                                           "the steps (QCC_IDS_READY), see ids_after_wait for the same steps without",
        "gpu_launches": launches_per_step * args.steps,
        "e2e": {"value": round(bytes_ / e2e_step_s / 1e9, 3), "unit": "GB/s",
                "us_per_layer": round(e2e_step_s * 1e6, 2),
                "h2d_bytes_per_step": x_bytes + id_bytes,
                "d2h_bytes_per_step": y_host.numel() * 2},
        "roofline": roofline,
        "clocks": clock_summary,
        "ids_after_wait": {"us_per_layer": round(late_us, 3), "gbs": round(bytes_ / (late_us * 1e-6) / 1e9, 1),
                           "note": "same steps without QCC_IDS_READY: each step reads its ids only after the "
                                   "step before has finished (ids produced on the stream, e.g. by the selector)"},
    }
    if parity is not None:
        line["parity"] = parity
    if sweep is not None:
        line["sweep"] = sweep
    if selector is not None:
        line["selector_ffn"] = selector
    if offload is not None:
        line["offload"] = offload
    if dense_oracle is not None:
        line.update(dense_oracle)
    if prefill is not None:
        line["prefill"] = prefill
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
