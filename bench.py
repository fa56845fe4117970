#!/usr/bin/env python
"""Decode throughput of the optiz-qwen hybrid hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload hybrid|serving]

Workload "hybrid" (default): one decode token for B=64 sequences at context 4096
through the 24-layer Qwen3.5 hybrid stack's hot path (18 Gated-DeltaNet
recurrent steps + 6 x [append-quantize + split-KV INT4 paged attention], 3:1
interleave; Hq 8 / Hkv 2 / head_dim 256; GDN 16 heads x 128).  Each rank runs
its own batch (weak scaling, no data-path collective).  Workload "serving":
B=1024 ragged sequences, context U[256, 8192], sharded across ranks by byte
cost (strong scaling).

The timed region replays a CUDA graph of every launch of a step, with all
inputs resident in HBM (the working set, ~2 GB, is far larger than the 126 MB
L2, so no flush is needed).  ``e2e`` times the host-facing call
``HybridDecodeStack.step`` (pinned host inputs -> device, step, outputs -> host).
Under torchrun every rank times its region between barriers; rank 0 prints the
max over ranks.
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

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

FALLBACK_HBM_GBS = 6650.0
METRIC = "decode tokens/s (hybrid 24-layer hot path: GDN step + INT4 paged attention)"


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["hybrid", "serving", "longctx"], default="hybrid")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the timed CPU baseline sample")
    return ap.parse_args(argv)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
    return FALLBACK_HBM_GBS, "profiling-recipe fallback 6.65 TB/s (of fallback)"


def dram_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` at the bench workload, from the committed ncu summary."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(kernel, {}).get("dram_bytes_per_launch")


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu_index)], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------- distributed plumbing
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_pg(world, local):
    import datetime

    import torch
    import torch.distributed as dist

    if world > 1 and not dist.is_initialized():
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return dist if world > 1 else None


def max_over_ranks(value: float, dist, device):
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist, device):
    import torch

    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


# ---------------------------------------------------------------------------- workloads
def serving_lengths(batch=1024, lo=256, hi=8192, seed=3):
    import numpy as np

    return np.random.default_rng(seed).integers(lo, hi + 1, size=batch).tolist()


def build_stack(args, world, rank, device):
    from optiz_qwen_b200.hybrid import HybridDecodeStack, HybridShape
    from optiz_qwen_b200.serving import shard_by_cost

    if args.workload == "hybrid":
        shape = HybridShape(batch=64, context=4096)
        stack = HybridDecodeStack(shape, device=device, seed=1 + rank, page_seed=1)
        desc = {"workload": "hybrid decode step: B=64 per GPU at context 4096, 24 layers = 18 Gated-DeltaNet "
                            "(16 heads x 128, fp32 state) + 6 full attention (Hq 8 / Hkv 2 / head_dim 256, "
                            "INT4 paged KV, page 64, permuted pages), 3:1 interleave, hidden 2048",
                "batch_per_gpu": 64, "global_batch": 64 * world, "context": 4096, "layers": 24,
                "context_held": "each step appends the new token at slot 4096 and attends over 4097",
                "l2": "no flush: ~2 GB per-step working set > 126 MB L2", "parallelism": f"dp{world} (sequences)"}
        return stack, 64 * world, desc
    lengths = serving_lengths()
    shards = shard_by_cost(lengths, world)
    mine = [lengths[i] for i in shards[rank]]
    shape = HybridShape(batch=len(mine), context=mine)
    stack = HybridDecodeStack(shape, device=device, seed=3 + rank, page_seed=3)
    desc = {"workload": "batched serving: B=1024 ragged sequences, context U[256,8192] (seed 3), sharded by byte "
                        "cost across GPUs, 24-layer hybrid hot path", "global_batch": 1024,
            "batch_this_rank": len(mine), "layers": 24, "l2": "no flush: working set far above L2",
            "parallelism": f"sequence-sharded x{world}"}
    return stack, 1024, desc


def time_graph(graph, reps, device):
    import torch

    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        graph.replay()
    e.record()
    torch.cuda.synchronize(device)
    return s.elapsed_time(e) / reps


def run_b200(args):
    import torch

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_pg(world, local)
    hbm_peak, peak_src = peaks()

    stack, global_batch, desc = build_stack(args, world, rank, device)
    stack.fill_inputs()
    counts = stack.counts()
    graph = stack.capture()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier(dist, device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index if world == 1 else local) as clocks:
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize(device)
    barrier(dist, device)
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, dist, device)
    value = global_batch * 1000.0 / ms

    # per-kernel device time: graphs holding only one kernel kind, same shapes and state
    kernels = {}
    reps = max(20, min(200, args.steps // 5))
    for kind, name, launches in (("gdn", "gdn_recurrent", len(stack.gdn)),
                                 ("attn", "decode_attn_int4_paged", len(stack.attn)),
                                 ("append", "append_quant_int4", len(stack.attn))):
        g = stack.capture((kind,))
        for _ in range(3):
            g.replay()
        per_step = time_graph(g, reps, device)
        us = per_step * 1000.0 / launches
        nbytes = counts.per_kernel[name]
        kernels[name] = {"us_per_launch": round(us, 2), "launches_per_step": launches,
                         "bytes_per_launch": nbytes, "GB_s": round(nbytes / us / 1e3, 1),
                         "frac_of_hbm": round(nbytes / us / 1e3 / hbm_peak, 4),
                         "share_of_step": round(per_step / ms_local, 3)}
        del g
    dominant = max((k for k in kernels if k != "append_quant_int4"),
                   key=lambda k: kernels[k]["us_per_launch"] * kernels[k]["launches_per_step"])
    dk = kernels[dominant]

    # end to end through the host-facing call: pinned inputs -> device -> step -> host
    stack.graph = graph
    for _ in range(3):
        stack.step()
    torch.cuda.synchronize(device)
    barrier(dist, device)
    e_steps = max(10, args.steps // 4)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(e_steps):
        stack.step()
        torch.cuda.current_stream(device).synchronize()   # the caller reads the step's outputs
    e2.record()
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / e_steps, dist, device)

    step_bytes = counts.attn_bytes + counts.gdn_bytes + counts.append_bytes
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak" if args.workload == "hybrid" else "strong", "vs_baseline": None,
        "dtype": "int4 KV codes x bf16/fp16 tensor-core dots, fp32 softmax/accumulate; fp32 GDN state",
        "data": "synthetic, seeded (config-0 distributions)", "config": desc,
        "clocks": clocks.summary(),
        "e2e": {"value": round(global_batch * 1000.0 / e2e_ms, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": counts.h2d_bytes, "d2h_bytes_per_step": counts.d2h_bytes,
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": counts.launches * args.steps,
        "roofline": {"bound": "hbm", "kernel": dominant, "achieved": dk["GB_s"], "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(dk["GB_s"] / hbm_peak, 4), "traffic": dram_traffic(dominant),
                     "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": dk["bytes_per_launch"]},
        "kernels": kernels,
        "step_hbm": {"bytes_per_step_per_gpu": step_bytes, "GB_s": round(step_bytes / ms_local / 1e6, 1),
                     "frac": round(step_bytes / ms_local / 1e6 / hbm_peak, 4)},
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(stack.shape, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph, stack
    if dist is not None:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- CPU legs (oracle port)
class OracleStep:
    """The oracle (numpy restatement of the reference's CPU torch path) over a sample of sequences:
    per attention layer the reference quantiser on the new token, dequantisation of the whole
    INT4 cache and fp32 attention; per GDN layer the recurrent gated delta rule."""

    def __init__(self, shape, seqs: int, layer_fraction: float = 1.0, seed: int = 0):
        import numpy as np

        rng = np.random.default_rng(seed)
        self.shape = shape
        self.seqs = seqs
        ctx = max(shape.lengths)
        hkv, d, h, dk = shape.num_kv_heads, shape.head_dim, shape.gdn_heads, shape.gdn_dim
        self.n_attn = max(1, round(shape.layer_types.count("full_attention") * layer_fraction))
        self.n_gdn = max(1, round(shape.layer_types.count("linear_attention") * layer_fraction))
        self.scale_layers = (shape.layer_types.count("full_attention") + shape.layer_types.count(
            "linear_attention")) / (self.n_attn + self.n_gdn)
        self.codes = rng.integers(0, 256, (hkv, 2, ctx + 1, d // 2), dtype=np.uint8)
        self.meta = (rng.random((hkv, 4, ctx + 1)) * 0.4).astype(np.float16)
        self.q = rng.standard_normal((1, shape.num_heads, d)).astype(np.float32)
        self.knew = rng.standard_normal((1, hkv, 1, d)).astype(np.float32)
        self.state = (0.02 * rng.standard_normal((1, h, dk, dk))).astype(np.float32)
        self.gq = rng.standard_normal((1, 1, h, dk)).astype(np.float32)
        self.gg = -np.logaddexp(0, rng.standard_normal((1, 1, h))).astype(np.float32)
        self.gb = (1 / (1 + np.exp(-rng.standard_normal((1, 1, h))))).astype(np.float32)

    def one_sequence(self) -> None:
        from oracle import attention as oattn
        from oracle import gdn as ogdn
        from oracle import kv_quant as kq

        for _ in range(self.n_attn):
            kq.quantize_tokens_int4(self.knew)
            k = kq.dequantize_tokens_int4(self.codes[:, 0], self.meta[:, 0], self.meta[:, 1])
            v = kq.dequantize_tokens_int4(self.codes[:, 1], self.meta[:, 2], self.meta[:, 3])
            oattn.decode_attention(self.q, [k], [v], self.shape.head_dim ** -0.5)
        for _ in range(self.n_gdn):
            ogdn.recurrent_gated_delta_rule(self.gq, self.gq, self.gq, self.gg, self.gb, self.state, True, True)

    def run(self, pool) -> float:
        """Process `seqs` sequences on the thread pool; return seconds per full 24-layer token."""
        t0 = time.perf_counter()
        list(pool.map(lambda _: self.one_sequence(), range(self.seqs)))
        return (time.perf_counter() - t0) * self.scale_layers / self.seqs


def cpu_baseline(shape, budget_s: float):
    import concurrent.futures as cf

    cores = os.cpu_count() or 1
    step = OracleStep(shape, seqs=cores)
    with cf.ThreadPoolExecutor(cores) as pool:
        step.run(pool)                                     # warm-up
        t0, times = time.perf_counter(), []
        while time.perf_counter() - t0 < budget_s or not times:
            times.append(step.run(pool))
    sec_per_token = statistics.median(times)
    return {"value": round(1.0 / sec_per_token, 2), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{cores} sequences per pass on {cores} threads, full 24-layer stack at context "
                      f"{max(shape.lengths)}, {len(times)} passes in {time.perf_counter() - t0:.1f} s; "
                      "numpy oracle of the reference's CPU torch path"}


def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    import concurrent.futures as cf

    from optiz_qwen_b200.hybrid import HybridShape

    if args.workload == "hybrid":
        shape = HybridShape(batch=64, context=4096)
        desc = {"workload": "hybrid decode step: B=64 per GPU at context 4096, 24 layers (18 GDN + 6 full "
                            "attention), sampled on the host CPU", "global_batch": 64 * world}
    else:
        shape = HybridShape(batch=1024, context=serving_lengths())
        desc = {"workload": "batched serving: B=1024 ragged, context U[256,8192], sampled on the host CPU",
                "global_batch": 1024}
    cores = os.cpu_count() or 1
    # size the per-step sample so warmup + steps stay within ~3 minutes
    probe = OracleStep(shape, seqs=1)
    with cf.ThreadPoolExecutor(cores) as pool:
        t_seq = probe.run(pool)
        budget_per_step = 150.0 / max(1, args.steps + args.warmup)
        frac = min(1.0, budget_per_step / max(t_seq, 1e-9))
        seqs = max(1, min(cores, int(budget_per_step / max(t_seq, 1e-9))))
        step = OracleStep(shape, seqs=seqs, layer_fraction=frac if seqs == 1 else 1.0)
        for _ in range(args.warmup):
            step.run(pool)
        times = [step.run(pool) for _ in range(args.steps)]
    sec_per_token = statistics.mean(times)
    value = 1.0 / sec_per_token
    sample = (f"per step {step.seqs} sequence(s) x {step.n_attn} attention + {step.n_gdn} GDN layers on "
              f"{cores} threads, scaled to the 24-layer stack; numpy oracle of the reference's CPU torch path")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec_per_token * 1000 * step.seqs, 3),
            "higher_is_better": True, "scaling": "weak" if args.workload == "hybrid" else "strong",
            "vs_baseline": None, "dtype": "fp32 (numpy)", "data": "synthetic, seeded", "config": desc,
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_longctx(args):
    """Config 2: one sequence at context 131072, 6 attention layers, KV range split across the ranks;
    per layer: append on the tail rank, partial attention, NCCL all-gather of (out, lse), LSE merge."""
    import torch

    from optiz_qwen_b200.context_parallel import ContextParallelDecoder

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_pg(world, local)
    hbm_peak, peak_src = peaks()
    length, layers = 131072, 6
    gen = torch.Generator(device=device)
    gen.manual_seed(2 * 1000 + rank)
    decs = []
    for _ in range(layers):
        d = ContextParallelDecoder(2, 256, rank=rank, world=world, device=device)
        d.prefill_random(length, generator=gen, capacity_tokens=0, page_seed=2)
        decs.append(d)
    q = torch.randn((1, 8, 256), generator=gen, device=device).to(torch.bfloat16)

    def step():
        for d in decs:
            d.decode(q)

    # one step, NCCL all-gathers included, captured in a CUDA graph after an eager warm-up
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream(device).wait_stream(side)
    barrier(dist, device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier(dist, device)
    steps = max(10, min(args.steps, 500))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize(device)
    barrier(dist, device)
    ms = max_over_ranks(start.elapsed_time(end) / steps, dist, device)
    kv_bytes = length * 2 * 264 * layers
    line = {"metric": METRIC, "value": round(1000.0 / ms, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int4 KV codes x int8/fp16 tensor-core dots, fp32 softmax/merge",
            "data": "synthetic, seeded",
            "config": {"workload": "long context: B=1, context 131072, 6 full-attention layers (Hq 8 / Hkv 2 / D 256), "
                                   "KV range split evenly across GPUs, NCCL all-gather of fp32 (out, lse) partials "
                                   "+ LSE merge per layer, step captured in a CUDA graph", "global_batch": 1},
            "step_hbm": {"kv_bytes_per_step_total": kv_bytes,
                         "GB_s_per_gpu": round(kv_bytes / world / ms / 1e6, 1),
                         "frac_per_gpu": round(kv_bytes / world / ms / 1e6 / hbm_peak, 4), "peak_source": peak_src}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph                                  # release the graph holding NCCL calls first
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.destroy_process_group()


def main(argv=None):
    args = parse_args(argv)
    if args.workload == "longctx" and args.impl != "reference":
        run_longctx(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
