#!/usr/bin/env python
"""Decode throughput of the optiz-qwen hybrid hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload hybrid|serving|longctx|prefill]

Workload "hybrid" (default): one decode token for B=64 sequences at context 4096
through the 24-layer Qwen3.5 hybrid stack's hot path (18 Gated-DeltaNet
recurrent steps + 6 x [append-quantize + split-KV INT4 paged attention], 3:1
interleave; Hq 8 / Hkv 2 / head_dim 256; GDN 16 heads x 128).  Each rank runs
its own batch (weak scaling, no data-path collective).  Workload "serving":
B=1024 ragged sequences, context U[256, 8192], sharded across ranks by byte
cost (strong scaling).  Workload "longctx": one sequence at context 131072 with
the KV range split across ranks.  Workload "prefill": the chunked GDN prefill on
the tensor cores (B=8, T=8192, 16 heads of 128, 18 layers) followed by 256
recurrent decode steps from the resulting states.

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


EPILOGUES = "attention * sigmoid(gate) and GDN gated RMSNorm, fused into the kernels' stores"
GATES_DESC = {"given": "g and beta given (the hook's arguments)",
              "fused": "g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) computed in the GDN kernel"}


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["hybrid", "serving", "longctx", "prefill"], default="hybrid")
    ap.add_argument("--exchange", choices=["nvlink", "nccl"], default="nvlink",
                    help="long-context exchange of the partials across GPUs: the NVLink exchange kernel "
                         "(peer stores, one launch per layer) or NCCL all-gather + merge")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kv-bits", type=int, choices=[4, 8], default=4,
                    help="hybrid/serving: width of the paged KV cache codes (8: the reference's k_bits=8 preset)")
    ap.add_argument("--append", choices=["fused", "separate"], default="fused",
                    help="the new token's append-quantize: inside the attention launch, or its own launch")
    ap.add_argument("--serving-order", choices=["longest-first", "index"], default="longest-first",
                    help="order of a serving shard's sequences in the batch (the attention launch's CTA order)")
    ap.add_argument("--no-early-gdn", action="store_true",
                    help="start a GDN step right after an attention launch only once that launch has finished")
    ap.add_argument("--no-early-attn", action="store_true",
                    help="launch attention only after the GDN layer ahead of it has finished")
    ap.add_argument("--conv", choices=["separate", "fused"], default=None,
                    help="hybrid/serving: feed each GDN layer its raw projection output and run its causal conv1d "
                         "update (separate kernel, or fused into the GDN step)")
    ap.add_argument("--epilogues", action="store_true",
                    help="hybrid/serving: include the layers' output epilogues (attention * sigmoid(gate), GDN "
                         "gated RMSNorm), fused into the kernels' stores; the CPU legs run them too")
    ap.add_argument("--small", action="store_true",
                    help="reduced case for ncu captures: prefill B=4, T=8192, 2 layers, 8 decode steps; hybrid B=8")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the timed CPU baseline sample")
    ap.add_argument("--gates", choices=["given", "fused"], default="given",
                    help="hybrid/serving: GDN steps take g and beta (the hook's arguments), or the raw gate "
                         "projections with the gate arithmetic in the kernel")
    ap.add_argument("--no-sub-records", action="store_true",
                    help="hybrid workload: skip the serving and long-context sub-records")
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
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while the GPU is under the bench's load
    (the timed loop, the per-kernel timings and the end-to-end loop, back to back)."""

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
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
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


APPEND_DESC = {"fused": "the new token quantised into the cache by the attention launch itself",
               "separate": "the new token quantised into the cache by its own append launch"}


def build_stack(args, world, rank, device):
    from optiz_qwen_b200.hybrid import HybridDecodeStack, HybridShape
    from optiz_qwen_b200.serving import shard_by_cost

    if args.workload == "hybrid":
        bsz = 8 if args.small else 64   # (--small: the profiling case, B = 8)
        shape = HybridShape(batch=bsz, context=4096)
        stack = HybridDecodeStack(shape, device=device, seed=1 + rank, page_seed=1, conv=args.conv,
                                  epilogues=args.epilogues, kv_bits=args.kv_bits, gates=args.gates,
                                  fused_append=args.append == "fused", early_attention=not args.no_early_attn)
        desc = {"gdn_conv": f"causal conv1d update ({args.conv})" if args.conv else "q/k/v given post-conv",
                "gdn_gates": GATES_DESC[args.gates], "append": APPEND_DESC[args.append],
                "epilogues": EPILOGUES if args.epilogues else "none",
                "workload": f"hybrid decode step: B={bsz} per GPU at context 4096, 24 layers = 18 Gated-DeltaNet "
                            "(16 heads x 128, fp32 state) + 6 full attention (Hq 8 / Hkv 2 / head_dim 256, "
                            f"INT{args.kv_bits} paged KV, page 64, permuted pages), 3:1 interleave, hidden 2048",
                "batch_per_gpu": bsz, "global_batch": bsz * world, "context": 4096, "layers": 24,
                "context_held": "each step appends the new token at slot 4096 and attends over 4097",
                "l2": "no flush: ~2 GB per-step working set > 126 MB L2", "parallelism": f"dp{world} (sequences)"}
        return stack, bsz * world, desc
    lengths = serving_lengths()
    shards = shard_by_cost(lengths, world)
    from optiz_qwen_b200.serving import longest_first

    order = longest_first(lengths, shards[rank]) if args.serving_order == "longest-first" else shards[rank]
    mine = [lengths[i] for i in order]
    shape = HybridShape(batch=len(mine), context=mine)
    stack = HybridDecodeStack(shape, device=device, seed=3 + rank, page_seed=3, conv=args.conv,
                              epilogues=args.epilogues, kv_bits=args.kv_bits, gates=args.gates,
                              fused_append=args.append == "fused", early_attention=not args.no_early_attn)
    desc = {"gdn_conv": f"causal conv1d update ({args.conv})" if args.conv else "q/k/v given post-conv",
            "gdn_gates": GATES_DESC[args.gates], "append": APPEND_DESC[args.append],
            "epilogues": EPILOGUES if args.epilogues else "none",
            "workload": "batched serving: B=1024 ragged sequences, context U[256,8192] (seed 3), sharded by byte "
                        f"cost across GPUs, 24-layer hybrid hot path, INT{args.kv_bits} paged KV", "global_batch": 1024,
            "batch_this_rank": len(mine), "layers": 24, "l2": "no flush: working set far above L2",
            "batch_order": "longest context first" if args.serving_order == "longest-first" else "by index",
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


def ranks_gather(value: float, dist, device) -> list[float]:
    """Every rank's value, in rank order (one all-gather; a one-element list on one process)."""
    if dist is None:
        return [value]
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    out = torch.empty(dist.get_world_size(), dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(out, t)
    return out.tolist()


def time_host_step(stack, steps, device, dist):
    """ms per call of the host-facing step (pinned inputs -> device, kernels, outputs -> host, the
    caller waiting for the outputs every step), max over ranks."""
    import torch

    for _ in range(3):
        stack.step()
    torch.cuda.synchronize(device)
    barrier(dist, device)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(steps):
        stack.step()
        torch.cuda.current_stream(device).synchronize()   # the caller reads the step's outputs
    e2.record()
    torch.cuda.synchronize(device)
    return max_over_ranks(s2.elapsed_time(e2) / steps, dist, device)


def time_copies_only(stack, steps, device, dist):
    """The host-facing step's transfers alone (same copies, streams and grouping, no kernels):
    ms per step, max over ranks.  The floor e2e cannot go below on this host."""
    import torch

    graph = stack.capture_io(kinds=())
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(device)
    barrier(dist, device)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(steps):
        graph.replay()
        torch.cuda.current_stream(device).synchronize()
    e2.record()
    torch.cuda.synchronize(device)
    del graph
    return max_over_ranks(s2.elapsed_time(e2) / steps, dist, device)


def measure_serving(args, world, rank, device, dist, hbm_peak):
    """Batched serving (B = 1024 ragged contexts, U[256, 8192], seed 3) sharded by byte cost over the
    ranks (strong scaling): device-timed step, per-rank spread, e2e through the host-facing step."""
    import torch

    sub = argparse.Namespace(**{**vars(args), "workload": "serving"})
    stack, global_batch, desc = build_stack(sub, world, rank, device)
    stack.fill_inputs()
    counts = stack.counts()
    graph = stack.capture()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier(dist, device)
    steps = max(10, min(args.steps, 100))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        graph.replay()
    e.record()
    torch.cuda.synchronize(device)
    barrier(dist, device)
    ms_local = s.elapsed_time(e) / steps
    per_rank = ranks_gather(ms_local, dist, device)
    ms = max(per_rank)
    stack.graph = graph
    e2e_ms = time_host_step(stack, max(10, steps // 4), device, dist)
    step_bytes = counts.attn_bytes + counts.gdn_bytes + counts.append_bytes
    out = {"workload": desc["workload"], "global_batch": global_batch, "batch_this_rank": stack.shape.batch,
           "scaling": "strong", "steps": steps, "ms_per_step": round(ms, 4),
           "tokens_per_s": round(global_batch * 1000.0 / ms, 1),
           "rank_ms": {"min": round(min(per_rank), 4), "max": round(max(per_rank), 4)},
           "hbm_frac_rank0": round(step_bytes / ms_local / 1e6 / hbm_peak, 4),
           "e2e": {"tokens_per_s": round(global_batch * 1000.0 / e2e_ms, 1), "ms_per_step": round(e2e_ms, 4),
                   "h2d_bytes_per_step_per_rank": counts.h2d_bytes,
                   "d2h_bytes_per_step_per_rank": counts.d2h_bytes}}
    del graph, stack
    torch.cuda.empty_cache()
    return out


def measure_longctx(args, world, rank, device, dist, hbm_peak):
    """Long context (B = 1, context 131072, 6 attention layers, seed 2): the KV range split across the
    ranks, per layer the partial attention and the exchange + LSE merge, the step in a CUDA graph."""
    import torch

    from optiz_qwen_b200.context_parallel import ContextParallelDecoder, PeerExchange

    length, layers = 131072, 6
    gen = torch.Generator(device=device)
    gen.manual_seed(2 * 1000 + rank)
    # NVLink exchange kernel (one call site per layer) or the NCCL all-gather + merge
    exchange = (PeerExchange(8, 256, rank=rank, world=world, device=device, sites=layers)
                if world > 1 and args.exchange == "nvlink" else None)
    decs = []
    for layer in range(layers):
        d = ContextParallelDecoder(2, 256, rank=rank, world=world, device=device, exchange=exchange, site=layer)
        # (d.early stays off: an early launch behind the previous layer's merge measured slower here,
        # 0.176 against 0.162 ms per step)
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
    del graph                                  # (a graph holding NCCL calls goes before the group does)
    torch.cuda.synchronize(device)
    if exchange is not None:
        exchange.close()
    how = ("NVLink exchange kernel: peer stores + flag + LSE merge in one launch" if exchange is not None
           else "NCCL all-gather of the partials + LSE merge kernel")
    return {"workload": "long context: B=1, context 131072, 6 full-attention layers (Hq 8 / Hkv 2 / D 256), "
                        "KV range split evenly across GPUs, per layer partial attention + exchange of fp32 "
                        f"(out, lse) ({how}) (one GPU: the attention kernel writes the output), step in a "
                        "CUDA graph",
            "exchange": "none (one GPU)" if world == 1 else args.exchange,
            "scaling": "strong", "steps": steps, "ms_per_step": round(ms, 4), "tokens_per_s": round(1000.0 / ms, 1),
            "kv_bytes_per_step_total": kv_bytes, "GB_s_per_gpu": round(kv_bytes / world / ms / 1e6, 1),
            "hbm_frac_per_gpu": round(kv_bytes / world / ms / 1e6 / hbm_peak, 4)}


def run_b200(args):
    import torch

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_pg(world, local)
    hbm_peak, peak_src = peaks()

    stack, global_batch, desc = build_stack(args, world, rank, device)
    stack.early_gdn_after_attn = stack.early_gdn_after_attn and not args.no_early_gdn
    stack.fill_inputs()
    counts = stack.counts()
    graph = stack.capture()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier(dist, device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # clocks are sampled from here through the last loaded phase (the timed loop alone is too short
    # for nvidia-smi's sampling at small step counts)
    clocks = ClockSampler(device.index if world == 1 else local).__enter__()
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
    kinds = [("gdn", "gdn_recurrent", len(stack.gdn)),
             ("attn", f"decode_attn_int{stack.kv_bits}_paged", len(stack.attn))]
    if not stack.fused_append:
        kinds.append(("append", f"append_quant_int{stack.kv_bits}", len(stack.attn)))
    for kind, name, launches in kinds:
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
    dominant = max((k for k in kernels if not k.startswith("append_quant")),
                   key=lambda k: kernels[k]["us_per_launch"] * kernels[k]["launches_per_step"])
    dk = kernels[dominant]

    # end to end through the host-facing call: pinned inputs -> device -> step -> host
    stack.graph = graph
    e_steps = max(10, args.steps // 4)
    e2e_ms = time_host_step(stack, e_steps, device, dist)
    copy_ms = time_copies_only(stack, e_steps, device, dist)
    del graph, stack
    torch.cuda.empty_cache()

    extra = {}
    if args.workload == "hybrid" and not args.no_sub_records:
        extra["serving"] = measure_serving(args, world, rank, device, dist, hbm_peak)
        extra["longctx"] = measure_longctx(args, world, rank, device, dist, hbm_peak)
        pre = measure_prefill(args, world, rank, device, dist, hbm_peak, peak_src, 3)
        rf = pre["roofline"]
        extra["prefill"] = {"workload": pre["config"]["workload"], "scaling": "weak", "steps": pre["steps"],
                            "ms_per_step": pre["ms_per_step"], "tokens_per_s": pre["value"],
                            "us_per_layer": rf["us_per_launch"], "GB_s": rf["achieved"], "hbm_frac": rf["frac"],
                            "tensor": rf["tensor"], "decode_tail": pre["decode_tail"], "e2e": pre["e2e"]}
    clocks.__exit__(None, None, None)

    step_bytes = counts.attn_bytes + counts.gdn_bytes + counts.append_bytes
    line = {
        "metric": METRIC if args.kv_bits == 4 else METRIC.replace("INT4", "INT8"), "value": round(value, 1),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak" if args.workload == "hybrid" else "strong", "vs_baseline": None,
        "dtype": (f"int{args.kv_bits} KV codes: q.k as u8 x s8 integer MMA (q in 21-bit fixed point per head, "
                  "three 8-bit digits), p.v as fp16 MMA (P' as fp16 + fp16 remainder, codes as exact fp16 "
                  "subnormals), fp32 softmax / accumulate; GDN fp32 state, bf16 q/k/v"),
        "data": "synthetic, seeded (config-0 distributions)", "config": desc,
        "clocks": clocks.summary(),
        "e2e": {"value": round(global_batch * 1000.0 / e2e_ms, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": counts.h2d_bytes * world, "d2h_bytes_per_step": counts.d2h_bytes * world,
                "ms_per_step": round(e2e_ms, 4),
                # the same transfers with no kernels: what the host's copy bandwidth allows
                "copies_only_ms_per_step": round(copy_ms, 4),
                "host_GB_s_copies_only": round((counts.h2d_bytes + counts.d2h_bytes) * world / copy_ms / 1e6, 1)},
        "gpu_launches": counts.launches * args.steps,
        "roofline": {"bound": "hbm", "kernel": dominant, "achieved": dk["GB_s"], "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(dk["GB_s"] / hbm_peak, 4),
                     # the committed capture is of the default workload's launch; other shapes have none
                     "traffic": dram_traffic(dominant) if args.workload == "hybrid" else None,
                     "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": dk["bytes_per_launch"]},
        "kernels": kernels,
        "step_hbm": {"bytes_per_step_per_gpu": step_bytes, "GB_s": round(step_bytes / ms_local / 1e6, 1),
                     "frac": round(step_bytes / ms_local / 1e6 / hbm_peak, 4)},
        **extra,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        from optiz_qwen_b200.hybrid import HybridShape

        shape = HybridShape(batch=64, context=4096) if args.workload == "hybrid" else HybridShape(
            batch=1024, context=serving_lengths())
        line["cpu_baseline"] = cpu_baseline(shape, args.cpu_seconds, args.epilogues, bits=args.kv_bits)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- CPU legs (oracle port)
class OracleStep:
    """The oracle (numpy restatement of the reference's CPU torch path) over a sample of sequences:
    per attention layer the reference quantiser on the new token, dequantisation of the whole
    INT4 cache and fp32 attention; per GDN layer the decode branch's gate arithmetic and the
    recurrent gated delta rule."""

    def __init__(self, shape, seqs: int, layer_fraction: float = 1.0, seed: int = 0, epilogues: bool = False,
                 bits: int = 4):
        import numpy as np

        rng = np.random.default_rng(seed)
        self.shape = shape
        self.epilogues = epilogues
        self.seqs = seqs
        ctx = max(shape.lengths)
        hkv, d, h, dk = shape.num_kv_heads, shape.head_dim, shape.gdn_heads, shape.gdn_dim
        self.n_attn = max(1, round(shape.layer_types.count("full_attention") * layer_fraction))
        self.n_gdn = max(1, round(shape.layer_types.count("linear_attention") * layer_fraction))
        self.scale_layers = (shape.layer_types.count("full_attention") + shape.layer_types.count(
            "linear_attention")) / (self.n_attn + self.n_gdn)
        self.bits = bits
        self.codes = rng.integers(0, 256, (hkv, 2, ctx + 1, d * bits // 8), dtype=np.uint8)
        self.meta = (rng.random((hkv, 4, ctx + 1)) * 0.4).astype(np.float16)
        self.q = rng.standard_normal((1, shape.num_heads, d)).astype(np.float32)
        self.knew = rng.standard_normal((1, hkv, 1, d)).astype(np.float32)
        self.state = (0.02 * rng.standard_normal((1, h, dk, dk))).astype(np.float32)
        self.gq = rng.standard_normal((1, 1, h, dk)).astype(np.float32)
        # raw gate projections; A_log = dt_bias = 0 as in the GPU stack (g = -softplus(a))
        self.ga = rng.standard_normal((1, 1, h)).astype(np.float32)
        self.gbr = rng.standard_normal((1, 1, h)).astype(np.float32)
        self.gparam = np.zeros(h, np.float32)
        self.gate = rng.standard_normal((1, shape.num_heads, d)).astype(np.float32)
        self.z = rng.standard_normal((1, 1, h, dk)).astype(np.float32)
        self.norm_w = (1.0 + 0.1 * rng.standard_normal(dk)).astype(np.float32)

    def one_sequence(self) -> None:
        from oracle import attention as oattn
        from oracle import epilogue as ep
        from oracle import gdn as ogdn
        from oracle import kv_quant as kq

        for _ in range(self.n_attn):
            quant, deq = ((kq.quantize_tokens_int4, kq.dequantize_tokens_int4) if self.bits == 4
                          else (kq.quantize_tokens_int8, kq.dequantize_tokens_int8))
            quant(self.knew)
            k = deq(self.codes[:, 0], self.meta[:, 0], self.meta[:, 1])
            v = deq(self.codes[:, 1], self.meta[:, 2], self.meta[:, 3])
            o, _ = oattn.decode_attention(self.q, [k], [v], self.shape.head_dim ** -0.5)
            if self.epilogues:
                ep.sigmoid_gate(o, self.gate, rnd=kq.round_bf16)
        for _ in range(self.n_gdn):
            g, beta = ogdn.decay_gates(self.ga, self.gbr, self.gparam, self.gparam, rnd=kq.round_bf16)
            o, _ = ogdn.recurrent_gated_delta_rule(self.gq, self.gq, self.gq, g, beta, self.state, True, True)
            if self.epilogues:
                ep.rmsnorm_gated(kq.round_bf16(o), self.z, self.norm_w, 1e-6, rnd=kq.round_bf16)

    def run(self, pool) -> float:
        """Process `seqs` sequences on the thread pool; return seconds per full 24-layer token."""
        t0 = time.perf_counter()
        list(pool.map(lambda _: self.one_sequence(), range(self.seqs)))
        return (time.perf_counter() - t0) * self.scale_layers / self.seqs


def cpu_baseline(shape, budget_s: float, epilogues: bool = False, bits: int = 4):
    import concurrent.futures as cf

    cores = os.cpu_count() or 1
    step = OracleStep(shape, seqs=cores, epilogues=epilogues, bits=bits)
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
                            "attention), sampled on the host CPU", "global_batch": 64 * world,
                "epilogues": EPILOGUES if args.epilogues else "none"}
    else:
        shape = HybridShape(batch=1024, context=serving_lengths())
        desc = {"workload": "batched serving: B=1024 ragged, context U[256,8192], sampled on the host CPU",
                "global_batch": 1024}
    cores = os.cpu_count() or 1
    # size the per-step sample so warmup + steps stay within ~3 minutes
    probe = OracleStep(shape, seqs=1, epilogues=args.epilogues)
    with cf.ThreadPoolExecutor(cores) as pool:
        t_seq = probe.run(pool)
        budget_per_step = 150.0 / max(1, args.steps + args.warmup)
        frac = min(1.0, budget_per_step / max(t_seq, 1e-9))
        seqs = max(1, min(cores, int(budget_per_step / max(t_seq, 1e-9))))
        step = OracleStep(shape, seqs=seqs, layer_fraction=frac if seqs == 1 else 1.0, epilogues=args.epilogues,
                          bits=args.kv_bits)
        for _ in range(args.warmup):
            step.run(pool)
        times = [step.run(pool) for _ in range(args.steps)]
    sec_per_token = statistics.mean(times)
    value = 1.0 / sec_per_token
    sample = (f"per step {step.seqs} sequence(s) x {step.n_attn} attention + {step.n_gdn} GDN layers on "
              f"{cores} threads, scaled to the 24-layer stack; numpy oracle of the reference's CPU torch path")
    line = {"impl": "reference", "metric": METRIC if args.kv_bits == 4 else METRIC.replace("INT4", "INT8"),
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec_per_token * 1000 * step.seqs, 3),
            "higher_is_better": True, "scaling": "weak" if args.workload == "hybrid" else "strong",
            "vs_baseline": None, "dtype": "fp32 (numpy)", "data": "synthetic, seeded", "config": desc,
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            # one host process on rank 0 whatever the GPU count: the same CPU figure at every N
            "ranks": f"rank 0 alone, one process on {cores} host threads, for all {world} GPU rank(s)"}
    print(json.dumps(line), flush=True)


def run_longctx(args):
    """Config 2 on its own (``--workload longctx``): one sequence at context 131072, 6 attention
    layers, KV range split across the ranks."""
    import torch

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_pg(world, local)
    hbm_peak, peak_src = peaks()
    rec = measure_longctx(args, world, rank, device, dist, hbm_peak)
    line = {"metric": METRIC, "value": rec["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
            "steps": rec["steps"], "warmup": args.warmup, "ms_per_step": rec["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 KV codes: q.k as u8 x s8 integer MMA, p.v as fp16 MMA; fp32 softmax / merge",
            "data": "synthetic, seeded", "config": {"workload": rec["workload"], "global_batch": 1},
            "step_hbm": {"kv_bytes_per_step_total": rec["kv_bytes_per_step_total"],
                         "GB_s_per_gpu": rec["GB_s_per_gpu"], "frac_per_gpu": rec["hbm_frac_per_gpu"],
                         "peak_source": peak_src}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


PREFILL_METRIC = "GDN chunked prefill tokens/s (tensor-core WY form, 18 layers) + recurrent decode tail"


def _prefill_inputs(b, t, h, d, gen, device):
    import torch

    q, k, v = (torch.randn((b, t, h, d), generator=gen, device=device).to(torch.bfloat16) for _ in range(3))
    beta = torch.sigmoid(torch.randn((b, t, h), generator=gen, device=device))
    g = -torch.nn.functional.softplus(torch.randn((b, t, h), generator=gen, device=device))
    return q, k, v, g, beta


def prefill_cpu_baseline(budget_s: float, t: int = 512):
    """The oracle's chunked form (numpy restatement of torch_chunk_gated_delta_rule) on one head; its
    matrix products run on numpy's BLAS threads (all host cores)."""
    import numpy as np

    from oracle import gdn as ogdn

    try:
        from threadpoolctl import threadpool_info

        cores = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except ImportError:
        cores = os.cpu_count() or 1
    rng = np.random.default_rng(4)
    q, k, v = (rng.standard_normal((1, t, 1, 128), dtype=np.float32) for _ in range(3))
    g = -np.logaddexp(0, rng.standard_normal((1, t, 1))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((1, t, 1))))).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((1, 1, 128, 128))).astype(np.float32)
    ogdn.chunk_gated_delta_rule(q, k, v, g, beta, 64, s0, True, True)
    t0, n = time.perf_counter(), 0
    while time.perf_counter() - t0 < budget_s or n == 0:
        ogdn.chunk_gated_delta_rule(q, k, v, g, beta, 64, s0, True, True)
        n += 1
    sec = (time.perf_counter() - t0) / n                 # seconds per head-layer of t tokens
    # whole workload: every token runs 16 heads x 18 layers
    return {"value": round(t / sec / (16 * 18), 2), "unit": "prefill tokens/s", "cores": cores, "kind": "port",
            "sample": f"one head, T={t}, {n} runs in {time.perf_counter() - t0:.1f} s (numpy BLAS on {cores} "
                      "threads), scaled to 16 heads x 18 layers per token; numpy chunked oracle of "
                      "torch_chunk_gated_delta_rule"}


def run_prefill(args):
    """Config 4 on its own (``--workload prefill``): see ``measure_prefill``."""
    import torch

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_pg(world, local)
    hbm_peak, peak_src = peaks()
    line = measure_prefill(args, world, rank, device, dist, hbm_peak, peak_src, max(3, min(args.steps, 40)))
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = prefill_cpu_baseline(min(args.cpu_seconds, 15.0))
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def measure_prefill(args, world, rank, device, dist, hbm_peak, peak_src, steps: int) -> dict:
    """Config 4: chunked GDN prefill (B=8, T=8192, H=16, d=128, 18 layers) on the tensor cores, then
    256 recurrent decode steps from the prefill's final states.  Weak scaling: every rank runs its own
    batch of 8 sequences, with no data-path collective.  Returns the bench line (no CPU baseline)."""
    import torch

    from optiz_qwen_b200 import cabi
    from optiz_qwen_b200.gdn.gated_delta_rule import chunk_gated_delta_rule

    tflops_peak = None
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        d = json.loads(pk.read_text())
        tflops_peak = float(d.get("bf16_tflops_sustained") or d.get("bf16_tflops") or 0) or None
    b, t, h, d, layers, tail = (4, 8192, 16, 128, 2, 8) if args.small else (8, 8192, 16, 128, 18, 256)
    gen = torch.Generator(device=device)
    gen.manual_seed(4 * 1000 + rank)
    ins = [_prefill_inputs(b, t, h, d, gen, device) for _ in range(layers)]
    s0 = [0.02 * torch.randn((b, h, d, d), generator=gen, device=device) for _ in range(layers)]
    states = [torch.empty_like(x) for x in s0]
    out = torch.empty((b, t, h, d), dtype=torch.bfloat16, device=device)
    dq = [_prefill_inputs(b, 1, h, d, gen, device) for _ in range(tail)]
    dout = torch.empty((b, 1, h, d), dtype=torch.bfloat16, device=device)

    # the two-phase form's per-chunk workspace, shared by the layers (they run in order)
    chunk_ws = torch.empty(cabi.gdn_chunk_workspace_bytes(b, t, h), dtype=torch.uint8, device=device)

    def prefill():
        for (q, k, v, g, beta), si, so in zip(ins, s0, states):
            cabi.gdn_chunk_fwd(q, k, v, g, beta, initial_state=si, final_state=so, out=out, use_qk_l2norm=True,
                               workspace=chunk_ws)

    def decode_tail():
        for step, (q, k, v, g, beta) in enumerate(dq):
            for li, st in enumerate(states):
                # every launch but the first follows another layer's GDN step (see HybridDecodeStack)
                cabi.gdn_recurrent(q, k, v, g, beta, initial_state=st, final_state=st, out=dout, use_qk_l2norm=True,
                                   prefetch_state=layers > 1 and (step > 0 or li > 0))

    prefill()
    decode_tail()
    torch.cuda.synchronize(device)
    graphs = {}
    for name, fn in (("prefill", prefill), ("decode", decode_tail)):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        graphs[name] = gr
    for _ in range(max(3, args.warmup)):
        graphs["prefill"].replay()
        graphs["decode"].replay()
    barrier(dist, device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with ClockSampler(device.index) as clocks:
        ev[0].record()
        for _ in range(steps):
            graphs["prefill"].replay()
        ev[1].record()
        for _ in range(steps):
            graphs["decode"].replay()
        ev[2].record()
        torch.cuda.synchronize(device)
    barrier(dist, device)
    pre_ms = max_over_ranks(ev[0].elapsed_time(ev[1]) / steps, dist, device)
    dec_ms = max_over_ranks(ev[1].elapsed_time(ev[2]) / steps, dist, device)
    layer_us = pre_ms * 1000.0 / layers
    bytes_layer = b * t * h * 1032                       # q, k, v, o bf16 + g, beta fp32 per token-head
    flops_layer = b * h * (t // 64) * (10 * 64 * 64 * d + 6 * 64 * d * d)
    gbs = bytes_layer / layer_us / 1e3
    tflops = flops_layer / layer_us / 1e6

    # end to end, one layer through the hook: pinned host inputs -> device -> prefill -> output + state to host
    q, k, v, g, beta = (x.cpu().pin_memory() for x in ins[0])
    s_host = s0[0].cpu().pin_memory()
    o_host = torch.empty((b, t, h, d), dtype=torch.bfloat16).pin_memory()
    st_host = torch.empty((b, h, d, d), dtype=torch.float32).pin_memory()
    def e2e_layer():
        dev = [x.to(device, non_blocking=True) for x in (q, k, v, g, beta, s_host)]
        o, st = chunk_gated_delta_rule(*dev[:3], g=dev[3], beta=dev[4], initial_state=dev[5], output_final_state=True,
                                       use_qk_l2norm_in_kernel=True)
        o_host.copy_(o, non_blocking=True)
        st_host.copy_(st, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
    e2e_layer()
    e_steps = 5
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(e_steps):
        e2e_layer()
    e2.record()
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / e_steps, dist, device)
    h2d = sum(x.numel() * x.element_size() for x in (q, k, v, g, beta, s_host))
    d2h = o_host.numel() * 2 + st_host.numel() * 4

    tokens = b * t * world
    line = {
        "metric": PREFILL_METRIC, "value": round(tokens * 1000.0 / pre_ms, 1), "unit": "prefill tokens/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(pre_ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 q/k/v; fp32 state and WY factors as split bf16 hi+lo tensor-core operands, fp32 accumulate",
        "data": "synthetic, seeded (config-0 distributions)",
        "config": {"workload": f"GDN chunked prefill: B={b} x T={t} per GPU, {h} heads, dk=dv={d}, chunk 64, "
                               f"{layers} layers; then {tail} recurrent decode steps x {layers} layers from the final "
                               "states" + (" (reduced profiling case)" if args.small else ""),
                   "global_batch": b * world, "seq_len": t, "l2": "inputs 805 MB per layer, far above L2"},
        "clocks": clocks.summary(),
        "decode_tail": {"ms_per_step": round(dec_ms / tail, 4), "tokens_per_s": round(b * world * tail * 1000.0 / dec_ms, 1),
                        "state_GB_s": round(layers * b * h * d * d * 8 / (dec_ms / tail) / 1e6, 1)},
        "e2e": {"value": round(b * t * world * 1000.0 / e2e_ms / layers, 1), "unit": "prefill tokens/s",
                "h2d_bytes_per_step": h2d * layers, "d2h_bytes_per_step": d2h * layers,
                "note": "one layer through chunk_gated_delta_rule with pinned host buffers, scaled to 18 layers"},
        "gpu_launches": 2 * layers * steps,  # per layer: the per-chunk factors, then the state walk
        "roofline": {"bound": "hbm", "kernel": "gdn_chunk", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(gbs / hbm_peak, 4), "traffic": dram_traffic("gdn_chunk"), "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": bytes_layer, "us_per_launch": round(layer_us, 1),
                     "tensor": {"achieved_tflops": round(tflops, 1), "peak_tflops": tflops_peak,
                                "frac": round(tflops / tflops_peak, 4) if tflops_peak else None,
                                "algorithmic_flops_per_launch": flops_layer}},
    }
    del graphs
    torch.cuda.synchronize(device)
    return line


def main(argv=None):
    args = parse_args(argv)
    if args.workload == "longctx" and args.impl != "reference":
        run_longctx(args)
        return
    if args.workload == "prefill":
        if args.impl != "reference":
            run_prefill(args)
        elif int(os.environ.get("RANK", "0")) == 0:
            base = prefill_cpu_baseline(min(args.cpu_seconds, 60.0))
            print(json.dumps({"impl": "reference", "metric": PREFILL_METRIC, "value": base["value"],
                              "unit": base["unit"], "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
                              "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                              "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (numpy)",
                              "data": "synthetic, seeded",
                              "config": {"workload": "GDN chunked prefill (B=8, T=8192, 16 heads, 18 layers), "
                                                     "sampled on the host CPU", "global_batch": 8},
                              "cpu_baseline": base,
                              "e2e": {"value": base["value"], "unit": base["unit"], "h2d_bytes_per_step": 0,
                                      "d2h_bytes_per_step": 0}}), flush=True)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
