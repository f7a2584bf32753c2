#!/usr/bin/env python
"""AI.IF filter throughput on B200: rows/s of the Qwen3-4B FP8 prefill path.

Workload: Qwen3-4B-shaped FP8 model with seeded
random-init weights; rows = a shared 64-token instruction prefix plus a
lognormal(5.3, 0.6) suffix clipped to [32, 2048], ids uniform in
[1000, 150000), a one-token question tail; tree attention, 16-token KV
pages, the reference's chunk budget (110,376 tokens). A step is one
chunk: one forward pass over the next rows of the rank's contiguous slice
and the answer readout.

Measurements (one JSON line on rank 0):
- value: rows/s with every chunk's inputs already in HBM (chunks packed
  and uploaded before the timed region), device-timed with CUDA events,
  max over ranks, rows summed over ranks;
- e2e: rows/s through the public API (quail_b200.api.B200Executor.filter)
  from host token lists: prefix tree, packing, pinned H2D copies, forward
  passes, D2H of bits and margins, the NCCL all-gather of results (N>1);
- roofline: the FP8 GEMM (the dominant kernel), algorithmic FLOPs per
  launch over CUDA-event launch time, against 2x the measured sustained
  bf16 dense peak (B200's FP8:bf16 dense ratio);
- cpu_baseline: the CPU oracle (a restatement of the reference's torch
  path) on a bounded sample of the same rows on the host cores;
- other_scales: the same timed chunks in the other scale mode (--scales:
  ue8m0 by default, the power-of-two scales vLLM's DeepGEMM path uses and
  the block-scaled MMA applies; fp32 keeps the loaded block scales).

--impl reference runs the reference arm: the reference's computation
restated on the host CPU (the oracle), timed per step on a bounded sample.
"""

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "AI.IF rows/sec (Qwen3-4B FP8 filter, config 1)"
UNIT = "rows/s"
SCALES_UE8M0 = ("ue8m0: power-of-two activation and weight block scales (weights "
                "re-quantised at load), block-scaled MMA; the mode vLLM selects for "
                "DeepGEMM (is_deep_gemm_e8m0_used), the only one its sm_100 GEMM takes")
SCALES_FP32 = "fp32: activation and weight block scales as computed / loaded"


# DRAM bytes (read + write) per GEMM launch, averaged over the 144 launches
# of one config-1 chunk (o, down: qb_gemm_fp8_bs; qkv with q/k norm, rotary
# and KV append: qb_gemm_fp8_qknorm_rope; gate_up: qb_gemm_fp8_silu_quant;
# x 36 layers). A profile constant, not measured in this run: ncu's
# dram__bytes_read.sum + dram__bytes_write.sum over the launch list of this
# bench's own workload (one pass per launch).
GEMM_DRAM_BYTES_PER_LAUNCH = 1.7174e9
GEMM_TRAFFIC_SOURCE = ("profile constant: ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                       "mean over the GEMM launches of one config-1 chunk")


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--pages", type=int, default=16384)
    p.add_argument("--cpu-rows", type=int, default=4,
                   help="config-1 rows 0..n-1 (the prefix parent and n-1 borrowing rows) "
                        "of the CPU baseline's sample")
    p.add_argument("--ref-rows", type=int, default=1,
                   help="config-1 rows per step of the reference arm's CPU sample")
    p.add_argument("--e2e-rows", type=int, default=25000,
                   help="rows of the rank's share run end to end (the whole share when "
                        "it is smaller)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--budget", type=int, default=0)
    p.add_argument("--scales", default="ue8m0", choices=["ue8m0", "fp32"],
                   help="quantiser / GEMM scale mode: ue8m0 (power-of-two scales on the "
                        "block-scaled MMA; DeepGEMM's mode on sm_100) or fp32")
    p.add_argument("--other-steps", type=int, default=6,
                   help="timed chunks of the other scale mode, reported beside the "
                        "headline (0: skip)")
    return p.parse_args()


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "MEASURED_PEAKS.json"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, \
        "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.devices = devices
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", ",".join(map(str, self.devices))],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def rows_needed(wl, lo, hi, chunks, budget):
    """Rows of [lo, hi) whose fresh tokens fill `chunks` chunks, plus 5%.

    A borrowing row puts only its suffix and question tail into a chunk
    (the shared prefix pages are the tree parent's), so the estimate counts
    those tokens, row by row, until `chunks` budgets are covered."""
    fresh = np.cumsum(wl.fresh_row_tokens(lo, hi)) + wl.prefix_tokens
    n = int(np.searchsorted(fresh, chunks * budget)) + 1
    return min(hi - lo, int(n * 1.05) + 64)


def pack_chunks(torch, arena, docs, questions, budget, n_chunks, device):
    """Pack chunks through the real filter loop without computing them.

    Packs until n_chunks + 1 chunks exist, so the first n_chunks were each
    closed by the budget (a stream's last chunk holds only what was left),
    or until the rows run out. Returns (chunks in launch order, whether the
    first n_chunks are all closed by the budget). The arena's page tables
    evolve exactly as in a real run of a single-stage filter: the pages of
    chunk i are freed once chunk i+1 is launched."""
    from quail_b200 import loop
    from quail_b200.pipeline import ModelPipeline
    from quail_b200.tokens import prefix_tree

    chunks = []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            chunks.append(chunk)
            return len(chunk.layout)

    class Answers:
        def submit(self, n):
            return [1] * n

        def result(self, handle):
            return handle

    stream = loop.FilterStream(torch, arena, Recorder(), Answers(), docs, questions, budget,
                               arena_writes=True, attention_mode="tree",
                               prefix_tree=prefix_tree(docs, 16), device=device)
    while len(chunks) < n_chunks + 1 and not stream.done:
        stream.next()
    full = len(chunks) > n_chunks
    return chunks[:n_chunks], full


def prepack(torch, arena, wl, lo, hi, budget, n_chunks, device):
    """n_chunks budget-filled chunks from the rows [lo, hi) of the workload.

    Starts from the rows_needed estimate and doubles the row count (with
    a fresh arena) until the packer closes n_chunks chunks on the budget.
    Raises when even the whole slice gives fewer than n_chunks chunks.
    Returns (chunks, rows used)."""
    n_rows = rows_needed(wl, lo, hi, n_chunks, budget)
    while True:
        docs = wl.docs[lo:lo + n_rows]
        chunks, full = pack_chunks(torch, arena, docs, wl.questions, budget, n_chunks, device)
        if full or (n_rows == hi - lo and len(chunks) == n_chunks):
            return chunks, n_rows
        if n_rows == hi - lo:
            raise RuntimeError(f"rows [{lo}, {hi}) pack only {len(chunks)} chunks for "
                               f"{n_chunks} steps")
        del chunks
        arena.reset()
        n_rows = min(hi - lo, 2 * n_rows)


def cpu_baseline(torch, weights, wl, rows, page_tokens=16, ue8m0=False):
    """The CPU oracle over a bounded sample (rows 0..rows-1 of the workload)."""
    from oracle import forward as of
    from oracle import numerics as nx
    from quail_b200 import loop
    from quail_b200.arena import KVArena
    from quail_b200.tokens import prefix_tree

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    # the baseline times the reference's algorithm at BLAS speed (the
    # oracle's fast mode), not the bit-exact tensor-core model
    nx.MODE["exact"] = False
    nx.MODE["ue8m0"] = ue8m0
    cpu_w = weights.to("cpu")
    docs = [wl.docs[i] for i in range(rows)]
    arena = KVArena(1, 4096, page_tokens, 1, 8, device=None)
    hosts = []

    class Rec:
        tree_attention = True

        def forward_chunk(self, chunk):
            hosts.append(chunk.host)
            return len(chunk.layout)

    class Ans:
        def submit(self, n):
            return [1] * n

        def result(self, h):
            return h

    loop.run_filter(torch, arena, Rec(), Ans(), docs, wl.questions, 1 << 20, arena_writes=True,
                    attention_mode="tree", prefix_tree=prefix_tree(docs, 16), device="cpu")
    cfg = cpu_w.config
    _, ans_w, tc, fc = cpu_w.answer_rows()

    def run_once():
        cpu_arena = of.CpuArena(cfg.n_layers, 4096 * page_tokens, cfg.n_kv, cfg.head_dim)
        for host in hosts:
            nx.answer_margin(of.forward_chunk(cpu_w, host, cpu_arena), ans_w, tc, fc)

    return run_once, cores, sum(len(h.final_indices) for h in hosts), \
        sum(h.tokens for h in hosts)


def reference_arm(args):
    """The reference's path restated on the host CPU (the oracle port)."""
    world, rank, _ = setup_dist(args)
    if rank != 0:
        return
    import torch

    from quail_b200.model import QWEN3_4B, random_weights
    from quail_b200.workload import config1

    wl = config1()
    weights = random_weights(QWEN3_4B, seed=0, device="cpu")
    ue8m0 = args.scales == "ue8m0"
    if ue8m0:
        # vLLM's load-time re-quantisation to power-of-two block scales
        from oracle import numerics as nx
        from quail_b200.model import LINEARS
        for layer in weights.layers:
            for wn, sn in LINEARS:
                q, sc = nx.requant_weight_ue8m0(getattr(layer, wn), getattr(layer, sn))
                setattr(layer, wn, q)
                setattr(layer, sn, sc)
    run_once, cores, rows, tokens = cpu_baseline(torch, weights, wl, args.ref_rows, ue8m0=ue8m0)
    for _ in range(args.warmup):
        run_once()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run_once()
    dt = time.perf_counter() - t0
    value = rows * args.steps / dt
    sample = f"{rows} config-1 rows ({tokens} tokens, one tree chunk) per step"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1000 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (fp8 codes dequantised on the CPU)",
        "data": "synthetic (seeded, config-1 shapes)",
        "config": {"workload": "config1: Qwen3-4B FP8 AI.IF filter, host CPU oracle sample",
                   "sample_rows": rows, "sample_tokens": tokens, "scales": args.scales},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}))


def main():
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    world, rank, local = setup_dist(args)
    import torch
    import torch.distributed as dist

    from quail_b200 import _native as nat
    from quail_b200.api import B200Executor
    from quail_b200.model import QWEN3_4B
    from quail_b200.workload import config1, token_shard

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                device_id=dev)
    cfg = QWEN3_4B
    wl = config1()
    budget = args.budget or cfg.max_chunk_tokens
    ex = B200Executor(torch, cfg, args.pages, device=dev, seed=0, scales=args.scales)
    lo, hi = token_shard(wl.row_tokens(), rank, world)

    # ---- device-resident timing: chunks packed and uploaded beforehand ----
    chunks, n_rows = prepack(torch, ex.arena, wl, lo, hi, budget, args.warmup + args.steps,
                             ex.device)
    docs = wl.docs[lo:lo + n_rows]
    torch.cuda.synchronize()

    def run(chunk):
        normed = ex.pipeline.forward_chunk(chunk)
        return ex.answer_rows.margins(normed)

    for chunk in chunks[:args.warmup]:
        run(chunk)
    torch.cuda.synchronize()
    timed = chunks[args.warmup:]
    sampler = ClockSampler([local]) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.5)
    ex.pipeline.engine.gemm_events = []
    launches0 = nat.LAUNCHES["count"]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    outs = [run(chunk) for chunk in timed]
    e1.record()
    torch.cuda.synchronize()
    launches = nat.LAUNCHES["count"] - launches0
    clocks = sampler.stop() if sampler else None
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    gemm = ex.pipeline.engine.gemm_events
    ex.pipeline.engine.gemm_events = None
    gemm_ms = sum(a.elapsed_time(b) for a, b, _, _ in gemm)
    gemm_flops = sum(f for _, _, f, _ in gemm)
    gemm_bytes = sum(nb for _, _, _, nb in gemm)
    rows_timed = sum(len(c.layout) for c in timed)
    tokens_timed = sum(c.tokens for c in timed)
    status = nat.kernel_status(local)
    vals = torch.tensor([ms, rows_timed, tokens_timed, gemm_ms, gemm_flops, len(gemm), status],
                        dtype=torch.float64, device=dev)
    if world > 1:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vals.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms, gemm_ms_max = float(mx[0]), float(mx[3])
        rows_all, tokens_all = float(sm[1]), float(sm[2])
        status = int(mx[6])
    else:
        rows_all, tokens_all = float(rows_timed), float(tokens_timed)
    del outs

    # ---- the other scale mode on the same chunks (fresh seed-0 weights) ----
    other = None
    n_other = min(args.other_steps, args.steps)
    if n_other > 0:
        from quail_b200.model import random_weights, requant_ue8m0
        from quail_b200.pipeline import build_pipeline
        o_ue8m0 = args.scales != "ue8m0"
        w_other = random_weights(cfg, seed=0, device=dev)
        if o_ue8m0:
            requant_ue8m0(w_other)
        pipe_other = build_pipeline(torch, w_other, ex.arena, ue8m0=o_ue8m0)
        pipe_other.forward_chunk(chunks[0])
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        pipe_other.engine.gemm_events = []
        o0 = torch.cuda.Event(enable_timing=True)
        o1 = torch.cuda.Event(enable_timing=True)
        o0.record()
        for chunk in timed[:n_other]:
            pipe_other.forward_chunk(chunk)
        o1.record()
        torch.cuda.synchronize()
        o_ms = o0.elapsed_time(o1)
        o_gemm = pipe_other.engine.gemm_events
        o_gemm_ms = sum(a.elapsed_time(b) for a, b, _, _ in o_gemm)
        o_flops = sum(f for _, _, f, _ in o_gemm)
        o_rows = sum(len(c.layout) for c in timed[:n_other])
        ov = torch.tensor([o_ms, o_rows, o_gemm_ms, o_flops], dtype=torch.float64, device=dev)
        if world > 1:
            omx = ov.clone()
            dist.all_reduce(omx, op=dist.ReduceOp.MAX)
            osm = ov.clone()
            dist.all_reduce(osm, op=dist.ReduceOp.SUM)
            o_ms, o_rows = float(omx[0]), float(osm[1])
        other = {"scales": "ue8m0" if o_ue8m0 else "fp32", "steps": n_other,
                 "value": o_rows / (o_ms / 1000.0), "ms_per_step": o_ms / n_other,
                 "gemm_tflops": o_flops / (o_gemm_ms / 1000.0) / 1e12 if o_gemm_ms else None}
        del pipe_other, w_other, o_gemm

    # ---- end to end through the public API, host inputs ----
    e2e = None
    if not args.no_e2e:
        ex.reset_arena()
        e2e_docs = wl.docs[lo:lo + min(hi - lo, args.e2e_rows)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = ex.filter(e2e_docs, wl.questions, budget=budget, attention="tree")
        if world > 1:
            # ranks hold different row counts: size-aware gather of (bit, margin)
            from quail_b200.distributed import gather_rows
            gather_rows(torch, dist, res.bits, dev)
            gather_rows(torch, dist, res.margins, dev)
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - t0
        t = torch.tensor([e2e_s, len(e2e_docs), res.h2d_bytes, res.d2h_bytes, res.chunks],
                         dtype=torch.float64, device=dev)
        if world > 1:
            mx = t.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            sm = t.clone()
            dist.all_reduce(sm, op=dist.ReduceOp.SUM)
            e2e_s, e2e_rows = float(mx[0]), float(sm[1])
        else:
            e2e_rows = float(t[1])
        e2e = {"value": e2e_rows / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": int(res.h2d_bytes / max(res.chunks, 1)),
               "d2h_bytes_per_step": int(res.d2h_bytes / max(res.chunks, 1)),
               "rows": int(e2e_rows), "seconds": e2e_s,
               "host_seconds": {k: round(v, 4) for k, v in sorted(res.timing.items())},
               "forward_seconds": round(res.gpu_s, 4),
               "note": "host token lists -> prefix tree, packing, pinned H2D, forward, "
                       "D2H bits+margins" + (", NCCL all-gather" if world > 1 else "")}

    # ---- CPU baseline (rank 0, N=1) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        run_once, cores, rows, tokens = cpu_baseline(torch, ex.weights, wl, args.cpu_rows,
                                                     ue8m0=args.scales == "ue8m0")
        t0 = time.perf_counter()
        run_once()
        dt = time.perf_counter() - t0
        cpu = {"value": rows / dt, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"rows 0..{rows - 1} of config 1 ({tokens} tokens, one tree chunk) "
                         f"through the CPU oracle, {dt:.1f} s"}

    ue8m0 = args.scales == "ue8m0"
    if rank == 0:
        peaks, src = measured_peaks()
        peak = 2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms else 0.0
        line = {
            "metric": METRIC, "value": rows_all / (ms / 1000.0), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": ("fp8-e4m3 GEMMs with UE8M0 (power-of-two) block scales" if ue8m0 else
                      "fp8-e4m3 GEMMs with fp32 block scales")
                     + ", bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded config-1 rows; random-init Qwen3-4B FP8 weights)",
            "config": {"workload": "config1: Qwen3-4B FP8 AI.IF filter, tree attention",
                       "scales": (SCALES_UE8M0 if ue8m0 else SCALES_FP32),
                       "rows_per_rank_timed": rows_timed, "chunk_budget_tokens": budget,
                       "parallelism": f"dp{world} (token-balanced contiguous row slices)",
                       "prefill_tokens_per_s": tokens_all / (ms / 1000.0),
                       "l2": "inputs larger than L2 (>=0.5 GB activations per chunk)",
                       "status_word": status},
            "roofline": {"bound": "tensor",
                         "kernel": "qb_gemm_fp8_bs + qb_gemm_fp8_qknorm_rope + "
                                   "qb_gemm_fp8_silu_quant (all GEMMs)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak if peak else None,
                         "traffic": GEMM_DRAM_BYTES_PER_LAUNCH,
                         "traffic_source": GEMM_TRAFFIC_SOURCE,
                         "algorithmic_bytes": gemm_bytes / max(len(gemm), 1),
                         "peak_source": f"2 x bf16_tflops_sustained of {src} (of measured)",
                         "launches": len(gemm), "gemm_ms": gemm_ms,
                         "gemm_share_of_step": gemm_ms / ms if ms else None},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clocks, "other_scales": other,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
