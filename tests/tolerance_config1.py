"""Agreement of the B200 path with the reference's semantics on config-1 rows.

The parity tests hold the kernels to the exact oracle bit for bit. This
script measures the other number north_star asks for: how far the kernels'
yes-minus-no margins are from the reference's algorithm computed the usual
way - the oracle's fast mode (fp32 BLAS partial sums per 128-deep K block,
torch's exp2 and reductions), which is FlashAttention / DeepGEMM semantics
without the kernels' fixed rounding orders - on the full 36-layer Qwen3-4B
FP8 model over config-1 rows.

Two steps, so the CPU half runs off the GPU box:

    python tests/tolerance_config1.py gpu --rows 64 --out margins.npz
    python tests/tolerance_config1.py cpu --gpu margins.npz --out summary.json

--depths 1,2,4,8,16,36 repeats both steps on the model cut to its first L
layers (the same weights), which shows how the difference grows with
depth.

``gpu`` runs B200Executor.filter over config-1 rows 0..N-1 (seeded
random-init weights, tree attention, the bench's chunk budget) and saves
the margins; ``cpu`` packs the same rows through the same host loop, runs
every chunk through the oracle's forward pass in fast mode on the CPU and
writes max / mean / percentile |margin difference|, the share within the
0.05 bar and the decision agreement where the reference's |margin| > 0.1.
"""

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def gpu(args):
    import torch

    from quail_b200.api import B200Executor
    from quail_b200.model import QWEN3_4B
    from quail_b200.workload import config1

    from quail_b200.model import random_weights

    wl = config1()
    docs = [wl.docs[i] for i in range(args.rows)]
    # generated on the CPU and copied, so both steps hold the same weights
    # (the CPU and CUDA generators give different numbers)
    full = random_weights(QWEN3_4B, seed=0, device="cpu").to(torch.device("cuda"))
    if args.scales == "ue8m0":
        from quail_b200.model import requant_ue8m0
        requant_ue8m0(full)
    out = {"rows": np.arange(args.rows)}
    for depth in depths(args):
        cfg, weights = truncated(QWEN3_4B, full, depth)
        ex = B200Executor(torch, cfg, 4096, weights=weights, scales=args.scales)
        res = ex.filter(docs, wl.questions, budget=QWEN3_4B.max_chunk_tokens)
        out[f"margins_L{depth}"] = res.margins
        del ex
    if len(depths(args)) == 1:
        out["margins"] = out[f"margins_L{depths(args)[0]}"]
    np.savez(args.out, **out)
    print(json.dumps({"rows": args.rows, "depths": depths(args), "out": args.out}))


def depths(args):
    return [int(d) for d in args.depths.split(",")] if args.depths else [36]


def truncated(cfg, weights, depth):
    """(config, Weights) of the first `depth` layers, tensors shared."""
    import dataclasses

    from quail_b200.model import Weights

    if depth == cfg.n_layers:
        return cfg, weights
    c = dataclasses.replace(cfg, name=f"{cfg.name}-L{depth}", n_layers=depth)
    w = Weights(c, weights.embed, weights.final_norm, weights.cos_sin)
    w.layers = weights.layers[:depth]
    return c, w


def cpu(args):
    import torch

    from oracle import forward as of
    from oracle import numerics as nx
    from quail_b200 import loop
    from quail_b200.arena import KVArena
    from quail_b200.model import QWEN3_4B, random_weights
    from quail_b200.tokens import prefix_tree
    from quail_b200.workload import config1

    got = np.load(args.gpu)
    n = len(got["rows"])
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    nx.MODE["exact"] = False
    wl = config1()
    docs = [wl.docs[i] for i in range(n)]
    full = random_weights(QWEN3_4B, seed=0, device="cpu")
    if args.scales == "ue8m0":
        from quail_b200.model import LINEARS
        nx.MODE["ue8m0"] = True
        for layer in full.layers:
            for wn, sn in LINEARS:
                q, sc = nx.requant_weight_ue8m0(getattr(layer, wn), getattr(layer, sn))
                setattr(layer, wn, q)
                setattr(layer, sn, sc)
    summaries = []
    for depth in depths(args):
        cfg, weights = truncated(QWEN3_4B, full, depth)
        summaries.append(compare(torch, of, nx, loop, KVArena, prefix_tree, wl, docs, weights,
                                 got[f"margins_L{depth}"] if f"margins_L{depth}" in got.files
                                 else got["margins"]))
    text = json.dumps(summaries if len(summaries) > 1 else summaries[0], indent=1)
    Path(args.out).write_text(text + "\n")
    print(text)


def compare(torch, of, nx, loop, KVArena, prefix_tree, wl, docs, weights, m_gpu):
    from quail_b200.model import QWEN3_4B

    n = len(docs)
    cfg = weights.config
    _, ans_w, tc, fc = weights.answer_rows()
    arena = KVArena(1, 4096, 16, 1, 8, device=None)
    cpu_arena = of.CpuArena(cfg.n_layers, 4096 * 16, cfg.n_kv, cfg.head_dim)
    want = np.full(n, np.nan, dtype=np.float32)
    t0 = time.perf_counter()

    class Oracle:
        tree_attention = True

        def forward_chunk(self, chunk):
            return chunk.host

    class Answers:
        def submit(self, host):
            normed = of.forward_chunk(weights, host, cpu_arena)
            margin, _ = nx.answer_margin(normed, ans_w, tc, fc)
            for (doc, _stage), m in zip(host.layout, margin.numpy()):
                want[doc] = m
            return [1] * len(host.layout)

        def result(self, h):
            return h

    loop.run_filter(torch, arena, Oracle(), Answers(), docs, wl.questions,
                    QWEN3_4B.max_chunk_tokens, arena_writes=True, attention_mode="tree",
                    prefix_tree=prefix_tree(docs, 16), device="cpu")
    m_gpu = m_gpu.astype(np.float64)
    m_ref = want.astype(np.float64)
    d = np.abs(m_gpu - m_ref)
    sure = np.abs(m_ref) > 0.1
    summary = {
        "what": "|margin(B200 kernels) - margin(oracle fast mode: fp32 BLAS GEMMs, torch "
                "exp2 and reductions)|, Qwen3-4B FP8 (first %d layers, seeded random-init "
                "weights), config-1 rows 0..%d, tree attention, %s scales"
                % (cfg.n_layers, n - 1, "ue8m0" if nx.MODE["ue8m0"] else "fp32"),
        "layers": cfg.n_layers, "rows": n,
        "max_abs_diff": float(d.max()), "mean_abs_diff": float(d.mean()),
        "median_abs_diff": float(np.median(d)), "p90_abs_diff": float(np.quantile(d, 0.9)),
        "within_0.05": float(np.mean(d <= 0.05)),
        "mean_abs_margin_ref": float(np.abs(m_ref).mean()),
        "decided_rows": int(sure.sum()),
        "decision_agreement_where_ref_abs_margin_gt_0.1":
            float(np.mean((m_gpu[sure] > 0) == (m_ref[sure] > 0))) if sure.any() else None,
        "decision_agreement_all": float(np.mean((m_gpu > 0) == (m_ref > 0))),
        "cpu_seconds": time.perf_counter() - t0,
    }
    return summary


def main():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("step", choices=["gpu", "cpu"])
    p.add_argument("--rows", type=int, default=64)
    p.add_argument("--gpu", default="margins.npz")
    p.add_argument("--out", default="out")
    p.add_argument("--scales", default="fp32", choices=["fp32", "ue8m0"])
    p.add_argument("--depths", default="",
                   help="comma-separated layer counts (default: the full 36)")
    args = p.parse_args()
    (gpu if args.step == "gpu" else cpu)(args)


if __name__ == "__main__":
    main()
