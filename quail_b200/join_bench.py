"""AI join throughput on one GPU: config 2 (Qwen3-4B FP8, two-level prefix sharing).

``python -m quail_b200.join_bench [--left N] [--right M] [--cpu]`` runs
``B200Executor.join`` over the first N left rows of config 2, each streaming
every one of the M right rows (pairs = N x M). Config 2 shards by left row,
so a GPU's share is a contiguous run of anchors against the whole right
table; N anchors out of 200 is one GPU's slice of a larger run. One
untimed warm-up join of one anchor precedes the timed one.

``--workload exists --outer N`` runs config 4's EXISTS variant instead: N
outer rows (64-token shared prefix | 512-token context), each against its
own 8 candidate documents of 4096-16384 tokens (pairs = 8 N). By default
the scoring short-circuits per outer row on its first positive margin
(``exists_stop``: the outer rows' candidate streams interleave one
candidate per outer row per chunk, and the candidates of an outer row not
yet launched when one answers TRUE are skipped); ``--no-stop`` scores every
candidate as the reference's join does (gate_group keeps an outer row with
any TRUE answer). It reports outer rows/s, the candidate pairs skipped and
the EXISTS survivors as well.

Prints one JSON line:

- ``e2e``: pairs/s through the public call (prefix tree, admission and
  packing on the host, pinned H2D, the forwards, D2H of the answer bits),
  timed on the wall clock around the call after a device synchronize;
- ``value``: pairs/s over the summed CUDA-event time of the forwards
  (``gpu_s``), the device-side rate;
- tokens: logical prompt tokens of the pairs, fresh tokens packed (the
  instruction and each left document are computed once per GPU), tokens
  read from borrowed pages;
- ``cpu_baseline`` (``--cpu``): the CPU oracle (BLAS mode, all host cores)
  on one anchor against the first ``--cpu-partners`` right rows.
"""

import argparse
import json
import os
import time

from quail_b200.api import B200Executor
from quail_b200.model import QWEN3_4B
from quail_b200.workload import config2, config4_exists


def cpu_sample(torch, weights, wl, partners, page_tokens=16):
    """(seconds, pairs, tokens) of the CPU oracle on anchor 0 x partners."""
    from oracle import forward as of
    from oracle import numerics as nx
    from quail_b200 import loop
    from quail_b200.arena import KVArena
    from quail_b200.tokens import prefix_tree

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    nx.MODE["exact"] = False
    cpu_w = weights.to("cpu")
    anchors = [wl.anchors[0]]
    sufs = [wl.partners[:partners]]
    arena = KVArena(1, 4096, page_tokens, 1, 8, device=None)
    hosts = []

    class Rec:
        tree_attention = True
        canvas_ids = ()

        def forward_chunk(self, chunk):
            hosts.append(chunk.host)
            return len(chunk.host.final_indices)  # one answer per final row

    class Ans:
        dtype = None

        def submit(self, n):
            return [1] * n

        def result(self, h):
            return h

    loop.run_join(torch, arena, Rec(), Ans(), anchors, sufs, 1 << 20, attention_mode="tree",
                  prefix_tree=prefix_tree(anchors, page_tokens), device="cpu")
    cfg = cpu_w.config
    _, ans_w, tc, fc = cpu_w.answer_rows()
    t0 = time.perf_counter()
    cpu_arena = of.CpuArena(cfg.n_layers, 4096 * page_tokens, cfg.n_kv, cfg.head_dim)
    for host in hosts:
        nx.answer_margin(of.forward_chunk(cpu_w, host, cpu_arena), ans_w, tc, fc)
    return time.perf_counter() - t0, partners, sum(h.tokens for h in hosts)


def exists_main(torch, args):
    """Config 4's EXISTS variant: outer rows 1..N against their candidates."""
    wl = config4_exists()
    ex = B200Executor(torch, QWEN3_4B, args.pages)
    budget = args.budget or None
    # warm-up: outer row 0 against two of its candidates
    ex.join([wl.anchors[0]], [wl.candidates(0)[:2]], budget=budget)
    ex.reset_arena()
    outer = list(range(1, 1 + args.outer))
    anchors = [wl.anchors[a] for a in outer]
    suffixes, partners = [], []
    for a in outer:
        first = len(suffixes)
        suffixes.extend(wl.candidates(a))
        partners.append([list(range(first, len(suffixes)))])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    res = ex.join(anchors, [suffixes], budget=budget, partners=partners,
                  exists_stop=not args.no_stop)
    wall = time.perf_counter() - t0
    pairs = len(suffixes)
    logical = sum(len(anchors[i]) * wl.n_candidates for i in range(len(anchors))) + sum(
        len(x) for x in suffixes)
    survivors = res.survivors("semi")
    return {
        "metric": "EXISTS outer rows/s (Qwen3-4B FP8, config 4 EXISTS variant)",
        "unit": "outer rows/s", "value": len(outer) / res.gpu_s, "e2e": len(outer) / wall,
        "pairs_per_s": pairs / res.gpu_s, "outer_rows": len(outer), "pairs": pairs,
        "pairs_skipped": res.skipped_pairs, "pairs_scored": pairs - res.skipped_pairs,
        "exists_survivors": len(survivors), "gpu_s": res.gpu_s, "wall_s": wall,
        "chunks": res.chunks, "logical_tokens": logical, "fresh_tokens": res.fresh_tokens,
        "borrowed_tokens": res.borrowed_tokens,
        "prefill_tokens_per_s": res.fresh_tokens / res.gpu_s,
        "h2d_bytes": res.h2d_bytes, "d2h_bytes": res.d2h_bytes,
        "config": {"workload": f"config4 EXISTS: outer rows 1..{len(outer)}, "
                               f"{wl.n_candidates} candidates each, tree attention, "
                               + ("every candidate scored" if args.no_stop else
                                  "short-circuit per outer row on the first TRUE"),
                   "budget": budget or ex.budget},
        "data": "synthetic (seeded config-4 EXISTS shapes; random-init Qwen3-4B FP8 weights)",
    }


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--workload", choices=["config2", "exists"], default="config2")
    p.add_argument("--outer", type=int, default=4, help="EXISTS outer rows timed")
    p.add_argument("--no-stop", action="store_true",
                   help="EXISTS: score every candidate (no short-circuit)")
    p.add_argument("--left", type=int, default=8, help="anchors (left rows) timed")
    p.add_argument("--right", type=int, default=500, help="partners (right rows)")
    p.add_argument("--pages", type=int, default=16384)
    p.add_argument("--budget", type=int, default=0)
    p.add_argument("--cpu", action="store_true")
    p.add_argument("--cpu-partners", type=int, default=2)
    args = p.parse_args(argv)
    import torch

    if args.workload == "exists":
        print(json.dumps(exists_main(torch, args)))
        return
    wl = config2(right=args.right)
    ex = B200Executor(torch, QWEN3_4B, args.pages)
    budget = args.budget or None
    ex.join([wl.anchors[0]], [wl.partners], budget=budget)  # warm-up
    ex.reset_arena()
    anchors = [wl.anchors[i] for i in range(1, 1 + args.left)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    res = ex.join(anchors, [wl.partners], budget=budget)
    wall = time.perf_counter() - t0
    pairs = len(anchors) * len(wl.partners)
    answered = sum(len(row) for row in res.answers[0].values())
    logical = wl.logical_tokens(1, 1 + args.left)
    line = {
        "metric": "AI join pairs/s (Qwen3-4B FP8, config 2)", "unit": "pairs/s",
        "value": pairs / res.gpu_s, "e2e": pairs / wall, "pairs": pairs, "answered": answered,
        "gpu_s": res.gpu_s, "wall_s": wall, "chunks": res.chunks,
        "logical_tokens": logical, "fresh_tokens": res.fresh_tokens,
        "borrowed_tokens": res.borrowed_tokens,
        "prefill_tokens_per_s": res.fresh_tokens / res.gpu_s,
        "h2d_bytes": res.h2d_bytes, "d2h_bytes": res.d2h_bytes,
        "config": {"workload": f"config2: {args.left} left x {args.right} right rows, tree "
                               f"attention, one GPU's slice", "budget": budget or ex.budget},
        "data": "synthetic (seeded config-2 shapes; random-init Qwen3-4B FP8 weights)",
    }
    if args.cpu:
        dt, n, tokens = cpu_sample(torch, ex.weights, wl, args.cpu_partners)
        line["cpu_baseline"] = {"value": n / dt, "unit": "pairs/s",
                                "cores": len(os.sched_getaffinity(0)), "kind": "port",
                                "sample": f"anchor 0 x {n} partners ({tokens} tokens) through "
                                          f"the CPU oracle, {dt:.1f} s"}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
