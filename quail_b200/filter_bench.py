"""AI.IF filter throughput on one GPU for a BASELINE configuration's shape.

``python -m quail_b200.filter_bench --config 3 [--rows N]`` runs
``B200Executor.filter`` over the first N rows of the configuration (config 3:
Qwen3-32B FP8, 96-token shared prefix, suffixes lognormal(5.5, 0.5) in
[64, 2048]; config 1: the bench's Qwen3-4B workload) after an untimed
warm-up filter of a few rows, and prints one JSON line (config 4: the
long-document filter, suffixes of 4096-16384 tokens, attention about 30%
of its FLOPs):

- ``e2e``: rows/s through the public call (prefix tree, admission and
  packing on the host, pinned H2D, the forwards, D2H of bits and margins),
  wall clock around the call after a device synchronize;
- ``value``: rows/s over the summed CUDA-event time of the forwards;
- fresh prefill tokens/s and the GEMM FLOP rate implied by 2 x the model's
  linear parameters per fresh token, against 2 x the measured sustained
  bf16 peak (FP8 dense) of MEASURED_PEAKS.json; the attention pairs and the
  attention share of the FLOPs, and the total FLOP rate (both over the
  whole forward time).

bench.py stays the headline (config 1); this module measures the other
filter configurations with the same kernels.
"""

import argparse
import json
import time

from quail_b200.api import B200Executor
from quail_b200.kernel_bench import peaks
from quail_b200.model import QWEN3_4B, QWEN3_32B
from quail_b200.workload import config1, config3, config4

CONFIGS = {1: (config1, QWEN3_4B), 3: (config3, QWEN3_32B), 4: (config4, QWEN3_4B)}


def linear_params(cfg) -> int:
    per_layer = (cfg.hidden * (cfg.n_q + 2 * cfg.n_kv) * cfg.head_dim
                 + cfg.n_q * cfg.head_dim * cfg.hidden + cfg.hidden * 2 * cfg.inter
                 + cfg.inter * cfg.hidden)
    return cfg.n_layers * per_layer


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS))
    p.add_argument("--rows", type=int, default=2000)
    p.add_argument("--pages", type=int, default=16384)
    args = p.parse_args(argv)
    import torch

    make, cfg = CONFIGS[args.config]
    wl = make()
    ex = B200Executor(torch, cfg, args.pages)
    ex.filter([wl.docs[i] for i in range(2 if args.config == 4 else 8)], wl.questions)
    ex.reset_arena()
    docs = [wl.docs[i] for i in range(8, 8 + args.rows)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    res = ex.filter(docs, wl.questions)
    wall = time.perf_counter() - t0
    flops = 2.0 * linear_params(cfg) * res.fresh_tokens
    _, fp8_peak, src = peaks()
    gemm_tflops = flops / res.gpu_s / 1e12
    # (query, key) pairs: each row past the shared prefix (and the question
    # row) attends every earlier key of its document, 4 n_q d FLOP per pair
    # and layer
    pairs = 0
    shared = wl.prefix_tokens
    for d in docs:
        n = len(d) + 1
        pairs += n * (n + 1) // 2 - shared * (shared + 1) // 2
    attn_flops = 4.0 * cfg.n_q * cfg.head_dim * cfg.n_layers * pairs
    print(json.dumps({
        "metric": f"AI.IF rows/sec ({cfg.name}, config {args.config})", "unit": "rows/s",
        "value": len(docs) / res.gpu_s, "e2e": len(docs) / wall, "rows": len(docs),
        "gpu_s": res.gpu_s, "wall_s": wall, "chunks": res.chunks,
        "fresh_tokens": res.fresh_tokens, "borrowed_tokens": res.borrowed_tokens,
        "prefill_tokens_per_s": res.fresh_tokens / res.gpu_s,
        "linear_tflops_per_s": gemm_tflops, "linear_frac_of_fp8_peak": gemm_tflops / fp8_peak,
        "attention_pairs": pairs, "attention_share_of_flops": attn_flops / (attn_flops + flops),
        "total_tflops_per_s": (flops + attn_flops) / res.gpu_s / 1e12,
        "peaks": src, "h2d_bytes": res.h2d_bytes, "d2h_bytes": res.d2h_bytes,
        "config": {"workload": f"config{args.config}: rows 8..{8 + len(docs) - 1}, tree "
                               f"attention", "budget": ex.budget},
        "data": f"synthetic (seeded config-{args.config} shapes; random-init {cfg.name} "
                "weights)",
    }))


if __name__ == "__main__":
    main()
