"""Per-kernel timing of the sm_100a library on one GPU.

``python -m quail_b200.kernel_bench <op> [options]`` launches one entry
point ``--warmup`` times untimed, then ``--iters`` times between CUDA
events on the launching stream, and prints one JSON line: mean ms per
launch, the algorithmic bytes or FLOPs of one launch and the achieved rate
against the measured peaks (MEASURED_PEAKS.json beside the repository
root, when present). Inputs are random device tensors of the Qwen3-4B
config-1 shapes; they exist only to be read, so values do not matter.

The same command with ``--warmup 0 --iters 1..3`` is the small case that
a profiler capture of one kernel runs on.

Ops:
  gemm       qb_gemm_fp8_bs on (m, n, k); default the 4B qkv projection
  gate_up    qb_gemm_fp8_silu_quant on (m, inter, hidden) beside the unfused
             qb_gemm_fp8_bs (n = 2 inter) + qb_silu_mul_quant pair
  qkv_rope   qb_gemm_fp8_qknorm_rope on m rows beside the unfused
             qb_gemm_fp8_bs + qb_qknorm_rope pair (with the KV append)
  layer      the four GEMMs of one 4B layer back to back (m rows)
  silu       qb_silu_mul_quant on (rows, inter)
  norm       qb_add_rmsnorm_quant on (rows, hidden)
  rope       qb_qknorm_rope with the fused KV append on rows
  attention  qb_tree_attention on one packed config-1 chunk (--budget tokens)
"""

import argparse
import json
from pathlib import Path

import numpy as np

from quail_b200 import _native as nat

ROOT = Path(__file__).resolve().parent.parent

# --ue8m0: the UE8M0 scale mode (power-of-two scales, block-scaled MMA)
UE8M0 = 0


def peaks():
    """(HBM GB/s, FP8 dense TFLOP/s, source) from MEASURED_PEAKS.json."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        hbm = float(p.get("hbm_gbs") or 6650.0)
        bf16 = float(p.get("bf16_tflops_sustained") or p.get("bf16_tflops") or 1400.0)
        return hbm, 2.0 * bf16, "measured"
    return 6650.0, 2.0 * 1400.0, "fallback"


def time_launches(torch, launch, warmup, iters):
    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        launch()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / max(iters, 1)


def _pow2(torch, x):
    return torch.exp2(torch.ceil(torch.log2(x))) if UE8M0 else x


def fp8_rows(torch, rows, k):
    q = (torch.randn(rows, k, device="cuda") * 2).to(torch.float8_e4m3fn)
    scale = _pow2(torch, torch.rand(k // 128, rows, device="cuda") * 0.01 + 0.001)
    return q, scale


def fp8_weight(torch, n, k):
    w = torch.randn(n, k, device="cuda").to(torch.float8_e4m3fn)
    s = _pow2(torch, torch.rand(n // 128, k // 128, device="cuda") * 0.02 + 0.001)
    return w, s


def gemm_launcher(torch, m, n, k):
    a, a_s = fp8_rows(torch, m, k)
    w, w_s = fp8_weight(torch, n, k)
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")

    def launch():
        nat.call("qb_gemm_fp8_bs", nat.ptr(a), nat.ptr(a_s), m, nat.ptr(w), nat.ptr(w_s),
                 nat.ptr(out), m, n, k, UE8M0, nat.stream_handle(torch))
    return launch


def op_gemm(torch, args):
    m, n, k = args.m, args.n, args.k
    launch = gemm_launcher(torch, m, n, k)
    ms = time_launches(torch, launch, args.warmup, args.iters)
    flops = 2.0 * m * n * k
    return {"shape": [m, n, k], "ms": ms, "tflops": flops / ms / 1e9, "bound": "tensor",
            "algorithmic": flops}


def op_gate_up(torch, args):
    m, inter, k = args.m, args.inter, args.hidden
    a, a_s = fp8_rows(torch, m, k)
    w, w_s = fp8_weight(torch, 2 * inter, k)
    q = torch.empty(m, inter, dtype=torch.float8_e4m3fn, device="cuda")
    s = torch.empty(inter // 128, m, dtype=torch.float32, device="cuda")
    gu = torch.empty(m, 2 * inter, dtype=torch.bfloat16, device="cuda")

    def fused():
        nat.call("qb_gemm_fp8_silu_quant", nat.ptr(a), nat.ptr(a_s), m, nat.ptr(w),
                 nat.ptr(w_s), nat.ptr(q), nat.ptr(s), m, m, inter, k, UE8M0,
                 nat.stream_handle(torch))

    def unfused():
        nat.call("qb_gemm_fp8_bs", nat.ptr(a), nat.ptr(a_s), m, nat.ptr(w), nat.ptr(w_s),
                 nat.ptr(gu), m, 2 * inter, k, UE8M0, nat.stream_handle(torch))
        nat.call("qb_silu_mul_quant", nat.ptr(gu), m, inter, nat.ptr(q), nat.ptr(s), m,
                 UE8M0, nat.stream_handle(torch))
    ms = time_launches(torch, fused, args.warmup, args.iters)
    ms_unfused = time_launches(torch, unfused, args.warmup, args.iters)
    flops = 2.0 * m * 2 * inter * k
    return {"shape": [m, inter, k], "ms": ms, "tflops": flops / ms / 1e9, "bound": "tensor",
            "algorithmic": flops, "ms_unfused": ms_unfused}


def op_qkv_rope(torch, args):
    from quail_b200.model import QWEN3_4B as cfg, rotary_cache
    m, k = args.m, cfg.hidden
    n = (cfg.n_q + 2 * cfg.n_kv) * cfg.head_dim
    a, a_s = fp8_rows(torch, m, k)
    w, w_s = fp8_weight(torch, n, k)
    pos = torch.arange(m, device="cuda", dtype=torch.int64) % 2048
    cos_sin = rotary_cache(cfg, "cuda")
    qw = torch.ones(cfg.head_dim, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(m, cfg.n_q * cfg.head_dim, dtype=torch.bfloat16, device="cuda")
    kk = torch.empty(m, cfg.n_kv * cfg.head_dim, dtype=torch.bfloat16, device="cuda")
    v = torch.empty_like(kk)
    kp = torch.empty_like(kk)
    vp = torch.empty_like(kk)
    row_dst = torch.arange(m, device="cuda", dtype=torch.int64)
    qkv = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    st = nat.stream_handle(torch)

    def fused():
        nat.call("qb_gemm_fp8_qknorm_rope", nat.ptr(a), nat.ptr(a_s), m, nat.ptr(w), nat.ptr(w_s),
                 m, k, nat.ptr(pos), nat.ptr(cos_sin), cos_sin.shape[0], nat.ptr(qw), nat.ptr(qw),
                 1e-6, cfg.n_q, cfg.n_kv, cfg.head_dim, nat.ptr(q), nat.ptr(kk), nat.ptr(v),
                 nat.ptr(row_dst), nat.ptr(kp), nat.ptr(vp), m, UE8M0, st)

    def unfused():
        nat.call("qb_gemm_fp8_bs", nat.ptr(a), nat.ptr(a_s), m, nat.ptr(w), nat.ptr(w_s),
                 nat.ptr(qkv), m, n, k, UE8M0, st)
        nat.call("qb_qknorm_rope", nat.ptr(qkv), n, nat.ptr(pos), nat.ptr(cos_sin),
                 cos_sin.shape[0], nat.ptr(qw), nat.ptr(qw), 1e-6, m, cfg.n_q, cfg.n_kv,
                 cfg.head_dim, nat.ptr(q), nat.ptr(kk), nat.ptr(v), nat.ptr(row_dst), nat.ptr(kp),
                 nat.ptr(vp), m, st)
    ms = time_launches(torch, fused, args.warmup, args.iters)
    ms_unfused = time_launches(torch, unfused, args.warmup, args.iters)
    flops = 2.0 * m * n * k
    return {"rows": m, "ms": ms, "tflops": flops / ms / 1e9, "bound": "tensor",
            "algorithmic": flops, "ms_unfused": ms_unfused}


def op_layer(torch, args):
    from quail_b200.model import QWEN3_4B as cfg
    m = args.m
    shapes = [((cfg.n_q + 2 * cfg.n_kv) * cfg.head_dim, cfg.hidden),
              (cfg.hidden, cfg.n_q * cfg.head_dim),
              (2 * cfg.inter, cfg.hidden), (cfg.hidden, cfg.inter)]
    launches = [gemm_launcher(torch, m, n, k) for n, k in shapes]

    def launch():
        for f in launches:
            f()
    ms = time_launches(torch, launch, args.warmup, args.iters)
    flops = sum(2.0 * m * n * k for n, k in shapes)
    return {"rows": m, "ms": ms, "tflops": flops / ms / 1e9, "bound": "tensor",
            "algorithmic": flops}


def op_silu(torch, args):
    rows, inter = args.rows, args.inter
    gate_up = torch.randn(rows, 2 * inter, device="cuda").to(torch.bfloat16)
    q = torch.empty(rows, inter, dtype=torch.float8_e4m3fn, device="cuda")
    s = torch.empty(inter // 128, rows, dtype=torch.float32, device="cuda")

    def launch():
        nat.call("qb_silu_mul_quant", nat.ptr(gate_up), rows, inter, nat.ptr(q), nat.ptr(s),
                 rows, UE8M0, nat.stream_handle(torch))
    ms = time_launches(torch, launch, args.warmup, args.iters)
    nbytes = rows * (4 * inter + inter + 4 * (inter // 128))
    return {"shape": [rows, inter], "ms": ms, "gbs": nbytes / ms / 1e6, "bound": "hbm",
            "algorithmic": nbytes}


def op_norm(torch, args):
    rows, h = args.rows, args.hidden
    hidden = torch.randn(rows, h, device="cuda").to(torch.bfloat16)
    residual = torch.randn(rows, h, device="cuda").to(torch.bfloat16)
    w = torch.ones(h, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(rows, h, dtype=torch.float8_e4m3fn, device="cuda")
    s = torch.empty(h // 128, rows, dtype=torch.float32, device="cuda")

    def launch():
        nat.call("qb_add_rmsnorm_quant", nat.ptr(hidden), nat.ptr(residual), nat.ptr(w), 1e-6,
                 rows, h, nat.ptr(q), nat.ptr(s), rows, UE8M0, nat.stream_handle(torch))
    ms = time_launches(torch, launch, args.warmup, args.iters)
    nbytes = rows * (2 * h + 2 * h + 2 * h + h + 4 * (h // 128))
    return {"shape": [rows, h], "ms": ms, "gbs": nbytes / ms / 1e6, "bound": "hbm",
            "algorithmic": nbytes}


def op_rope(torch, args):
    from quail_b200.model import QWEN3_4B as cfg, rotary_cache
    rows = args.rows
    d = cfg.head_dim
    width = (cfg.n_q + 2 * cfg.n_kv) * d
    qkv = torch.randn(rows, width, device="cuda").to(torch.bfloat16)
    pos = torch.arange(rows, device="cuda", dtype=torch.int64) % 2048
    cos_sin = rotary_cache(cfg, "cuda")
    qw = torch.ones(d, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(rows, cfg.n_q * d, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(rows, cfg.n_kv * d, dtype=torch.bfloat16, device="cuda")
    v = torch.empty_like(k)
    pool_rows = rows
    kp = torch.empty(pool_rows, cfg.n_kv * d, dtype=torch.bfloat16, device="cuda")
    vp = torch.empty_like(kp)
    row_dst = torch.arange(rows, device="cuda", dtype=torch.int64)

    def launch():
        nat.call("qb_qknorm_rope", nat.ptr(qkv), width, nat.ptr(pos), nat.ptr(cos_sin),
                 cos_sin.shape[0], nat.ptr(qw), nat.ptr(qw), 1e-6, rows, cfg.n_q, cfg.n_kv, d,
                 nat.ptr(q), nat.ptr(k), nat.ptr(v), nat.ptr(row_dst), nat.ptr(kp), nat.ptr(vp),
                 pool_rows, nat.stream_handle(torch))
    ms = time_launches(torch, launch, args.warmup, args.iters)
    kv = cfg.n_kv * d * 2
    nbytes = rows * (width * 2 + cfg.n_q * d * 2 + 2 * kv + 2 * kv + 8 + 8)
    return {"rows": rows, "ms": ms, "gbs": nbytes / ms / 1e6, "bound": "hbm",
            "algorithmic": nbytes}


def op_attention(torch, args):
    """One packed config-1 tree chunk: the layer-0 attention of the forward."""
    from quail_b200 import loop
    from quail_b200.arena import KVArena
    from quail_b200.engine import Engine
    from quail_b200.model import QWEN3_4B
    from quail_b200.pipeline import ModelPipeline
    from quail_b200.tokens import prefix_tree
    from quail_b200.workload import config1

    cfg = QWEN3_4B
    wl = config1(rows=args.doc_rows)
    arena = KVArena(1, args.pages, 16, cfg.n_kv, cfg.head_dim, device=torch.device("cuda"))
    arena.pools.normal_()
    chunks = []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            chunks.append(chunk)
            return len(chunk.layout)

    class Answers:
        def submit(self, n):
            return [1] * n

        def result(self, h):
            return h

    docs = wl.docs
    stream = loop.FilterStream(torch, arena, Recorder(), Answers(), docs, wl.questions,
                               args.budget, arena_writes=True, attention_mode="tree",
                               prefix_tree=prefix_tree(docs, 16), device=torch.device("cuda"))
    # the second chunk reads resident prefixes of the first, as in a steady run
    while len(chunks) < 2 and not stream.done:
        stream.next()
    chunk = chunks[-1]
    meta = chunk.meta
    rows = chunk.input_ids.shape[0]
    d = cfg.head_dim
    q = torch.randn(rows, cfg.n_q * d, device="cuda").to(torch.bfloat16)
    k = torch.randn(rows, cfg.n_kv * d, device="cuda").to(torch.bfloat16)
    v = torch.randn(rows, cfg.n_kv * d, device="cuda").to(torch.bfloat16)
    eng = Engine(torch, arena, cfg, ue8m0=UE8M0)

    def launch():
        meta["layer"] = 0
        eng.attention_tree(q, k, v, meta)
    ms = time_launches(torch, launch, args.warmup, args.iters)
    cu = np.asarray(meta["cu_a"].cpu())
    seg = np.diff(cu)
    pairs = float(np.sum(seg * (seg + 1) / 2.0))
    reads = meta["reads"]
    if reads is not None:
        cu_q = np.asarray(reads["cu_q"].cpu())
        used = np.asarray(reads["used"].cpu())
        pairs += float(np.sum(np.diff(cu_q) * used))
    flops = 4.0 * d * cfg.n_q * pairs
    return {"rows": rows, "segments": int(len(seg)), "ms": ms, "tflops": flops / ms / 1e9,
            "bound": "tensor (bf16)", "algorithmic": flops, "pairs": pairs}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("op", choices=["gemm", "gate_up", "qkv_rope", "layer", "silu", "norm",
                                  "rope", "attention"])
    p.add_argument("--m", type=int, default=65536)
    p.add_argument("--n", type=int, default=6144)
    p.add_argument("--k", type=int, default=2560)
    p.add_argument("--rows", type=int, default=65536)
    p.add_argument("--inter", type=int, default=9728)
    p.add_argument("--hidden", type=int, default=2560)
    p.add_argument("--budget", type=int, default=110376)
    p.add_argument("--doc-rows", type=int, default=2000)
    p.add_argument("--pages", type=int, default=16384)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--ue8m0", action="store_true",
                   help="UE8M0 scale mode: power-of-two scales, block-scaled MMA")
    args = p.parse_args(argv)
    global UE8M0
    UE8M0 = int(args.ue8m0)
    import torch
    torch.manual_seed(0)
    result = globals()["op_" + args.op](torch, args)
    hbm, fp8, source = peaks()
    if "gbs" in result:
        result["frac"] = result["gbs"] / hbm
    elif result["bound"] == "tensor":
        result["frac"] = result["tflops"] / fp8
    result.update(op=args.op, peaks=source, status=nat.kernel_status())
    print(json.dumps(result))


if __name__ == "__main__":
    main()
