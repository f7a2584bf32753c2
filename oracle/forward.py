"""CPU restatement of Qwen3Pipeline.forward_chunk. Test infrastructure only.

Follows quail/backends/quail/executor/models/qwen3.py:46-77 layer by layer
and Engine.attention_tree / attention_unified
(quail/backends/quail/executor/attention.py:835-953) over a CPU copy of the
KV arena, driven by a packed chunk's host metadata (quail_b200.loop.HostChunk
or the same dict layout). Weights are a quail_b200.model.Weights on the CPU.
"""

import torch

from oracle import numerics as nx


class CpuArena:
    """bf16 K/V pools on the CPU: [n_layers, 2, rows, n_kv, d]."""

    def __init__(self, n_layers, pool_rows, n_kv, head_dim, page_tokens=16):
        self.pools = torch.zeros((n_layers, 2, pool_rows, n_kv * head_dim),
                                 dtype=torch.bfloat16)
        self.page_tokens = page_tokens

    def kv(self, layer):
        return self.pools[layer, 0], self.pools[layer, 1]


def _t(a, dtype=torch.int64):
    return torch.as_tensor(a).to(dtype)


def _paged_rows(table_row, used, page_tokens):
    j = torch.arange(used)
    pages = _t(table_row)[j // page_tokens]
    return pages * page_tokens + j % page_tokens


def tree_attention(q, k, v, meta, kp, vp, cfg, page_tokens):
    """Calls A and B plus merge_attn_quant (attention.py:835-870)."""
    rows = q.shape[0]
    scale = cfg.head_dim ** -0.5
    cu = [int(x) for x in meta["cu_a"]]
    out_a = torch.empty(rows, cfg.n_q * cfg.head_dim, dtype=torch.bfloat16)
    lse_a = torch.empty(rows, cfg.n_q)
    for s0, s1 in zip(cu[:-1], cu[1:]):
        n = s1 - s0
        mask = torch.ones(n, n, dtype=torch.bool).tril()
        o, l = nx.attention_heads(q[s0:s1], k[s0:s1], v[s0:s1], cfg.n_q, cfg.n_kv, scale,
                                  mask)
        out_a[s0:s1], lse_a[s0:s1] = o, l
    reads = meta["reads"]
    if reads is None:
        return nx.quant_groups(out_a.to(torch.float32))
    rrows = _t(reads["rows"])
    cu_q = [int(x) for x in reads["cu_q"]]
    out_b = torch.empty(len(rrows), cfg.n_q * cfg.head_dim, dtype=torch.bfloat16)
    lse_b = torch.empty(len(rrows), cfg.n_q)
    for g, (r0, r1) in enumerate(zip(cu_q[:-1], cu_q[1:])):
        used = int(reads["used"][g])
        prow = _paged_rows(reads["table"][g], used, page_tokens)
        o, l = nx.attention_heads(q[rrows[r0:r1]], kp[prow], vp[prow], cfg.n_q, cfg.n_kv,
                                  scale)
        out_b[r0:r1], lse_b[r0:r1] = o, l
    return nx.merge_attn_quant(out_a, lse_a, out_b, lse_b, _t(reads["source"]), cfg.n_q,
                               cfg.head_dim)


def unified_attention(q, k, v, meta, kp, vp, cfg, page_tokens):
    """Scatter, tail copy, one causal paged call, quant (attention.py:878-953)."""
    u = meta["unified"]
    scale = cfg.head_dim ** -0.5
    src, dst = _t(u["src"]), _t(u["dst"])
    kp[dst], vp[dst] = k[src], v[src]
    if u["tail_src"] is not None:
        ts, td = _t(u["tail_src"]), _t(u["tail_dst"])
        kp[td], vp[td] = kp[ts].clone(), vp[ts].clone()
    rows = q.shape[0]
    out = torch.empty(rows, cfg.n_q * cfg.head_dim, dtype=torch.bfloat16)
    cu = [int(x) for x in u["cu_q"]]
    for s, (r0, r1) in enumerate(zip(cu[:-1], cu[1:])):
        used = int(u["used"][s])
        n = r1 - r0
        prow = _paged_rows(u["table"][s], used, page_tokens)
        qpos = torch.arange(n)[:, None] + (used - n)
        mask = torch.arange(used)[None, :] <= qpos
        o, _ = nx.attention_heads(q[r0:r1], kp[prow], vp[prow], cfg.n_q, cfg.n_kv, scale, mask)
        out[r0:r1] = o
    return nx.quant_groups(out.to(torch.float32))


def forward_chunk(weights, chunk, arena: CpuArena, return_hidden=False):
    """Final-normed bf16 rows of chunk.final_indices, on the CPU."""
    cfg = weights.config
    ids = _t(chunk.input_ids)
    pos = _t(chunk.positions)
    meta = chunk.meta
    tree = chunk.attention_mode == "tree"
    hidden = residual = None
    for layer_index, layer in enumerate(weights.layers):
        if layer_index == 0:
            residual, xq, xs = nx.embed_rmsnorm_quant(ids, weights.embed, layer.input_ln, cfg.eps)
        else:
            residual, xq, xs = nx.add_rmsnorm_quant(hidden, residual, layer.input_ln, cfg.eps)
        qkv = nx.gemm_fp8_bs(xq, xs, layer.qkv_w, layer.qkv_s)
        q, k, v = nx.qk_norm_rope(qkv, pos, weights.cos_sin, layer.q_norm, layer.k_norm,
                                  cfg.eps, cfg.n_q, cfg.n_kv, cfg.head_dim)
        kp, vp = arena.kv(layer_index)
        if tree:
            if meta["kv_src"] is not None:
                src, dst = _t(meta["kv_src"]), _t(meta["kv_dst"])
                kp[dst], vp[dst] = k[src], v[src]
            oq, os_ = tree_attention(q, k, v, meta, kp, vp, cfg, arena.page_tokens)
        else:
            oq, os_ = unified_attention(q, k, v, meta, kp, vp, cfg, arena.page_tokens)
        hidden = nx.gemm_fp8_bs(oq, os_, layer.o_w, layer.o_s)
        residual, gq, gs = nx.add_rmsnorm_quant(hidden, residual, layer.post_ln, cfg.eps)
        gate_up = nx.gemm_fp8_bs(gq, gs, layer.gate_up_w, layer.gate_up_s)
        dq, ds = nx.silu_mul_quant(gate_up)
        hidden = nx.gemm_fp8_bs(dq, ds, layer.down_w, layer.down_s)
    normed = nx.final_norm(hidden, residual, _t(chunk.final_indices), weights.final_norm,
                           cfg.eps)
    if return_hidden:
        return normed, hidden, residual
    return normed
