"""The Qwen3 forward pass over the B200 kernels, behind Quail's pipeline seam.

``ModelPipeline`` is Quail's contract between the chunk loop and a model
(quail/backends/quail/executor/models/base.py:11-47); ``Qwen3Pipeline``
runs the layer order of quail/backends/quail/executor/models/qwen3.py:46-77
with every op on libquailb200:

    embed + RMSNorm + quant        (layer 0)  | add + RMSNorm + quant (later)
    QKV GEMM -> q/k norm + rotary + paged KV append
    attention (tree or unified) -> fp8 o_proj input
    O GEMM -> add + RMSNorm + quant -> gate_up GEMM -> SiLU*up + quant
    -> down GEMM
    final add + RMSNorm on the answer rows only

forward_chunk returns the final-normed bf16 rows of chunk.final_indices.
"""

from quail_b200.engine import Engine


class ModelPipeline:
    """The chunk loop's view of one model family (Quail's attribute set)."""

    engine = None
    max_chunk_tokens = None
    warm_tokens = (64, 128, 256, 512, 1024, 2048)
    canvas_ids = ()
    canvas_answer_row = 0
    needs_pages = False
    tree_attention = True
    gemm_warmup = False

    def forward_chunk(self, chunk):
        raise NotImplementedError

    def linears(self):
        raise NotImplementedError


class Qwen3Pipeline(ModelPipeline):
    """Qwen3 FP8 forward passes on sm_100a kernels."""

    def __init__(self, torch, weights, arena, ue8m0=False):
        self.torch = torch
        self.weights = weights
        self.cfg = weights.config
        self.arena = arena
        # ue8m0: the UE8M0 scale mode (Engine.use_ue8m0); the weights' block
        # scales must be powers of two (model.requant_ue8m0)
        self.engine = Engine(torch, arena, self.cfg, ue8m0=ue8m0)
        self.tree_attention = True
        self.max_chunk_tokens = self.cfg.max_chunk_tokens
        self.layers = weights.layers
        # a list records every op's output of the next forward passes as
        # (layer, name, tensor); parity diagnostics only
        self.trace = None
        # the qkv GEMM carries the q/k norm, rotary and KV append when a
        # 256-column tile holds two whole heads (n_q + 2 n_kv even)
        self.fused_qkv = self.cfg.head_dim == 128 and (self.cfg.n_q + 2 * self.cfg.n_kv) % 2 == 0

    def linears(self):
        layer = self.layers[0]
        return ((layer.qkv_w, layer.qkv_s), (layer.o_w, layer.o_s),
                (layer.gate_up_w, layer.gate_up_s), (layer.down_w, layer.down_s))

    def forward_chunk(self, chunk):
        eng = self.engine
        w = self.weights
        meta = chunk.meta
        meta["layer"] = 0
        rows = chunk.tokens
        tree = chunk.attention_mode == "tree"
        row_dst = None
        if tree and meta["kv_src"] is not None and meta["kv_src"].numel():
            row_dst = eng.kv_row_map(meta["kv_src"], meta["kv_dst"], rows)
        hidden = None
        residual = None
        trace = self.trace
        for index, layer in enumerate(self.layers):
            if index == 0:
                residual, x = eng.embed_norm_quant(chunk.input_ids, w.embed, layer.input_ln)
            else:
                if trace is not None:
                    trace.append((index, "residual_in", residual.clone()))
                x = eng.norm_quant(hidden, layer.input_ln, residual)
            if self.fused_qkv:
                # qkv GEMM + q/k norm + rotary + KV append in one kernel
                q, k, v = eng.gemm_qknorm_rope(x, layer.qkv_w, layer.qkv_s, chunk.positions,
                                               w.cos_sin, layer.q_norm, layer.k_norm,
                                               meta["layer"], row_dst)
                qkv = None
                if trace is not None:
                    # the bf16 qkv the fused kernel never writes, for the trace
                    qkv = eng.gemm(x, layer.qkv_w, layer.qkv_s)
            else:
                qkv = eng.gemm(x, layer.qkv_w, layer.qkv_s)
                q, k, v = eng.qk_norm_rope(qkv, chunk.positions, w.cos_sin, layer.q_norm,
                                           layer.k_norm, meta["layer"], row_dst)
            if tree:
                o_in = eng.attention_tree(q, k, v, meta)
            else:
                o_in = eng.attention_unified(q, k, v, meta)
            hidden = eng.gemm(o_in, layer.o_w, layer.o_s)
            if trace is not None:
                trace.extend([(index, "x", x), (index, "qkv", qkv), (index, "q", q),
                              (index, "k", k), (index, "v", v), (index, "o_in", o_in),
                              (index, "o", hidden), (index, "residual_mid_in",
                                                     residual.clone())])
            x = eng.norm_quant(hidden, layer.post_ln, residual)
            # gate_up GEMM + SiLU quantisation in one kernel
            x2 = eng.gemm_silu_quant(x, layer.gate_up_w, layer.gate_up_s)
            hidden = eng.gemm(x2, layer.down_w, layer.down_s)
            if trace is not None:
                # the bf16 gate_up the fused kernel never writes, for the trace
                gate_up = eng.gemm(x, layer.gate_up_w, layer.gate_up_s)
                trace.extend([(index, "g_in", x), (index, "gate_up", gate_up),
                              (index, "d_in", x2), (index, "down", hidden)])
        return eng.final_norm(hidden, residual, chunk.final_indices, w.final_norm)


def build_pipeline(torch, weights, arena, ue8m0=False):
    """The pipeline for weights.config (Quail's build_pipeline seam)."""
    return Qwen3Pipeline(torch, weights, arena, ue8m0=ue8m0)
