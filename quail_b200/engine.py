"""Torch-facing wrappers of the sm_100a kernels: one method per fused op.

Engine mirrors the primitives Quail's forward loop calls
(quail/backends/quail/executor/attention.py:84-953): norm_quant, gemm,
qk_norm_rope, attention (tree or unified) and activation_quant, plus the
final norm. Every method launches libquailb200 kernels on the current CUDA
stream; tensors are allocated by torch's caching allocator and passed down
as raw pointers. There is no fallback: a missing library raises on import
of quail_b200._native.load().
"""

from quail_b200 import _native as nat

GROUP = 128


class QuantRows:
    """fp8 rows plus their group-major scales: scale[g * ld + row]."""

    __slots__ = ("q", "scale", "ld")

    def __init__(self, q, scale, ld):
        self.q = q
        self.scale = scale
        self.ld = ld


class Engine:
    """Kernels, quantisation and attention over the paged arena.

    Args:
        torch: the torch module.
        arena: KVArena the attention reads and the KV append writes.
        cfg: ModelConfig of the loaded weights.
        ue8m0: the reference's UE8M0 scale mode (Engine.use_ue8m0, from
            vLLM's is_deep_gemm_e8m0_used; quail/backends/quail/executor/
            attention.py:115): power-of-two activation scales from every
            quantiser, and GEMMs on the block-scaled MMA. The weights'
            scales must then be powers of two (model.requant_ue8m0).
    """

    def __init__(self, torch, arena, cfg, ue8m0=False):
        self.torch = torch
        self.arena = arena
        self.cfg = cfg
        self.use_ue8m0 = bool(ue8m0)
        self.num_q_heads = cfg.n_q
        self.num_kv_heads = cfg.n_kv
        self.head_dim = cfg.head_dim
        self.softmax_scale = cfg.head_dim ** -0.5
        # a list turns on per-launch CUDA events around every GEMM:
        # (start, end, flops, algorithmic bytes) tuples, read by bench.py's
        # roofline
        self.gemm_events = None
        nat.load()

    def _stream(self):
        return nat.stream_handle(self.torch)

    def _quant_buffers(self, rows, width):
        t = self.torch
        q = t.empty((rows, width), dtype=t.float8_e4m3fn, device="cuda")
        scale = t.empty((width // GROUP, max(rows, 1)), dtype=t.float32, device="cuda")
        return QuantRows(q, scale, max(rows, 1))

    # ---- norms and quantisation ---------------------------------------------

    def embed_norm_quant(self, ids, embed, norm_w):
        """Layer 0: (residual = embed[ids], quantised RMSNorm of it)."""
        t = self.torch
        rows, h = ids.shape[0], embed.shape[1]
        residual = t.empty((rows, h), dtype=t.bfloat16, device="cuda")
        out = self._quant_buffers(rows, h)
        nat.call("qb_embed_rmsnorm_quant", nat.ptr(ids), rows, nat.ptr(embed), embed.shape[0],
                 h, nat.ptr(norm_w), self.cfg.eps, nat.ptr(residual), nat.ptr(out.q),
                 nat.ptr(out.scale), out.ld, int(self.use_ue8m0), self._stream())
        return residual, out

    def norm_quant(self, hidden, norm_w, residual):
        """residual += hidden (bf16 store); quantised RMSNorm of the sum."""
        rows, h = hidden.shape
        out = self._quant_buffers(rows, h)
        nat.call("qb_add_rmsnorm_quant", nat.ptr(hidden), nat.ptr(residual), nat.ptr(norm_w),
                 self.cfg.eps, rows, h, nat.ptr(out.q), nat.ptr(out.scale), out.ld,
                 int(self.use_ue8m0), self._stream())
        return out

    def activation_quant(self, gate_up):
        """silu(gate) * up, quantised."""
        rows, two_i = gate_up.shape
        out = self._quant_buffers(rows, two_i // 2)
        nat.call("qb_silu_mul_quant", nat.ptr(gate_up), rows, two_i // 2, nat.ptr(out.q),
                 nat.ptr(out.scale), out.ld, int(self.use_ue8m0), self._stream())
        return out

    # ---- GEMM ------------------------------------------------------------------

    def gemm(self, x: QuantRows, weight, weight_scale):
        t = self.torch
        m, k = x.q.shape
        n = weight.shape[0]
        out = t.empty((m, n), dtype=t.bfloat16, device="cuda")
        timed = self.gemm_events is not None
        if timed:
            start, end = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
            start.record()
        nat.call("qb_gemm_fp8_bs", nat.ptr(x.q), nat.ptr(x.scale), x.ld, nat.ptr(weight),
                 nat.ptr(weight_scale), nat.ptr(out), m, n, k, int(self.use_ue8m0),
                 self._stream())
        if timed:
            end.record()
            # algorithmic bytes: A and W once, C once, both scale arrays
            nbytes = m * k + n * k + 2 * m * n + 4 * (m * (k // 128) + (n // 128) * (k // 128))
            self.gemm_events.append((start, end, 2.0 * m * n * k, nbytes))
        return out

    def gemm_silu_quant(self, x: QuantRows, weight, weight_scale):
        """activation_quant(gemm(x, gate_up)) in one kernel: the quantised
        silu(gate) * up, without the bf16 gate_up intermediate."""
        t = self.torch
        m, k = x.q.shape
        inter = weight.shape[0] // 2
        out = self._quant_buffers(m, inter)
        timed = self.gemm_events is not None
        if timed:
            start, end = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
            start.record()
        nat.call("qb_gemm_fp8_silu_quant", nat.ptr(x.q), nat.ptr(x.scale), x.ld,
                 nat.ptr(weight), nat.ptr(weight_scale), nat.ptr(out.q), nat.ptr(out.scale),
                 out.ld, m, inter, k, int(self.use_ue8m0), self._stream())
        if timed:
            end.record()
            n = 2 * inter
            # A and W once, the fp8 product and its scales once, both input scales
            nbytes = (m * k + n * k + m * inter + 4 * m * (inter // 128)
                      + 4 * (m * (k // 128) + (n // 128) * (k // 128)))
            self.gemm_events.append((start, end, 2.0 * m * n * k, nbytes))
        return out

    # ---- rotary + KV append -------------------------------------------------

    def kv_row_map(self, kv_src, kv_dst, rows):
        """Per-row arena destination (-1: not written) of the tree KV append."""
        t = self.torch
        row_dst = t.empty(max(rows, 1), dtype=t.int64, device="cuda")
        nat.call("qb_kv_row_map", nat.ptr(kv_src), nat.ptr(kv_dst), kv_src.shape[0], rows,
                 self.arena.pool_rows, nat.ptr(row_dst), self._stream())
        return row_dst

    def qk_norm_rope(self, qkv, positions, cos_sin, q_w, k_w, layer, row_dst=None):
        """(q, k, v) after per-head norm and rotary; appends KV where row_dst >= 0."""
        t = self.torch
        cfg = self.cfg
        rows = qkv.shape[0]
        q = t.empty((rows, cfg.n_q * cfg.head_dim), dtype=t.bfloat16, device="cuda")
        k = t.empty((rows, cfg.n_kv * cfg.head_dim), dtype=t.bfloat16, device="cuda")
        v = t.empty_like(k)
        kp = vp = None
        if row_dst is not None:
            kp, vp = self.arena.layer_kv(layer)
        nat.call("qb_qknorm_rope", nat.ptr(qkv), qkv.stride(0), nat.ptr(positions),
                 nat.ptr(cos_sin), cos_sin.shape[0], nat.ptr(q_w), nat.ptr(k_w), cfg.eps, rows,
                 cfg.n_q, cfg.n_kv, cfg.head_dim, nat.ptr(q), nat.ptr(k), nat.ptr(v),
                 nat.ptr(row_dst), nat.ptr(kp), nat.ptr(vp), self.arena.pool_rows,
                 self._stream())
        return q, k, v

    def gemm_qknorm_rope(self, x: QuantRows, weight, weight_scale, positions, cos_sin, q_w, k_w,
                         layer, row_dst=None):
        """qk_norm_rope(gemm(x, qkv)) in one kernel: (q, k, v), KV appended
        where row_dst >= 0; the bf16 qkv intermediate is never written."""
        t = self.torch
        cfg = self.cfg
        m, k_dim = x.q.shape
        q = t.empty((m, cfg.n_q * cfg.head_dim), dtype=t.bfloat16, device="cuda")
        k = t.empty((m, cfg.n_kv * cfg.head_dim), dtype=t.bfloat16, device="cuda")
        v = t.empty_like(k)
        kp = vp = None
        if row_dst is not None:
            kp, vp = self.arena.layer_kv(layer)
        timed = self.gemm_events is not None
        if timed:
            start, end = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
            start.record()
        nat.call("qb_gemm_fp8_qknorm_rope", nat.ptr(x.q), nat.ptr(x.scale), x.ld, nat.ptr(weight),
                 nat.ptr(weight_scale), m, k_dim, nat.ptr(positions), nat.ptr(cos_sin),
                 cos_sin.shape[0], nat.ptr(q_w), nat.ptr(k_w), cfg.eps, cfg.n_q, cfg.n_kv,
                 cfg.head_dim, nat.ptr(q), nat.ptr(k), nat.ptr(v), nat.ptr(row_dst), nat.ptr(kp),
                 nat.ptr(vp), self.arena.pool_rows, int(self.use_ue8m0), self._stream())
        if timed:
            end.record()
            n = weight.shape[0]
            # A and W once, q/k/v once, both scale arrays (the pool copy aside)
            nbytes = m * k_dim + n * k_dim + 2 * m * n + 4 * (m * (k_dim // 128)
                                                            + (n // 128) * (k_dim // 128))
            self.gemm_events.append((start, end, 2.0 * m * n * k_dim, nbytes))
        return q, k, v

    def kv_scatter(self, src_k, src_v, src, dst, layer, src_rows):
        kp, vp = self.arena.layer_kv(layer)
        row = self.cfg.n_kv * self.cfg.head_dim
        nat.call("qb_kv_scatter", nat.ptr(src_k), nat.ptr(src_v), nat.ptr(src), nat.ptr(dst),
                 src.shape[0], row, src_rows, nat.ptr(kp), nat.ptr(vp), self.arena.pool_rows,
                 self._stream())

    # ---- attention ---------------------------------------------------------------

    def attention_tree(self, q, k, v, meta):
        """Tree path: causal own segment + resident reads, merged and quantised."""
        cfg = self.cfg
        rows = q.shape[0]
        layer = meta["layer"]
        out = self._quant_buffers(rows, cfg.n_q * cfg.head_dim)
        reads = meta["reads"]
        kp, vp = self.arena.layer_kv(layer)
        tiles = meta["tiles"]
        if reads is not None:
            table = reads["table"]
            args = (nat.ptr(reads["cu_q"]), nat.ptr(reads["used"]), nat.ptr(table),
                    table.shape[0], table.shape[1], nat.ptr(reads["source"]))
        else:
            args = (None, None, None, 0, 0, None)
        nat.call("qb_tree_attention", nat.ptr(q), nat.ptr(k), nat.ptr(v), rows, cfg.n_q,
                 cfg.n_kv, cfg.head_dim, nat.ptr(meta["cu_a"]), meta["cu_a"].shape[0] - 1,
                 nat.ptr(tiles), tiles.shape[0], *args, nat.ptr(kp), nat.ptr(vp),
                 self.arena.n_pages, self.arena.page_tokens, self.softmax_scale,
                 nat.ptr(out.q), nat.ptr(out.scale), out.ld, int(self.use_ue8m0),
                 self._stream())
        meta["layer"] += 1
        return out

    def attention_unified(self, q, k, v, meta):
        """Unified path: scatter current KV, one causal paged call, quantised."""
        cfg = self.cfg
        rows = q.shape[0]
        layer = meta["layer"]
        u = meta["unified"]
        if u is None:
            raise ValueError("the B200 unified path needs arena pages")
        if u["src"].numel():
            self.kv_scatter(k, v, u["src"], u["dst"], layer, rows)
        if u["tail_src"] is not None:
            kp, vp = self.arena.layer_kv(layer)
            self.kv_scatter(kp, vp, u["tail_src"], u["tail_dst"], layer, self.arena.pool_rows)
        out = self._quant_buffers(rows, cfg.n_q * cfg.head_dim)
        kp, vp = self.arena.layer_kv(layer)
        table, tiles = u["table"], u["tiles"]
        nat.call("qb_unified_attention", nat.ptr(q), rows, cfg.n_q, cfg.n_kv, cfg.head_dim,
                 nat.ptr(u["cu_q"]), u["cu_q"].shape[0] - 1, nat.ptr(tiles), tiles.shape[0],
                 nat.ptr(u["used"]), nat.ptr(table), table.shape[1], nat.ptr(kp), nat.ptr(vp),
                 self.arena.n_pages, self.arena.page_tokens, self.softmax_scale,
                 nat.ptr(out.q), nat.ptr(out.scale), out.ld, int(self.use_ue8m0),
                 self._stream())
        meta["layer"] += 1
        return out

    # ---- the end of the pass -------------------------------------------------------

    def final_norm(self, hidden, residual, finals, weight):
        t = self.torch
        n = finals.shape[0]
        h = hidden.shape[1]
        normed = t.empty((n, h), dtype=t.bfloat16, device="cuda")
        nat.call("qb_final_norm", nat.ptr(hidden), nat.ptr(residual), hidden.shape[0], h,
                 nat.ptr(finals), n, nat.ptr(weight), self.cfg.eps, nat.ptr(normed),
                 self._stream())
        return normed
