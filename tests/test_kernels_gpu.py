"""Per-kernel parity on the GPU: each libquailb200 entry point, called
through the C ABI, against the CPU oracle on the same seeded inputs.

The bar is bit equality. The kernels fix every rounding step (explicit
__f*_rn operations, one summation order per reduction, FMA-only exp2 / ln)
and the oracle (oracle/numerics.py in exact mode, oracle/tcmodel.c)
restates those steps, with tensor-core products under the accumulation
model measured on the B200 (tests/test_oracle_model.py). So fp8 codes,
scales, bf16 outputs, KV pool rows and margins must match bit for bit.
"""

import dataclasses

import numpy as np
import pytest
import torch

from oracle import forward as of
from oracle import numerics as nx
from quail_b200 import _native as nat
from quail_b200 import loop
from quail_b200.arena import KVArena
from quail_b200.engine import Engine, QuantRows
from quail_b200.model import TINY, random_weights
from quail_b200.tokens import prefix_tree

pytestmark = pytest.mark.gpu


def bits(t):
    t = t.detach().cpu().contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


def assert_bits_equal(got, want, what=""):
    g, w = bits(got), bits(want)
    assert g.shape == w.shape, (what, g.shape, w.shape)
    diff = int((g != w).sum())
    assert diff == 0, f"{what}: {diff} of {g.numel()} elements differ"


def codes_close(got, want, **_):
    assert_bits_equal(got, want, "fp8 codes")


def fp8_rows_close(q_got, s_got, q_ref, s_ref, **_):
    assert_bits_equal(s_got, s_ref, "scales")
    assert_bits_equal(q_got, q_ref, "fp8 codes")


def bf16_close(got, want, **_):
    assert_bits_equal(got, want, "bf16")


@pytest.fixture(scope="module")
def dev():
    torch.manual_seed(0)
    return torch.device("cuda")


def assert_status_clean():
    assert nat.kernel_status(torch.cuda.current_device()) == 0


class _Arena:
    pool_rows = 64


def engine_for(cfg, arena=None):
    return Engine(torch, arena or _Arena(), cfg)


@pytest.mark.parametrize("rows,hidden", [(1, 512), (37, 512), (300, 2560)])
def test_embed_rmsnorm_quant(dev, rows, hidden):
    g = torch.Generator().manual_seed(rows)
    embed = (0.02 * torch.randn(1000, hidden, generator=g)).to(torch.bfloat16)
    w = (1 + 0.05 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    ids = torch.randint(0, 1000, (rows,), generator=g)
    cfg = TINY
    eng = engine_for(cfg)
    res, out = eng.embed_norm_quant(ids.to(dev), embed.to(dev), w.to(dev))
    r_ref, q_ref, s_ref = nx.embed_rmsnorm_quant(ids, embed, w, cfg.eps)
    assert torch.equal(res.cpu().view(torch.int16), r_ref.view(torch.int16))
    codes_close(out.q, q_ref)
    assert_bits_equal(out.scale[:, :rows], s_ref, "scales")
    assert_status_clean()


@pytest.mark.parametrize("rows,hidden", [(1, 512), (77, 2560), (5, 5120)])
def test_add_rmsnorm_quant(dev, rows, hidden):
    g = torch.Generator().manual_seed(hidden + rows)
    x = (2 * torch.randn(rows, hidden, generator=g)).to(torch.bfloat16)
    r = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    eng = engine_for(TINY)
    r_dev = r.to(dev)
    out = eng.norm_quant(x.to(dev), w.to(dev), r_dev)
    r_ref, q_ref, s_ref = nx.add_rmsnorm_quant(x, r, w, TINY.eps)
    assert torch.equal(r_dev.cpu().view(torch.int16), r_ref.view(torch.int16))
    codes_close(out.q, q_ref)
    assert_bits_equal(out.scale[:, :rows], s_ref, "scales")


@pytest.mark.parametrize("rows,inter", [(3, 1024), (129, 9728)])
def test_silu_mul_quant(dev, rows, inter):
    g = torch.Generator().manual_seed(inter)
    gu = (3 * torch.randn(rows, 2 * inter, generator=g)).to(torch.bfloat16)
    eng = engine_for(TINY)
    out = eng.activation_quant(gu.to(dev))
    q_ref, s_ref = nx.silu_mul_quant(gu)
    codes_close(out.q, q_ref, max_frac=0.003)
    assert_bits_equal(out.scale[:, :rows], s_ref, "scales")


def _fp8_operands(g, m, n, k):
    a = torch.randn(m, k, generator=g) * (1 + torch.rand(m, 1, generator=g))
    aq, as_ = nx.quant_groups(a)
    wq = torch.randn(n, k, generator=g).to(torch.float8_e4m3fn)
    ws = torch.exp(np.log(0.02) + 0.3 * torch.randn(n // 128, k // 128, generator=g))
    return aq, as_, wq, ws


@pytest.mark.parametrize("m,n,k", [(1, 256, 256), (7, 384, 512), (128, 256, 128),
                                   (300, 1024, 2560), (257, 2560, 4096), (1000, 512, 9728)])
def test_gemm_fp8_block_scaled(dev, m, n, k):
    g = torch.Generator().manual_seed(m * 7 + n + k)
    aq, as_, wq, ws = _fp8_operands(g, m, n, k)
    eng = engine_for(TINY)
    x = QuantRows(aq.to(dev), as_.to(dev).contiguous(), m)
    out = eng.gemm(x, wq.to(dev), ws.to(dev))
    torch.cuda.synchronize()
    ref = nx.gemm_fp8_bs(aq, as_, wq, ws)
    bf16_close(out, ref, ulps=1)
    assert_status_clean()


@pytest.mark.parametrize("m,inter,k,oracle", [(1, 128, 256, True), (7, 384, 512, True),
                                              (300, 1024, 2560, True), (257, 9728, 2560, False),
                                              (4096 + 5, 2048, 256, False)])
def test_gemm_silu_quant(dev, m, inter, k, oracle):
    """gate_up GEMM + SiLU quantisation in one kernel: the same fp8 codes and
    scales as the bf16 GEMM followed by qb_silu_mul_quant (and the oracle)."""
    g = torch.Generator().manual_seed(m + inter + k)
    aq, as_, wq, ws = _fp8_operands(g, m, 2 * inter, k)
    eng = engine_for(TINY)
    x = QuantRows(aq.to(dev), as_.to(dev).contiguous(), m)
    out = eng.gemm_silu_quant(x, wq.to(dev), ws.to(dev))
    torch.cuda.synchronize()
    assert_status_clean()
    if oracle:
        q_ref, s_ref = nx.silu_mul_quant(nx.gemm_fp8_bs(aq, as_, wq, ws))
        assert_bits_equal(out.scale[:, :m], s_ref, "scales")
        assert_bits_equal(out.q, q_ref, "fp8 codes")
    if inter % 256 == 0:
        ref = eng.activation_quant(eng.gemm(x, wq.to(dev), ws.to(dev)))
        assert_bits_equal(out.scale[:, :m], ref.scale[:, :m], "scales vs unfused")
        assert_bits_equal(out.q, ref.q, "fp8 codes vs unfused")


@pytest.mark.parametrize("cfg_name,m,runs", [("tiny", 1, False), ("tiny", 300, False),
                                             ("tiny", 300, True), ("mixed", 300, True),
                                             ("4b", 517, False), ("4b", 517, True),
                                             ("32b", 130, True)])
def test_gemm_qknorm_rope_matches_unfused(dev, cfg_name, m, runs):
    """qkv GEMM + q/k norm + rotary + KV append in one kernel: the same q, k,
    v and pool rows, bit for bit, as qb_gemm_fp8_bs then qb_qknorm_rope.
    runs: KV destinations in consecutive runs (two of them, the second from
    a row that is not a multiple of 32: box stores and per-row stores) instead
    of every other row at random. mixed: 6 q and 3 kv heads, so one tile
    holds the last k head and the first v head."""
    from quail_b200.model import QWEN3_4B, QWEN3_32B, rotary_cache
    cfg = {"tiny": TINY, "4b": QWEN3_4B, "32b": QWEN3_32B,
           "mixed": dataclasses.replace(TINY, n_q=6, n_kv=3)}[cfg_name]
    g = torch.Generator().manual_seed(m + cfg.hidden)
    n = (cfg.n_q + 2 * cfg.n_kv) * cfg.head_dim
    aq, as_, wq, ws = _fp8_operands(g, m, n, cfg.hidden)
    x = QuantRows(aq.to(dev), as_.to(dev).contiguous(), m)
    pos = torch.randint(0, 4000, (m,), generator=g).to(dev)
    cos_sin = rotary_cache(cfg, dev)
    qw = (1 + 0.1 * torch.randn(cfg.head_dim, generator=g)).to(torch.bfloat16).to(dev)
    kw = (1 + 0.1 * torch.randn(cfg.head_dim, generator=g)).to(torch.bfloat16).to(dev)
    pool_rows = 2 * m + 16
    arenas = [KVArena(1, (pool_rows + 15) // 16, 16, cfg.n_kv, cfg.head_dim, device=dev)
              for _ in range(2)]
    for a in arenas:
        a.pools.zero_()
    row_dst = torch.full((m,), -1, dtype=torch.int64)
    if runs:
        cut = (m * 2) // 3 + 5
        row_dst[:cut] = 3 + torch.arange(cut)
        row_dst[cut:] = m + 8 + torch.arange(m - cut)
    else:
        row_dst[::2] = torch.randperm(arenas[0].pool_rows, generator=g)[: (m + 1) // 2]
    assert int(row_dst.max()) < arenas[0].pool_rows
    row_dst = row_dst.to(dev)
    eng_f = Engine(torch, arenas[0], cfg)
    q_f, k_f, v_f = eng_f.gemm_qknorm_rope(x, wq.to(dev), ws.to(dev), pos, cos_sin, qw, kw, 0,
                                           row_dst)
    eng_u = Engine(torch, arenas[1], cfg)
    qkv = eng_u.gemm(x, wq.to(dev), ws.to(dev))
    q_u, k_u, v_u = eng_u.qk_norm_rope(qkv, pos, cos_sin, qw, kw, 0, row_dst)
    torch.cuda.synchronize()
    assert_status_clean()
    assert_bits_equal(q_f, q_u, "q")
    assert_bits_equal(k_f, k_u, "k")
    assert_bits_equal(v_f, v_u, "v")
    assert_bits_equal(arenas[0].pools, arenas[1].pools, "KV pools")


def test_gemm_qknorm_rope_bad_indices_flag_like_unfused(dev):
    """A position past the rotary cache and a KV destination past the pool:
    the fused kernel flags STATUS_BAD_INDEX, reads cos/sin row 0 and skips
    the append, as qb_qknorm_rope does; every output equals the pair's."""
    cfg = TINY
    m = 96
    g = torch.Generator().manual_seed(41)
    n = (cfg.n_q + 2 * cfg.n_kv) * cfg.head_dim
    aq, as_, wq, ws = _fp8_operands(g, m, n, cfg.hidden)
    x = QuantRows(aq.to(dev), as_.to(dev).contiguous(), m)
    from quail_b200.model import rotary_cache
    cos_sin = rotary_cache(cfg, dev)
    pos = torch.randint(0, 100, (m,), generator=g)
    pos[5] = cos_sin.shape[0]
    pos = pos.to(dev)
    qw = torch.ones(cfg.head_dim, dtype=torch.bfloat16, device=dev)
    arenas = [KVArena(1, 16, 16, cfg.n_kv, cfg.head_dim, device=dev) for _ in range(2)]
    for a in arenas:
        a.pools.zero_()
    row_dst = torch.arange(m, dtype=torch.int64)
    row_dst[37] = arenas[0].pool_rows + 3
    row_dst = row_dst.to(dev)
    out = []
    for fused, arena in ((True, arenas[0]), (False, arenas[1])):
        eng = Engine(torch, arena, cfg)
        assert_status_clean()
        if fused:
            q, k, v = eng.gemm_qknorm_rope(x, wq.to(dev), ws.to(dev), pos, cos_sin, qw, qw, 0,
                                           row_dst)
        else:
            qkv = eng.gemm(x, wq.to(dev), ws.to(dev))
            q, k, v = eng.qk_norm_rope(qkv, pos, cos_sin, qw, qw, 0, row_dst)
        torch.cuda.synchronize()
        assert nat.kernel_status(torch.cuda.current_device()) == 1 << 9  # STATUS_BAD_INDEX
        out.append((q, k, v))
    for (name, a), b in zip((("q", out[0][0]), ("k", out[0][1]), ("v", out[0][2])), out[1]):
        assert_bits_equal(a, b, name)
    assert_bits_equal(arenas[0].pools, arenas[1].pools, "KV pools")


def test_gemm_large_against_dequantised_matmul(dev):
    """A full 4B QKV-shaped GEMM against fp32 torch on the dequantised operands."""
    g = torch.Generator(device="cuda").manual_seed(5)
    m, n, k = 4096 + 77, 6144, 2560
    a = torch.randn(m, k, device=dev, generator=g)
    g2 = torch.Generator().manual_seed(6)
    aq, as_ = nx.quant_groups(a.cpu())
    wq = torch.randn(n, k, generator=g2).to(torch.float8_e4m3fn)
    ws = torch.exp(np.log(0.02) + 0.3 * torch.randn(n // 128, k // 128, generator=g2))
    eng = engine_for(TINY)
    out = eng.gemm(QuantRows(aq.to(dev), as_.to(dev), m), wq.to(dev), ws.to(dev))
    a_deq = nx.dequant(aq, as_).to(dev)
    w_deq = (wq.float() * ws.repeat_interleave(128, 0).repeat_interleave(128, 1)).to(dev)
    ref = (a_deq @ w_deq.t())
    err = (out.float() - ref).abs()
    assert float((err / (ref.abs() + 1e-2 * ref.abs().mean())).max()) < 0.02
    assert float(err.mean() / ref.abs().mean()) < 2e-3
    assert_status_clean()


def test_qk_norm_rope_and_kv_append(dev):
    cfg = TINY
    rows = 50
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(rows, cfg.qkv_width, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (rows,), generator=g)
    w = random_weights(cfg, seed=1, device="cpu")
    qw, kw = w.layers[0].q_norm, w.layers[0].k_norm
    arena = KVArena(cfg.n_layers, 16, 16, cfg.n_kv, cfg.head_dim, device=dev)
    arena.pools.zero_()
    eng = Engine(torch, arena, cfg)
    src = torch.tensor([0, 5, 7, 49], dtype=torch.int64)
    dst = torch.tensor([3, 200, 0, 255], dtype=torch.int64)
    row_dst = eng.kv_row_map(src.to(dev), dst.to(dev), rows)
    q, k, v = eng.qk_norm_rope(qkv.to(dev), pos.to(dev), w.cos_sin.to(dev), qw.to(dev),
                               kw.to(dev), 1, row_dst)
    q_ref, k_ref, v_ref = nx.qk_norm_rope(qkv, pos, w.cos_sin, qw, kw, cfg.eps, cfg.n_q,
                                          cfg.n_kv)
    assert_bits_equal(q, q_ref, "q")
    assert_bits_equal(k, k_ref, "k")
    assert_bits_equal(v, v_ref, "v")
    kp, vp = arena.layer_kv(1)
    kp = kp.reshape(-1, cfg.n_kv * cfg.head_dim).cpu()
    vp = vp.reshape(-1, cfg.n_kv * cfg.head_dim).cpu()
    assert torch.equal(kp[dst], k.cpu()[src])
    assert torch.equal(vp[dst], v.cpu()[src])
    untouched = torch.ones(kp.shape[0], dtype=torch.bool)
    untouched[dst] = False
    assert int(kp[untouched].abs().sum()) == 0
    assert_status_clean()


# GQA groups of 2 and 4 (one and two 128-row M tiles) and 8 (Qwen3-32B's
# grouping: 64 query heads over 8 KV heads); the tcgen05 kernel takes even
# groups only (every Qwen3 shape), an odd one is rejected before launch
ATTN_CONFIGS = {"g2": TINY, "g4": dataclasses.replace(TINY, name="tiny-g4", n_q=8),
                "g8": dataclasses.replace(TINY, name="tiny-g8", n_q=16, n_kv=2)}


def test_attention_rejects_odd_gqa_groups(dev):
    cfg = dataclasses.replace(TINY, name="tiny-g3", n_q=3, n_kv=1)
    _, arena, chunks = _attention_case("tree", dev, cfg=cfg)
    eng = Engine(torch, arena, cfg)
    chunk = chunks[0]
    rows = chunk.tokens
    q = torch.zeros(rows, cfg.n_q * cfg.head_dim, device=dev, dtype=torch.bfloat16)
    kv = torch.zeros(rows, cfg.n_kv * cfg.head_dim, device=dev, dtype=torch.bfloat16)
    chunk.meta["layer"] = 0
    with pytest.raises(ValueError, match="query heads per KV head"):
        eng.attention_tree(q, kv, kv, chunk.meta)
    assert_status_clean()


def _attention_case(mode, dev, seed=0, cfg=TINY, long=False):
    """A packed chunk (our packer) with random q/k/v and random resident KV.
    long: two documents past a thousand tokens (config 4's regime: many key
    tiles per query tile, query tiles deep into a causal segment)."""
    rng = np.random.default_rng(seed)
    prefix = rng.integers(1000, 2000, 64).tolist()
    lens = rng.integers(1, 150, 4 if long else 12)
    docs = [prefix + rng.integers(1000, 2000, int(n)).tolist() for n in lens]
    docs.append(prefix + rng.integers(1000, 2000, 300).tolist())
    if long:
        docs += [prefix + rng.integers(1000, 2000, n).tolist() for n in (1200, 700)]
    arena = KVArena(cfg.n_layers, 200, 16, cfg.n_kv, cfg.head_dim, device=dev)
    g = torch.Generator(device="cuda").manual_seed(seed)
    arena.pools.copy_(torch.randn(arena.pools.shape, device=dev, generator=g))
    chunks = []

    class Capture:
        tree_attention = True

        def forward_chunk(self, chunk):
            chunks.append(chunk)
            return chunk

    class Answers:
        def submit(self, chunk):
            return [1] * len(chunk.layout)

        def result(self, h):
            return h

    # two stages so the second chunk has kept groups reading their own pages
    loop.run_filter(torch, arena, Capture(), Answers(), docs, [[7, 8], [7, 9, 9]], 3000,
                    arena_writes=True, attention_mode=mode, prefix_tree=prefix_tree(docs, 16),
                    device=dev)
    return cfg, arena, chunks


@pytest.mark.parametrize("case", sorted(ATTN_CONFIGS) + ["long"])
@pytest.mark.parametrize("mode", ["tree", "unified"])
def test_attention_against_oracle(dev, mode, case):
    cfg, arena, chunks = _attention_case(mode, dev, cfg=ATTN_CONFIGS.get(case, TINY),
                                         long=case == "long")
    eng = Engine(torch, arena, cfg)
    scale = cfg.head_dim ** -0.5
    checked = 0
    for chunk in chunks:
        rows = chunk.tokens
        g = torch.Generator(device="cuda").manual_seed(rows)
        q = torch.randn(rows, cfg.n_q * cfg.head_dim, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(rows, cfg.n_kv * cfg.head_dim, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(rows, cfg.n_kv * cfg.head_dim, device=dev, generator=g).to(torch.bfloat16)
        meta = chunk.meta
        meta["layer"] = 0
        kp, vp = arena.layer_kv(0)
        kp2 = kp.reshape(-1, cfg.n_kv * cfg.head_dim)
        vp2 = vp.reshape(-1, cfg.n_kv * cfg.head_dim)
        host = chunk.host
        if mode == "tree":
            if meta["kv_src"] is not None:
                kp2[meta["kv_dst"]] = k[meta["kv_src"]]
                vp2[meta["kv_dst"]] = v[meta["kv_src"]]
            kp_ref, vp_ref = kp2.cpu().clone(), vp2.cpu().clone()
            out = eng.attention_tree(q, k, v, meta)
            q_ref, s_ref = of.tree_attention(q.cpu(), k.cpu(), v.cpu(), host.meta, kp_ref,
                                             vp_ref, cfg, arena.page_tokens)
        else:
            kp_ref, vp_ref = kp2.cpu().clone(), vp2.cpu().clone()
            out = eng.attention_unified(q, k, v, meta)
            q_ref, s_ref = of.unified_attention(q.cpu(), k.cpu(), v.cpu(), host.meta, kp_ref,
                                                vp_ref, cfg, arena.page_tokens)
            assert torch.equal(kp2.cpu(), kp_ref) and torch.equal(vp2.cpu(), vp_ref)
        torch.cuda.synchronize()
        fp8_rows_close(out.q, out.scale[:, :rows], q_ref, s_ref)
        checked += 1
        assert scale > 0
    assert checked >= 2
    assert_status_clean()


def test_final_norm_and_answer_margin(dev):
    cfg = TINY
    g = torch.Generator().manual_seed(11)
    rows = 40
    hidden = torch.randn(rows, cfg.hidden, generator=g).to(torch.bfloat16)
    residual = torch.randn(rows, cfg.hidden, generator=g).to(torch.bfloat16)
    finals = torch.tensor([3, 0, 39, 17], dtype=torch.int64)
    w = random_weights(cfg, seed=2, device="cpu")
    eng = engine_for(cfg)
    normed = eng.final_norm(hidden.to(dev), residual.to(dev), finals.to(dev),
                            w.final_norm.to(dev))
    ref = nx.final_norm(hidden, residual, finals, w.final_norm, cfg.eps)
    assert_bits_equal(normed, ref, "normed")
    from quail_b200.readout import AnswerRows
    wd = w.to(dev)
    rows_obj = AnswerRows(torch, wd)
    margin, bits = rows_obj.margins(normed)
    allowed, ans_w, tc, fc = w.answer_rows()
    m_ref, b_ref = nx.answer_margin(normed.cpu(), ans_w, tc, fc)
    assert_bits_equal(margin, m_ref, "margins")
    assert_bits_equal(bits, b_ref, "bits")
    assert_status_clean()


def test_answer_score_readout(dev):
    """AI.SCORE: fp32 yes/no logits and sigmoid, through AsyncScores, against
    the oracle bit for bit and torch's fp32 sigmoid within float tolerance."""
    cfg = TINY
    g = torch.Generator().manual_seed(12)
    rows = 57
    normed = torch.randn(rows, cfg.hidden, generator=g).to(torch.bfloat16)
    w = random_weights(cfg, seed=3, device="cpu")
    from quail_b200.readout import AnswerRows, AsyncScores
    scorer = AsyncScores(torch, AnswerRows(torch, w.to(dev)))
    got = scorer.result(scorer.submit(normed.to(dev)))
    allowed, ans_w, tc, fc = w.answer_rows()
    ref = nx.answer_score(normed, ans_w, tc, fc)
    assert got.dtype == np.float32 and got.shape == (rows,)
    assert np.array_equal(got.view(np.int32), ref.numpy().view(np.int32))
    logits = normed.float() @ ans_w.float().t()
    plain = torch.sigmoid(logits[:, tc].amax(1) - logits[:, fc].amax(1))
    assert float((torch.from_numpy(got) - plain).abs().max()) < 1e-5
    assert_status_clean()
