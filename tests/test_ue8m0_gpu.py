"""The UE8M0 scale mode on the GPU against the oracle, bit for bit.

The reference's quantisers and GEMMs have a UE8M0 mode (Engine.use_ue8m0,
set from vLLM's is_deep_gemm_e8m0_used; quail/backends/quail/executor/
attention.py:115, 151, 315-316, 350-351, 467-468): every quantiser scale is
the least power of two at or above max(amax, 1e-10) / 448, the weights are
re-quantised to power-of-two block scales at load (vLLM's
requant_weight_ue8m0_inplace), and DeepGEMM's sm_100 GEMM applies the
scales in the block-scaled MMA, accumulating the whole K in fp32. Here:

- the quantisers (embedding norm, residual-add norm, SiLU product) in the
  mode, codes and scales;
- the weight re-quantisation kernel;
- the block-scaled GEMM (tcgen05 kind::mxf8f6f4) and its fused SiLU and
  q/k norm + rotary epilogues, against the oracle's accumulation model;
- a scale that is not a power of two: the status bit, no fault;
- the TINY and a 2-layer 4B-width model end to end through run_filter.
"""

import numpy as np
import pytest
import torch

from oracle import forward as of
from oracle import numerics as nx
from quail_b200 import _native as nat
from quail_b200 import loop
from quail_b200.arena import KVArena
from quail_b200.engine import Engine, QuantRows
from quail_b200.model import QWEN3_4B, TINY, random_weights, requant_ue8m0, scales_are_ue8m0
from quail_b200.pipeline import Qwen3Pipeline
from quail_b200.readout import AnswerRows, AsyncAnswers
from quail_b200.tokens import prefix_tree

pytestmark = pytest.mark.gpu

STATUS_BAD_SCALE = 0x400


@pytest.fixture(autouse=True)
def ue8m0_oracle():
    nx.MODE["ue8m0"] = True
    yield
    nx.MODE["ue8m0"] = False


def bits(t):
    t = t.detach().cpu().contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


def assert_bits_equal(got, want, what=""):
    g, w = bits(got), bits(want)
    assert g.shape == w.shape, (what, g.shape, w.shape)
    diff = int((g != w).sum())
    assert diff == 0, f"{what}: {diff} of {g.numel()} elements differ"


def assert_pow2(scales):
    b = bits(scales.float())
    assert int(((b & 0x807FFFFF) != 0).sum()) == 0


class _Arena:
    pool_rows = 64


def engine(cfg=TINY, arena=None):
    return Engine(torch, arena or _Arena(), cfg, ue8m0=True)


def status():
    return nat.kernel_status(torch.cuda.current_device())


def test_exact_power_of_two_scale():
    s = torch.tensor([1.0, 1.0000001, 0.75, 2.0 ** -40, 3.0e38, float("inf")])
    got = nx.ue8m0_scale(s)
    assert got.tolist()[:4] == [1.0, 2.0, 1.0, 2.0 ** -40]
    assert got[4] == float("inf") and got[5] == float("inf")


@pytest.mark.parametrize("rows,hidden", [(1, 512), (300, 2560)])
def test_embed_rmsnorm_quant_ue8m0(rows, hidden):
    g = torch.Generator().manual_seed(rows)
    embed = (0.02 * torch.randn(1000, hidden, generator=g)).to(torch.bfloat16)
    w = (1 + 0.05 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    ids = torch.randint(0, 1000, (rows,), generator=g)
    res, out = engine().embed_norm_quant(ids.cuda(), embed.cuda(), w.cuda())
    r_ref, q_ref, s_ref = nx.embed_rmsnorm_quant(ids, embed, w, TINY.eps)
    assert_bits_equal(res, r_ref, "residual")
    assert_bits_equal(out.scale[:, :rows], s_ref, "scales")
    assert_bits_equal(out.q, q_ref, "codes")
    assert_pow2(s_ref)


@pytest.mark.parametrize("rows,hidden", [(77, 2560), (5, 5120)])
def test_add_rmsnorm_quant_ue8m0(rows, hidden):
    g = torch.Generator().manual_seed(hidden + rows)
    x = (2 * torch.randn(rows, hidden, generator=g)).to(torch.bfloat16)
    r = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    r_dev = r.cuda()
    out = engine().norm_quant(x.cuda(), w.cuda(), r_dev)
    r_ref, q_ref, s_ref = nx.add_rmsnorm_quant(x, r, w, TINY.eps)
    assert_bits_equal(r_dev, r_ref, "residual")
    assert_bits_equal(out.scale[:, :rows], s_ref, "scales")
    assert_bits_equal(out.q, q_ref, "codes")


@pytest.mark.parametrize("rows,inter", [(3, 1024), (129, 9728)])
def test_silu_mul_quant_ue8m0(rows, inter):
    g = torch.Generator().manual_seed(inter)
    gu = (3 * torch.randn(rows, 2 * inter, generator=g)).to(torch.bfloat16)
    out = engine().activation_quant(gu.cuda())
    q_ref, s_ref = nx.silu_mul_quant(gu)
    assert_bits_equal(out.scale[:, :rows], s_ref, "scales")
    assert_bits_equal(out.q, q_ref, "codes")


@pytest.mark.parametrize("n,k", [(256, 128), (512, 640), (2560, 9728)])
def test_requant_weight_matches_oracle(n, k):
    g = torch.Generator().manual_seed(n + k)
    w = torch.randn(n, k, generator=g).to(torch.float8_e4m3fn)
    s = torch.exp(np.log(0.02) + 0.3 * torch.randn(n // 128, k // 128, generator=g))
    w_dev, s_dev = w.cuda(), s.cuda()
    nat.call("qb_requant_weight_ue8m0", nat.ptr(w_dev), nat.ptr(s_dev), n, k,
             nat.stream_handle(torch))
    q_ref, s_ref = nx.requant_weight_ue8m0(w, s)
    assert_bits_equal(s_dev, s_ref, "scales")
    assert_bits_equal(w_dev, q_ref, "codes")
    assert_pow2(s_dev)


def _operands(g, m, n, k, spread=0):
    """ue8m0 activations from the quantiser; weights re-quantised from
    lognormal block scales; spread > 0 widens the codes' exponents."""
    a = torch.randn(m, k, generator=g) * (1 + torch.rand(m, 1, generator=g))
    if spread:
        a = a * torch.exp2(torch.randint(-spread, spread + 1, (m, k), generator=g).float())
    aq, as_ = nx.quant_groups(a)
    w = torch.randn(n, k, generator=g)
    if spread:
        w = w * torch.exp2(torch.randint(-spread, spread + 1, (n, k), generator=g).float())
    wq = w.clamp(-448, 448).to(torch.float8_e4m3fn)
    ws = torch.exp(np.log(0.02) + 0.3 * torch.randn(n // 128, k // 128, generator=g))
    wq, ws = nx.requant_weight_ue8m0(wq, ws)
    return aq, as_, wq, ws


@pytest.mark.parametrize("m,n,k,spread", [(1, 256, 128, 0), (7, 512, 512, 0),
                                          (300, 1024, 2560, 0), (257, 2560, 4096, 0),
                                          (130, 512, 1024, 4), (64, 256, 9728, 6)])
def test_gemm_ue8m0_matches_oracle(m, n, k, spread):
    g = torch.Generator().manual_seed(m * 7 + n + k + spread)
    aq, as_, wq, ws = _operands(g, m, n, k, spread)
    x = QuantRows(aq.cuda(), as_.cuda().contiguous(), m)
    out = engine().gemm(x, wq.cuda(), ws.cuda())
    torch.cuda.synchronize()
    assert_bits_equal(out, nx.gemm_fp8_bs(aq, as_, wq, ws), "bf16")
    assert status() == 0


def test_gemm_ue8m0_random_exponents():
    """Power-of-two scales over a wide exponent range (not from a
    quantiser): the scale exponents enter the accumulation model."""
    g = torch.Generator().manual_seed(11)
    m, n, k = 96, 512, 1024
    aq = (torch.randn(m, k, generator=g) * 8).to(torch.float8_e4m3fn)
    wq = (torch.randn(n, k, generator=g) * 8).to(torch.float8_e4m3fn)
    as_ = torch.exp2(torch.randint(-30, 8, (k // 128, m), generator=g).float())
    ws = torch.exp2(torch.randint(-20, 4, (n // 128, k // 128), generator=g).float())
    out = engine().gemm(QuantRows(aq.cuda(), as_.cuda(), m), wq.cuda(), ws.cuda())
    torch.cuda.synchronize()
    assert_bits_equal(out, nx.gemm_fp8_bs(aq, as_, wq, ws), "bf16")
    assert status() == 0


def test_gemm_ue8m0_rejects_scales_that_are_not_powers_of_two():
    """A scale with mantissa bits sets the status bit; the call still ends
    normally and the device stays usable."""
    g = torch.Generator().manual_seed(3)
    aq, as_, wq, ws = _operands(g, 64, 256, 256)
    as_bad = as_.clone()
    as_bad[0, 5] *= 1.5
    assert status() == 0
    engine().gemm(QuantRows(aq.cuda(), as_bad.cuda(), 64), wq.cuda(), ws.cuda())
    torch.cuda.synchronize()
    assert status() == STATUS_BAD_SCALE
    assert status() == 0
    out = engine().gemm(QuantRows(aq.cuda(), as_.cuda(), 64), wq.cuda(), ws.cuda())
    torch.cuda.synchronize()
    assert_bits_equal(out, nx.gemm_fp8_bs(aq, as_, wq, ws), "bf16")


def test_gemm_ue8m0_rejects_odd_widths():
    with pytest.raises(ValueError, match="multiple of 256"):
        nat.call("qb_gemm_fp8_bs", None, None, 8, None, None, None, 8, 384, 256, 1, None)


@pytest.mark.parametrize("m,inter,k", [(1, 128, 256), (300, 1024, 2560), (257, 9728, 2560)])
def test_gemm_silu_quant_ue8m0(m, inter, k):
    g = torch.Generator().manual_seed(m + inter + k)
    aq, as_, wq, ws = _operands(g, m, 2 * inter, k)
    out = engine().gemm_silu_quant(QuantRows(aq.cuda(), as_.cuda(), m), wq.cuda(), ws.cuda())
    torch.cuda.synchronize()
    gu = nx.gemm_fp8_bs(aq, as_, wq, ws)
    q_ref, s_ref = nx.silu_mul_quant(gu)
    assert_bits_equal(out.scale[:, :m], s_ref, "scales")
    assert_bits_equal(out.q, q_ref, "codes")
    assert status() == 0


@pytest.mark.parametrize("m", [5, 300])
def test_gemm_qknorm_rope_ue8m0(m):
    from quail_b200.model import rotary_cache
    cfg = QWEN3_4B
    g = torch.Generator().manual_seed(m)
    n = cfg.qkv_width
    aq, as_, wq, ws = _operands(g, m, n, cfg.hidden)
    pos = torch.randint(0, 4096, (m,), generator=g)
    cos_sin = rotary_cache(cfg, "cpu")
    q_w = (1 + 0.05 * torch.randn(128, generator=g)).to(torch.bfloat16)
    k_w = (1 + 0.05 * torch.randn(128, generator=g)).to(torch.bfloat16)
    eng = engine(cfg)
    q, k, v = eng.gemm_qknorm_rope(QuantRows(aq.cuda(), as_.cuda(), m), wq.cuda(), ws.cuda(),
                                   pos.cuda(), cos_sin.cuda(), q_w.cuda(), k_w.cuda(), 0)
    torch.cuda.synchronize()
    qkv = nx.gemm_fp8_bs(aq, as_, wq, ws)
    q_ref, k_ref, v_ref = nx.qk_norm_rope(qkv, pos, cos_sin, q_w, k_w, cfg.eps, cfg.n_q, cfg.n_kv)
    assert_bits_equal(q, q_ref, "q")
    assert_bits_equal(k, k_ref, "k")
    assert_bits_equal(v, v_ref, "v")
    assert status() == 0


def rows_with_prefix(seed, n, prefix_len, lo, hi, vocab_lo, vocab_hi):
    rng = np.random.default_rng(seed)
    prefix = rng.integers(vocab_lo, vocab_hi, prefix_len).tolist()
    lens = rng.integers(lo, hi + 1, n)
    docs = [prefix + rng.integers(vocab_lo, vocab_hi, int(s)).tolist() for s in lens]
    question = [int(np.random.default_rng(3).integers(vocab_lo, vocab_hi))]
    return docs, [question]


def _filter_parity(cfg, weights, docs, questions, budget, n_pages, mode):
    dev = torch.device("cuda")
    requant_ue8m0(weights)
    assert scales_are_ue8m0(weights)
    arena = KVArena(cfg.n_layers, n_pages, 16, cfg.n_kv, cfg.head_dim, device=dev)
    arena.pools.zero_()
    pipe = Qwen3Pipeline(torch, weights, arena, ue8m0=True)
    ans = AsyncAnswers(torch, AnswerRows(torch, weights), keep_margins=True)
    hosts = []
    loop.run_filter(torch, arena, pipe, ans, docs, questions, budget, arena_writes=True,
                    attention_mode=mode, prefix_tree=prefix_tree(docs, 16), device=dev,
                    on_chunk=lambda host, groups: hosts.append(host))
    torch.cuda.synchronize()
    assert status() == 0
    cpu_w = weights.to("cpu")
    cpu_arena = of.CpuArena(cfg.n_layers, arena.pool_rows, cfg.n_kv, cfg.head_dim)
    _, ans_w, tc, fc = cpu_w.answer_rows()
    compared = 0
    for host, got in zip(hosts, ans.margins):
        want, _ = nx.answer_margin(of.forward_chunk(cpu_w, host, cpu_arena), ans_w, tc, fc)
        want = want.numpy().astype(np.float32)
        assert np.array_equal(got.view(np.int32), want.view(np.int32)), (got, want)
        compared += len(want)
    assert compared == len(docs)


@pytest.mark.parametrize("mode", ["tree", "unified"])
def test_tiny_filter_ue8m0_matches_oracle(mode):
    cfg = TINY
    weights = random_weights(cfg, seed=0, device="cuda")
    docs, questions = rows_with_prefix(1, 48, 64, 16, 200, 16, cfg.vocab)
    _filter_parity(cfg, weights, docs, questions, 1500, 400, mode)


def test_4b_width_two_layers_ue8m0_matches_oracle():
    """The 4B shapes (hidden 2560, 32 / 8 heads, inter 9728) with two layers
    and a short vocabulary: every kernel of the 4B path in the mode."""
    import dataclasses
    cfg = dataclasses.replace(QWEN3_4B, name="qwen3-4b-2l", n_layers=2, vocab=4096)
    weights = random_weights(cfg, seed=2, device="cuda")
    docs, questions = rows_with_prefix(4, 6, 64, 32, 200, 16, cfg.vocab)
    _filter_parity(cfg, weights, docs, questions, 2048, 400, "tree")
