"""Per-op CPU restatements (torch fp32 on the CPU). Test infrastructure only.

Every function names the reference code it restates. Values cross op
boundaries in the dtypes the reference stores (bf16 activations, fp8 e4m3
codes with fp32 scales), so roundings happen where the reference's do.
Scales are returned group-major, (width / 128, rows), as the kernels
write them.

Two modes (MODE["exact"]):
- exact (default, the parity oracle): every reduction in the order the
  sm_100a kernels use, tensor-core products under the measured accumulation
  model, exp2 / ln by the FMA-only methods both sides share (oracle/tc.py,
  oracle/tcmodel.c). Agrees with the kernels bit for bit.
- fast (the CPU baseline): the same algorithm with torch's own reductions,
  fp32 BLAS GEMMs and exp; agrees to the last bits, runs at BLAS speed.

MODE["ue8m0"] selects the reference's UE8M0 scale mode (Engine.use_ue8m0,
quail/backends/quail/executor/attention.py:115): power-of-two quantiser
scales and the GEMMs' whole-K accumulation of the block-scaled MMA.
"""

import numpy as np
import torch

from oracle import tc

GROUP = 128
FP8_MAX = 448.0
MODE = {"exact": True, "ue8m0": False}


def _to_bf16(x):
    return x.to(torch.bfloat16)


def _to_fp8(x):
    return x.to(torch.float8_e4m3fn)


# Every narrowing conversion goes through these two hooks: round to nearest
# even, as the compiled kernels (cvt.rn) do. The golden-vector test swaps in
# the conversions of the Triton interpreter that produced the vectors.
CONVERT = {"bf16": _to_bf16, "fp8": _to_fp8}


def to_bf16(x):
    return CONVERT["bf16"](x)


def to_fp8(x):
    return CONVERT["fp8"](x)


def bf16(x):
    """Round fp32 to bf16 and back (round to nearest even)."""
    return to_bf16(x).to(torch.float32)


def _sumsq_rows(x):
    if MODE["exact"]:
        return tc.sumsq_rows(x)[:, None]
    return (x * x).sum(dim=-1, keepdim=True)


def _sigmoid(x):
    if MODE["exact"]:
        return tc.sigmoid(x)
    return 1.0 / (1.0 + torch.exp(-x))


def fma(a, b, c):
    """fp32 a * b + c with one rounding (CUDA's fmaf / FFMA)."""
    return tc.fma(a, b, c)


def ue8m0_scale(scale):
    """The UE8M0 mode's scale: exp2(ceil(log2(scale))) for fp32 scale > 0,
    taken exactly as the least power of two >= scale (from the bits: a
    power of two, inf and NaN stay). The reference computes it through
    log2 (attention.py:315-316, 350-351, 467-468; vLLM's
    per_token_group_quant_fp8 with use_ue8m0); a float log2 can round to
    an integer for a scale a few ulps above a power of two, which the exact
    form does not."""
    b = scale.to(torch.float32).contiguous().view(torch.int32)
    up = (b & 0x7F800000) + 0x800000
    keep = ((b & 0x7FFFFF) == 0) | (b >= 0x7F800000)
    return torch.where(keep, b, up).view(torch.float32)


def quant_groups(y):
    """1x128 fp8 quantisation of fp32 rows.

    The per-group quantiser shared by vLLM's per_token_group_quant_fp8 and
    Quail's fused Triton kernels (quail/backends/quail/executor/
    attention.py:315-323, 348-355, 461-469): scale = max(amax, 1e-10) / 448,
    q = clamp(y / scale, -448, 448) cast to e4m3 (nearest even).
    Returns (codes float8_e4m3fn [rows, width], scales f32 [width/128, rows]).
    """
    rows, width = y.shape
    g = y.reshape(rows, width // GROUP, GROUP)
    amax = g.abs().amax(dim=2)
    scale = torch.clamp(amax, min=1e-10) / FP8_MAX
    if MODE["ue8m0"]:
        scale = ue8m0_scale(scale)
    q = torch.clamp(g / scale[:, :, None], -FP8_MAX, FP8_MAX)
    return to_fp8(q.reshape(rows, width)), scale.t().contiguous()


def dequant(codes, scales):
    """fp32 values of fp8 codes with group-major scales."""
    rows, width = codes.shape
    s = scales.t().reshape(rows, width // GROUP, 1)
    return (codes.to(torch.float32).reshape(rows, width // GROUP, GROUP) * s).reshape(rows, width)


def sqrt(x):
    """IEEE (correctly rounded) fp32 square root, as CUDA's sqrtf computes it.
    torch's CPU sqrt is not correctly rounded for float32; numpy's is."""
    x = x.to(torch.float32).contiguous()
    return torch.from_numpy(np.sqrt(x.numpy()))


def _rstd(total, width, eps):
    return 1.0 / sqrt(total / width + eps)


def rms_norm_bf16(x, w, eps):
    """vLLM rms_norm on bf16 rows (vllm/ir/ops/layernorm.py rms_norm):
    fp32 variance, x * rsqrt(var + eps) rounded to bf16, times the bf16
    weight, rounded to bf16."""
    x = x.to(torch.float32)
    y = bf16(x * _rstd(_sumsq_rows(x), x.shape[-1], eps))
    return bf16(y * w.to(torch.float32))


def embed_rmsnorm_quant(ids, embed, w, eps):
    """Layer 0: embedding gather, vLLM rms_norm, per-group quant
    (models/qwen3.py:51, 55-57; attention.py:143-151, 763-766)."""
    residual = embed[ids]
    q, s = quant_groups(rms_norm_bf16(residual, w, eps))
    return residual, q, s


def add_rmsnorm_quant(hidden, residual, w, eps):
    """Triton add_rms_norm_quant (attention.py:326-359): x = hidden +
    residual in fp32; residual stored as bf16(x); y = x * rstd * w in fp32
    from the unrounded x; per-group quant. Returns (new residual, q, s)."""
    x = hidden.to(torch.float32) + residual.to(torch.float32)
    y = x * _rstd(_sumsq_rows(x), x.shape[-1], eps) * w.to(torch.float32)
    q, s = quant_groups(y)
    return to_bf16(x), q, s


def silu_mul_quant(gate_up):
    """Triton silu_mul_quant (attention.py:301-323): y = g * sigmoid(g) * u
    in fp32 from the bf16 halves; per-group quant."""
    half = gate_up.shape[1] // 2
    g = gate_up[:, :half].to(torch.float32)
    u = gate_up[:, half:].to(torch.float32)
    y = g * _sigmoid(g) * u
    return quant_groups(y)


def gemm_fp8_bs(a_codes, a_scales, w_codes, w_scales):
    """DeepGEMM fp8_gemm_nt as Quail calls it (attention.py:129-141): per
    128-deep K block an fp32 partial product of the fp8 codes, promoted
    with acc = fma(partial, a_scale[kb, m] * w_scale[n/128, kb], acc) in K
    order (DeepGEMM's promotion), bf16 output. a_scales is group-major
    (K/128, M). Exact mode: the partials follow the tensor cores'
    accumulation (tcmodel.c); fast mode: fp32 BLAS partials."""
    if MODE["ue8m0"]:
        return gemm_fp8_mx(a_codes, a_scales, w_codes, w_scales)
    if MODE["exact"]:
        return tc.gemm_fp8(a_codes, a_scales, w_codes, w_scales)
    m, k = a_codes.shape
    n = w_codes.shape[0]
    kb = k // GROUP
    a = a_codes.to(torch.float32).reshape(m, kb, GROUP).permute(1, 0, 2)
    w = w_codes.to(torch.float32).reshape(n, kb, GROUP).permute(1, 2, 0)
    acc = torch.zeros(m, n, dtype=torch.float32)
    ws = w_scales.to(torch.float32).repeat_interleave(GROUP, dim=0)  # [n, kb]
    for b in range(kb):
        acc = acc + (a[b] @ w[b]) * (a_scales[b][:, None] * ws[:, b][None, :])
    return to_bf16(acc)


def gemm_fp8_mx(a_codes, a_scales, w_codes, w_scales):
    """fp8_gemm_nt in the UE8M0 mode on sm_100 (DeepGEMM's block-scaled
    kernels): every scale a power of two, applied to the products, one fp32
    accumulation over the whole K, bf16 output. Exact mode: the tensor
    cores' accumulation per K=32 step (tcmodel.c gemm_mx); fast mode: the
    exactly scaled operands through an fp32 BLAS GEMM."""
    if MODE["exact"]:
        return tc.gemm_mx(a_codes, a_scales, w_codes, w_scales)
    m, k = a_codes.shape
    n = w_codes.shape[0]
    a = dequant(a_codes, a_scales)
    ws = w_scales.to(torch.float32).repeat_interleave(GROUP, 0).repeat_interleave(GROUP, 1)
    w = w_codes.to(torch.float32) * ws[:n, :k]
    return to_bf16(a @ w.t())


def requant_weight_ue8m0(w_codes, w_scales):
    """A block-scaled fp8 weight re-quantised to power-of-two block scales,
    as vLLM does at load time when DeepGEMM uses UE8M0 (vllm 0.22,
    model_executor/layers/quantization/utils/fp8_utils.py
    requant_weight_ue8m0_inplace, through deep_gemm.py per_block_cast_to_fp8):
    x = code * scale (fp32) per 128 x 128 block; s = max(amax, 1e-4) / 448
    raised to a power of two; codes = e4m3(x / s). Returns (codes, scales)."""
    n, k = w_codes.shape
    nb, kb = n // GROUP, k // GROUP
    x = (w_codes.to(torch.float32).reshape(nb, GROUP, kb, GROUP)
         * w_scales.to(torch.float32)[:, None, :, None])
    amax = x.abs().amax(dim=(1, 3)).clamp(min=1e-4)
    s = ue8m0_scale(amax / FP8_MAX)
    q = to_fp8(x / s[:, None, :, None]).reshape(n, k)
    return q, s


def qk_norm_rope(qkv, positions, cos_sin, q_w, k_w, eps, n_q, n_kv, head_dim=128):
    """Triton qk_norm_rope (attention.py:363-409): per-head RMSNorm of q
    and k in fp32, times the weight, neox rotary with cos | sin of the bf16
    cache row; bf16 outputs. Also returns v, the raw slice (qwen3.py:63-64)."""
    rows = qkv.shape[0]
    half = head_dim // 2
    cs = cos_sin[positions].to(torch.float32)
    cos, sin = cs[:, None, :half], cs[:, None, half:]

    def norm_rope(x, w, heads):
        x = x.reshape(rows, heads, head_dim).to(torch.float32)
        if MODE["exact"]:
            ss = tc.sumsq_heads(x).reshape(rows, heads, 1)
        else:
            ss = (x * x).sum(-1, keepdim=True)
        rstd = 1.0 / sqrt(ss / head_dim + eps)
        wf = w.to(torch.float32)
        a = x[..., :half] * rstd * wf[:half]
        b = x[..., half:] * rstd * wf[half:]
        out = torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)
        return to_bf16(out).reshape(rows, heads * head_dim)

    qw = n_q * head_dim
    kw = n_kv * head_dim
    q = norm_rope(qkv[:, :qw], q_w, n_q)
    k = norm_rope(qkv[:, qw:qw + kw], k_w, n_kv)
    v = qkv[:, qw + kw:qw + 2 * kw].contiguous()
    return q, k, v


# FlashAttention's algorithm (Dao, FlashAttention-2, 2023): keys in blocks,
# a running row max m, P = exp2(s * scale * log2 e - m * scale * log2 e)
# (an FFMA) rounded to bf16 before the PV product, row sums from the fp32 P,
# the accumulator rescaled when m grows, out = acc * (1 / l) rounded to bf16,
# lse = m * scale + ln(l). KEY_BLOCK is the key block of the sm_100a kernel.
# Exact mode follows the kernel: exp2 is its softmax exp2 (tc.exp2_soft),
# and the row sum is eight partials (key j of a block goes to partial j % 8,
# in key order, each partial rescaled by alpha per block) combined as
# ((l0 + l1) + (l2 + l3)) + ((l4 + l5) + (l6 + l7)).
KEY_BLOCK = 64
LOG2E_F = 1.44269504088896341


def attend(q, k, v, scale, mask=None):
    """Softmax attention for one query head (FlashAttention numerics).

    q [nq, d], k/v [nk, d] (bf16 values); mask [nq, nk] True = visible.
    Returns (out bf16 [nq, d], lse f32 [nq]) with lse the natural
    log-sum-exp of the scaled scores, FlashAttention's softmax_lse
    (attention.py:802-818, return_softmax_lse=True)."""
    nq, nk = q.shape[0], k.shape[0]
    exact = MODE["exact"]
    sl2 = torch.tensor(scale, dtype=torch.float32) * torch.tensor(LOG2E_F, dtype=torch.float32)
    if exact:
        s = tc.mma_bf16(q, k)
    else:
        s = q.to(torch.float32) @ k.to(torch.float32).t()
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    m = torch.full((nq,), float("-inf"))
    lq = torch.zeros(nq, 8)
    acc = torch.zeros(nq, v.shape[1])
    exp2 = tc.exp2_soft if exact else torch.exp2
    for j0 in range(0, nk, KEY_BLOCK):
        sb = s[:, j0:j0 + KEY_BLOCK]
        nb = sb.shape[1]
        if nb < KEY_BLOCK:
            sb = torch.cat([sb, torch.full((nq, KEY_BLOCK - nb), float("-inf"))], dim=1)
        m_new = torch.maximum(m, sb.amax(dim=1))
        seen = m_new > float("-inf")
        alpha = torch.where(seen, exp2((m - m_new) * sl2), torch.ones(nq))
        msl = torch.where(seen, m_new * sl2, torch.zeros(nq))
        if exact:
            p = exp2(tc.fma(sb, sl2.expand_as(sb), (-msl)[:, None].expand_as(sb)))
        else:
            p = exp2(sb * sl2 - msl[:, None])
        # eight row-sum partials: key 8 n + i of the block goes to partial i
        lq = lq * alpha[:, None]
        pv = p.reshape(nq, 8, 8)
        for n8 in range(8):
            lq = lq + pv[:, n8, :]
        acc = acc * alpha[:, None]
        pb = bf16(p)
        vb = torch.zeros(KEY_BLOCK, v.shape[1], dtype=torch.bfloat16)
        vb[:nb] = v[j0:j0 + nb]
        if exact:
            acc = tc.mma_bf16(pb, vb.t(), acc)
        else:
            acc = acc + pb @ vb.to(torch.float32)
        m = m_new
    l = ((lq[:, 0] + lq[:, 1]) + (lq[:, 2] + lq[:, 3])) + \
        ((lq[:, 4] + lq[:, 5]) + (lq[:, 6] + lq[:, 7]))
    out = acc * (1.0 / l)[:, None]
    if exact:
        lse = tc.fma(m, torch.full_like(m, scale), tc.ln(l))
    else:
        lse = m * scale + torch.log(l)
    return to_bf16(out), lse


def attention_heads(q, k, v, n_q, n_kv, scale, mask=None, head_dim=128):
    """attend() over every query head with grouped KV heads.

    q [nq, n_q*d]; k, v [nk, n_kv*d]. Returns (out bf16 [nq, n_q*d],
    lse f32 [nq, n_q])."""
    nq, nk = q.shape[0], k.shape[0]
    qh = q.reshape(nq, n_q, head_dim)
    kh = k.reshape(nk, n_kv, head_dim)
    vh = v.reshape(nk, n_kv, head_dim)
    group = n_q // n_kv
    outs, lses = [], []
    for h in range(n_q):
        o, l = attend(qh[:, h], kh[:, h // group], vh[:, h // group], scale, mask)
        outs.append(o)
        lses.append(l)
    return torch.stack(outs, dim=1).reshape(nq, n_q * head_dim), torch.stack(lses, dim=1)


def merge_attn_quant(out_a, lse_a, out_b, lse_b, source, n_q, head_dim=128):
    """Triton merge_attn_quant (attention.py:432-473): w = bf16(sigmoid(
    lse_b - lse_a)); merged = bf16(a + (b - a) * w); rows with source < 0
    keep a; per-head (128-column) quantisation. out_b/lse_b are indexed by
    source. Returns (q, scales)."""
    rows = out_a.shape[0]
    a = out_a.to(torch.float32).reshape(rows, n_q, head_dim)
    has_b = source >= 0
    safe = torch.clamp(source, min=0).long()
    b = out_b.to(torch.float32).reshape(-1, n_q, head_dim)[safe]
    lb = lse_b[safe]
    w = bf16(_sigmoid(lb - lse_a))
    merged = bf16(a + (b - a) * w[:, :, None])
    y = torch.where(has_b[:, None, None], merged, a)
    return quant_groups(y.reshape(rows, n_q * head_dim))


def final_norm(hidden, residual, finals, w, eps):
    """index_select of the answer rows + vLLM fused_add_rms_norm
    (models/qwen3.py:72-77; vllm/ir/ops/layernorm.py fused_add_rms_norm):
    x = hidden + residual in fp32, rstd from the unrounded x,
    bf16(bf16(x * rstd) * w)."""
    x = hidden[finals].to(torch.float32) + residual[finals].to(torch.float32)
    y = bf16(x * _rstd(_sumsq_rows(x), x.shape[-1], eps))
    return to_bf16(y * w.to(torch.float32))


def answer_score(normed, ans_w, true_cols, false_cols):
    """AsyncScores.submit (readout.py:88-111): fp32 scores of the retained head
    rows (no bf16 rounding), max per class, sigmoid(yes - no) in fp32."""
    if MODE["exact"]:
        raw = tc.dot_rows(normed.to(torch.float32), ans_w.to(torch.float32))
    else:
        raw = normed.to(torch.float32) @ ans_w.to(torch.float32).t()
    t = raw[:, list(true_cols)].amax(dim=1)
    f = raw[:, list(false_cols)].amax(dim=1)
    return tc.sigmoid(t - f) if MODE["exact"] else torch.sigmoid(t - f)


def answer_margin(normed, ans_w, true_cols, false_cols):
    """AnswerRows.logits + AsyncAnswers.submit (readout.py:45-49, 70-80):
    bf16 scores of the retained head rows (fp32 accumulate), max per class,
    margin = t - f, bit = t > f."""
    if MODE["exact"]:
        raw = tc.dot_rows(normed.to(torch.float32), ans_w.to(torch.float32))
    else:
        raw = normed.to(torch.float32) @ ans_w.to(torch.float32).t()
    scores = bf16(raw)
    t = scores[:, list(true_cols)].amax(dim=1)
    f = scores[:, list(false_cols)].amax(dim=1)
    return t - f, (t > f).to(torch.uint8)
