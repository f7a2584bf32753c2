"""Pin the CPU oracle against the reference's own Triton kernels.

tests/golden/kernels.npz holds inputs and outputs of Quail's fused Triton
kernels (quail/backends/quail/executor/attention.py:293-642) run under
TRITON_INTERPRET=1 (tests/golden/make_golden.py). The oracle's
restatements must reproduce them: bf16 outputs exactly, fp8 codes exactly
(or one code step where a float division lands on a rounding tie) and
fp32 scales to the last bit or one ulp.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import numerics as nx

GOLDEN = Path(__file__).resolve().parent / "golden" / "kernels.npz"


def interpreter_bf16(x):
    """fp32 -> bf16 as the Triton interpreter does it: truncation."""
    x = x.to(torch.float32).contiguous()
    return (x.view(torch.int32) & ~0xFFFF).view(torch.float32).to(torch.bfloat16)


def interpreter_fp8(x):
    """fp32 -> e4m3 as the Triton interpreter does it: nearest, ties away
    from zero (the compiled cvt.rn rounds ties to even; ties are frequent
    in the UE8M0 mode, where q = y * 2^-e is exact), except that the carry
    of a round-up into the next binade is ORed into the exponent: when the
    pre-carry biased exponent is odd the carry is lost and the result is
    half the correctly rounded power of two."""
    xd = x.to(torch.float64)
    a = xd.abs()
    _, e2 = torch.frexp(a)
    quantum = torch.exp2(torch.clamp(e2 - 1, min=-6).to(torch.float64) - 3)
    k = a / quantum
    tie = (k - torch.floor(k)) == 0.5
    away = (torch.sign(xd) * (torch.floor(k) + 1) * quantum).to(torch.float32)
    rne = torch.where(tie, away, x.to(torch.float32)).to(torch.float8_e4m3fn)
    code = rne.view(torch.uint8)
    r = rne.to(torch.float32)
    mantissa_zero = (code & 0x7) == 0
    biased_exp = (code >> 3) & 0xF
    carried = mantissa_zero & (r.abs() > x.abs()) & (r != 0)
    lost = carried & (biased_exp % 2 == 0) & (biased_exp > 1)
    half = (r / 2).to(torch.float8_e4m3fn).view(torch.uint8)
    return torch.where(lost, half, code).view(torch.float8_e4m3fn)


@pytest.fixture()
def interpreter_rounding(monkeypatch):
    """The vectors came from the Triton interpreter; emulate its conversions
    so the comparison checks the fp32 arithmetic bit for bit. The compiled
    kernels (Triton's and ours) round to nearest even (cvt.rn)."""
    monkeypatch.setitem(nx.CONVERT, "bf16", interpreter_bf16)
    monkeypatch.setitem(nx.CONVERT, "fp8", interpreter_fp8)


@pytest.fixture(scope="module")
def vec():
    raw = np.load(GOLDEN)
    out = {}
    for name in raw.files:
        if name.endswith("__bf16"):
            out[name[:-6]] = torch.from_numpy(raw[name]).view(torch.bfloat16)
        else:
            out[name] = torch.from_numpy(raw[name])
    return out


def fp8_codes_close(got, want, max_frac=0.005):
    """fp8 codes equal except on a few elements sitting on a rounding tie.

    A last-ulp difference in a scale (fp32 reduction order) can move an
    element across a rounding boundary: one code step, or, on a boundary
    where the interpreter's carry rule applies, its halved power of two.
    """
    g = got.view(torch.uint8).to(torch.int32)
    w = want.view(torch.uint8).to(torch.int32)
    diff = g != w
    gv = got.view(torch.float8_e4m3fn).to(torch.float32)[diff]
    wv = want.view(torch.float8_e4m3fn).to(torch.float32)[diff]
    one_step = (g - w).abs()[diff] <= 1
    carry = (torch.maximum(gv.abs(), wv.abs()) == 2 * torch.minimum(gv.abs(), wv.abs()))
    assert bool((one_step | carry).all())
    assert float(diff.float().mean()) <= max_frac


def test_add_rmsnorm_quant(vec, interpreter_rounding):
    r_out, q, s = nx.add_rmsnorm_quant(vec["norm_x"], vec["norm_r_in"], vec["norm_w"], 1e-6)
    assert torch.equal(r_out.view(torch.int16), vec["norm_r_out"].view(torch.int16))
    fp8_codes_close(q, vec["norm_q"])
    torch.testing.assert_close(s, vec["norm_s"], rtol=5e-7, atol=0)


def test_qk_norm_rope(vec, interpreter_rounding):
    qkv = vec["rope_qkv"]
    q, k, v = nx.qk_norm_rope(qkv, vec["rope_pos"], vec["rope_cs"], vec["rope_qw"],
                              vec["rope_kw"], 1e-6, 4, 2)
    # bf16 outputs: allow one bf16 step on a few elements (fp32 reduction order)
    for got, want in ((q, vec["rope_q"]), (k, vec["rope_k"])):
        g = got.view(torch.int16).to(torch.int32)
        w = want.view(torch.int16).to(torch.int32)
        d = (g - w).abs()
        assert int(d.max()) <= 1
        assert float((d > 0).float().mean()) < 0.01
    assert torch.equal(v, qkv[:, 6 * 128:])


def test_silu_mul_quant(vec, interpreter_rounding):
    q, s = nx.silu_mul_quant(vec["silu_gu"])
    fp8_codes_close(q, vec["silu_q"])
    torch.testing.assert_close(s, vec["silu_s"], rtol=3e-7, atol=0)


def test_merge_attn_quant(vec, interpreter_rounding):
    q, s = nx.merge_attn_quant(vec["merge_a"].reshape(6, 512), vec["merge_la"],
                               vec["merge_b"].reshape(4, 512), vec["merge_lb"],
                               vec["merge_src"], 4)
    fp8_codes_close(q, vec["merge_q"])
    torch.testing.assert_close(s, vec["merge_s"], rtol=2e-7, atol=0)


@pytest.fixture
def ue8m0_mode():
    nx.MODE["ue8m0"] = True
    yield
    nx.MODE["ue8m0"] = False


def test_add_rmsnorm_quant_ue8m0(vec, interpreter_rounding, ue8m0_mode):
    """UE8M0=True: the scales are powers of two, equal to the reference's."""
    _, q, s = nx.add_rmsnorm_quant(vec["norm_x"], vec["norm_r_in"], vec["norm_w"], 1e-6)
    assert torch.equal(s, vec["norm_s_ue8m0"])
    fp8_codes_close(q, vec["norm_q_ue8m0"])


def test_silu_mul_quant_ue8m0(vec, interpreter_rounding, ue8m0_mode):
    q, s = nx.silu_mul_quant(vec["silu_gu"])
    assert torch.equal(s, vec["silu_s_ue8m0"])
    fp8_codes_close(q, vec["silu_q_ue8m0"])


def test_merge_attn_quant_ue8m0(vec, interpreter_rounding, ue8m0_mode):
    q, s = nx.merge_attn_quant(vec["merge_a"].reshape(6, 512), vec["merge_la"],
                               vec["merge_b"].reshape(4, 512), vec["merge_lb"],
                               vec["merge_src"], 4)
    assert torch.equal(s, vec["merge_s_ue8m0"])
    fp8_codes_close(q, vec["merge_q_ue8m0"])


def test_requant_weight_ue8m0_matches_vllm():
    """The oracle's load-time re-quantisation against vLLM's own
    requant_weight_ue8m0_inplace (tests/golden/requant_ue8m0.npz), zero,
    full-range and tiny blocks included: codes and scales bit for bit."""
    d = np.load(GOLDEN.parent / "requant_ue8m0.npz")
    w = torch.from_numpy(d["w"]).view(torch.float8_e4m3fn)
    q, s = nx.requant_weight_ue8m0(w, torch.from_numpy(d["s"]))
    assert torch.equal(s, torch.from_numpy(d["s_ue8m0"]))
    assert torch.equal(q.view(torch.uint8), torch.from_numpy(d["w_ue8m0"]))


def test_kv_row_scatter(vec):
    kp = torch.zeros(10, 2, 128, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    kp[vec["scat_dst"]] = vec["scat_k"][vec["scat_src"]]
    vp[vec["scat_dst"]] = vec["scat_v"][vec["scat_src"]]
    assert torch.equal(kp.view(torch.int16), vec["scat_kpool"].view(torch.int16))
    assert torch.equal(vp.view(torch.int16), vec["scat_vpool"].view(torch.int16))


def test_quant_roundtrip_bounds():
    g = torch.Generator().manual_seed(0)
    y = torch.randn(8, 256, generator=g) * 5
    q, s = nx.quant_groups(y)
    back = nx.dequant(q, s)
    # e4m3 has a 3-bit mantissa: relative error <= 2^-4 of each group's max
    err = (back - y).abs().reshape(8, 2, 128).amax(-1)
    assert bool((err <= s.t() * 448 * 2 ** -4 + 1e-12).all())


def test_gemm_restatement_matches_dequantised_product():
    g = torch.Generator().manual_seed(1)
    a = torch.randn(5, 256, generator=g)
    aq, as_ = nx.quant_groups(a)
    w = torch.randn(256, 256, generator=g).to(torch.float8_e4m3fn)
    ws = torch.rand(2, 2, generator=g) + 0.5
    out = nx.gemm_fp8_bs(aq, as_, w, ws).float()
    ref = nx.dequant(aq, as_) @ (w.float() * ws.repeat_interleave(128, 0)
                                 .repeat_interleave(128, 1)).t()
    torch.testing.assert_close(out, ref, rtol=1e-2, atol=1e-2)
