"""Model shapes and seeded random-init weights for the Qwen3 FP8 path.

No checkpoint is loaded (no network, no weights on disk): every model is a
random initialisation of the Qwen3 architecture, seeded so the oracle and
the kernels see the same numbers. The layout follows vLLM's loaded Qwen3
module as Quail reads it (quail/backends/quail/executor/models/qwen3.py:
24-44): a fused QKV projection with q | k | v output rows, a merged
gate_up projection with gate rows first, FP8 e4m3 weights with one fp32
scale per 128 x 128 block (``weight_scale_inv``), bf16 norms, bf16
embeddings tied to the output head, and a bf16 rotary cos | sin cache.

Weight codes are e4m3(N(0, 1)); block scales are exp(N(ln 0.02, 0.3));
norm weights are bf16(1 + 0.05 N(0, 1)); embeddings are bf16(N(0, 0.02)).
"""

import math
from dataclasses import dataclass, field

GROUP = 128


@dataclass(frozen=True)
class ModelConfig:
    """Shape of one Qwen3-architecture decoder."""

    name: str
    n_layers: int
    hidden: int
    n_q: int
    n_kv: int
    head_dim: int
    inter: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    max_pos: int = 40960
    fp8: bool = True
    true_ids: tuple = (10, 12, 14, 16)
    false_ids: tuple = (11, 13, 15, 17)

    @property
    def qkv_width(self) -> int:
        return (self.n_q + 2 * self.n_kv) * self.head_dim

    @property
    def linear_params(self) -> int:
        """Parameters of the four linears of one layer."""
        h, d = self.hidden, self.head_dim
        return (h * self.qkv_width + self.n_q * d * h
                + h * 2 * self.inter + self.inter * h)

    @property
    def gemm_flops_per_token(self) -> float:
        """2 x linear parameters over all layers (Quail's dense_decoder_cost)."""
        return 2.0 * self.linear_params * self.n_layers

    @property
    def kv_bytes_per_token(self) -> int:
        """bf16 K and V over all layers (kappa)."""
        return self.n_layers * self.n_kv * self.head_dim * 2 * 2

    @property
    def max_chunk_tokens(self) -> int:
        """The reference's int32 element-offset cap (models/qwen3.py:35-38)."""
        widest = max(self.qkv_width, 2 * self.inter)
        return (2 ** 31 - 1) // widest


# The kernel-test model: every kernel path of the 4B model at small widths.
TINY = ModelConfig("tiny-fp8", n_layers=2, hidden=512, n_q=4, n_kv=2, head_dim=128,
                   inter=1024, vocab=4096, max_pos=8192)
QWEN3_4B = ModelConfig("qwen3-4b-fp8", n_layers=36, hidden=2560, n_q=32, n_kv=8,
                       head_dim=128, inter=9728, vocab=151936)
QWEN3_32B = ModelConfig("qwen3-32b-fp8", n_layers=64, hidden=5120, n_q=64, n_kv=8,
                        head_dim=128, inter=25600, vocab=151936)
MODELS = {m.name: m for m in (TINY, QWEN3_4B, QWEN3_32B)}


@dataclass
class Layer:
    input_ln: object
    post_ln: object
    q_norm: object
    k_norm: object
    qkv_w: object
    qkv_s: object
    o_w: object
    o_s: object
    gate_up_w: object
    gate_up_s: object
    down_w: object
    down_s: object


@dataclass
class Weights:
    config: ModelConfig
    embed: object          # bf16 [vocab, hidden], tied output head
    final_norm: object     # bf16 [hidden]
    cos_sin: object        # bf16 [max_pos, head_dim]
    layers: list = field(default_factory=list)

    @property
    def device(self):
        return self.embed.device

    def answer_rows(self):
        """(allowed ids, retained head rows, true cols, false cols).

        The rows Quail's retain_answer_head keeps
        (quail/backends/quail/executor/model.py:112-134; readout.py:27-38).
        """
        torch = _torch()
        cfg = self.config
        allowed = sorted(set(cfg.true_ids) | set(cfg.false_ids))
        rows = self.embed.index_select(
            0, torch.tensor(allowed, device=self.device)).contiguous()
        true_cols = [i for i, t in enumerate(allowed) if t in set(cfg.true_ids)]
        false_cols = [i for i, t in enumerate(allowed) if t in set(cfg.false_ids)]
        return allowed, rows, true_cols, false_cols

    def to(self, device):
        """A copy of every tensor on another device (the oracle runs on CPU)."""
        def move(x):
            return x.to(device)
        out = Weights(self.config, move(self.embed), move(self.final_norm),
                      move(self.cos_sin))
        for layer in self.layers:
            out.layers.append(Layer(**{k: move(v) for k, v in layer.__dict__.items()}))
        return out


def _torch():
    import torch
    return torch


#: the fp8 linears of a Layer: (weight attribute, block-scale attribute)
LINEARS = (("qkv_w", "qkv_s"), ("o_w", "o_s"), ("gate_up_w", "gate_up_s"),
           ("down_w", "down_s"))


def scales_are_ue8m0(weights) -> bool:
    """True when every block scale of every linear is a power of two."""
    torch = _torch()
    for layer in weights.layers:
        for _, sn in LINEARS:
            bits = getattr(layer, sn).contiguous().view(torch.int32)
            if bool(((bits & 0x807FFFFF) != 0).any()):
                return False
    return True


def requant_ue8m0(weights):
    """Re-quantise every linear to power-of-two block scales in place (the
    UE8M0 mode's load-time step: vLLM's requant_weight_ue8m0_inplace, here
    qb_requant_weight_ue8m0 on the weights' GPU). Returns weights."""
    from quail_b200 import _native as nat
    torch = _torch()
    for layer in weights.layers:
        for wn, sn in LINEARS:
            w, sc = getattr(layer, wn), getattr(layer, sn)
            if not (w.is_contiguous() and sc.is_contiguous()):
                raise ValueError(f"{wn}/{sn}: contiguous tensors needed")
            nat.call("qb_requant_weight_ue8m0", nat.ptr(w), nat.ptr(sc), w.shape[0],
                     w.shape[1], nat.stream_handle(torch))
    return weights


def rotary_cache(cfg: ModelConfig, device="cpu"):
    """vLLM's neox rotary cache: cos | sin of pos * theta^(-2i/d), cast to bf16.

    Restates RotaryEmbedding._compute_cos_sin_cache (vLLM
    model_executor/layers/rotary_embedding/base.py): fp32 on the CPU, then
    the model dtype.
    """
    torch = _torch()
    d = cfg.head_dim
    inv_freq = 1.0 / (cfg.rope_theta ** (
        torch.arange(0, d, 2, dtype=torch.float) / d))
    t = torch.arange(cfg.max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1)
    return cache.to(torch.bfloat16).to(device)


def _fp8_linear(gen, n_out, n_in, device):
    torch = _torch()
    codes = torch.randn(n_out, n_in, generator=gen, device=device,
                        dtype=torch.float32).to(torch.float8_e4m3fn)
    scales = torch.exp(math.log(0.02) + 0.3 * torch.randn(
        n_out // GROUP, n_in // GROUP, generator=gen, device=device,
        dtype=torch.float32))
    return codes, scales


def _norm(gen, n, device):
    torch = _torch()
    w = 1.0 + 0.05 * torch.randn(n, generator=gen, device=device)
    return w.to(torch.bfloat16)


def random_weights(cfg: ModelConfig, seed: int = 0, device="cpu", embed_std=0.02,
                   branch_scale=1.0, final_norm_scale=1.0) -> Weights:
    """Seeded random-init weights of a Qwen3 FP8 model.

    The same (cfg, seed, device type) always gives the same weights; CPU
    and CUDA generators differ, so the oracle copies the device weights.
    """
    torch = _torch()
    if not cfg.fp8:
        raise ValueError("the B200 path runs the FP8 models only")
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    h, d = cfg.hidden, cfg.head_dim
    embed = (embed_std * torch.randn(cfg.vocab, h, generator=gen, device=device)
             ).to(torch.bfloat16)
    final_norm = (_norm(gen, h, device).float() * final_norm_scale).to(torch.bfloat16)
    w = Weights(cfg, embed, final_norm, rotary_cache(cfg, device))
    for _ in range(cfg.n_layers):
        qkv_w, qkv_s = _fp8_linear(gen, cfg.qkv_width, h, device)
        o_w, o_s = _fp8_linear(gen, h, cfg.n_q * d, device)
        gu_w, gu_s = _fp8_linear(gen, 2 * cfg.inter, h, device)
        dn_w, dn_s = _fp8_linear(gen, h, cfg.inter, device)
        o_s *= branch_scale
        dn_s *= branch_scale
        w.layers.append(Layer(
            input_ln=_norm(gen, h, device), post_ln=_norm(gen, h, device),
            q_norm=_norm(gen, d, device), k_norm=_norm(gen, d, device),
            qkv_w=qkv_w, qkv_s=qkv_s, o_w=o_w, o_s=o_s,
            gate_up_w=gu_w, gate_up_s=gu_s, down_w=dn_w, down_s=dn_s))
    return w
