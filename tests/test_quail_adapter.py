"""The Quail-side adapter (quail_b200/quail_adapter.py), on the CPU.

- weights_from_vllm over a stand-in of vLLM's loaded Qwen3 module: the
  Weights share its tensors, and shapes the kernels do not take are
  rejected;
- the backend's support check and the registration, with stand-ins for
  Quail's classes;
- with the reference checkout present, the same registration against
  Quail's own ExtensionRegistry, DeviceSpec, QuailBackend and Qwen3 model
  specs (in a child process, so the stand-in for Quail's SQL dependency
  stays out of this one). Skipped where the reference is absent.
"""

import subprocess
import sys
import textwrap
from dataclasses import dataclass
from pathlib import Path
from types import SimpleNamespace as NS

import pytest
import torch

from quail_b200 import quail_adapter as qa
from quail_b200.model import TINY, random_weights

ROOT = Path(__file__).resolve().parent.parent
REFERENCE = Path("/root/reference")


def fake_vllm(weights):
    """vLLM's Qwen3ForCausalLM attribute layout around quail_b200 tensors."""
    layers = []
    for L in weights.layers:
        attn = NS(qkv_proj=NS(weight=L.qkv_w, weight_scale_inv=L.qkv_s),
                  o_proj=NS(weight=L.o_w, weight_scale_inv=L.o_s),
                  q_norm=NS(weight=L.q_norm), k_norm=NS(weight=L.k_norm),
                  rotary_emb=NS(cos_sin_cache=weights.cos_sin.float()))
        mlp = NS(gate_up_proj=NS(weight=L.gate_up_w, weight_scale_inv=L.gate_up_s),
                 down_proj=NS(weight=L.down_w, weight_scale_inv=L.down_s))
        layers.append(NS(self_attn=attn, mlp=mlp, input_layernorm=NS(weight=L.input_ln),
                         post_attention_layernorm=NS(weight=L.post_ln)))
    return NS(model=NS(embed_tokens=NS(weight=weights.embed), norm=NS(weight=weights.final_norm),
                       layers=layers))


def test_weights_from_vllm_shares_tensors():
    w = random_weights(TINY, seed=3, device="cpu")
    got = qa.weights_from_vllm(fake_vllm(w), TINY, torch)
    assert got.embed is w.embed and got.final_norm is w.final_norm
    assert torch.equal(got.cos_sin, w.cos_sin)
    for a, b in zip(got.layers, w.layers):
        for name in ("qkv_w", "qkv_s", "o_w", "o_s", "gate_up_w", "gate_up_s", "down_w",
                     "down_s", "input_ln", "post_ln", "q_norm", "k_norm"):
            assert getattr(a, name) is getattr(b, name), name


def test_weights_from_vllm_rejects_other_layouts():
    w = random_weights(TINY, seed=3, device="cpu")
    m = fake_vllm(w)
    m.model.layers[1].mlp.gate_up_proj.weight = w.layers[1].gate_up_w.t()   # [K, N]
    with pytest.raises(ValueError, match="gate_up_proj"):
        qa.weights_from_vllm(m, TINY, torch)
    m = fake_vllm(w)
    m.model.layers[0].mlp.down_proj.weight_scale_inv = w.layers[0].down_s[:, :1]
    with pytest.raises(ValueError, match="block scales"):
        qa.weights_from_vllm(m, TINY, torch)
    m = fake_vllm(w)
    m.model.layers = m.model.layers[:1]
    with pytest.raises(ValueError, match="layers"):
        qa.weights_from_vllm(m, TINY, torch)


@dataclass(frozen=True)
class _Result:
    supported: bool
    reason: str = None

    @classmethod
    def accept(cls):
        return cls(True)

    @classmethod
    def reject(cls, reason):
        return cls(False, reason)


class _QuailBackend:
    name = "quail"

    def supports(self, model, device, gpu_count):
        return _Result.reject("the reference's check")


@dataclass(frozen=True)
class _Device:
    name: str
    mem_bytes: float
    hbm_bw: float
    peak_flops: float
    bf16_flops: float = 0.0


class _Registry:
    def __init__(self):
        self.items = {}

    def register_device(self, d):
        self.items["device", d.name] = d
        return self

    def register_backend(self, b):
        self.items["backend", b.name] = b
        return self


def test_backend_support_check_and_registration():
    reg = qa.register(_Registry(), _Device, _QuailBackend, _Result)
    dev, backend = reg.items["device", "b200"], reg.items["backend", "quail-b200"]
    assert isinstance(backend, _QuailBackend)
    assert dev.peak_flops == 4.5e15 and dev.mem_bytes == 180e9
    qwen = NS(arch="qwen3", weight_precision="fp8", name="qwen3-4b-fp8")
    assert backend.supports(qwen, dev, 8).supported
    assert backend.supports(qwen, dev, 1).supported
    assert not backend.supports(qwen, dev, 3).supported
    assert not backend.supports(qwen, NS(name="h100-sxm"), 1).supported
    gemma = NS(arch="diffusion_gemma", weight_precision="fp8", name="g")
    assert "Qwen3" in backend.supports(gemma, dev, 1).reason
    bf16 = NS(arch="qwen3", weight_precision="bf16", name="q")
    assert not backend.supports(bf16, dev, 1).supported


@pytest.mark.skipif(not (REFERENCE / "quail").is_dir(), reason="reference checkout absent")
def test_registration_with_quails_own_classes():
    script = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(ROOT)!r})
        from tests.golden import make_golden as mg
        mg._install_reference({str(REFERENCE)!r})
        from quail.extensions import ExtensionRegistry
        from quail.specs import QWEN3_4B_FP8, QWEN3_32B_FP8
        from quail.specs.h100_sxm import H100_SXM
        from quail.backends.quail.backend import QuailBackend
        from quail_b200 import quail_adapter as qa
        reg = qa.register(ExtensionRegistry())
        dev = reg._registrations["device", "b200"]
        backend = reg._registrations["backend", "quail-b200"]
        assert isinstance(backend, QuailBackend)
        assert backend.supports(QWEN3_4B_FP8, dev, 8).supported
        assert backend.supports(QWEN3_32B_FP8, dev, 1).supported
        assert not backend.supports(QWEN3_4B_FP8, H100_SXM, 1).supported
        assert not QuailBackend().supports(QWEN3_4B_FP8, dev, 1).supported
        print("ok", dev.attn_flops)
    """)
    out = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True,
                         cwd=str(ROOT), timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.startswith("ok 2250000000000000")
