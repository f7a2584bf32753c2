"""The Quail-side adapter: what a Quail process registers to select this path.

Three seams of the reference meet quail_b200 here:

- ``device_spec()``: the ``b200`` DeviceSpec the planner prices plans
  against (quail/specs/base.py:168-193; the reference ships h100-sxm and
  rtx-pro-6000 specs, quail/specs/h100_sxm.py), with the dense peaks of
  one B200;
- ``backend_class()``: a QuailBackend subclass named ``quail-b200`` whose
  ``supports`` accepts the Qwen3 architecture on ``b200`` with 1, 2, 4 or
  8 GPUs - the reference's QuailBackend.supports rejects every device but
  h100-sxm and rtx-pro-6000 (quail/backends/quail/backend.py:333-344) -
  and inherits planning and execution unchanged;
- ``weights_from_vllm()``: vLLM's loaded Qwen3 module (the object Quail's
  worker builds, quail/backends/quail/worker.py:46-148) as quail_b200
  Weights, tensors shared, not copied.

``register(registry)`` adds the device and the backend to Quail's
ExtensionRegistry (quail/extensions.py:102-108). Quail itself is imported
only when these functions run, so this module loads without it.
"""

from quail_b200.model import Layer, Weights

#: one B200: 180 GB HBM3e at 7.7 TB/s, dense FP8 4.5 PFLOP/s, dense bf16
#: 2.25 PFLOP/s (NVIDIA's doubled figures are 2:4 sparsity)
B200_DEVICE = dict(name="b200", mem_bytes=180e9, hbm_bw=7.7e12, peak_flops=4.5e15,
                   bf16_flops=2.25e15)

BACKEND_NAME = "quail-b200"
GPU_COUNTS = (1, 2, 4, 8)


def device_spec(DeviceSpec=None):
    """Quail's DeviceSpec for one B200 (DeviceSpec: the class to build,
    Quail's own by default)."""
    if DeviceSpec is None:
        from quail.specs.base import DeviceSpec
    return DeviceSpec(**B200_DEVICE)


def backend_class(QuailBackend=None, SupportResult=None):
    """A QuailBackend subclass that runs the Qwen3 FP8 path on b200.

    Planning, request preparation and execution are Quail's; only the
    support check differs. The classes default to Quail's own."""
    if QuailBackend is None:
        from quail.backends.quail.backend import QuailBackend
    if SupportResult is None:
        from quail.planner.physical_optimizer import SupportResult

    class B200QuailBackend(QuailBackend):
        name = BACKEND_NAME

        def supports(self, model, device, gpu_count):
            if device.name != B200_DEVICE["name"]:
                return SupportResult.reject(f"{BACKEND_NAME} runs on b200 only, not "
                                            f"{device.name!r}")
            if getattr(model, "arch", None) != "qwen3":
                return SupportResult.reject(f"{BACKEND_NAME} runs the Qwen3 FP8 path, not "
                                            f"architecture {getattr(model, 'arch', None)!r}")
            if getattr(model, "weight_precision", "fp8") != "fp8":
                return SupportResult.reject(f"{BACKEND_NAME} needs FP8 block-scaled weights")
            if gpu_count not in GPU_COUNTS:
                return SupportResult.reject(f"{BACKEND_NAME} runs on 1, 2, 4 or 8 GPUs")
            return SupportResult.accept()

    return B200QuailBackend


def register(registry, DeviceSpec=None, QuailBackend=None, SupportResult=None):
    """Register the b200 device and the quail-b200 backend; returns registry."""
    cls = backend_class(QuailBackend, SupportResult)
    return registry.register_device(device_spec(DeviceSpec)).register_backend(cls())


def weights_from_vllm(model, cfg, torch=None):
    """vLLM's loaded Qwen3 module as quail_b200 Weights.

    vLLM's layout is the one the kernels take (quail/backends/quail/
    executor/models/qwen3.py:24-44): qkv_proj rows q | k | v, gate_up_proj
    gate rows first, fp8 weights [N, K] with fp32 ``weight_scale_inv``
    [N/128, K/128], bf16 norms and embeddings (tied head), and the rotary
    module's cos | sin cache, cast to bf16 as Quail's qk_norm_rope reads it.
    Raises ValueError on a shape the kernels do not take.
    """
    if torch is None:
        import torch
    m = model.model
    layers = list(m.layers)
    if len(layers) != cfg.n_layers:
        raise ValueError(f"model has {len(layers)} layers, config {cfg.name} has "
                         f"{cfg.n_layers}")
    cos_sin = layers[0].self_attn.rotary_emb.cos_sin_cache.to(torch.bfloat16)
    w = Weights(cfg, m.embed_tokens.weight, m.norm.weight, cos_sin)

    def linear(lin, n, k, what):
        weight = lin.weight
        scale = getattr(lin, "weight_scale_inv", None)
        if scale is None:
            scale = getattr(lin, "weight_scale", None)
        if tuple(weight.shape) != (n, k):
            raise ValueError(f"{what}: weight {tuple(weight.shape)}, expected [N, K] = "
                             f"{(n, k)} (K-major)")
        if scale is None or tuple(scale.shape) != (n // 128, k // 128):
            raise ValueError(f"{what}: block scales must be [N/128, K/128] = "
                             f"{(n // 128, k // 128)}")
        return weight, scale

    h, d = cfg.hidden, cfg.head_dim
    for i, layer in enumerate(layers):
        a, f = layer.self_attn, layer.mlp
        qkv_w, qkv_s = linear(a.qkv_proj, cfg.qkv_width, h, f"layer {i} qkv_proj")
        o_w, o_s = linear(a.o_proj, h, cfg.n_q * d, f"layer {i} o_proj")
        gu_w, gu_s = linear(f.gate_up_proj, 2 * cfg.inter, h, f"layer {i} gate_up_proj")
        dn_w, dn_s = linear(f.down_proj, h, cfg.inter, f"layer {i} down_proj")
        w.layers.append(Layer(
            input_ln=layer.input_layernorm.weight, post_ln=layer.post_attention_layernorm.weight,
            q_norm=a.q_norm.weight, k_norm=a.k_norm.weight, qkv_w=qkv_w, qkv_s=qkv_s,
            o_w=o_w, o_s=o_s, gate_up_w=gu_w, gate_up_s=gu_s, down_w=dn_w, down_s=dn_s))
    return w
