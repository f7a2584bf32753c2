"""CPU oracle of the AI.IF prefill path - TEST INFRASTRUCTURE ONLY.

This package restates, in plain torch-CPU fp32 arithmetic, the numerics
of the reference's Qwen3 forward pass (Quail's Engine and Qwen3Pipeline,
quail/backends/quail/executor/{attention.py,models/qwen3.py,readout.py}).
It is the checker the parity tests, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg of ``bench.py`` compare the CUDA kernels against; the
product path (quail_b200) never imports it.

Pinning: the fused elementwise kernels (norm+quant, qk-norm+rope, SiLU
quant, LSE merge+quant) are pinned against golden vectors produced by the
reference's own Triton kernels run under TRITON_INTERPRET=1
(tests/golden/make_golden.py). The GEMM (DeepGEMM fp8_gemm_nt), the
FlashAttention calls, vLLM's RMSNorm ops and the rotary cache come from
third-party libraries that are not in the reference tree; they are
restated from their published algorithms and are "parity unpinned" by
reference-produced vectors.
"""
