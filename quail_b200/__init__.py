"""quail_b200: Quail's AI.IF / AI_FILTER prefill hot path on B200 (sm_100a).

Host side (Python, mirroring Quail's executor seams): the prefix tree
(tokens), the paged KV arena (arena), filter admission (pack), the
overlapped chunk loop (loop), the Qwen3 pipeline (pipeline), the answer
readout (readout) and multi-GPU row sharding (distributed). Device side:
libquailb200.so, the sm_100a kernels behind the C ABI in
include/quail_b200.h, loaded by quail_b200._native.
"""

__version__ = "0.1.0"
