"""ctypes binding of libquailb200.so, the sm_100a kernel library.

The library is the only compute path: there is no CPU or torch fallback.
Loading fails loudly when the shared object is missing; build it with
``python -m quail_b200.build`` (or ``__graft_entry__.build()``).

Every wrapper here checks the library's int status and raises
``ValueError`` for a rejected argument and ``RuntimeError`` for a CUDA
failure, with the library's own message.
"""

import ctypes
import os
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libquailb200.so"

QB_OK = 0
QB_ERR_INVALID = 1
QB_ERR_CUDA = 2
QB_ERR_DEVICE = 3
QB_ERR_TIMEOUT = 4

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_F32 = ctypes.c_float

# name -> argument types; every entry point returns int
SIGNATURES = {
    "qb_version": [],
    "qb_last_error": [],
    "qb_kernel_status": [_I32, _P],
    "qb_set_wait_limit": [_I32, ctypes.c_uint64],
    "qb_embed_rmsnorm_quant": [_P, _I64, _P, _I64, _I64, _P, _F32, _P, _P, _P, _I64, _I32, _P],
    "qb_add_rmsnorm_quant": [_P, _P, _P, _F32, _I64, _I64, _P, _P, _I64, _I32, _P],
    "qb_gemm_fp8_bs": [_P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _I32, _P],
    "qb_qknorm_rope": [_P, _I64, _P, _P, _I64, _P, _P, _F32, _I64, _I32, _I32, _I32,
                       _P, _P, _P, _P, _P, _P, _I64, _P],
    "qb_kv_row_map": [_P, _P, _I64, _I64, _I64, _P, _P],
    "qb_kv_scatter": [_P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _I64, _P],
    "qb_tree_attention": [_P, _P, _P, _I64, _I32, _I32, _I32, _P, _I64, _P, _I64,
                          _P, _P, _P, _I64, _I64, _P, _P, _P, _I64, _I32, _F32,
                          _P, _P, _I64, _I32, _P],
    "qb_tree_attention_tiles": [_P, _I64, _P, _I64, _P],
    "qb_unified_attention": [_P, _I64, _I32, _I32, _I32, _P, _I64, _P, _I64, _P, _P, _I64,
                             _P, _P, _I64, _I32, _F32, _P, _P, _I64, _I32, _P],
    "qb_silu_mul_quant": [_P, _I64, _I64, _P, _P, _I64, _I32, _P],
    "qb_gemm_fp8_silu_quant": [_P, _P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _P],
    "qb_gemm_fp8_qknorm_rope": [_P, _P, _I64, _P, _P, _I64, _I64, _P, _P, _I64, _P, _P, _F32,
                                _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _I64, _I32, _P],
    "qb_requant_weight_ue8m0": [_P, _P, _I64, _I64, _P],
    "qb_final_norm": [_P, _P, _I64, _I64, _P, _I64, _P, _F32, _P, _P],
    "qb_answer_margin": [_P, _I64, _I64, _P, _I32, _P, _I32, _P, _I32, _P, _P, _P],
    "qb_answer_score": [_P, _I64, _I64, _P, _I32, _P, _I32, _P, _I32, _P, _P],
}

_lib = None


class KernelError(RuntimeError):
    """A CUDA failure or a bounded device wait that gave up."""


def load():
    """The loaded library; raises ImportError when it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    path = os.environ.get("QUAIL_B200_LIBRARY", str(LIBRARY))
    if not Path(path).exists():
        raise ImportError(
            f"{path} is missing: build the sm_100a kernels with "
            f"`python -m quail_b200.build` before using quail_b200")
    lib = ctypes.CDLL(path)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_char_p if name == "qb_last_error" else ctypes.c_int
    _lib = lib
    return lib


def exported_symbols():
    """The entry points this binding expects the library to export."""
    return sorted(SIGNATURES)


def check(status: int, what: str) -> None:
    if status == QB_OK:
        return
    msg = load().qb_last_error().decode(errors="replace")
    if status == QB_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise KernelError(f"{what} failed ({status}): {msg}")


# entry points that launch a kernel; LAUNCHES counts them per process
LAUNCHING = frozenset(n for n in SIGNATURES if n not in (
    "qb_version", "qb_last_error", "qb_kernel_status", "qb_set_wait_limit",
    "qb_tree_attention_tiles"))
LAUNCHES = {"count": 0}


def call(name: str, *args) -> None:
    """Call one entry point and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)
    if name in LAUNCHING:
        LAUNCHES["count"] += 1


def ptr(tensor):
    """Device pointer of a tensor (None -> NULL)."""
    return None if tensor is None else ctypes.c_void_p(tensor.data_ptr())


def stream_handle(torch, device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def kernel_status(device: int = 0) -> int:
    """Read and clear the device status word (synchronises the device)."""
    out = ctypes.c_uint32(0)
    call("qb_kernel_status", device, ctypes.byref(out))
    return out.value


def set_wait_limit(device: int = 0, limit_ns: int = 0) -> None:
    """Shorten (or, with 0, restore to one second) the kernels' bounded
    waits on a device; a diagnostic for tests of the give-up path."""
    call("qb_set_wait_limit", device, limit_ns)


def version() -> tuple:
    v = load().qb_version()
    return (v >> 16, (v >> 8) & 0xFF, v & 0xFF)
