"""ctypes wrapper of oracle/libqbmodel.so (oracle/tcmodel.c). Test infrastructure.

Builds the library on first use when it is missing (gcc is in the image).
Arrays are torch CPU tensors; results are new tensors.
"""

import ctypes

import torch

from oracle import build as _build

_lib = None
_P = ctypes.c_void_p
_I = ctypes.c_int64


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(str(path))
        L.qbm_gemm_fp8.argtypes = [_P, _P, _I, _P, _P, _P, _I, _I, _I]
        L.qbm_gemm_fp8_f32.argtypes = [_P, _P, _I, _P, _P, _P, _I, _I, _I]
        L.qbm_gemm_mx.argtypes = [_P, _P, _I, _P, _P, _P, _I, _I, _I]
        L.qbm_gemm_mx_f32.argtypes = [_P, _P, _I, _P, _P, _P, _I, _I, _I]
        L.qbm_mma_bf16.argtypes = [_P, _P, _P, _P, _I, _I, _I]
        for name in ("qbm_exp2f_array", "qbm_exp2s_array", "qbm_sigmoidf_array",
                     "qbm_lnf_array"):
            getattr(L, name).argtypes = [_P, _P, _I]
        L.qbm_fmaf_array.argtypes = [_P, _P, _P, _P, _I]
        L.qbm_sumsq_rows.argtypes = [_P, _I, _I, _P]
        L.qbm_sumsq_heads.argtypes = [_P, _I, _P]
        L.qbm_dot_rows.argtypes = [_P, _P, _I, _I, _I, _P]
        for name in ("qbm_exp2f", "qbm_lnf", "qbm_sigmoidf", "qbm_expf"):
            getattr(L, name).argtypes = [ctypes.c_float]
            getattr(L, name).restype = ctypes.c_float
        _lib = L
    return _lib


def _c(t, dtype=None):
    t = t.detach().contiguous()
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def gemm_fp8(a_codes, a_scales, w_codes, w_scales):
    """The kernel's FP8 block-scaled GEMM, bit for bit: bf16 [M, N]."""
    a = _c(a_codes).view(torch.uint8)
    w = _c(w_codes).view(torch.uint8)
    as_ = _c(a_scales, torch.float32)
    ws = _c(w_scales, torch.float32)
    m, k = a.shape
    n = w.shape[0]
    out = torch.empty(m, n, dtype=torch.int16)
    lib().qbm_gemm_fp8(_p(a), _p(as_), as_.shape[1], _p(w), _p(ws), _p(out), m, n, k)
    return out.view(torch.bfloat16)


def gemm_fp8_f32(a_codes, a_scales, w_codes, w_scales):
    """gemm_fp8's fp32 accumulator, before the bf16 rounding."""
    a = _c(a_codes).view(torch.uint8)
    w = _c(w_codes).view(torch.uint8)
    as_ = _c(a_scales, torch.float32)
    ws = _c(w_scales, torch.float32)
    m, k = a.shape
    n = w.shape[0]
    out = torch.empty(m, n, dtype=torch.float32)
    lib().qbm_gemm_fp8_f32(_p(a), _p(as_), as_.shape[1], _p(w), _p(ws), _p(out), m, n, k)
    return out


def gemm_mx(a_codes, a_scales, w_codes, w_scales, f32=False):
    """The kernel's UE8M0-mode GEMM (block-scaled MMA over the whole K),
    bit for bit: bf16 [M, N] (f32: the accumulator before rounding)."""
    a = _c(a_codes).view(torch.uint8)
    w = _c(w_codes).view(torch.uint8)
    as_ = _c(a_scales, torch.float32)
    ws = _c(w_scales, torch.float32)
    m, k = a.shape
    n = w.shape[0]
    if f32:
        out = torch.empty(m, n, dtype=torch.float32)
        lib().qbm_gemm_mx_f32(_p(a), _p(as_), as_.shape[1], _p(w), _p(ws), _p(out), m, n, k)
        return out
    out = torch.empty(m, n, dtype=torch.int16)
    lib().qbm_gemm_mx(_p(a), _p(as_), as_.shape[1], _p(w), _p(ws), _p(out), m, n, k)
    return out.view(torch.bfloat16)


def mma_bf16(a, b, c0=None):
    """Chain of mma.sync bf16 K=16 steps: C0 + a @ b^T under the tensor-core model.

    a [M, K] bf16, b [N, K] bf16, c0 [M, N] f32 or None -> f32 [M, N]."""
    a = _c(a, torch.bfloat16).view(torch.int16)
    b = _c(b, torch.bfloat16).view(torch.int16)
    m, k = a.shape
    n = b.shape[0]
    out = torch.empty(m, n, dtype=torch.float32)
    c = None if c0 is None else _c(c0, torch.float32)
    lib().qbm_mma_bf16(_p(a), _p(b), None if c is None else _p(c), _p(out), m, n, k)
    return out


def _unary(name, x):
    x = _c(x, torch.float32)
    y = torch.empty_like(x)
    getattr(lib(), name)(_p(x), _p(y), x.numel())
    return y


def exp2(x):
    return _unary("qbm_exp2f_array", x)


def exp2_soft(x):
    """The attention softmax's exp2 (the kernel's qexp2s)."""
    return _unary("qbm_exp2s_array", x)


def sigmoid(x):
    return _unary("qbm_sigmoidf_array", x)


def ln(x):
    return _unary("qbm_lnf_array", x)


def fma(a, b, c):
    a, b, c = torch.broadcast_tensors(_c(a, torch.float32), _c(b, torch.float32),
                                      _c(c, torch.float32))
    a, b, c = a.contiguous(), b.contiguous(), c.contiguous()
    y = torch.empty_like(a)
    lib().qbm_fmaf_array(_p(a), _p(b), _p(c), _p(y), a.numel())
    return y


def sumsq_rows(x):
    """Row sums of squares in the norm kernels' order: f32 [rows]."""
    x = _c(x, torch.float32)
    rows, h = x.shape
    out = torch.empty(rows, dtype=torch.float32)
    lib().qbm_sumsq_rows(_p(x), rows, h, _p(out))
    return out


def sumsq_heads(x):
    """Per-head (128-wide) sums of squares in the rotary kernel's order."""
    x = _c(x, torch.float32).reshape(-1, 128)
    out = torch.empty(x.shape[0], dtype=torch.float32)
    lib().qbm_sumsq_heads(_p(x), x.shape[0], _p(out))
    return out


def dot_rows(y, w):
    """Dot products in the answer kernel's order: f32 [rows, n_ids]."""
    y = _c(y, torch.float32)
    w = _c(w, torch.float32)
    out = torch.empty(y.shape[0], w.shape[0], dtype=torch.float32)
    lib().qbm_dot_rows(_p(y), _p(w), y.shape[0], w.shape[0], y.shape[1], _p(out))
    return out
