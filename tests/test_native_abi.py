"""The C ABI: the library loads and exports every entry point the header
declares, and argument checks reject bad calls before any launch (these
calls touch no GPU, so they run on the CPU-only test host)."""

import ctypes
import re
from pathlib import Path

import pytest

from quail_b200 import _native as nat

HEADER = Path(__file__).resolve().parent.parent / "include" / "quail_b200.h"


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(qb_\w+)\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    if not nat.LIBRARY.exists():
        from quail_b200 import build
        build.build()
    return nat.load()


def test_header_and_binding_agree():
    assert header_functions() == nat.exported_symbols()


def test_library_exports_every_declared_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), name


def test_version(lib):
    assert nat.version() >= (0, 1, 0)


def test_invalid_gemm_shapes_are_rejected_before_launch(lib):
    with pytest.raises(ValueError, match="multiple of 128"):
        nat.call("qb_gemm_fp8_bs", None, None, 8, None, None, None, 8, 256, 100, 0, None)
    with pytest.raises(ValueError, match="multiple of 128"):
        nat.call("qb_gemm_fp8_bs", None, None, 8, None, None, None, 8, 200, 256, 0, None)
    with pytest.raises(ValueError, match="a_scale_ld"):
        nat.call("qb_gemm_fp8_bs", None, None, 4, None, None, None, 8, 256, 256, 0, None)
    unaligned = ctypes.c_void_p(0x1001)
    with pytest.raises(ValueError, match="aligned"):
        nat.call("qb_gemm_fp8_bs", unaligned, unaligned, 8, unaligned, unaligned,
                 unaligned, 8, 256, 256, 0, None)


def test_invalid_fused_silu_gemm_calls_are_rejected(lib):
    with pytest.raises(ValueError, match="inter must be a multiple of 128"):
        nat.call("qb_gemm_fp8_silu_quant", None, None, 8, None, None, None, None, 8, 8, 100,
                 256, 0, None)
    with pytest.raises(ValueError, match="scale_ld"):
        nat.call("qb_gemm_fp8_silu_quant", None, None, 8, None, None, None, None, 4, 8, 128,
                 256, 0, None)
    unaligned = ctypes.c_void_p(0x1001)
    with pytest.raises(ValueError, match="aligned"):
        nat.call("qb_gemm_fp8_silu_quant", unaligned, unaligned, 8, unaligned, unaligned,
                 unaligned, unaligned, 8, 8, 128, 256, 0, None)


def test_invalid_fused_qkv_calls_are_rejected(lib):
    # 3 + 2 * 1 heads: a 256-column tile would split a head
    with pytest.raises(ValueError, match="even"):
        nat.call("qb_gemm_fp8_qknorm_rope", None, None, 8, None, None, 8, 256, None, None, 10,
                 None, None, 1e-6, 3, 1, 128, None, None, None, None, None, None, 0, 0, None)
    with pytest.raises(ValueError, match="head_dim"):
        nat.call("qb_gemm_fp8_qknorm_rope", None, None, 8, None, None, 8, 256, None, None, 10,
                 None, None, 1e-6, 4, 2, 64, None, None, None, None, None, None, 0, 0, None)
    # the rotary table and norm weights are copied 16 bytes at a time: a
    # 4-byte aligned cos_sin (enough for qb_qknorm_rope) is refused here
    ok16, four = ctypes.c_void_p(0x1000), ctypes.c_void_p(0x1004)
    with pytest.raises(ValueError, match="16-byte aligned"):
        nat.call("qb_gemm_fp8_qknorm_rope", ok16, ok16, 8, ok16, ok16, 8, 256, ok16, four, 10,
                 ok16, ok16, 1e-6, 4, 2, 128, ok16, ok16, ok16, None, None, None, 0, 0, None)
    with pytest.raises(ValueError, match="16-byte aligned"):
        nat.call("qb_gemm_fp8_qknorm_rope", ok16, ok16, 8, ok16, ok16, 8, 256, ok16, ok16, 10,
                 four, ok16, 1e-6, 4, 2, 128, ok16, ok16, ok16, None, None, None, 0, 0, None)
    # a KV pool whose rows do not fit a 32-bit TMA coordinate
    with pytest.raises(ValueError, match="pool_rows"):
        nat.call("qb_gemm_fp8_qknorm_rope", ok16, ok16, 8, ok16, ok16, 8, 256, ok16, ok16, 10,
                 ok16, ok16, 1e-6, 4, 2, 128, ok16, ok16, ok16, ok16, ok16, ok16, 1 << 31, 0, None)


def test_invalid_attention_and_norm_calls_are_rejected(lib):
    with pytest.raises(ValueError, match="head_dim"):
        nat.call("qb_tree_attention", None, None, None, 4, 4, 2, 64, None, 1, None, 1,
                 None, None, None, 0, 0, None, None, None, 0, 16, 0.1, None, None, 4, 0, None)
    with pytest.raises(ValueError, match="multiple of n_kv"):
        nat.call("qb_unified_attention", None, 4, 6, 4, 128, None, 1, None, 1, None, None,
                 1, None, None, 1, 16, 0.1, ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 0,
                 None)
    with pytest.raises(ValueError, match="multiple of 256"):
        nat.call("qb_add_rmsnorm_quant", None, None, None, 1e-6, 4, 300, None, None, 4, 0, None)
    with pytest.raises(ValueError, match="n_ids"):
        nat.call("qb_answer_margin", None, 1, 512, None, 17, None, 1, None, 1, None, None,
                 None)
    with pytest.raises(ValueError, match="128"):
        nat.call("qb_qknorm_rope", None, 768, None, None, 10, None, None, 1e-6, 2, 4, 2, 64,
                 None, None, None, None, None, None, 0, None)


def test_tiles_helper_runs_on_host(lib):
    cu = (ctypes.c_int32 * 4)(0, 70, 70, 200)
    out = (ctypes.c_int32 * 20)()
    n = ctypes.c_int64(0)
    nat.call("qb_tree_attention_tiles", cu, 3, out, 10, ctypes.byref(n))
    assert n.value == 2 + 3
    pairs = [(out[2 * i], out[2 * i + 1]) for i in range(n.value)]
    assert pairs == [(0, 0), (0, 64), (2, 70), (2, 134), (2, 198)]
