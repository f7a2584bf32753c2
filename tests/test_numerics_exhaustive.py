"""The branch-free fast paths of the kernels' numerics, checked exhaustively
on the GPU against the exact forms (tests/numerics_check.cu): Markstein's
reciprocal over every normal d, the fast sigmoid over every fp32 pattern,
the quantisation scale over every group max, the saturating quantiser
over 2^30 values and the softmax exp2 over every x <= 1. Any mismatch
breaks bit parity with the oracle."""

import ctypes
import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
NAMES = ["rcp_rn_normal_x2", "sigmoidf_ref_x2_fast", "group_scale", "quant2_sat",
         "qexp2f_x2_softmax"]


def test_fast_numerics_paths_are_exact(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    so = tmp_path / "numerics_check.so"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-shared", "-I",
                    str(ROOT / "include"), "-I", str(ROOT / "quail_b200" / "csrc"), "-o", str(so),
                    str(HERE / "numerics_check.cu")], check=True)
    lib = ctypes.CDLL(str(so))
    bad = (ctypes.c_ulonglong * 5)()
    first = (ctypes.c_uint * 5)()
    assert lib.qbn_run_checks(bad, first) == 0
    report = {n: (int(bad[i]), hex(first[i])) for i, n in enumerate(NAMES)}
    assert all(int(b) == 0 for b in bad), report
