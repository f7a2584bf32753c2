"""The branch-free fast paths of the kernels' numerics, checked exhaustively
on the GPU against the exact forms (tests/numerics_check.cu): Markstein's
reciprocal over every normal d, the fast sigmoid over every fp32 pattern,
the quantisation scale over every group max, the saturating quantiser
over 2^30 values, and the attention softmax's exp2: its packed form against
the scalar one over every x <= 1, within 5e-7 relative of CUDA's exp2f on
[-125, 1] (its own bound 1.7e-7 plus exp2f's 2 ulp), and equal to the oracle's C restatement (oracle/tcmodel.c
qbm_exp2s) on 2^24 sampled inputs and the edges. Any mismatch breaks bit
parity with the oracle."""

import ctypes
import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
NAMES = ["rcp_rn_normal_x2", "sigmoidf_ref_x2_fast", "group_scale", "quant2_sat",
         "qexp2s_x2", "qexp2s_error_bound"]


@pytest.fixture(scope="module")
def checks(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    so = tmp_path_factory.mktemp("numerics") / "numerics_check.so"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-shared", "-I",
                    str(ROOT / "include"), "-I", str(ROOT / "quail_b200" / "csrc"), "-o", str(so),
                    str(HERE / "numerics_check.cu")], check=True)
    return ctypes.CDLL(str(so))


def test_softmax_exp2_matches_the_oracle(checks):
    import numpy as np
    import torch

    from oracle import tc
    rng = np.random.default_rng(5)
    x = np.concatenate([
        -rng.exponential(8.0, 1 << 23).astype(np.float32),
        rng.uniform(-130.0, 1.0, 1 << 23).astype(np.float32),
        np.array([0.0, -0.0, 1.0, 0.5, -0.5, -125.5, -126.0, -126.5, -126.49999, -126.50001,
                  -127.0, -150.0, -1e30, -np.inf, np.nan], dtype=np.float32)])
    y = np.empty_like(x)
    lib = checks
    lib.qbn_exp2s.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    assert lib.qbn_exp2s(x.ctypes.data, y.ctypes.data, x.size) == 0
    want = tc.exp2_soft(torch.from_numpy(x)).numpy()
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(y), nan)
    diff = np.flatnonzero(y[~nan].view(np.uint32) != want[~nan].view(np.uint32))
    assert diff.size == 0, (diff.size, x[~nan][diff[:5]], y[~nan][diff[:5]], want[~nan][diff[:5]])


def test_fast_numerics_paths_are_exact(checks):
    lib = checks
    bad = (ctypes.c_ulonglong * 6)()
    first = (ctypes.c_uint * 6)()
    assert lib.qbn_run_checks(bad, first) == 0
    report = {n: (int(bad[i]), hex(first[i])) for i, n in enumerate(NAMES)}
    assert all(int(b) == 0 for b in bad), report
