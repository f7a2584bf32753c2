"""Measure the B200 tensor cores' fp32 accumulation and save it as a fixture.

Needs a B200: builds tests/golden/tensorcore_probe.cu (the library's GEMM
instantiated with an fp32 output, plus one mma.sync m16n8k16 bf16 per
launch) and records, for seeded operands with a wide exponent spread:

- gemm_s{3,6}_*: e4m3 codes a [64, 128], w [64, 128] and the fp32
  accumulator of one 128-deep block (four tcgen05 K=32 MMAs, unit scales);
- mx_s{3,6}_*: the UE8M0 mode's block-scaled MMA (kind::mxf8f6f4): codes
  a [64, 512], w [64, 512], power-of-two scales with random exponents
  (a_scale [4, 64], w_scale [1, 4]) and the fp32 accumulator of the whole
  K (sixteen K=32 steps);
- mma_*: bf16 A [16, 16], B [16, 8], fp32 C and the fp32 D = C + A B of one
  mma.sync;
- tcf16_m{0,1}_r*: tcgen05 kind::f16 (bf16) chains of four K=16 MMAs in the
  tcgen05 attention's layouts: bf16 A [128, 64], B [64, 64] read K-major
  (mode 0, N = 64) or V [64, 128] read MN-major (mode 1, N = 128), the fp32
  C preloaded into TMEM (NaN placeholder: not loaded) and D.

tests/test_oracle_model.py checks that oracle/tcmodel.c reproduces every
output bit for bit. Run: python tests/golden/make_tensorcore_probe.py
[output .npz, default tests/golden/tensorcore_probe.npz]
"""

import ctypes
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def build(tmp):
    so = Path(tmp) / "probe.so"
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-I",
                    str(ROOT / "include"), "-o", str(so), str(HERE / "tensorcore_probe.cu"),
                    str(ROOT / "quail_b200" / "csrc" / "capi.cu")], check=True)
    return ctypes.CDLL(str(so))


def operands(rng, shape, spread):
    x = rng.standard_normal(shape) * np.exp2(rng.integers(-spread, spread + 1, shape))
    return np.clip(x, -400, 400).astype(np.float32)


def main():
    dev = torch.device("cuda")
    rng = np.random.default_rng(0)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        lib = build(tmp)
        P = ctypes.c_void_p
        stream = P(torch.cuda.current_stream().cuda_stream)
        for spread in (3, 6):
            a = torch.from_numpy(operands(rng, (128, 128), spread)).to(torch.float8_e4m3fn)
            w = torch.from_numpy(operands(rng, (256, 128), spread)).to(torch.float8_e4m3fn)
            A, W = a.to(dev), w.to(dev)
            AS, WS = torch.ones(1, 128, device=dev), torch.ones(2, 1, device=dev)
            res = torch.zeros(128, 256, device=dev)
            assert lib.probe_gemm_f32(P(A.data_ptr()), P(AS.data_ptr()), ctypes.c_int64(128),
                                      P(W.data_ptr()), P(WS.data_ptr()), P(res.data_ptr()),
                                      ctypes.c_int64(128), ctypes.c_int64(256),
                                      ctypes.c_int64(128), stream) == 0
            torch.cuda.synchronize()
            out[f"gemm_s{spread}_a"] = a.view(torch.uint8).numpy()[:64]
            out[f"gemm_s{spread}_w"] = w.view(torch.uint8).numpy()[:64]
            out[f"gemm_s{spread}_out"] = res.cpu().numpy()[:64, :64]
        reps = 96
        A = np.zeros((reps, 16, 16), np.float32)
        B = np.zeros((reps, 16, 8), np.float32)
        C = np.zeros((reps, 16, 8), np.float32)
        af = np.zeros((reps, 32, 4), np.uint32)
        bfr = np.zeros((reps, 32, 2), np.uint32)
        cf = np.zeros((reps, 32, 4), np.float32)
        for r in range(reps):
            s = (0, 4, 8)[r % 3]
            ta = torch.from_numpy(operands(rng, (16, 16), s)).to(torch.bfloat16)
            tb = torch.from_numpy(operands(rng, (16, 8), s)).to(torch.bfloat16)
            A[r], B[r] = ta.float().numpy(), tb.float().numpy()
            C[r] = 0 if r % 4 == 0 else operands(rng, (16, 8), s)
            ba = ta.view(torch.int16).numpy().astype(np.uint16).astype(np.uint32)
            bb = tb.view(torch.int16).numpy().astype(np.uint16).astype(np.uint32)
            for t in range(32):
                g, q = t // 4, t % 4
                af[r, t] = [ba[g, 2 * q] | ba[g, 2 * q + 1] << 16,
                            ba[g + 8, 2 * q] | ba[g + 8, 2 * q + 1] << 16,
                            ba[g, 2 * q + 8] | ba[g, 2 * q + 9] << 16,
                            ba[g + 8, 2 * q + 8] | ba[g + 8, 2 * q + 9] << 16]
                bfr[r, t] = [bb[2 * q, g] | bb[2 * q + 1, g] << 16,
                             bb[2 * q + 8, g] | bb[2 * q + 9, g] << 16]
                cf[r, t] = [C[r, g, 2 * q], C[r, g, 2 * q + 1], C[r, g + 8, 2 * q],
                            C[r, g + 8, 2 * q + 1]]
        ad = torch.from_numpy(af.view(np.int32)).to(dev)
        bd = torch.from_numpy(bfr.view(np.int32)).to(dev)
        cd = torch.from_numpy(cf).to(dev)
        dd = torch.zeros_like(cd)
        assert lib.probe_mma(P(ad.data_ptr()), P(bd.data_ptr()), P(cd.data_ptr()),
                             P(dd.data_ptr()), reps, stream) == 0
        torch.cuda.synchronize()
        dn = dd.cpu().numpy()
        D = np.zeros((reps, 16, 8), np.float32)
        for t in range(32):
            g, q = t // 4, t % 4
            D[:, g, 2 * q], D[:, g, 2 * q + 1] = dn[:, t, 0], dn[:, t, 1]
            D[:, g + 8, 2 * q], D[:, g + 8, 2 * q + 1] = dn[:, t, 2], dn[:, t, 3]
        out.update(mma_A=A, mma_B=B, mma_C=C, mma_D=D)
        # tcgen05 kind::f16: mode 0 = S (B K-major, N 64), mode 1 = PV (B = V
        # MN-major, N 128); C preloaded in TMEM (zero for r % 4 == 1) or not
        for mode in (0, 1):
            n = 64 if mode == 0 else 128
            for r in range(6):
                s = (0, 4, 8)[r % 3]
                use_c = 0 if r % 4 == 0 else 1
                ta = torch.from_numpy(operands(rng, (128, 64), s)).to(torch.bfloat16)
                tb = torch.from_numpy(operands(rng, (64, n), s)).to(torch.bfloat16)
                c = np.zeros((128, n), np.float32)
                if use_c and r % 4 != 1:
                    c = operands(rng, (128, n), s)
                ad, bd = ta.to(dev), tb.to(dev)
                cd = torch.from_numpy(c).to(dev)
                dd = torch.zeros(128, n, device=dev)
                assert lib.probe_tc_f16(mode, P(ad.data_ptr()), P(bd.data_ptr()),
                                        P(cd.data_ptr()), P(dd.data_ptr()), use_c, stream) == 0
                torch.cuda.synchronize()
                key = f"tcf16_m{mode}_r{r}"
                out[key + "_a"] = ta.view(torch.int16).numpy()
                out[key + "_b"] = tb.view(torch.int16).numpy()
                out[key + "_c"] = c if use_c else np.full((1,), np.nan, np.float32)
                out[key + "_d"] = dd.cpu().numpy()
        # separate stream: the entries above keep their operands
        rng_mx = np.random.default_rng(1)
        for spread in (3, 6):
            a = torch.from_numpy(operands(rng_mx, (128, 512), spread)).to(torch.float8_e4m3fn)
            w = torch.from_numpy(operands(rng_mx, (256, 512), spread)).to(torch.float8_e4m3fn)
            a_s = np.exp2(rng_mx.integers(-12, 5, (4, 128))).astype(np.float32)
            w_s = np.exp2(rng_mx.integers(-12, 5, (2, 4))).astype(np.float32)
            A, W = a.to(dev), w.to(dev)
            AS, WS = torch.from_numpy(a_s).to(dev), torch.from_numpy(w_s).to(dev)
            res = torch.zeros(128, 256, device=dev)
            assert lib.probe_gemm_mx_f32(P(A.data_ptr()), P(AS.data_ptr()), ctypes.c_int64(128),
                                         P(W.data_ptr()), P(WS.data_ptr()), P(res.data_ptr()),
                                         ctypes.c_int64(128), ctypes.c_int64(256),
                                         ctypes.c_int64(512), stream) == 0
            torch.cuda.synchronize()
            out[f"mx_s{spread}_a"] = a.view(torch.uint8).numpy()[:64]
            out[f"mx_s{spread}_w"] = w.view(torch.uint8).numpy()[:64]
            out[f"mx_s{spread}_as"] = np.ascontiguousarray(a_s[:, :64])
            out[f"mx_s{spread}_ws"] = w_s[:1]
            out[f"mx_s{spread}_out"] = res.cpu().numpy()[:64, :64]
    dest = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "tensorcore_probe.npz"
    np.savez_compressed(dest, **out)


if __name__ == "__main__":
    main()
