// Tensor-core numerics probes for tests/golden/make_tensorcore_probe.py (test
// infrastructure, not part of the library): tcgen05 f8f6f4 partials in fp32
// and one mma.sync m16n8k16 bf16. Bounds: every index below is within the
// buffers the host allocates (checked in probe.py).
#include "../../quail_b200/csrc/gemm_fp8.cu"

extern "C" int probe_gemm_f32(const void* a, const float* as, int64_t ld, const void* w,
                              const float* ws, float* out, int64_t m, int64_t n, int64_t k,
                              void* stream) {
    CUtensorMap ma, mb, mc;
    memset(&mc, 0, sizeof(mc));  // no TMA store on the fp32 path
    if (make_map(&ma, a, m, k, BM) || make_map(&mb, w, n, k, 256)) return 1;
    cudaFuncSetAttribute(gemm_fp8_bs_kernel<256, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Cfg<256>::SMEM);
    uint32_t* status = device_status_ptr();
    int64_t tiles = ((m + BM - 1) / BM) * (n / 256);
    gemm_fp8_bs_kernel<256, float><<<(int)(tiles < 148 ? tiles : 148), NUM_THREADS, Cfg<256>::SMEM,
                                     (cudaStream_t)stream>>>(ma, mb, mc, as, ld, ws, out, (int)m, (int)n,
                                                             (int)k, status);
    return cudaGetLastError() != cudaSuccess;
}

// one warp: D[16x8] = A[16x16] B[16x8] + C, fragments in the PTX layout
__global__ void mma_probe(const uint32_t* a_frag, const uint32_t* b_frag, const float* c_frag,
                          float* d_frag) {
    const int t = threadIdx.x;
    float c[4] = {c_frag[4 * t], c_frag[4 * t + 1], c_frag[4 * t + 2], c_frag[4 * t + 3]};
    uint32_t a[4] = {a_frag[4 * t], a_frag[4 * t + 1], a_frag[4 * t + 2], a_frag[4 * t + 3]};
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b_frag[2 * t]), "r"(b_frag[2 * t + 1]));
    for (int i = 0; i < 4; ++i) d_frag[4 * t + i] = c[i];
}

extern "C" int probe_mma(const uint32_t* a, const uint32_t* b, const float* c, float* d, int reps,
                         void* stream) {
    for (int r = 0; r < reps; ++r)
        mma_probe<<<1, 32, 0, (cudaStream_t)stream>>>(a + r * 128, b + r * 64, c + r * 128, d + r * 128);
    return cudaGetLastError() != cudaSuccess;
}
