// Tensor-core numerics probes for tests/golden/make_tensorcore_probe.py (test
// infrastructure, not part of the library): tcgen05 f8f6f4 partials and the
// block-scaled (UE8M0) accumulator in fp32, and one mma.sync m16n8k16 bf16. Bounds: every index below is within the
// buffers the host allocates (checked in probe.py).
#include "../../quail_b200/csrc/gemm_fp8.cu"

// The library's GEMM kernel with an fp32 output (the accumulator before
// the bf16 rounding): MX = false, the promoted 128-deep partials; MX = true,
// the UE8M0 mode's whole-K block-scaled accumulator. n % 256 == 0.
template <bool MX>
static int probe_f32(const void* a, const float* as, int64_t ld, const void* w, const float* ws,
                     float* out, int64_t m, int64_t n, int64_t k, void* stream) {
    using C = Cfg<256, MAX_STAGES, false, false, false, MX>;
    CUtensorMap ma, mb, mc;
    memset(&mc, 0, sizeof(mc));  // no TMA store on the fp32 path
    if (make_map(&ma, a, m, k, BM) || make_map(&mb, w, n, k, 256)) return 1;
    auto kern = gemm_fp8_bs_kernel<256, float, MAX_STAGES, false, false, false, MX>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    uint32_t* status = device_status_ptr();
    RopeArgs none;
    memset(&none, 0, sizeof(none));
    const int64_t tiles = ((m + BM - 1) / BM) * (n / 256);
    kern<<<(int)(tiles < 148 ? tiles : 148), NUM_THREADS, C::SMEM, (cudaStream_t)stream>>>(
        ma, mb, mc, as, ld, ws, out, nullptr, 0, (int)m, (int)n, (int)k, status, none);
    return cudaGetLastError() != cudaSuccess;
}

extern "C" int probe_gemm_f32(const void* a, const float* as, int64_t ld, const void* w,
                              const float* ws, float* out, int64_t m, int64_t n, int64_t k,
                              void* stream) {
    return probe_f32<false>(a, as, ld, w, ws, out, m, n, k, stream);
}

extern "C" int probe_gemm_mx_f32(const void* a, const float* as, int64_t ld, const void* w,
                                 const float* ws, float* out, int64_t m, int64_t n, int64_t k,
                                 void* stream) {
    return probe_f32<true>(a, as, ld, w, ws, out, m, n, k, stream);
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

// ---- tcgen05 kind::f16 (bf16 -> fp32) in the tcgen05 attention layouts ----
// One block of 128 threads: A [128 x 64] K-major (128-byte swizzle), B either
// [64 x 64] K-major (mode 0: S = Q K^T, N = 64) or V [64 keys x 128] read
// MN-major (mode 1: O = P V, N = 128, the two 64-column halves 8 KB apart);
// D = (C if use_c) + four chained K=16 MMAs. All smem and TMEM indices stay
// inside the arrays below (128 rows x at most 128 columns).

__device__ __forceinline__ uint64_t probe_mn_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void probe_mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                              uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void probe_tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

__global__ void __launch_bounds__(128, 1)
tc_f16_probe(const uint16_t* a, const uint16_t* b, const float* c, float* d, int mode, int use_c,
             uint32_t* status) {
    __shared__ __align__(1024) uint8_t sa[128 * 128];
    __shared__ __align__(1024) uint8_t sb[2 * 64 * 128];
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_base;
    const int t = threadIdx.x, warp = t >> 5;
    const int n = mode == 0 ? 64 : 128;
    for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4*>(sa + t * 128 + ((j ^ (t & 7)) << 4)) =
            *reinterpret_cast<const uint4*>(a + t * 64 + j * 8);
    if (t < 64) {
        if (mode == 0) {
            for (int j = 0; j < 8; ++j)
                *reinterpret_cast<uint4*>(sb + t * 128 + ((j ^ (t & 7)) << 4)) =
                    *reinterpret_cast<const uint4*>(b + t * 64 + j * 8);
        } else {
            for (int h = 0; h < 2; ++h)
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<uint4*>(sb + h * 8192 + t * 128 + ((j ^ (t & 7)) << 4)) =
                        *reinterpret_cast<const uint4*>(b + t * 128 + h * 64 + j * 8);
        }
    }
    if (t == 0) {
        mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(
                         smem_u32(&tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    if (use_c) {
        for (int c0 = 0; c0 < n; c0 += 16) {
            uint32_t r[16];
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(c[t * n + c0 + i]);
            probe_tmem_st16(tm + lane_addr + (uint32_t)c0, r);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (t == 0) {
        const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (mode ? (1u << 16) : 0u) |
                               ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
        for (int ks = 0; ks < 4; ++ks) {
            const uint64_t ad = sw128_desc(smem_u32(sa)) + (uint64_t)(2 * ks);
            const uint64_t bd = mode == 0 ? sw128_desc(smem_u32(sb)) + (uint64_t)(2 * ks)
                                          : probe_mn_desc(smem_u32(sb) + ks * 2048, 8192, 1024);
            probe_mma_f16(tm, ad, bd, idesc, (ks > 0 || use_c) ? 1u : 0u);
        }
        mma_commit(&bar);
    }
    int flag = 0;
    mbar_wait(&bar, 0, &flag, status, 1u);
    tc_fence_after();
    for (int c0 = 0; c0 < n; c0 += 16) {
        uint32_t r[16];
        tmem_ld16_nowait(tm + lane_addr + (uint32_t)c0, r);
        tmem_wait_ld();
        for (int i = 0; i < 16; ++i) d[t * n + c0 + i] = __uint_as_float(r[i]);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tm)
                     : "memory");
}

extern "C" int probe_tc_f16(int mode, const void* a, const void* b, const float* c, float* d,
                            int use_c, void* stream) {
    uint32_t* status = device_status_ptr();
    tc_f16_probe<<<1, 128, 0, (cudaStream_t)stream>>>((const uint16_t*)a, (const uint16_t*)b, c,
                                                     d, mode, use_c, status);
    return cudaGetLastError() != cudaSuccess;
}
