// Exhaustive GPU checks of the branch-free fast paths in
// quail_b200/csrc/common.cuh against the exact forms they stand in for.
// Built and run by tests/test_numerics_exhaustive.py; every check counts
// mismatching outputs (bit patterns) and must count zero.
//
//   0  rcp_rn_normal_x2 vs __frcp_rn, every d in [2^-126, 2^126)
//   1  sigmoidf_ref_x2_fast (+ exact redo when rare) vs sigmoidf_ref,
//      every fp32 bit pattern
//   2  group_scale vs max(a, 1e-10) / 448 by __fdiv_rn, every a >= +0 (and
//      the positive NaNs)
//   3  quant2_sat (+ the group bound and exact redo) vs quant2, e4m3 codes,
//      on 64 group scales x 2^24 values of the group each
//   4  qexp2s_x2 (the attention softmax's packed exp2) vs qexp2s, every
//      x <= 1 (every negative float, zeros, positives up to 1.0, -inf, NaNs)
//   5  qexp2s against CUDA's exp2f, every x in [-125, 1]: a relative
//      difference above 5e-7 counts (the polynomial's bound, 1.7e-7, plus
//      exp2f's own maximum error of 2 ulp, 2.4e-7)
// qbn_exp2s(x, y, n) evaluates qexp2s on the GPU for the oracle comparison.
#include "common.cuh"

using namespace qb;

namespace {

__device__ unsigned long long g_bad[6];
__device__ unsigned int g_first[6];

__device__ void record(int which, uint32_t bits) {
    atomicAdd(&g_bad[which], 1ull);
    atomicMin(&g_first[which], bits);
}

__device__ __forceinline__ uint32_t mix(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

__global__ void check_rcp(uint32_t lo, uint32_t hi) {
    const uint64_t n = hi - lo;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t ba = lo + (uint32_t)i, bb = hi - 1u - (uint32_t)i;
        float a = __uint_as_float(ba), b = __uint_as_float(bb);
        const float wa = __frcp_rn(a), wb = __frcp_rn(b);
        rcp_rn_normal_x2(a, b);
        if (__float_as_uint(a) != __float_as_uint(wa)) record(0, ba);
        if (__float_as_uint(b) != __float_as_uint(wb)) record(0, bb);
    }
}

__global__ void check_sigmoid() {
    const uint64_t n = 1ull << 32;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t ba = (uint32_t)i, bb = mix((uint32_t)i);
        const float ga = __uint_as_float(ba), gb = __uint_as_float(bb);
        float a = ga, b = gb;
        bool rare = false;
        sigmoidf_ref_x2_fast(a, b, rare);
        if (rare) {
            a = ga;
            b = gb;
            sigmoidf_ref_x2(a, b);
        }
        if (__float_as_uint(a) != __float_as_uint(sigmoidf_ref(ga))) record(1, ba);
        if (__float_as_uint(b) != __float_as_uint(sigmoidf_ref(gb))) record(1, bb);
    }
}

__global__ void check_scale() {
    const uint64_t n = 1ull << 31;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t ba = (uint32_t)i;
        const float a = __uint_as_float(ba);
        const float want = __fdiv_rn(fmaxf(a, 1e-10f), QB_FP8_MAX);
        if (__float_as_uint(group_scale(a)) != __float_as_uint(want)) record(2, ba);
    }
}

// block b: one group max amax_b; its 2^24 values y with |y| <= amax_b (a
// third scaled uniforms, a third random bit patterns under amax, a third
// small values down to the subnormals, zeros of both signs among them)
__global__ void check_quant(const float* amaxes) {
    const float amax = amaxes[blockIdx.y];
    const float scale = group_scale(amax);
    const GroupDivider dv(scale);
    const uint32_t per_block = (1u << 24) / gridDim.x;
    for (uint32_t i = threadIdx.x; i < per_block; i += blockDim.x) {
        const uint32_t k = blockIdx.x * per_block + i;
        const uint32_t h = mix(k * 2654435761u + blockIdx.y);
        float y[2];
        for (int j = 0; j < 2; ++j) {
            const uint32_t r = mix(h + j * 0x9E3779B9u);
            const int kind = (int)((k + j) % 3);
            float v;
            if (kind == 0) {
                v = __fmul_rn(amax, __fmul_rn((float)(r >> 8), 0x1p-24f));
            } else if (kind == 1) {
                v = __uint_as_float(r & 0x7FFFFFFFu);
                if (!(v <= amax)) v = __fmul_rn(amax, 0.5f);
            } else {
                v = __uint_as_float((r & 0x3FFFFFFFu) >> 4);  // below 2^-64, subnormals too
                if ((r & 0xFF) == 0) v = 0.0f;
            }
            y[j] = (r & 0x100u) ? -v : v;
        }
        float a = y[0], b = y[1];
        bool rare = !(amax < 0x1p+100f);
        dv.quant2_sat(a, b, rare);
        if (rare) {
            a = y[0];
            b = y[1];
            dv.quant2(a, b);
        }
        float wa = y[0], wb = y[1];
        dv.quant2(wa, wb);
        if (fp8x2(a, b) != fp8x2(wa, wb)) record(3, __float_as_uint(y[0]));
    }
}

// all bit patterns with sign 1 (negatives, -0, -inf, NaNs) and the
// non-negative ones up to 1.0f
__global__ void check_exp2s() {
    const uint64_t n = (1ull << 31) + 0x3F800001ull;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t ba = i < (1ull << 31) ? (uint32_t)i | 0x80000000u
                                              : (uint32_t)(i - (1ull << 31));
        const uint32_t bb = ba ^ 0x00400001u;  // a second lane value nearby
        const float xa = __uint_as_float(ba);
        const float xb = (__uint_as_float(bb) <= 1.0f || __uint_as_float(bb) != __uint_as_float(bb))
                             ? __uint_as_float(bb) : xa;
        float a = xa, b = xb;
        qexp2s_x2(a, b);
        const float wa = qexp2s(xa);
        const bool nan_a = wa != wa;
        if (nan_a ? (a == a) : (__float_as_uint(a) != __float_as_uint(wa))) record(4, ba);
        const float wb = qexp2s(xb);
        const bool nan_b = wb != wb;
        if (nan_b ? (b == b) : (__float_as_uint(b) != __float_as_uint(wb)))
            record(4, __float_as_uint(xb));
        if (xa >= -125.0f && xa <= 1.0f) {
            const float e = exp2f(xa);
            if (fabsf(wa - e) > 5e-7f * e) record(5, ba);
        }
    }
}

__global__ void exp2s_kernel(const float* x, float* y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        y[i] = qexp2s(x[i]);
}

}  // namespace

// bad[6], first[6] (host): mismatch counts and the smallest mismatching
// input bits of each check. Returns a cudaError_t.
extern "C" int qbn_run_checks(unsigned long long* bad, unsigned int* first) {
    unsigned long long zero[6] = {0, 0, 0, 0, 0, 0};
    unsigned int ones[6] = {0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu,
                            0xFFFFFFFFu};
    cudaMemcpyToSymbol(g_bad, zero, sizeof(zero));
    cudaMemcpyToSymbol(g_first, ones, sizeof(ones));
    check_rcp<<<148 * 8, 256>>>(0x00800000u, 0x7E800000u);
    check_sigmoid<<<148 * 8, 256>>>();
    check_scale<<<148 * 8, 256>>>();
    float amax_host[64];
    for (int i = 0; i < 64; ++i) {
        // group maxima from 2^-40 to 2^99, odd mantissas
        const int e = -40 + (i * 139) / 63;
        amax_host[i] = ldexpf(1.0f + (float)((i * 37) % 64) / 64.0f, e);
    }
    amax_host[63] = 1e-10f;  // the scale floor
    float* amax_dev = nullptr;
    cudaMalloc(&amax_dev, sizeof(amax_host));
    cudaMemcpy(amax_dev, amax_host, sizeof(amax_host), cudaMemcpyHostToDevice);
    check_quant<<<dim3(256, 64), 256>>>(amax_dev);
    check_exp2s<<<148 * 8, 256>>>();
    cudaError_t err = cudaDeviceSynchronize();
    cudaFree(amax_dev);
    if (err != cudaSuccess) return (int)err;
    cudaMemcpyFromSymbol(bad, g_bad, sizeof(zero));
    cudaMemcpyFromSymbol(first, g_first, sizeof(ones));
    return (int)cudaGetLastError();
}

// y[i] = qexp2s(x[i]) on the GPU (host arrays of n floats). Returns a
// cudaError_t.
extern "C" int qbn_exp2s(const float* x, float* y, int64_t n) {
    float *dx = nullptr, *dy = nullptr;
    cudaError_t err = cudaMalloc(&dx, n * sizeof(float));
    if (err == cudaSuccess) err = cudaMalloc(&dy, n * sizeof(float));
    if (err == cudaSuccess) err = cudaMemcpy(dx, x, n * sizeof(float), cudaMemcpyHostToDevice);
    if (err == cudaSuccess) {
        exp2s_kernel<<<148 * 4, 256>>>(dx, dy, n);
        err = cudaDeviceSynchronize();
    }
    if (err == cudaSuccess) err = cudaMemcpy(y, dy, n * sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(dx);
    cudaFree(dy);
    return (int)err;
}
