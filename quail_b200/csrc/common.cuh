// Shared helpers for the sm_100a kernels of libquailb200.
//
// Every exported entry point is extern "C", takes plain pointers and sizes,
// runs on the caller's stream and returns an int status (QB_OK = 0). The
// message of the last failure on the calling host thread is kept for
// qb_last_error().
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/quail_b200.h"

typedef __nv_bfloat16 bf16;
typedef __nv_bfloat162 bf162;

// fp8 e4m3 has no infinity; the quantisers clamp to this before the cast.
#define QB_FP8_MAX 448.0f
// the quantisation group: 128 consecutive columns of one row share a scale.
#define QB_GROUP 128

namespace qb {

void set_error(const char* fmt, ...);

// Checks a launch; returns QB_ERR_CUDA with the CUDA message on failure.
int launch_status(const char* what);

// Device address of the status word bounded waits report into (current device).
uint32_t* device_status_ptr();

// Status bits a kernel ORs into the status word when a bounded wait gives up.
enum : uint32_t {
    STATUS_GEMM_PRODUCER = 1u << 0,
    STATUS_GEMM_MMA = 1u << 1,
    STATUS_GEMM_EPILOGUE = 1u << 2,
    STATUS_GEMM_DRAIN = 1u << 3,
    STATUS_BAD_TOKEN = 1u << 8,     // a token id outside [0, vocab)
    STATUS_BAD_INDEX = 1u << 9,     // a page, row or segment index out of range
};

inline int invalid(const char* what) {
    set_error("%s", what);
    return QB_ERR_INVALID;
}

inline bool aligned(const void* p, size_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

// ---- numerics shared by the kernels -------------------------------------

__device__ __forceinline__ float bf16_round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}

// The reference quantiser (per_token_group_quant_fp8 and the fused Triton
// kernels): scale = max(amax, 1e-10) / 448; q = clamp(y / scale, +-448),
// rounded to nearest even e4m3.
__device__ __forceinline__ float group_scale(float amax) {
    return fmaxf(amax, 1e-10f) / QB_FP8_MAX;
}

__device__ __forceinline__ float quant_clamp(float y, float scale) {
    float q = y / scale;
    return fminf(fmaxf(q, -QB_FP8_MAX), QB_FP8_MAX);
}

// two floats -> two e4m3 bytes (low byte = first value)
__device__ __forceinline__ uint16_t fp8x2(float a, float b) {
    __nv_fp8x2_storage_t s = __nv_cvt_float2_to_fp8x2(make_float2(a, b),
                                                       __NV_SATFINITE, __NV_E4M3);
    return static_cast<uint16_t>(s);
}

// ---- exp2 / exp / sigmoid / ln by fixed FMA-only methods -----------------
// Every transcendental on the path goes through these, so a CPU restatement
// with the same operations rounds identically (CUDA's expf / logf differ
// from a CPU libm in the last bits, and one such bit moves a quantisation
// group's scale).
//   exp2: n = rint(x), f = x - n in [-1/2, 1/2], 2^f by the degree-7 Taylor
//         series sum (ln 2)^k f^k / k! in Horner form, times 2^n;
//   ln:   x = 2^e m with m in [sqrt(1/2), sqrt 2), ln m = 2 atanh(t),
//         t = (m - 1) / (m + 1), atanh(t) = t (1 + t^2/3 + ... + t^12/13).

__device__ __forceinline__ float qexp2f(float x) {
    if (!(x >= -149.0f)) return (x != x) ? x : 0.0f;
    if (x >= 128.0f) return __int_as_float(0x7f800000);
    const float n = rintf(x);
    const float f = __fsub_rn(x, n);
    float p = 0.0000152527338040598403f;
    p = __fmaf_rn(p, f, 0.000154035303933816099f);
    p = __fmaf_rn(p, f, 0.00133335581464284434f);
    p = __fmaf_rn(p, f, 0.00961812910762847716f);
    p = __fmaf_rn(p, f, 0.0555041086648215800f);
    p = __fmaf_rn(p, f, 0.240226506959100712f);
    p = __fmaf_rn(p, f, 0.693147180559945309f);
    p = __fmaf_rn(p, f, 1.0f);
    const int ni = (int)n;
    if (ni >= -126) return __fmul_rn(p, __int_as_float((ni + 127) << 23));
    return __fmul_rn(__fmul_rn(p, __int_as_float((ni + 126 + 127) << 23)),
                     __int_as_float(1 << 23));
}

__device__ __forceinline__ float qexpf(float x) {
    return qexp2f(__fmul_rn(x, 1.44269504088896341f));
}

__device__ __forceinline__ float sigmoidf_ref(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, qexpf(-x)));
}

// ln x for normal positive x
__device__ __forceinline__ float qlnf(float x) {
    const unsigned b = __float_as_uint(x);
    int e = (int)((b >> 23) & 0xFF) - 127;
    float m = __uint_as_float((b & 0x7FFFFFu) | 0x3F800000u);
    if (m > 1.41421356237309505f) {
        m = __fmul_rn(m, 0.5f);
        e += 1;
    }
    const float t = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
    const float t2 = __fmul_rn(t, t);
    float p = 1.0f / 13.0f;
    p = __fmaf_rn(p, t2, 1.0f / 11.0f);
    p = __fmaf_rn(p, t2, 1.0f / 9.0f);
    p = __fmaf_rn(p, t2, 1.0f / 7.0f);
    p = __fmaf_rn(p, t2, 1.0f / 5.0f);
    p = __fmaf_rn(p, t2, 1.0f / 3.0f);
    p = __fmaf_rn(p, t2, 1.0f);
    const float lnm = __fmul_rn(__fmul_rn(t, p), 2.0f);
    return __fmaf_rn((float)e, 0.693147180559945309f, lnm);
}

// Sum of squares of 8 values in a fixed order: x0*x0, then FMAs.
__device__ __forceinline__ float sumsq8(const float* x) {
    float ss = __fmul_rn(x[0], x[0]);
#pragma unroll
    for (int i = 1; i < 8; ++i) ss = __fmaf_rn(x[i], x[i], ss);
    return ss;
}

// unpack 8 bf16 held in a uint4 into floats
__device__ __forceinline__ void bf16x8_to_float(const uint4& v, float* f) {
    const bf162* h = reinterpret_cast<const bf162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __bfloat1622float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ uint4 float_to_bf16x8(const float* f) {
    uint4 v;
    bf162* h = reinterpret_cast<bf162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over the block in a fixed order: an xor butterfly inside each warp
// (every lane ends with the same bits), then the warp totals added in warp
// order. Every thread gets the result. scratch holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_warps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = scratch[0];
    for (int w = 1; w < n_warps; ++w) t = __fadd_rn(t, scratch[w]);
    return t;
}

}  // namespace qb
