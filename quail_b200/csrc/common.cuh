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

#include <atomic>

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
    STATUS_ATTN_LOAD = 1u << 4,     // tcgen05 attention: loader, MMA, softmax, correction
    STATUS_ATTN_MMA = 1u << 5,
    STATUS_ATTN_SOFTMAX = 1u << 6,
    STATUS_ATTN_CORRECTION = 1u << 7,
    STATUS_BAD_TOKEN = 1u << 8,     // a token id outside [0, vocab)
    STATUS_BAD_INDEX = 1u << 9,     // a page, row or segment index out of range
    STATUS_BAD_SCALE = 1u << 10,    // a UE8M0-mode scale that is not a power of two
};

inline int invalid(const char* what) {
    set_error("%s", what);
    return QB_ERR_INVALID;
}

// Devices a per-device "done once" flag covers (cudaGetDevice ids).
constexpr int MAX_DEVICES = 64;

// Raises a kernel's dynamic shared-memory limit once per device. `done`
// is the kernel's own array of MAX_DEVICES flags; several host threads may
// race here, and each then sets the same attribute (an idempotent call).
// Returns false when the CUDA call fails (its error is left for
// launch_status to report).
template <typename Kernel>
inline bool set_smem_once(std::atomic<bool>* done, Kernel kernel, int bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const bool cached = dev >= 0 && dev < MAX_DEVICES;
    if (cached && done[dev].load(std::memory_order_acquire)) return true;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess)
        return false;
    if (cached) done[dev].store(true, std::memory_order_release);
    return true;
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
// The division by 448 is Markstein's correction with r = RN(1/448)
// (q0 = RN(a r), e = a - 448 q0 exact by FMA, q = RN(q0 + e r)): the
// correctly rounded quotient for every a in [1e-10, inf] (checked against
// __fdiv_rn on all of them).
__device__ __forceinline__ float group_scale(float amax) {
    const float a = fmaxf(amax, 1e-10f);
    constexpr float r = 1.0f / QB_FP8_MAX;
    const float q0 = __fmul_rn(a, r);
    const float e = __fmaf_rn(-QB_FP8_MAX, q0, a);
    return a < INFINITY ? __fmaf_rn(e, r, q0) : q0;  // inf: e would be NaN
}

// The UE8M0 mode of the same quantisers (use_ue8m0: scale =
// exp2(ceil(log2(max(amax, 1e-10) / 448)))): the least power of two >= the
// fp32 scale above, taken exactly from its bits. q = y / scale is then the
// exact product y * 2^-e, rounded once by the e4m3 conversion.
__device__ __forceinline__ float ue8m0_scale(float amax) {
    const float s = group_scale(amax);
    const uint32_t b = __float_as_uint(s);
    if ((b & 0x7FFFFFu) == 0 || b >= 0x7F800000u) return s;  // a power of two, inf or NaN
    return __uint_as_float((b & 0x7F800000u) + 0x800000u);
}

// 1 / s for a UE8M0 scale s = 2^k (k in [-43, 127]; 0 for an infinite s,
// NaN for NaN), exactly
__device__ __forceinline__ float ue8m0_inverse(float s) {
    const uint32_t b = __float_as_uint(s);
    if (b >= 0x7F800000u) return b == 0x7F800000u ? 0.0f : s;
    if (b >= 0x7F000000u) return __uint_as_float(0x00400000u >> ((b >> 23) - 254u));  // 2^-127
    return __uint_as_float(0x7F000000u - b);
}

// y / scale for many y of one group: the correctly rounded quotient from
// one reciprocal per group by Markstein's correction (P. Markstein, IBM J.
// Res. Dev. 34(1), 1990): r = RN(1/s), q0 = RN(y r), e = y - s q0 (exact by
// FMA), q = RN(q0 + e r). The residual stays exact while |y| >= 2^-96 (no
// underflow); smaller, huge and non-finite y (and the sign of zero) take
// the IEEE division. Equal to y / scale bit for bit (checked against it on
// 4e8 random pairs over the range quantisation sees).
// out of line: rare paths stay out of the unrolled hot loops' code
static __device__ __noinline__ float div_slow(float y, float s) { return __fdiv_rn(y, s); }

struct GroupDivider {
    float s, r;
    __device__ __forceinline__ explicit GroupDivider(float scale) {
        s = scale;
        r = __frcp_rn(scale);
    }
    __device__ __forceinline__ float div(float y) const {
        const float a = fabsf(y);
        // (an infinite scale has r = 0, and the residual would be NaN)
        if (!(a >= 0x1p-96f && a < 0x1p+100f && s < INFINITY)) return div_slow(y, s);
        const float q0 = __fmul_rn(y, r);
        const float e = __fmaf_rn(-s, q0, y);
        return __fmaf_rn(e, r, q0);
    }
    __device__ __forceinline__ float quant(float y) const {
        return fminf(fmaxf(div(y), -QB_FP8_MAX), QB_FP8_MAX);
    }
    // quant of two values with f32x2 arithmetic (same bits as quant on each)
    __device__ __forceinline__ void quant2(float& a, float& b) const;
    // quant2 for the saturating e4m3 conversion, which clamps a finite
    // quotient to +-448 as quant2 does: RN(y / s) without the clamp. Exact
    // for |y| in [2^-96, 2^100); *rare is set for |y| < 2^-96 (zeros too: the
    // residual step would turn -0 into +0) and NaN. The caller checks the
    // upper bound once on the group max (!(amax < 2^100)) and redoes rare
    // values with quant2.
    __device__ __forceinline__ void quant2_sat(float& a, float& b, bool& rare) const;
};

// e4m3 byte -> its value (exact through half precision)
__device__ __forceinline__ float fp8_to_float(uint8_t c) {
    const __half_raw h = __nv_cvt_fp8_to_halfraw(c, __NV_E4M3);
    return __half2float(__half(h));
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
//   exp2: x clamped to [-150, 128], n = rint(x), f = x - n in [-1/2, 1/2],
//         2^f by the degree-7 Taylor series sum (ln 2)^k f^k / k! in Horner
//         form, times 2^n (a subnormal result in two steps);
//   ln:   x = 2^e m with m in [sqrt(1/2), sqrt 2), ln m = 2 atanh(t),
//         t = (m - 1) / (m + 1), atanh(t) = t (1 + t^2/3 + ... + t^12/13).

// ---- packed fp32 pairs (Blackwell f32x2: two IEEE operations per
// instruction, each rounded exactly as its scalar form) -----------------
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// x clamped to [-150, 128], NaN kept: 2^-150 rounds to 0 and 2^128 to inf,
// so the clamp is the whole range handling
__device__ __forceinline__ float exp2_clamp(float x) {
    float r;
    asm("max.NaN.f32 %0, %1, 0fC3160000;" : "=f"(r) : "f"(x));  // -150
    asm("min.NaN.f32 %0, %0, 0f43000000;" : "+f"(r));             // 128
    return r;
}

// 2^n for the exponent held in t = x + 1.5 * 2^23 (n >= -126)
__device__ __forceinline__ float exp2_scale(float t) {
    return __int_as_float((__float_as_int(t) - 0x4B400000 + 127) << 23);
}

__device__ __forceinline__ float exp2_finish(float p, float t) {
    const int ni = __float_as_int(t) - 0x4B400000;
    if (ni >= -126) return __fmul_rn(p, exp2_scale(t));
    return __fmul_rn(__fmul_rn(p, __int_as_float((ni + 126 + 127) << 23)),
                     __int_as_float(1 << 23));
}

__device__ __forceinline__ void GroupDivider::quant2(float& a, float& b) const {
    const float fa = fabsf(a), fb = fabsf(b);
    if (fa >= 0x1p-96f && fa < 0x1p+100f && fb >= 0x1p-96f && fb < 0x1p+100f && s < INFINITY) {
        const uint64_t y = f2pack(a, b), rr = f2pack(r, r);
        const uint64_t q0 = f2mul(y, rr);
        const uint64_t e = f2fma(f2pack(-s, -s), q0, y);
        f2unpack(f2fma(e, rr, q0), a, b);
    } else {
        a = div(a);
        b = div(b);
    }
    a = fminf(fmaxf(a, -QB_FP8_MAX), QB_FP8_MAX);
    b = fminf(fmaxf(b, -QB_FP8_MAX), QB_FP8_MAX);
}

__device__ __forceinline__ void GroupDivider::quant2_sat(float& a, float& b, bool& rare) const {
    rare |= !(fabsf(a) >= 0x1p-96f) | !(fabsf(b) >= 0x1p-96f);
    const uint64_t y = f2pack(a, b), rr = f2pack(r, r);
    const uint64_t q0 = f2mul(y, rr);
    const uint64_t e = f2fma(f2pack(-s, -s), q0, y);
    f2unpack(f2fma(e, rr, q0), a, b);
}

// 1 / d, correctly rounded, for two d in [2^-126, 2^126) (normal d with a
// normal reciprocal), by Markstein's correction of the hardware
// approximation: r0 = rcp.approx(d), e = RN(1 - d r0) (exact by FMA),
// r = RN(r0 + e r0). Equal to __frcp_rn on every float of that range
// (exhaustive check on the B200).
__device__ __forceinline__ void rcp_rn_normal_x2(float& a, float& b) {
    float ra, rb;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(ra) : "f"(a));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rb) : "f"(b));
    const uint64_t r = f2pack(ra, rb);
    const uint64_t e = f2fma(f2pack(-a, -b), r, f2pack(1.0f, 1.0f));
    f2unpack(f2fma(e, r, r), a, b);
}

// 2^f on [-1/2, 1/2]: Taylor coefficients (ln 2)^k / k!, k = 7 .. 0, Horner
#define QB_EXP2_POLY(STEP)                          \
    STEP(0.000154035303933816099f)                  \
    STEP(0.00133335581464284434f)                   \
    STEP(0.00961812910762847716f)                   \
    STEP(0.0555041086648215800f)                    \
    STEP(0.240226506959100712f)                     \
    STEP(0.693147180559945309f)                     \
    STEP(1.0f)
// a subnormal result on either lane (rare): out of line
static __device__ __noinline__ void exp2_finish_slow(float& a, float& b, float pa, float pb, float ta,
                                              float tb) {
    a = exp2_finish(pa, ta);
    b = exp2_finish(pb, tb);
}

constexpr float QB_EXP2_C7 = 0.0000152527338040598403f;

__device__ __forceinline__ float qexp2f(float x) {
    // n = rint(x) by adding and removing 1.5 * 2^23: the sum has unit
    // spacing, so it rounds x to the nearest integer (ties to even, the
    // shift being even) and its low mantissa bits hold n
    const float xc = exp2_clamp(x);
    const float t = __fadd_rn(xc, 12582912.0f);
    const float n = __fsub_rn(t, 12582912.0f);
    const float f = __fsub_rn(xc, n);
    float p = QB_EXP2_C7;
#define QB_STEP(c) p = __fmaf_rn(p, f, c);
    QB_EXP2_POLY(QB_STEP)
#undef QB_STEP
    return exp2_finish(p, t);
}

// two qexp2f at once with f32x2 arithmetic; the same bits as qexp2f on each
__device__ __forceinline__ void qexp2f_x2(float& a, float& b) {
    const uint64_t M = f2pack(12582912.0f, 12582912.0f);
    const uint64_t x = f2pack(exp2_clamp(a), exp2_clamp(b));
    const uint64_t t = f2add(x, M);
    const uint64_t f = f2sub(x, f2sub(t, M));
    uint64_t p = f2pack(QB_EXP2_C7, QB_EXP2_C7);
#define QB_STEP2(c) p = f2fma(p, f, f2pack(c, c));
    QB_EXP2_POLY(QB_STEP2)
#undef QB_STEP2
    float pa, pb, ta, tb;
    f2unpack(p, pa, pb);
    f2unpack(t, ta, tb);
    if (__float_as_int(ta) - 0x4B400000 >= -126 && __float_as_int(tb) - 0x4B400000 >= -126) {
        f2unpack(f2mul(p, f2pack(exp2_scale(ta), exp2_scale(tb))), a, b);
    } else {
        exp2_finish_slow(a, b, pa, pb, ta, tb);
    }
}

__device__ __forceinline__ float qexpf(float x) {
    return qexp2f(__fmul_rn(x, 1.44269504088896341f));
}

__device__ __forceinline__ float sigmoidf_ref(float x) {
    // __frcp_rn is the correctly rounded 1 / d, the same value as 1.0f / d
    return __frcp_rn(__fadd_rn(1.0f, qexpf(-x)));
}

// qexp2f_x2 without its rare branch, for x <= 1 (softmax exponents): x is
// clamped at -127, where n = -127 gives the scale bits 0 and so 2^x = 0
// without a select; *rare is set for x in [-150.5, -126.5) (a subnormal
// result, redone with qexp2f_x2 by the caller); x below -150.5 (masked
// keys: -inf) gives 0 as qexp2f does (2^-150.5 is under half the smallest
// subnormal), NaN stays NaN.
__device__ __forceinline__ void qexp2f_x2_softmax(float& a, float& b, bool& rare) {
    rare |= ((a < -126.5f) & (a >= -150.5f)) | ((b < -126.5f) & (b >= -150.5f));
    const uint64_t M = f2pack(12582912.0f, 12582912.0f);
    float ac, bc;
    asm("max.NaN.f32 %0, %1, 0fC2FE0000;" : "=f"(ac) : "f"(a));  // -127
    asm("max.NaN.f32 %0, %1, 0fC2FE0000;" : "=f"(bc) : "f"(b));
    const uint64_t x = f2pack(ac, bc);
    const uint64_t t = f2add(x, M);
    const uint64_t f = f2sub(x, f2sub(t, M));
    uint64_t p = f2pack(QB_EXP2_C7, QB_EXP2_C7);
#define QB_STEP6(c) p = f2fma(p, f, f2pack(c, c));
    QB_EXP2_POLY(QB_STEP6)
#undef QB_STEP6
    float ta, tb;
    f2unpack(t, ta, tb);
    constexpr uint32_t K = (127u - 0x4B400000u) << 23;  // 2^n bits: (bits(t) << 23) + K
    f2unpack(f2mul(p, f2pack(__uint_as_float((__float_as_uint(ta) << 23) + K),
                             __uint_as_float((__float_as_uint(tb) << 23) + K))),
             a, b);
}

// The attention softmax's exp2 (P and the rescale factor alpha): 2^x for
// x <= 1, -inf and NaN. n = rint(max(x, -127)), f = x - n in [-1/2, 1/2],
// 2^f by a degree-5 polynomial 1 + c1 f + ... + c5 f^5 fitted for least
// relative error on [-1/2, 1/2] (weighted least squares with Lawson
// iterations; max relative error 1.7e-7 in fp32 Horner, the accuracy class
// of the 2-ulp hardware ex2.approx FlashAttention's softmax uses), times
// 2^n. The constant term is exactly 1, so 2^0 = 1: a key tile that moves no
// row max (alpha = 2^0) leaves the row sums and the output unscaled. n = -127 gives the
// scale 0, so 2^x = 0 below -126.5 (FlashAttention's ex2 flushes subnormal
// results to zero as well). Four FMA steps fewer than qexp2f and no
// subnormal branch; the oracle's qbm_exp2s restates it bit for bit.
#define QB_EXP2S_POLY(STEP)        \
    STEP(0.009671512991189957f)    \
    STEP(0.05550733581185341f)     \
    STEP(0.24022242426872253f)    \
    STEP(0.6931470036506653f)     \
    STEP(1.0f)
constexpr float QB_EXP2S_C5 = 0.0013264724984765053f;

__device__ __forceinline__ void qexp2s_x2(float& a, float& b) {
    float ac, bc;
    asm("max.NaN.f32 %0, %1, 0fC2FE0000;" : "=f"(ac) : "f"(a));  // -127
    asm("max.NaN.f32 %0, %1, 0fC2FE0000;" : "=f"(bc) : "f"(b));
    const uint64_t M = f2pack(12582912.0f, 12582912.0f);
    const uint64_t x = f2pack(ac, bc);
    const uint64_t t = f2add(x, M);
    const uint64_t f = f2sub(x, f2sub(t, M));
    uint64_t p = f2pack(QB_EXP2S_C5, QB_EXP2S_C5);
#define QB_STEPS2(c) p = f2fma(p, f, f2pack(c, c));
    QB_EXP2S_POLY(QB_STEPS2)
#undef QB_STEPS2
    float ta, tb;
    f2unpack(t, ta, tb);
    constexpr uint32_t K = (127u - 0x4B400000u) << 23;  // 2^n bits: (bits(t) << 23) + K
    f2unpack(f2mul(p, f2pack(__uint_as_float((__float_as_uint(ta) << 23) + K),
                             __uint_as_float((__float_as_uint(tb) << 23) + K))),
             a, b);
}

__device__ __forceinline__ float qexp2s(float x) {
    float xc;
    asm("max.NaN.f32 %0, %1, 0fC2FE0000;" : "=f"(xc) : "f"(x));
    const float t = __fadd_rn(xc, 12582912.0f);
    const float f = __fsub_rn(xc, __fsub_rn(t, 12582912.0f));
    float p = QB_EXP2S_C5;
#define QB_STEPS(c) p = __fmaf_rn(p, f, c);
    QB_EXP2S_POLY(QB_STEPS)
#undef QB_STEPS
    constexpr uint32_t K = (127u - 0x4B400000u) << 23;
    return __fmul_rn(p, __uint_as_float((__float_as_uint(t) << 23) + K));
}

// max of three floats (NaN operands ignored, as fmaxf)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// two sigmoidf_ref at once (same bits on each)
__device__ __forceinline__ void sigmoidf_ref_x2(float& a, float& b) {
    float ea, eb;
    f2unpack(f2mul(f2pack(-a, -b), f2pack(1.44269504088896341f, 1.44269504088896341f)), ea, eb);
    qexp2f_x2(ea, eb);
    f2unpack(f2add(f2pack(1.0f, 1.0f), f2pack(ea, eb)), ea, eb);
    a = __frcp_rn(ea);
    b = __frcp_rn(eb);
}

// sigmoidf_ref_x2, branch-free: the same bits unless *rare is set, for
// x = -g log2(e) above 125 (1 + 2^x reaches 2^125.5: the reciprocal leaves
// rcp_rn_normal_x2's range) or NaN; the caller then redoes the pair with
// sigmoidf_ref_x2. Below, x is clamped at -127 instead of -150: n = rint(x)
// = -127 gives the scale bits 0, so 2^x becomes 0 there, and any 2^x under
// 2^-24 leaves 1 + 2^x = 1 exactly as qexp2f's value would.
__device__ __forceinline__ void sigmoidf_ref_x2_fast(float& a, float& b, bool& rare) {
    float xa, xb;
    f2unpack(f2mul(f2pack(a, b), f2pack(-1.44269504088896341f, -1.44269504088896341f)), xa, xb);
    rare |= !(xa <= 125.0f) | !(xb <= 125.0f);
    const uint64_t M = f2pack(12582912.0f, 12582912.0f);
    const uint64_t x = f2pack(fmaxf(xa, -127.0f), fmaxf(xb, -127.0f));
    const uint64_t t = f2add(x, M);
    const uint64_t f = f2sub(x, f2sub(t, M));
    uint64_t p = f2pack(QB_EXP2_C7, QB_EXP2_C7);
#define QB_STEP5(c) p = f2fma(p, f, f2pack(c, c));
    QB_EXP2_POLY(QB_STEP5)
#undef QB_STEP5
    float ta, tb;
    f2unpack(t, ta, tb);
    // 2^n: bits (n + 127) << 23, n = bits(t) - 0x4B400000, in one shift-add
    constexpr uint32_t K = (127u - 0x4B400000u) << 23;
    const uint64_t e = f2mul(p, f2pack(__uint_as_float((__float_as_uint(ta) << 23) + K),
                                       __uint_as_float((__float_as_uint(tb) << 23) + K)));
    float da, db;
    f2unpack(f2add(f2pack(1.0f, 1.0f), e), da, db);
    rcp_rn_normal_x2(da, db);
    a = da;
    b = db;
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

// (a, b) rounded to nearest even bf16, a in the low half
__device__ __forceinline__ uint32_t bf16x2_bits(float a, float b) {
    const bf162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// the two bf16 halves of u (low first) as floats, exactly
__device__ __forceinline__ float2 bf16x2_float2(uint32_t u) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
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
