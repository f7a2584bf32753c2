// RMSNorm + fp8 quantisation kernels (HBM-bound): the layer-0 embedding
// norm, the fused residual-add norm of every later norm, and the SiLU-gated
// product of the MLP. One 16-byte vector (8 bf16) per thread; a 128-column
// quantisation group is 16 consecutive lanes (a half warp).
#include "common.cuh"

namespace {

using namespace qb;

// Max |v| over the 16 lanes of a half warp (one quantisation group).
__device__ __forceinline__ float group_amax(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Quantise 8 values of one group slice; the half warp's lane 0 writes the
// scale. ue8m0: the power-of-two scale, q = y * 2^-e exactly.
__device__ __forceinline__ void quant_store8(const float* y, uint8_t* q_row, float* scale_out,
                                             int64_t scale_ld, int64_t row, int col8,
                                             bool ue8m0) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(y[i]));
    amax = group_amax(amax);
    const float scale = ue8m0 ? ue8m0_scale(amax) : group_scale(amax);
    const GroupDivider dv(scale);
    float q[8];
    bool rare = !(amax < 0x1p+100f);
    if (ue8m0) {
        const float inv = ue8m0_inverse(scale);
        const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
        for (int i = 0; i < 8; i += 2)
            f2unpack(f2mul(f2pack(y[i], y[i + 1]), inv2), q[i], q[i + 1]);
        rare = false;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            q[i] = y[i];
            q[i + 1] = y[i + 1];
            dv.quant2_sat(q[i], q[i + 1], rare);
        }
    }
    if (rare) {  // a zero, tiny or non-finite value: the exact path
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            q[i] = y[i];
            q[i + 1] = y[i + 1];
            dv.quant2(q[i], q[i + 1]);
        }
    }
    uint2 packed;
    uint16_t* p = reinterpret_cast<uint16_t*>(&packed);
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = fp8x2(q[2 * i], q[2 * i + 1]);
    *reinterpret_cast<uint2*>(q_row + col8 * 8) = packed;
    if ((threadIdx.x & 15) == 0) scale_out[(int64_t)(col8 / 16) * scale_ld + row] = scale;
}

// blockDim.x == hidden / 8; one row per block. 32 registers (the bound
// allows 2 x 1024 threads) keep six 320-thread blocks resident per SM for the
// 4B hidden size: the memory parallelism this HBM-bound kernel lives on.
template <bool UE8M0>
__global__ void __launch_bounds__(1024, 2) embed_rmsnorm_quant_kernel(const int64_t* __restrict__ ids,
                                           const bf16* __restrict__ embed, int64_t vocab,
                                           int hidden, const bf16* __restrict__ w, float eps,
                                           bf16* __restrict__ residual_out,
                                           uint8_t* __restrict__ q_out,
                                           float* __restrict__ scale_out, int64_t scale_ld,
                                           uint32_t* status) {
    __shared__ float scratch[32];
    const int64_t row = blockIdx.x;
    const int t = threadIdx.x;
    int64_t id = ids[row];
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < vocab) {
        raw = *reinterpret_cast<const uint4*>(embed + id * hidden + t * 8);
    } else if (t == 0) {
        atomicOr(status, STATUS_BAD_TOKEN);
    }
    *reinterpret_cast<uint4*>(residual_out + row * hidden + t * 8) = raw;
    float x[8];
    bf16x8_to_float(raw, x);
    const float total = block_sum(sumsq8(x), scratch);
    const float rstd = 1.0f / sqrtf(total / (float)hidden + eps);
    float wf[8];
    bf16x8_to_float(*reinterpret_cast<const uint4*>(w + t * 8), wf);
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = bf16_round(bf16_round(x[i] * rstd) * wf[i]);
    quant_store8(y, q_out + row * hidden, scale_out, scale_ld, row, t, UE8M0);
}

// blockDim.x == hidden / 8; one row per block; 32 registers as above.
template <bool UE8M0>
__global__ void __launch_bounds__(1024, 2) add_rmsnorm_quant_kernel(const bf16* __restrict__ hidden_in,
                                         bf16* __restrict__ residual,
                                         const bf16* __restrict__ w, float eps, int hidden,
                                         uint8_t* __restrict__ q_out,
                                         float* __restrict__ scale_out, int64_t scale_ld) {
    __shared__ float scratch[32];
    const int64_t row = blockIdx.x;
    const int t = threadIdx.x;
    const int64_t off = row * hidden + t * 8;
    float h[8], r[8], x[8];
    bf16x8_to_float(*reinterpret_cast<const uint4*>(hidden_in + off), h);
    bf16x8_to_float(*reinterpret_cast<const uint4*>(residual + off), r);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = h[i] + r[i];
    *reinterpret_cast<uint4*>(residual + off) = float_to_bf16x8(x);
    const float total = block_sum(sumsq8(x), scratch);
    const float rstd = 1.0f / sqrtf(total / (float)hidden + eps);
    float wf[8];
    bf16x8_to_float(*reinterpret_cast<const uint4*>(w + t * 8), wf);
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = __fmul_rn(__fmul_rn(x[i], rstd), wf[i]);
    quant_store8(y, q_out + row * hidden, scale_out, scale_ld, row, t, UE8M0);
}

// One warp per 256 outputs of one row (two quantisation groups).
template <bool UE8M0>
__global__ void silu_mul_quant_kernel(const bf16* __restrict__ gate_up, int64_t rows, int inter,
                                      uint8_t* __restrict__ q_out, float* __restrict__ scale_out,
                                      int64_t scale_ld) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int per_row = inter / 256;
    if (warp >= rows * per_row) return;  // whole warps exit together
    const int64_t row = warp / per_row;
    const int col8 = (int)(warp % per_row) * 32 + lane;  // 8-column vector index
    const bf16* base = gate_up + row * (int64_t)(2 * inter);
    float g[8], u[8], sg[8], y[8];
    bf16x8_to_float(*reinterpret_cast<const uint4*>(base + col8 * 8), g);
    bf16x8_to_float(*reinterpret_cast<const uint4*>(base + inter + col8 * 8), u);
    bool rare = false;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        sg[i] = g[i];
        sg[i + 1] = g[i + 1];
        sigmoidf_ref_x2_fast(sg[i], sg[i + 1], rare);
    }
    if (rare) {  // g below about -86 or NaN: the exact path
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            sg[i] = g[i];
            sg[i + 1] = g[i + 1];
            sigmoidf_ref_x2(sg[i], sg[i + 1]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        // y = (g * sigmoid(g)) * u, two lanes per instruction
        const uint64_t gs = f2mul(f2pack(g[i], g[i + 1]), f2pack(sg[i], sg[i + 1]));
        f2unpack(f2mul(gs, f2pack(u[i], u[i + 1])), y[i], y[i + 1]);
    }
    quant_store8(y, q_out + row * inter, scale_out, scale_ld, row, col8, UE8M0);
}

// One 128 x 128 weight block per block of 256 threads (64 codes each, in
// four 16-byte pieces of the block's rows): x = code * old scale (fp32),
// s = max(amax, 1e-4) / 448 raised to a power of two, codes = e4m3(x / s),
// in place.
__global__ void __launch_bounds__(256) requant_ue8m0_kernel(uint8_t* __restrict__ w,
                                                            float* __restrict__ w_scale,
                                                            int64_t k) {
    __shared__ float red[8];
    const int nb = blockIdx.y, kb = blockIdx.x, kbs = (int)(k / 128);
    const float s_old = w_scale[(int64_t)nb * kbs + kb];
    const int t = threadIdx.x;
    // piece p of thread t: row (t / 8) + 32 p, bytes 16 (t % 8) .. + 15
    uint4 raw[4];
    float amax = 0.0f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int64_t row = (int64_t)nb * 128 + (t >> 3) + 32 * p;
        raw[p] = *reinterpret_cast<const uint4*>(w + row * k + (int64_t)kb * 128 + (t & 7) * 16);
        const uint8_t* c = reinterpret_cast<const uint8_t*>(&raw[p]);
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(__fmul_rn(fp8_to_float(c[i]), s_old)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((t & 31) == 0) red[t >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
    float s = __fdiv_rn(fmaxf(amax, 1e-4f), QB_FP8_MAX);
    const uint32_t b = __float_as_uint(s);
    if ((b & 0x7FFFFFu) != 0 && b < 0x7F800000u) s = __uint_as_float((b & 0x7F800000u) + 0x800000u);
    const float inv = ue8m0_inverse(s);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint8_t* c = reinterpret_cast<const uint8_t*>(&raw[p]);
        uint4 o;
        uint16_t* op = reinterpret_cast<uint16_t*>(&o);
#pragma unroll
        for (int i = 0; i < 16; i += 2)
            op[i >> 1] = fp8x2(__fmul_rn(__fmul_rn(fp8_to_float(c[i]), s_old), inv),
                               __fmul_rn(__fmul_rn(fp8_to_float(c[i + 1]), s_old), inv));
        const int64_t row = (int64_t)nb * 128 + (t >> 3) + 32 * p;
        *reinterpret_cast<uint4*>(w + row * k + (int64_t)kb * 128 + (t & 7) * 16) = o;
    }
    if (t == 0) w_scale[(int64_t)nb * kbs + kb] = s;
}

int check_rows(int64_t rows, int64_t hidden, const char* who) {
    if (rows < 0) return invalid(who);
    if (hidden <= 0 || hidden % 256 != 0 || hidden / 8 > 1024) {
        set_error("%s: hidden %lld must be a positive multiple of 256 and <= 8192", who,
                  (long long)hidden);
        return QB_ERR_INVALID;
    }
    if (rows > 0x7fffffffLL) return invalid("rows exceed the grid limit");
    return QB_OK;
}

}  // namespace

extern "C" int qb_embed_rmsnorm_quant(const int64_t* ids, int64_t rows, const void* embed,
                                      int64_t vocab, int64_t hidden, const void* norm_w,
                                      float eps, void* residual_out, void* q_out,
                                      float* scale_out, int64_t scale_ld, int ue8m0,
                                      void* stream) {
    int st = check_rows(rows, hidden, "qb_embed_rmsnorm_quant");
    if (st) return st;
    if (scale_ld < rows) return invalid("qb_embed_rmsnorm_quant: scale_ld < rows");
    if (!aligned(embed, 16) || !aligned(residual_out, 16) || !aligned(norm_w, 16) ||
        !aligned(q_out, 8))
        return invalid("qb_embed_rmsnorm_quant: pointers must be 16-byte aligned (q_out 8)");
    if (rows == 0) return QB_OK;
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_embed_rmsnorm_quant: status word");
    (ue8m0 ? embed_rmsnorm_quant_kernel<true> : embed_rmsnorm_quant_kernel<false>)
        <<<(unsigned)rows, (unsigned)(hidden / 8), 0, (cudaStream_t)stream>>>(
            ids, (const bf16*)embed, vocab, (int)hidden, (const bf16*)norm_w, eps,
            (bf16*)residual_out, (uint8_t*)q_out, scale_out, scale_ld, status);
    return launch_status("qb_embed_rmsnorm_quant");
}

extern "C" int qb_add_rmsnorm_quant(const void* hidden, void* residual, const void* w, float eps,
                                    int64_t rows, int64_t hidden_dim, void* q_out,
                                    float* scale_out, int64_t scale_ld, int ue8m0,
                                    void* stream) {
    int st = check_rows(rows, hidden_dim, "qb_add_rmsnorm_quant");
    if (st) return st;
    if (scale_ld < rows) return invalid("qb_add_rmsnorm_quant: scale_ld < rows");
    if (!aligned(hidden, 16) || !aligned(residual, 16) || !aligned(w, 16) || !aligned(q_out, 8))
        return invalid("qb_add_rmsnorm_quant: pointers must be 16-byte aligned (q_out 8)");
    if (rows == 0) return QB_OK;
    (ue8m0 ? add_rmsnorm_quant_kernel<true> : add_rmsnorm_quant_kernel<false>)
        <<<(unsigned)rows, (unsigned)(hidden_dim / 8), 0, (cudaStream_t)stream>>>(
            (const bf16*)hidden, (bf16*)residual, (const bf16*)w, eps, (int)hidden_dim,
            (uint8_t*)q_out, scale_out, scale_ld);
    return launch_status("qb_add_rmsnorm_quant");
}

extern "C" int qb_silu_mul_quant(const void* gate_up, int64_t rows, int64_t inter, void* q_out,
                                 float* scale_out, int64_t scale_ld, int ue8m0, void* stream) {
    if (rows < 0 || inter <= 0 || inter % 256 != 0)
        return invalid("qb_silu_mul_quant: inter must be a positive multiple of 256");
    if (scale_ld < rows) return invalid("qb_silu_mul_quant: scale_ld < rows");
    if (!aligned(gate_up, 16) || !aligned(q_out, 8))
        return invalid("qb_silu_mul_quant: gate_up must be 16-byte aligned, q_out 8");
    if (rows == 0) return QB_OK;
    const int64_t warps = rows * (inter / 256);
    const int64_t blocks = (warps + 7) / 8;
    if (blocks > 0x7fffffffLL) return invalid("qb_silu_mul_quant: too many rows");
    (ue8m0 ? silu_mul_quant_kernel<true> : silu_mul_quant_kernel<false>)
        <<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
            (const bf16*)gate_up, rows, (int)inter, (uint8_t*)q_out, scale_out, scale_ld);
    return launch_status("qb_silu_mul_quant");
}

extern "C" int qb_requant_weight_ue8m0(void* w, float* w_scale, int64_t n, int64_t k,
                                       void* stream) {
    if (n <= 0 || k <= 0 || n % 128 != 0 || k % 128 != 0)
        return invalid("qb_requant_weight_ue8m0: n and k must be positive multiples of 128");
    if (!aligned(w, 16) || !w_scale)
        return invalid("qb_requant_weight_ue8m0: w must be 16-byte aligned, w_scale non-NULL");
    if (n / 128 > 65535) return invalid("qb_requant_weight_ue8m0: n too large");
    requant_ue8m0_kernel<<<dim3((unsigned)(k / 128), (unsigned)(n / 128)), 256, 0,
                           (cudaStream_t)stream>>>((uint8_t*)w, w_scale, k);
    return launch_status("qb_requant_weight_ue8m0");
}
