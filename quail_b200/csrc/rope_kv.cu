// Per-head q/k RMSNorm + neox rotary, the contiguous v copy, and the paged
// KV append, fused into one pass over the QKV GEMM output (HBM-bound).
// Lane l of a warp owns elements (2l, 2l+1) of the first half of a head and
// (64+2l, 65+2l) of the second half, so each rotary pair sits in one lane.
#include "common.cuh"

namespace {

using namespace qb;

constexpr int HEAD = 128;
constexpr int HALF = HEAD / 2;

// Normalise + rotate one head held as (a0, a1 | b0, b1) per lane and store it.
// The reference computes qa*cos - qb*sin with separate roundings; __fmul_rn /
// __fsub_rn / __fadd_rn keep the compiler from contracting them into FMAs.
__device__ __forceinline__ void norm_rope_head(const bf16* src, bf16* dst, bf16* pool_dst,
                                               const float2 w_a, const float2 w_b,
                                               const float2 c, const float2 s, float eps,
                                               int lane) {
    float2 a = __bfloat1622float2(*reinterpret_cast<const bf162*>(src + 2 * lane));
    float2 b = __bfloat1622float2(*reinterpret_cast<const bf162*>(src + HALF + 2 * lane));
    float ss = __fmul_rn(a.x, a.x);
    ss = __fmaf_rn(a.y, a.y, ss);
    ss = __fmaf_rn(b.x, b.x, ss);
    ss = __fmaf_rn(b.y, b.y, ss);
    ss = warp_sum(ss);
    const float rstd = 1.0f / sqrtf(ss / (float)HEAD + eps);
    a.x = __fmul_rn(__fmul_rn(a.x, rstd), w_a.x);
    a.y = __fmul_rn(__fmul_rn(a.y, rstd), w_a.y);
    b.x = __fmul_rn(__fmul_rn(b.x, rstd), w_b.x);
    b.y = __fmul_rn(__fmul_rn(b.y, rstd), w_b.y);
    const bf162 oa = __floats2bfloat162_rn(__fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(b.x, s.x)),
                                           __fsub_rn(__fmul_rn(a.y, c.y), __fmul_rn(b.y, s.y)));
    const bf162 ob = __floats2bfloat162_rn(__fadd_rn(__fmul_rn(b.x, c.x), __fmul_rn(a.x, s.x)),
                                           __fadd_rn(__fmul_rn(b.y, c.y), __fmul_rn(a.y, s.y)));
    *reinterpret_cast<bf162*>(dst + 2 * lane) = oa;
    *reinterpret_cast<bf162*>(dst + HALF + 2 * lane) = ob;
    if (pool_dst) {
        *reinterpret_cast<bf162*>(pool_dst + 2 * lane) = oa;
        *reinterpret_cast<bf162*>(pool_dst + HALF + 2 * lane) = ob;
    }
}

// One block (256 threads) per row.
__global__ void qknorm_rope_kernel(const bf16* __restrict__ qkv, int64_t qkv_ld,
                                   const int64_t* __restrict__ positions,
                                   const bf16* __restrict__ cos_sin, int64_t max_pos,
                                   const bf16* __restrict__ q_w, const bf16* __restrict__ k_w,
                                   float eps, int n_q, int n_kv, bf16* __restrict__ q_out,
                                   bf16* __restrict__ k_out, bf16* __restrict__ v_out,
                                   const int64_t* __restrict__ row_dst, bf16* __restrict__ k_pool,
                                   bf16* __restrict__ v_pool, int64_t pool_rows,
                                   uint32_t* status) {
    const int64_t row = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, n_warps = blockDim.x >> 5;
    int64_t pos = positions[row];
    if (pos < 0 || pos >= max_pos) {
        if (threadIdx.x == 0) atomicOr(status, STATUS_BAD_INDEX);
        pos = 0;
    }
    int64_t dst = row_dst ? row_dst[row] : -1;
    if (dst >= pool_rows) {
        if (threadIdx.x == 0) atomicOr(status, STATUS_BAD_INDEX);
        dst = -1;
    }
    const bf16* in = qkv + row * qkv_ld;
    const bf16* cs = cos_sin + pos * HEAD;
    const float2 c = __bfloat1622float2(*reinterpret_cast<const bf162*>(cs + 2 * lane));
    const float2 s = __bfloat1622float2(*reinterpret_cast<const bf162*>(cs + HALF + 2 * lane));
    const int kv_width = n_kv * HEAD;
    for (int h = warp; h < n_q + n_kv; h += n_warps) {
        const bool is_q = h < n_q;
        const bf16* w = is_q ? q_w : k_w;
        const float2 w_a = __bfloat1622float2(*reinterpret_cast<const bf162*>(w + 2 * lane));
        const float2 w_b = __bfloat1622float2(*reinterpret_cast<const bf162*>(w + HALF + 2 * lane));
        bf16* out = is_q ? q_out + row * (int64_t)(n_q * HEAD) + h * HEAD
                         : k_out + row * (int64_t)kv_width + (h - n_q) * HEAD;
        bf16* pool = (!is_q && dst >= 0) ? k_pool + dst * kv_width + (h - n_q) * HEAD : nullptr;
        norm_rope_head(in + h * HEAD, out, pool, w_a, w_b, c, s, eps, lane);
    }
    // v: n_kv * 128 bf16, 16 bytes per thread
    const bf16* v_in = in + (n_q + n_kv) * HEAD;
    for (int i = threadIdx.x; i < kv_width / 8; i += blockDim.x) {
        const uint4 val = *reinterpret_cast<const uint4*>(v_in + i * 8);
        *reinterpret_cast<uint4*>(v_out + row * kv_width + i * 8) = val;
        if (dst >= 0) *reinterpret_cast<uint4*>(v_pool + dst * kv_width + i * 8) = val;
    }
}

__global__ void kv_row_map_kernel(const int64_t* __restrict__ src, const int64_t* __restrict__ dst,
                                  int64_t n, int64_t rows, int64_t pool_rows,
                                  int64_t* __restrict__ row_dst, uint32_t* status) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t s = src[i], d = dst[i];
    if (s < 0 || s >= rows || d < 0 || d >= pool_rows) {
        atomicOr(status, STATUS_BAD_INDEX);
        return;
    }
    row_dst[s] = d;
}

// One block per copied row; 16 bytes per thread.
__global__ void kv_scatter_kernel(const bf16* __restrict__ src_k, const bf16* __restrict__ src_v,
                                  const int64_t* __restrict__ src, const int64_t* __restrict__ dst,
                                  int64_t row_elems, int64_t src_rows, bf16* dst_k, bf16* dst_v,
                                  int64_t dst_rows, uint32_t* status) {
    const int64_t i = blockIdx.x;
    const int64_t s = src[i], d = dst[i];
    if (s < 0 || s >= src_rows || d < 0 || d >= dst_rows) {
        if (threadIdx.x == 0) atomicOr(status, STATUS_BAD_INDEX);
        return;
    }
    for (int64_t e = threadIdx.x; e < row_elems / 8; e += blockDim.x) {
        *reinterpret_cast<uint4*>(dst_k + d * row_elems + e * 8) =
            *reinterpret_cast<const uint4*>(src_k + s * row_elems + e * 8);
        *reinterpret_cast<uint4*>(dst_v + d * row_elems + e * 8) =
            *reinterpret_cast<const uint4*>(src_v + s * row_elems + e * 8);
    }
}

}  // namespace

extern "C" int qb_qknorm_rope(const void* qkv, int64_t qkv_ld, const int64_t* positions,
                              const void* cos_sin, int64_t max_pos, const void* q_w,
                              const void* k_w, float eps, int64_t rows, int n_q, int n_kv,
                              int head_dim, void* q_out, void* k_out, void* v_out,
                              const int64_t* row_dst, void* k_pool, void* v_pool,
                              int64_t pool_rows, void* stream) {
    if (head_dim != HEAD) return invalid("qb_qknorm_rope: head_dim must be 128");
    if (rows < 0 || n_q <= 0 || n_kv <= 0 || n_q % n_kv != 0)
        return invalid("qb_qknorm_rope: bad head counts");
    if (qkv_ld < (int64_t)(n_q + 2 * n_kv) * HEAD || qkv_ld % 8 != 0)
        return invalid("qb_qknorm_rope: qkv_ld must cover q|k|v and be a multiple of 8");
    if (!aligned(qkv, 16) || !aligned(v_out, 16) || !aligned(q_out, 4) || !aligned(k_out, 4))
        return invalid("qb_qknorm_rope: qkv and v_out must be 16-byte aligned");
    if (row_dst && (!k_pool || !v_pool || !aligned(v_pool, 16) || !aligned(k_pool, 4)))
        return invalid("qb_qknorm_rope: KV append needs 16-byte aligned pools");
    if (max_pos <= 0) return invalid("qb_qknorm_rope: empty rotary cache");
    if (rows == 0) return QB_OK;
    if (rows > 0x7fffffffLL) return invalid("qb_qknorm_rope: too many rows");
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_qknorm_rope: status word");
    qknorm_rope_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)qkv, qkv_ld, positions, (const bf16*)cos_sin, max_pos, (const bf16*)q_w,
        (const bf16*)k_w, eps, n_q, n_kv, (bf16*)q_out, (bf16*)k_out, (bf16*)v_out, row_dst,
        (bf16*)k_pool, (bf16*)v_pool, pool_rows, status);
    return launch_status("qb_qknorm_rope");
}

extern "C" int qb_kv_row_map(const int64_t* src, const int64_t* dst, int64_t n, int64_t rows,
                             int64_t pool_rows, int64_t* row_dst, void* stream) {
    if (n < 0 || rows < 0) return invalid("qb_kv_row_map: negative size");
    if (rows == 0) return QB_OK;
    cudaError_t e = cudaMemsetAsync(row_dst, 0xff, rows * sizeof(int64_t), (cudaStream_t)stream);
    if (e != cudaSuccess) return launch_status("qb_kv_row_map: memset");
    if (n == 0) return QB_OK;
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_kv_row_map: status word");
    const int64_t blocks = (n + 255) / 256;
    kv_row_map_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(src, dst, n, rows,
                                                                         pool_rows, row_dst,
                                                                         status);
    return launch_status("qb_kv_row_map");
}

extern "C" int qb_kv_scatter(const void* src_k, const void* src_v, const int64_t* src,
                             const int64_t* dst, int64_t n, int64_t row_elems, int64_t src_rows,
                             void* dst_k, void* dst_v, int64_t dst_rows, void* stream) {
    if (n < 0 || row_elems <= 0 || row_elems % 8 != 0)
        return invalid("qb_kv_scatter: row_elems must be a positive multiple of 8");
    if (!aligned(src_k, 16) || !aligned(src_v, 16) || !aligned(dst_k, 16) || !aligned(dst_v, 16))
        return invalid("qb_kv_scatter: pointers must be 16-byte aligned");
    if (n == 0) return QB_OK;
    if (n > 0x7fffffffLL) return invalid("qb_kv_scatter: too many rows");
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_kv_scatter: status word");
    kv_scatter_kernel<<<(unsigned)n, 128, 0, (cudaStream_t)stream>>>(
        (const bf16*)src_k, (const bf16*)src_v, src, dst, row_elems, src_rows, (bf16*)dst_k,
        (bf16*)dst_v, dst_rows, status);
    return launch_status("qb_kv_scatter");
}
