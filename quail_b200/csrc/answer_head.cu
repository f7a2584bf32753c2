// The end of the forward pass and the answer readout, over answer rows only.
//  - final norm: gather each final row of hidden and residual, add them in
//    fp32, RMSNorm, bf16 output (the reference's index_select +
//    fused_add_rms_norm);
//  - answer margin: dot products of each normed row with the retained
//    TRUE/FALSE rows of the output head, bf16-rounded scores, per-class max,
//    margin and bit (the reference's F.linear + amax + compare).
// One block per row, one 16-byte vector (8 columns) per thread.
#include "common.cuh"

namespace {

using namespace qb;

constexpr int MAX_IDS = 16;

__global__ void final_norm_kernel(const bf16* __restrict__ hidden,
                                  const bf16* __restrict__ residual, int64_t rows, int hdim,
                                  const int64_t* __restrict__ finals,
                                  const bf16* __restrict__ final_w, float eps,
                                  bf16* __restrict__ normed_out, uint32_t* status) {
    __shared__ float scratch[32];
    const int64_t i = blockIdx.x;
    const int t = threadIdx.x;
    int64_t row = finals[i];
    if (row < 0 || row >= rows) {
        if (t == 0) atomicOr(status, STATUS_BAD_INDEX);
        row = 0;
    }
    float h[8], r[8], x[8];
    bf16x8_to_float(*reinterpret_cast<const uint4*>(hidden + row * hdim + t * 8), h);
    bf16x8_to_float(*reinterpret_cast<const uint4*>(residual + row * hdim + t * 8), r);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = h[j] + r[j];
    const float total = block_sum(sumsq8(x), scratch);
    const float rstd = 1.0f / sqrtf(total / (float)hdim + eps);
    float wf[8], y[8];
    bf16x8_to_float(*reinterpret_cast<const uint4*>(final_w + t * 8), wf);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = bf16_round(x[j] * rstd) * wf[j];
    *reinterpret_cast<uint4*>(normed_out + i * hdim + t * 8) = float_to_bf16x8(y);
}

// SCORE = false: bf16 scores, margin and bit (AI_FILTER / AI_JOIN);
// SCORE = true: fp32 scores, out = sigmoid(t - f) (AI.SCORE), bits unused.
template <bool SCORE>
__global__ void answer_margin_kernel(const bf16* __restrict__ normed, int hdim,
                                     const bf16* __restrict__ ans_w, int n_ids,
                                     const int32_t* __restrict__ true_cols, int n_true,
                                     const int32_t* __restrict__ false_cols, int n_false,
                                     float* __restrict__ margin_out,
                                     uint8_t* __restrict__ bits_out, uint32_t* status) {
    __shared__ float partial[32][MAX_IDS];
    __shared__ float scores[MAX_IDS];
    const int64_t i = blockIdx.x;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int n_warps = blockDim.x >> 5;
    float y[8];
    bf16x8_to_float(*reinterpret_cast<const uint4*>(normed + i * hdim + t * 8), y);
    for (int id = 0; id < n_ids; ++id) {
        float aw[8];
        bf16x8_to_float(*reinterpret_cast<const uint4*>(ans_w + (int64_t)id * hdim + t * 8), aw);
        float d = __fmul_rn(y[0], aw[0]);
#pragma unroll
        for (int j = 1; j < 8; ++j) d = __fmaf_rn(y[j], aw[j], d);
        d = warp_sum(d);
        if (lane == 0) partial[warp][id] = d;
    }
    __syncthreads();
    if (t < n_ids) {
        float s = 0.0f;
        for (int w = 0; w < n_warps; ++w) s = __fadd_rn(s, partial[w][t]);
        scores[t] = SCORE ? s : bf16_round(s);
    }
    __syncthreads();
    if (t == 0) {
        float best_t = -INFINITY, best_f = -INFINITY;
        for (int j = 0; j < n_true; ++j) {
            const int c = true_cols[j];
            if (c >= 0 && c < n_ids) best_t = fmaxf(best_t, scores[c]);
            else atomicOr(status, STATUS_BAD_INDEX);
        }
        for (int j = 0; j < n_false; ++j) {
            const int c = false_cols[j];
            if (c >= 0 && c < n_ids) best_f = fmaxf(best_f, scores[c]);
            else atomicOr(status, STATUS_BAD_INDEX);
        }
        if (SCORE) {
            margin_out[i] = sigmoidf_ref(__fsub_rn(best_t, best_f));
        } else {
            margin_out[i] = best_t - best_f;
            bits_out[i] = best_t > best_f ? 1 : 0;
        }
    }
}

int check_hdim(int64_t hdim, const char* who) {
    if (hdim <= 0 || hdim % 256 != 0 || hdim / 8 > 1024) {
        set_error("%s: hidden_dim must be a positive multiple of 256, at most 8192", who);
        return QB_ERR_INVALID;
    }
    return QB_OK;
}

}  // namespace

extern "C" int qb_final_norm(const void* hidden, const void* residual, int64_t rows,
                             int64_t hidden_dim, const int64_t* finals, int64_t n_finals,
                             const void* final_w, float eps, void* normed_out, void* stream) {
    int st = check_hdim(hidden_dim, "qb_final_norm");
    if (st) return st;
    if (n_finals < 0 || rows < 0) return invalid("qb_final_norm: negative size");
    if (!aligned(hidden, 16) || !aligned(residual, 16) || !aligned(final_w, 16) ||
        !aligned(normed_out, 16))
        return invalid("qb_final_norm: pointers must be 16-byte aligned");
    if (n_finals == 0) return QB_OK;
    if (n_finals > 0x7fffffffLL) return invalid("qb_final_norm: too many rows");
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_final_norm: status word");
    final_norm_kernel<<<(unsigned)n_finals, (unsigned)(hidden_dim / 8), 0, (cudaStream_t)stream>>>(
        (const bf16*)hidden, (const bf16*)residual, rows, (int)hidden_dim, finals,
        (const bf16*)final_w, eps, (bf16*)normed_out, status);
    return launch_status("qb_final_norm");
}

extern "C" int qb_answer_margin(const void* normed, int64_t n_rows, int64_t hidden_dim,
                                const void* ans_w, int n_ids, const int32_t* true_cols, int n_true,
                                const int32_t* false_cols, int n_false, float* margin_out,
                                uint8_t* bits_out, void* stream) {
    int st = check_hdim(hidden_dim, "qb_answer_margin");
    if (st) return st;
    if (n_ids <= 0 || n_ids > MAX_IDS) return invalid("qb_answer_margin: 1 <= n_ids <= 16");
    if (n_true <= 0 || n_false <= 0) return invalid("qb_answer_margin: empty answer class");
    if (n_rows < 0) return invalid("qb_answer_margin: negative size");
    if (!aligned(normed, 16) || !aligned(ans_w, 16))
        return invalid("qb_answer_margin: pointers must be 16-byte aligned");
    if (n_rows == 0) return QB_OK;
    if (n_rows > 0x7fffffffLL) return invalid("qb_answer_margin: too many rows");
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_answer_margin: status word");
    answer_margin_kernel<false><<<(unsigned)n_rows, (unsigned)(hidden_dim / 8), 0,
                                  (cudaStream_t)stream>>>(
        (const bf16*)normed, (int)hidden_dim, (const bf16*)ans_w, n_ids, true_cols, n_true,
        false_cols, n_false, margin_out, bits_out, status);
    return launch_status("qb_answer_margin");
}

extern "C" int qb_answer_score(const void* normed, int64_t n_rows, int64_t hidden_dim,
                               const void* ans_w, int n_ids, const int32_t* true_cols, int n_true,
                               const int32_t* false_cols, int n_false, float* score_out,
                               void* stream) {
    int st = check_hdim(hidden_dim, "qb_answer_score");
    if (st) return st;
    if (n_ids <= 0 || n_ids > MAX_IDS) return invalid("qb_answer_score: 1 <= n_ids <= 16");
    if (n_true <= 0 || n_false <= 0) return invalid("qb_answer_score: empty answer class");
    if (n_rows < 0) return invalid("qb_answer_score: negative size");
    if (!aligned(normed, 16) || !aligned(ans_w, 16))
        return invalid("qb_answer_score: pointers must be 16-byte aligned");
    if (n_rows == 0) return QB_OK;
    if (n_rows > 0x7fffffffLL) return invalid("qb_answer_score: too many rows");
    uint32_t* status = device_status_ptr();
    if (!status) return launch_status("qb_answer_score: status word");
    answer_margin_kernel<true><<<(unsigned)n_rows, (unsigned)(hidden_dim / 8), 0,
                                 (cudaStream_t)stream>>>(
        (const bf16*)normed, (int)hidden_dim, (const bf16*)ans_w, n_ids, true_cols, n_true,
        false_cols, n_false, score_out, nullptr, status);
    return launch_status("qb_answer_score");
}
