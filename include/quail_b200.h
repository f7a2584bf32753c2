/*
 * quail_b200.h - C ABI of libquailb200.so, the sm_100a (B200) kernels of
 * Quail's AI.IF / AI_FILTER prefill path.
 *
 * Conventions shared by every entry point:
 *   - plain device pointers and sizes only; no torch or C++ types;
 *   - every call is asynchronous on `stream` (a cudaStream_t passed as
 *     void*; NULL is the legacy default stream) and returns QB_OK (0) or a
 *     QB_ERR_* code; qb_last_error() gives the message of the last failure
 *     on the calling host thread;
 *   - argument checks (shapes, alignment, counts) happen on the host before
 *     any launch; a rejected call launches nothing;
 *   - bf16 is IEEE bfloat16 stored as uint16_t, fp8 is e4m3fn stored as
 *     uint8_t, and every "scale" array holds one float per 128-column group
 *     of a row, laid out group-major: scale[g * scale_ld + row]
 *     (the column-major (rows, width/128) layout of
 *     quail/backends/quail/executor/attention.py:153-156);
 *   - `ue8m0` selects the reference's UE8M0 scale mode (Engine.use_ue8m0,
 *     vLLM's is_deep_gemm_e8m0_used; quail/backends/quail/executor/
 *     attention.py:115, 151, 315-316, 350-351, 467-468): a quantiser's
 *     scale becomes exp2(ceil(log2(max(amax, 1e-10) / 448))), the least
 *     power of two at or above the fp32 scale (taken exactly from its
 *     bits), and the GEMMs take power-of-two scales on the block-scaled
 *     MMA path. 0 keeps the fp32 scales.
 *
 * Each function names the reference interface it replaces
 * (paths inside the animysore/quail repository).
 */
#ifndef QUAIL_B200_H
#define QUAIL_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QB_OK 0
#define QB_ERR_INVALID 1   /* bad argument: shape, alignment, count */
#define QB_ERR_CUDA 2      /* a CUDA runtime or driver call failed */
#define QB_ERR_DEVICE 3    /* the device is not sm_100 or lacks a feature */
#define QB_ERR_TIMEOUT 4   /* a kernel's bounded wait ran out (see qb_kernel_status) */

/* Bits of the device status word (qb_kernel_status). */
#define QB_STATUS_WAIT_GEMM 0x0Fu    /* a GEMM role's bounded wait gave up */
#define QB_STATUS_WAIT_ATTN 0xF0u    /* an attention role's bounded wait gave up */
#define QB_STATUS_BAD_TOKEN 0x100u   /* a token id outside [0, vocab) */
#define QB_STATUS_BAD_INDEX 0x200u   /* a page, row or segment index out of range */
#define QB_STATUS_BAD_SCALE 0x400u   /* a UE8M0-mode scale that is not a power of two */

/* Library version, (major << 16) | (minor << 8) | patch. */
int qb_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* qb_last_error(void);

/* Reads and clears the device status word the tcgen05 kernels set when a
 * bounded wait gives up (0 = no timeout seen). Synchronises the device,
 * then takes the word and leaves 0 in one atomic exchange on the device,
 * so no bit set meanwhile by another stream is lost. */
int qb_kernel_status(int device, uint32_t* status_out);

/* Sets how long the kernels' bounded waits on `device` wait before they give
 * up (ns; 0 restores the default of one second). Waits for copies and MMAs
 * a block already issued keep their own one-second limit, so a shortened
 * limit ends only the waits on other roles. A diagnostic for tests of the
 * give-up path (status bits, abort fan-out, TMEM freed); it synchronises the
 * device. Replaces nothing in the reference: Quail's workers detect a failed
 * GPU child on the host (quail/backends/quail/worker.py:382-384). */
int qb_set_wait_limit(int device, uint64_t limit_ns);

/*
 * Layer-0 input norm: hidden = embed[ids]; residual_out = hidden;
 * y = bf16(bf16(hidden * rsqrt(mean(hidden^2) + eps)) * norm_w);
 * q_out/scale_out = 1x128 fp8 quantisation of y.
 * Replaces Qwen3Pipeline.forward_chunk's embedding plus
 * Engine.norm_quant(hidden, norm) with residual=None
 * (quail/backends/quail/executor/models/qwen3.py:51,55-57;
 *  quail/backends/quail/executor/attention.py:763-766, 143-151, 158-175).
 * ids: int64 [rows]; embed: bf16 [vocab, hidden]; norm_w: bf16 [hidden];
 * residual_out: bf16 [rows, hidden]; q_out: fp8 [rows, hidden];
 * scale_out: f32 [hidden/128, scale_ld]. hidden % 256 == 0.
 */
int qb_embed_rmsnorm_quant(const int64_t* ids, int64_t rows, const void* embed,
                           int64_t vocab, int64_t hidden, const void* norm_w,
                           float eps, void* residual_out, void* q_out,
                           float* scale_out, int64_t scale_ld, int ue8m0,
                           void* stream);

/*
 * Fused residual add + RMSNorm + 1x128 fp8 quantisation:
 * x = hidden + residual (fp32); residual = bf16(x);
 * y = x * rsqrt(mean(x^2) + eps) * w (fp32); q_out/scale_out = quant(y).
 * Replaces the Triton add_rms_norm_quant kernel and its wrapper
 * Engine.custom_norm_quant (quail/backends/quail/executor/attention.py:326-359,
 * 658-671). hidden, residual: bf16 [rows, hidden_dim] (residual updated in
 * place); w: bf16 [hidden_dim]; q_out fp8 [rows, hidden_dim];
 * scale_out f32 [hidden_dim/128, scale_ld]. hidden_dim % 256 == 0.
 */
int qb_add_rmsnorm_quant(const void* hidden, void* residual, const void* w,
                         float eps, int64_t rows, int64_t hidden_dim, void* q_out,
                         float* scale_out, int64_t scale_ld, int ue8m0, void* stream);

/*
 * FP8 e4m3 GEMM with 1x128 activation scales and 128x128 weight scales on
 * tcgen05 tensor cores (TMEM accumulators, TMA-fed shared memory):
 * out[m, n] = bf16( sum_kb (sum_{k in kb} a[m,k] w[n,k]) * a_scale[kb, m]
 *                                                       * w_scale[n/128, kb] ).
 * Replaces Engine.gemm -> DeepGEMM fp8_gemm_nt
 * (quail/backends/quail/executor/attention.py:129-141).
 * a: fp8 [m, k] row-major; a_scale: f32 [k/128, a_scale_ld];
 * w: fp8 [n, k] row-major; w_scale: f32 [n/128, k/128]; out: bf16 [m, n].
 * Requires k % 128 == 0, n % 128 == 0, a and w 16-byte aligned.
 * ue8m0 != 0 (fp8_gemm_nt's is_deep_gemm_e8m0_used): every scale is a power
 * of two, applied by the block-scaled MMA (tcgen05 kind::mxf8f6f4) and
 * accumulated over the whole K in fp32:
 * out[m, n] = bf16( sum_k a[m,k] w[n,k] a_scale[k/128, m] w_scale[n/128, k/128] );
 * n % 256 == 0; a scale that is not a power of two sets QB_STATUS_BAD_SCALE.
 */
int qb_gemm_fp8_bs(const void* a, const float* a_scale, int64_t a_scale_ld,
                   const void* w, const float* w_scale, void* out, int64_t m,
                   int64_t n, int64_t k, int ue8m0, void* stream);

/*
 * Per-head RMSNorm of q and k, neox rotary from cos_sin[pos] (cos in the
 * first head_dim/2 columns, sin in the rest), and a contiguous copy of v.
 * When row_dst is given, row r's k (after rotary) and v are also appended
 * to the paged KV pools at pool row row_dst[r] (skipped where row_dst < 0).
 * Replaces the Triton qk_norm_rope kernel (Engine.custom_qk_norm_rope,
 * quail/backends/quail/executor/attention.py:363-409, 673-688), the v
 * slice + .contiguous() (models/qwen3.py:63-64, attention.py:793) and the
 * kv_row_scatter of the tree path (attention.py:725-736, 846-848).
 * qkv: bf16 [rows, qkv_ld] holding q | k | v heads; positions: int64 [rows];
 * cos_sin: bf16 [max_pos, head_dim]; q_w, k_w: bf16 [head_dim];
 * q_out: bf16 [rows, n_q*head_dim]; k_out, v_out: bf16 [rows, n_kv*head_dim];
 * row_dst: int64 [rows] or NULL; k_pool, v_pool: bf16 [pool_rows, n_kv*head_dim].
 * head_dim == 128.
 */
int qb_qknorm_rope(const void* qkv, int64_t qkv_ld, const int64_t* positions,
                   const void* cos_sin, int64_t max_pos, const void* q_w,
                   const void* k_w, float eps, int64_t rows, int n_q, int n_kv,
                   int head_dim, void* q_out, void* k_out, void* v_out,
                   const int64_t* row_dst, void* k_pool, void* v_pool,
                   int64_t pool_rows, void* stream);

/*
 * The qkv projection and qb_qknorm_rope in one kernel: the same bits as
 * qb_gemm_fp8_bs(a, w, n = (n_q + 2 n_kv) * 128) into a bf16 qkv followed by
 * qb_qknorm_rope(qkv, ...), without the bf16 [m, n] intermediate: q and k
 * normalised and rotated, v copied, k and v appended to the pools at
 * row_dst. Replaces engine.gemm(q_in, q_scale, attn.qkv_proj) +
 * custom_qk_norm_rope + the v slice + kv_row_scatter (quail/backends/quail/
 * executor/models/qwen3.py:61-64; attention.py:129-141, 363-409, 673-688,
 * 725-736). a, a_scale, a_scale_ld, w, w_scale: as qb_gemm_fp8_bs with
 * n = (n_q + 2 n_kv) * 128 weight rows (q | k | v heads), n_q + 2 n_kv even;
 * the rest as qb_qknorm_rope, with cos_sin, q_w and k_w 16-byte aligned and
 * pool_rows < 2^31. head_dim == 128.
 */
int qb_gemm_fp8_qknorm_rope(const void* a, const float* a_scale,
                            int64_t a_scale_ld, const void* w,
                            const float* w_scale, int64_t m, int64_t k,
                            const int64_t* positions, const void* cos_sin,
                            int64_t max_pos, const void* q_w, const void* k_w,
                            float eps, int n_q, int n_kv, int head_dim,
                            void* q_out, void* k_out, void* v_out,
                            const int64_t* row_dst, void* k_pool, void* v_pool,
                            int64_t pool_rows, int ue8m0, void* stream);

/*
 * Builds the per-row destination map the fused KV append reads:
 * row_dst[r] = dst[i] where src[i] == r, else -1.
 * Replaces nothing by itself; it turns the reference's (kv_src, kv_dst)
 * scatter lists (quail/backends/quail/executor/loop.py:521-533) into the
 * form qb_qknorm_rope takes. dst values must be < pool_rows.
 */
int qb_kv_row_map(const int64_t* src, const int64_t* dst, int64_t n,
                  int64_t rows, int64_t pool_rows, int64_t* row_dst,
                  void* stream);

/*
 * Row copy between KV row spaces: dst_k[dst[i]] = src_k[src[i]], same for v,
 * row_elems bf16 per row. Replaces the Triton kv_row_scatter kernel
 * (quail/backends/quail/executor/attention.py:415-427, 725-736), used by the
 * unified path for fresh rows and the kept tail copy (attention.py:933-938).
 */
int qb_kv_scatter(const void* src_k, const void* src_v, const int64_t* src,
                  const int64_t* dst, int64_t n, int64_t row_elems,
                  int64_t src_rows, void* dst_k, void* dst_v, int64_t dst_rows,
                  void* stream);

/*
 * The tree attention path, fused: causal attention of each cu_a segment
 * over its own rows (call A), non-causal attention of reader rows over the
 * resident KV pages their read group names (call B), the LSE merge with the
 * reference's bf16 roundings, and per-head fp8 quantisation of the o_proj
 * input. Replaces Engine.attention_tree: FA varlen calls A and B plus the
 * Triton merge_attn_quant kernel
 * (quail/backends/quail/executor/attention.py:835-870, 802-833, 432-473,
 * 738-759).
 * q: bf16 [rows, n_q, 128]; k, v: bf16 [rows, n_kv, 128];
 * cu_a: int32 [n_seg + 1]; tiles: int32 [n_tiles, 2] (segment, first row)
 * of 64-row query tiles (see qb_tree_attention_tiles), in any order;
 * read_cu_q: int32 [n_reads + 1]; read_used: int32 [n_reads];
 * read_table: int32 [n_reads, table_width] of page ids; source: int32 [rows]
 * (reader index of each row or -1); k_pool, v_pool: bf16
 * [n_pages * page_tokens, n_kv, 128]; q_out: fp8 [rows, n_q * 128];
 * scale_out: f32 [n_q, scale_ld].
 */
int qb_tree_attention(const void* q, const void* k, const void* v, int64_t rows,
                      int n_q, int n_kv, int head_dim, const int32_t* cu_a,
                      int64_t n_seg, const int32_t* tiles, int64_t n_tiles,
                      const int32_t* read_cu_q, const int32_t* read_used,
                      const int32_t* read_table, int64_t n_reads,
                      int64_t table_width, const int32_t* source,
                      const void* k_pool, const void* v_pool, int64_t n_pages,
                      int page_tokens, float softmax_scale, void* q_out,
                      float* scale_out, int64_t scale_ld, int ue8m0,
                      void* stream);

/*
 * The unified attention path: one causal paged call in which query
 * sequence s (rows cu_q[s] .. cu_q[s+1]) reads used[s] keys through block
 * table row s and its queries are the last cu_q[s+1] - cu_q[s] of them;
 * the bf16 output is fp8-quantised per head for o_proj. The caller first
 * scatters the chunk's KV into the pools (qb_kv_scatter). Replaces
 * Engine.attention_unified's paged FA call and the quant after it
 * (quail/backends/quail/executor/attention.py:878-953, 796-798).
 * q: bf16 [rows, n_q, 128]; tiles: int32 [n_tiles, 2] (sequence, first
 * row); table: int32 [n_seq, table_width]; pools as qb_tree_attention.
 */
int qb_unified_attention(const void* q, int64_t rows, int n_q, int n_kv,
                         int head_dim, const int32_t* cu_q, int64_t n_seq,
                         const int32_t* tiles, int64_t n_tiles,
                         const int32_t* used, const int32_t* table,
                         int64_t table_width, const void* k_pool,
                         const void* v_pool, int64_t n_pages, int page_tokens,
                         float softmax_scale, void* q_out, float* scale_out,
                         int64_t scale_ld, int ue8m0, void* stream);

/*
 * Host helper for qb_tree_attention: the (segment, first row) pairs of the
 * 64-row query tiles of every cu_a segment, in segment order, written to
 * tiles_host (2 int32 per tile; capacity tiles at most). Host pointers.
 * Replaces nothing in the reference: FA varlen derives its tiles on device.
 */
int qb_tree_attention_tiles(const int32_t* cu_a_host, int64_t n_seg,
                            int32_t* tiles_host, int64_t capacity,
                            int64_t* n_tiles);

/*
 * SiLU-gated product of the two halves of gate_up, 1x128 fp8 quantised:
 * y = g * sigmoid(g) * u (fp32). Replaces the Triton silu_mul_quant kernel
 * (Engine.custom_silu_quant, quail/backends/quail/executor/attention.py:
 * 301-323, 644-656). gate_up: bf16 [rows, 2 * inter]; q_out: fp8
 * [rows, inter]; scale_out: f32 [inter/128, scale_ld]. inter % 256 == 0.
 */
int qb_silu_mul_quant(const void* gate_up, int64_t rows, int64_t inter,
                      void* q_out, float* scale_out, int64_t scale_ld,
                      int ue8m0, void* stream);

/*
 * The MLP's gate_up projection and its SiLU-gated quantisation in one
 * kernel: the same bits as qb_gemm_fp8_bs(a, w, n = 2 * inter) into bf16
 * gate_up followed by qb_silu_mul_quant, without the bf16 [rows, 2 * inter]
 * intermediate. Replaces the MLP's engine.gemm(gate_up_proj) +
 * engine.activation_quant pair (quail/backends/quail/executor/models/
 * qwen3.py:69-70; Engine.gemm and custom_silu_quant, attention.py:129-140,
 * 644-656, 771-775). a, a_scale, a_scale_ld: as qb_gemm_fp8_bs;
 * w: fp8 [2 * inter, k] (gate rows, then up rows); w_scale: f32
 * [2 * inter / 128, k / 128]; q_out: fp8 [m, inter]; scale_out: f32
 * [inter / 128, scale_ld]. inter % 128 == 0, k % 128 == 0; a, w, q_out
 * 16-byte aligned.
 */
int qb_gemm_fp8_silu_quant(const void* a, const float* a_scale,
                           int64_t a_scale_ld, const void* w,
                           const float* w_scale, void* q_out, float* scale_out,
                           int64_t scale_ld, int64_t m, int64_t inter,
                           int64_t k, int ue8m0, void* stream);

/*
 * Re-quantises a block-scaled fp8 weight to power-of-two block scales, in
 * place, for the UE8M0 mode: per 128 x 128 block x = w * w_scale (fp32),
 * s = max(amax(|x|), 1e-4) / 448 raised to the least power of two at or
 * above it, w = e4m3(x / s), w_scale = s. Replaces vLLM's
 * requant_weight_ue8m0_inplace, which Quail's model load runs when
 * DeepGEMM uses UE8M0 scales (vllm/model_executor/layers/quantization/
 * utils/fp8_utils.py; the mode quail/backends/quail/executor/attention.py:
 * 115 reads). w: fp8 [n, k] row-major, 16-byte aligned; w_scale: f32
 * [n/128, k/128]. n, k multiples of 128.
 */
int qb_requant_weight_ue8m0(void* w, float* w_scale, int64_t n, int64_t k,
                            void* stream);

/*
 * Final norm over the answer rows only: for each final row f,
 * x = hidden[f] + residual[f] (fp32); rstd = rsqrt(mean(x^2) + eps);
 * normed_out[i] = bf16(bf16(x * rstd) * final_w).
 * Replaces the final index_select + fused_add_rms_norm of
 * Qwen3Pipeline.forward_chunk (quail/backends/quail/executor/models/
 * qwen3.py:72-77; attention.py:177-181).
 * hidden, residual: bf16 [rows, hidden_dim]; finals: int64 [n_finals];
 * final_w: bf16 [hidden_dim]; normed_out: bf16 [n_finals, hidden_dim].
 */
int qb_final_norm(const void* hidden, const void* residual, int64_t rows,
                  int64_t hidden_dim, const int64_t* finals, int64_t n_finals,
                  const void* final_w, float eps, void* normed_out, void* stream);

/*
 * The yes/no answer head over the retained output rows only:
 * scores[j] = bf16(normed . ans_w[j]) (fp32 accumulate);
 * t = max over true_cols, f = max over false_cols;
 * margin_out = t - f; bits_out = t > f.
 * Replaces AnswerRows.logits and AsyncAnswers.submit's bit
 * (quail/backends/quail/executor/readout.py:45-49, 70-80) over the rows
 * retain_answer_head keeps (executor/model.py:112-134), instead of the full
 * vocabulary head.
 * normed: bf16 [n_rows, hidden_dim]; ans_w: bf16 [n_ids, hidden_dim];
 * true_cols/false_cols: int32 indices into ans_w rows; margin_out:
 * f32 [n_rows]; bits_out: u8 [n_rows]. n_ids <= 16.
 */
int qb_answer_margin(const void* normed, int64_t n_rows, int64_t hidden_dim,
                     const void* ans_w, int n_ids, const int32_t* true_cols,
                     int n_true, const int32_t* false_cols, int n_false,
                     float* margin_out, uint8_t* bits_out, void* stream);

/*
 * AI.SCORE readout over the retained output rows: fp32 scores
 * normed . ans_w[j] (the same fixed summation order as qb_answer_margin,
 * no bf16 rounding), t = max over true_cols, f = max over false_cols,
 * score_out = sigmoid(t - f) in fp32. Replaces AsyncScores.submit
 * (quail/backends/quail/executor/readout.py:88-111: fp32 F.linear, amax per
 * class, torch.sigmoid(yes - no)).
 * normed: bf16 [n_rows, hidden_dim]; ans_w: bf16 [n_ids, hidden_dim];
 * score_out: f32 [n_rows]. n_ids <= 16.
 */
int qb_answer_score(const void* normed, int64_t n_rows, int64_t hidden_dim, const void* ans_w,
                    int n_ids, const int32_t* true_cols, int n_true, const int32_t* false_cols,
                    int n_false, float* score_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QUAIL_B200_H */
