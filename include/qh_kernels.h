/* SPDX-License-Identifier: MIT
 *
 * qh_kernels.h -- C-ABI of the non-matmul kernels of the hybrid forward pass
 * (the device counterparts of the reference's per-token fp32 code). The
 * host step driver (qwen.haiku_b200/csrc/qh_slm.c) chains them with the
 * matmul plans of qh_backend.h. Every call works on B sequences at once,
 * device pointers, asynchronous on `stream`, returns QH_OK or QH_ERR_*.
 *
 * Rounding follows the reference operation by operation: products and sums
 * the reference does in float are done with explicitly rounded float ops
 * (no FMA contraction), and its double-precision accumulations stay double.
 */
#ifndef QH_KERNELS_H
#define QH_KERNELS_H

#include <stdint.h>

#include "qh_sampler.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Token embedding from a Q6_K table of shape (hidden, vocab): h[b] = the
 * dequantized row tokens[b] (q6k_dequant_block, slm/tensor.c:988;
 * slm/qwen.c:885-907). */
int qh_embed_q6k(const void *d_table, int64_t hidden, const int32_t *d_tokens, int32_t B, float *d_h,
                 void *stream);

/* Token embedding from an F32 table of shape (hidden, vocab): h[b] = row
 * tokens[b] (tensor_get_rows on the fp32 view, slm/qwen.c:885-889). */
int qh_embed_f32(const float *d_table, int64_t hidden, const int32_t *d_tokens, int32_t B, float *d_h,
                 void *stream);

/* RMSNorm over rows of `dim` (tensor_rms_norm, slm/tensor.c:348-369):
 * y = x * (1 / sqrtf(float(sum(x*x) / dim) + eps)) * w, the sum of squares
 * accumulated in double. */
int qh_rmsnorm(const float *d_x, const float *d_w, int64_t dim, int64_t rows, float eps, float *d_y,
               void *stream);

/* h += mix over n floats (tensor_add, slm/tensor.c:285). */
int qh_add(float *d_h, const float *d_mix, int64_t n, void *stream);

/* out = silu(gate) * up over n floats (simd_silu_f32 + tensor_mul,
 * slm/qwen.c:952-955). */
int qh_swiglu(const float *d_gate, const float *d_up, float *d_out, int64_t n, void *stream);

/* Gated DeltaNet pre-processing for one layer, B sequences
 * (slm/qwen.c:357-475): push qkv into the conv ring slot pos % kk,
 * causal conv + SiLU, split into Q/K/V, per-head L2 norm of Q (scaled by
 * 1/sqrt(head_dim)) and K, beta = sigmoid(b), g = exp(ssm_a *
 * softplus(a + dt_bias)). The position is read from device memory (*d_pos)
 * here and in the attention kernels, so a whole step can be captured once
 * in a CUDA graph and replayed for every position.
 *   qkv [B][conv_dim], ring [B][kk][conv_dim], conv_w [conv_dim][kk],
 *   b, a [B][heads]; out q, k, v [B][heads*hd], beta, g [B][heads]. */
int qh_gdn_pre(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b,
               const float *d_a, const float *d_dt_bias, const float *d_ssm_a, int32_t B,
               int32_t heads, int32_t hd, int32_t kk, const int32_t *d_pos, float *d_q, float *d_k,
               float *d_v, float *d_beta, float *d_g, void *stream);

/* Gated DeltaNet recurrence (slm/qwen.c:499-557) over state [B][heads][hd
 * k][hd v]: state *= g; kv = state^T K; delta = (V - kv) * beta;
 * state += K delta^T; out = state^T Q -- both reductions over k in double,
 * in the reference's order. out [B][heads*hd]. */
int qh_gdn_recurrence(float *d_state, const float *d_q, const float *d_k, const float *d_v,
                      const float *d_beta, const float *d_g, int32_t B, int32_t heads, int32_t hd,
                      float *d_out, void *stream);

/* Gated RMSNorm per head (slm/qwen.c:571-598): y = ((x * rs) * w) * silu(z). */
int qh_gdn_gated_norm(const float *d_x, const float *d_z, const float *d_w, int32_t B, int32_t heads,
                      int32_t hd, float eps, float *d_y, void *stream);

/* Attention pre-processing for one layer (slm/model.c:831-913): split the
 * head-interleaved Q/gate projection, per-head RMSNorm of Q and K, partial
 * interleaved-MRoPE with the host-built cos/sin table rope[pos][rope_dim/2][2],
 * append K (roped) and V as fp16 at row *d_pos (< max_pos) of the layer's caches
 * [B][max_pos][kvh][hd]. qraw [B][2*nh*hd], k, v [B][kvh*hd] in; q [B][nh][hd],
 * gate [B][nh*hd] out. */
int qh_attn_pre(const float *d_qraw, const float *d_k, const float *d_v, const float *d_qnorm_w,
                const float *d_knorm_w, const float *d_rope, int32_t B, int32_t nh, int32_t kvh,
                int32_t hd, int32_t rope_dim, float eps, const int32_t *d_pos, int32_t max_pos,
                float *d_q, float *d_gate, uint16_t *d_kcache, uint16_t *d_vcache, void *stream);

/* Causal GQA attention of the new query over cache rows 0..*d_pos, then the
 * sigmoid output gate (tensor_attention, slm/tensor.c:1049-1102;
 * slm/model.c:940-947). ctx [B][nh*hd]. */
int qh_attn_decode(const float *d_q, const uint16_t *d_kcache, const uint16_t *d_vcache,
                   const float *d_gate, int32_t B, int32_t nh, int32_t kvh, int32_t hd,
                   const int32_t *d_pos, int32_t max_pos, float *d_ctx, void *stream);

/* Greedy pick per row (sample_argmax, slm/model.c:401-412): index of the
 * first maximum of logits [B][vocab]. */
int qh_argmax(const float *d_logits, int32_t B, int64_t vocab, int32_t *d_out, void *stream);

/* End of a device-driven decode step (the loop of slm_generate,
 * slm/model.c, kept on the device): with pos = ctl[0] and n_prompt = ctl[1],
 * picks[b][pos] = next[b]; tokens[b] = prompt[b][pos + 1] while pos + 1 <
 * n_prompt (teacher forcing through the prompt), else next[b]; then
 * ctl[0] = pos + 1. prompt and picks are [B][stride]. */
int qh_feed_next(const int32_t *d_next, const int32_t *d_prompt, int32_t B, int32_t stride, int32_t *d_ctl,
                 int32_t *d_tokens, int32_t *d_picks, void *stream);

/* ------------------------------------------------------------------------
 * Fused forms used by the decode step. Same arithmetic as the chains they
 * replace (bit-identical results), fewer launches and HBM round trips.
 * ---------------------------------------------------------------------- */

/* Every fused kernel below that ends in a Q8_K quantization writes xq for
 * K values x n_tok = B rows in the layout chosen by layout_tile: 0 = the
 * split layout of qh_backend.h (GEMV input), QH_Q8KT_TILE (64) = the tiled
 * layout of qh_q8kt_bytes (tensor-core GEMM input). */

/* Optional residual add, RMSNorm and Q8_K quantization in one launch:
 * with d_mix, h_out = h + mix and xq = Q8_K(rmsnorm(h_out) * w); without,
 * xq = Q8_K(rmsnorm(h) * w) and h_out is not touched (qh_add + qh_rmsnorm
 * + qh_quantize_q8k; slm/tensor.c:285, 348-369, 683-720). h_out must not
 * alias h. dim a multiple of 256, at most 4096. */
int qh_rmsnorm_q8k(const float *d_h, const float *d_mix, float *d_h_out, const float *d_w, int64_t dim, int32_t B,
                   float eps, void *d_xq, int32_t layout_tile, void *stream);

/* xq = Q8_K(silu(gate) * up) for B rows of ffn values (qh_swiglu +
 * qh_quantize_q8k; slm/qwen.c:952-955). */
int qh_swiglu_q8k(const float *d_gate, const float *d_up, int64_t ffn, int32_t B, void *d_xq, int32_t layout_tile,
                  void *stream);

/* The whole Gated DeltaNet mixer between its projections for one token per
 * sequence (slm/qwen.c:357-598): qh_gdn_pre + qh_gdn_recurrence +
 * qh_gdn_gated_norm (z is the attn_gate projection [B][heads*hd], norm_w
 * ssm_norm [hd]) + Q8_K of the result into xq (K = heads*hd, n_tok = B).
 * hd must be 128, heads even. */
int qh_gdn_fused(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b, const float *d_a,
                 const float *d_dt_bias, const float *d_ssm_a, float *d_state, const float *d_z,
                 const float *d_norm_w, int32_t B, int32_t heads, int32_t hd, int32_t kk, float eps,
                 const int32_t *d_pos, void *d_xq, int32_t layout_tile, void *stream);

/* ------------------------------------------------------------------------
 * Prompt chunks: n_tok tokens of each of n_seq sequences at once, rows
 * sequence-major (row = s * n_tok + j, position *d_pos + j). Each kernel
 * performs the per-token arithmetic of its decode counterpart, in the same
 * order, so a prompt run in chunks leaves the same caches and produces the
 * same activations as the prompt fed one token per step (the reference's
 * default prefill in slm_generate_raw, slm/slm.c:280-287).
 * ---------------------------------------------------------------------- */

/* qh_attn_pre for every prompt row: q/k norms, MRoPE at the row's position,
 * K and V appended to the caches at rows *d_pos .. *d_pos + n_tok - 1. */
int qh_attn_prefill_pre(const float *d_qraw, const float *d_k, const float *d_v, const float *d_qnorm_w,
                        const float *d_knorm_w, const float *d_rope, int32_t n_seq, int32_t n_tok, int32_t nh,
                        int32_t kvh, int32_t hd, int32_t rope_dim, float eps, const int32_t *d_pos, int32_t max_pos,
                        float *d_q, float *d_gate, uint16_t *d_kcache, uint16_t *d_vcache, void *stream);

/* Causal attention of every prompt row over cache rows 0 .. its position
 * (qh_attn_decode per row; needs hd 128 and a query group of 1, 2, 4 or 8). */
int qh_attn_prefill(const float *d_q, const uint16_t *d_kcache, const uint16_t *d_vcache, const float *d_gate,
                    int32_t n_seq, int32_t n_tok, int32_t nh, int32_t kvh, int32_t hd, const int32_t *d_pos,
                    int32_t max_pos, float *d_ctx, void *stream);

/* qh_gdn_fused for n_tok consecutive tokens of each sequence, in token
 * order, inside one launch (hd 128, conv kernel 4). */
int qh_gdn_prefill(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b, const float *d_a,
                   const float *d_dt_bias, const float *d_ssm_a, float *d_state, const float *d_z,
                   const float *d_norm_w, int32_t n_seq, int32_t n_tok, int32_t heads, int32_t hd, int32_t kk,
                   float eps, const int32_t *d_pos, void *d_xq, int32_t layout_tile, void *stream);

/* ------------------------------------------------------------------------
 * Chunked prefill (the reference's batched prompt path, slm_forward_batch,
 * slm/qwen.c:1018-1106, taken under LLM_USE_FORWARD_BATCH): its DeltaNet
 * layers (slm_forward_ssm_batch, slm/qwen.c:627-806) run the 64-token chunk
 * algebra of chunked_ssm_step_f32 (slm/chunked.c:287-523), which is not
 * bit-equal to the per-token recurrence; these two kernels reproduce it bit
 * for bit. Rows are sequence-major (row = s * n_tok + j, position
 * *d_pos + j); chunks of 64 start at each call's first token.
 * ---------------------------------------------------------------------- */

/* Conv ring, SiLU, per-head L2 norms, beta and g_log for n_tok tokens per
 * sequence (slm/qwen.c:652-715), in place: the head slices of each row of
 * qkv [rows][3*heads*hd] become Q * (qrs / sqrt(hd)), K * krs and silu(conv
 * V); b and a [rows][heads] become beta = sigmoid(b) and g_log = ssm_a *
 * softplus(a + dt_bias). The ring [n_seq][kk][3*heads*hd] is read at and
 * left for the chunk's positions, as qh_gdn_prefill. hd 128, kk 4. */
int qh_gdn_chunk_prep(float *d_qkv, float *d_ring, const float *d_conv_w, float *d_b, float *d_a,
                      const float *d_dt_bias, const float *d_ssm_a, int32_t n_seq, int32_t n_tok, int32_t heads,
                      int32_t hd, int32_t kk, const int32_t *d_pos, void *stream);

/* The chunked delta rule over n_tok tokens per sequence: for each head and
 * each chunk of <= 64 tokens, chunked_ssm_step_f32 (slm/chunked.c:287-523)
 * on qh_gdn_chunk_prep's rows, the state [n_seq][heads][hd k][hd v] (16-byte
 * aligned) carried across chunks. out [rows][heads*hd] receives the
 * per-token outputs before the gated norm (qh_gdn_gated_norm). hd 128. */
int qh_gdn_chunked(const float *d_qkv, const float *d_beta, const float *d_glog, float *d_state, int32_t n_seq,
                   int32_t n_tok, int32_t heads, int32_t hd, float *d_out, void *stream);

/* qh_gdn_fused without the quantization: the gated-norm output y fp32
 * [B][heads*hd] for qh_quantize_q8k / qh_quantize_q8kt. The heads are then
 * independent CTAs (no cluster pairs), which keeps more of them resident
 * when many sequences run. */
int qh_gdn_fused_y(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b, const float *d_a,
                   const float *d_dt_bias, const float *d_ssm_a, float *d_state, const float *d_z,
                   const float *d_norm_w, int32_t B, int32_t heads, int32_t hd, int32_t kk, float eps,
                   const int32_t *d_pos, float *d_y, void *stream);

/* qh_argmax + qh_feed_next over a grid of CTAs per row (sample_argmax,
 * slm/model.c:401-412). d_scratch holds per-slice partial maxima and ticket
 * counters: qh_argmax_feed_scratch_bytes bytes, zero-filled before the first
 * call (each call leaves the counters at zero). The size query returns -1
 * for bad arguments. */
int64_t qh_argmax_feed_scratch_bytes(int32_t B, int64_t vocab);
int qh_argmax_feed(const float *d_logits, int32_t B, int64_t vocab, void *d_scratch, int32_t *d_next,
                   const int32_t *d_prompt, int32_t stride, int32_t *d_ctl, int32_t *d_tokens, int32_t *d_picks,
                   void *stream);

/* Sampler settings of a sampled decode step, read from device memory so a
 * captured step serves any settings: the chain (qh_sampler.h) plus the
 * eos/eot masking of slm_generate_raw (slm/slm.c:303-322) -- while
 * pos - gen0 < min_new (tokens generated so far), logits[eos_id] and
 * logits[eot_id] are -inf during sampling and restored after (-1: none). */
typedef struct qh_sample_ctl {
    qh_sampler sp;
    int32_t eos_id, eot_id;
    int32_t min_new;
    int32_t gen0;  /* position of the first sampled step */
} qh_sample_ctl;

/* qh_sample + the device-side feed of a sampled decode step: per row the
 * pick goes to d_next, d_picks[row][pos], d_tokens (the next input) and is
 * appended to the row's history (d_hist [B][hist_stride], lengths d_hist_n);
 * the last row to finish advances d_ctl[0]. *d_ticket starts at zero and is
 * left at zero. */
int qh_sample_feed(float *d_logits, int32_t B, int64_t vocab, const qh_sample_ctl *d_sctl, int32_t *d_hist,
                   int32_t hist_stride, int32_t *d_hist_n, uint64_t *d_rng, int32_t *d_next, int32_t stride,
                   int32_t *d_ctl, int32_t *d_tokens, int32_t *d_picks, unsigned *d_ticket, void *stream);

/* expf (fn 0) or logf (fn 1) of the floats whose bit patterns are
 * first, first + 1, ..., first + n - 1 (wrapping at 2^32), as the device
 * kernels evaluate them (the host C library's values, bit for bit: the
 * reference calls expf/logf at slm/qwen.c:464-470, slm/model.c:943,
 * slm/tensor.c:315/491/1086, simd/simd.c:264-277, slm/sampler.c:105). For
 * checking those functions against the host library. */
int qh_libm_eval(int fn, uint32_t first, int64_t n, float *d_out, void *stream);

/* ---- Persistent decode step (one sequence) ------------------------------
 * A run of consecutive operations of slm_forward_step (slm/qwen.c:874-981)
 * for ONE sequence, executed as one cooperative launch of one CTA per SM
 * with a grid-wide barrier between phases, instead of one launch per
 * operation. Two kinds of phase:
 *   QH_STEP_MATVEC  form the Q8_K input row of xk values in every CTA --
 *     residual add + RMSNorm (QH_STEP_X_RESNORM: x = xa (+ xb), norm weight
 *     xw, eps; x written to xh_out by one CTA when xh_out is given; the
 *     operations of qh_rmsnorm_q8k), SwiGLU (QH_STEP_X_SWIGLU: silu(xa) * xb,
 *     as qh_swiglu_q8k) or plain quantization (QH_STEP_X_QUANT: xa, as
 *     qh_quantize_q8k) -- then out = W x for up to QH_STEP_MAX_PROJ
 *     K-quant weights (Q4_K, Q5_K, Q6_K; the values of qh_matmul_preq:
 *     tensor_matmul_*_f32, slm/tensor.c:827-1033);
 *   QH_STEP_GDN  one Gated DeltaNet token update for every head (the
 *     operations of qh_gdn_fused_y, slm/qwen.c:318-611), fp32 output rows y;
 *   QH_STEP_ATTN  one gated-attention token for every query head (the
 *     operations of qh_attn_pre + qh_attn_decode, slm/model.c:766-953):
 *     q/k RMSNorm, MRoPE, the fp16 K/V append at *d_pos, softmax attention
 *     over the cache, the sigmoid gate; fp32 output rows ctx. Not directly
 *     before a QH_STEP_GDN phase (they share a shared-memory region).
 * Weight tiles stream into shared memory ahead of the phase that reads them
 * (weights do not depend on activations), so a phase's time is its
 * dependency latency, not a launch's ramp. Outputs are bit-identical to the
 * launch-per-operation chain. Positions are read from *d_pos. Every wait in
 * the kernel is bounded; a timeout is reported through
 * qh_check_device_error. */
#define QH_STEP_MATVEC 0
#define QH_STEP_GDN 1
#define QH_STEP_ATTN 2
#define QH_STEP_X_RESNORM 1
#define QH_STEP_X_SWIGLU 2
#define QH_STEP_X_QUANT 3
#define QH_STEP_MAX_PROJ 8
/* Longest cache a QH_STEP_ATTN phase takes (its scores live in shared memory). */
#define QH_STEP_ATTN_MAX_POS 8192

typedef struct qh_step_proj {
    int32_t type;      /* QH_GGUF_Q4_K, QH_GGUF_Q5_K or QH_GGUF_Q6_K */
    const void *d_w;   /* GGUF blocks [out_f][k], 16-byte aligned */
    int64_t k, out_f;
    float *d_out;      /* [out_f] */
} qh_step_proj;

typedef struct qh_step_phase {
    int32_t kind;      /* QH_STEP_MATVEC or QH_STEP_GDN */
    /* QH_STEP_MATVEC */
    int32_t xform;     /* QH_STEP_X_* */
    int64_t xk;
    float eps;         /* RMSNorm epsilon (also the DeltaNet gated-norm epsilon) */
    const float *d_xa, *d_xb, *d_xw;
    float *d_xh_out;
    int32_t n_proj;
    qh_step_proj proj[QH_STEP_MAX_PROJ];
    /* optional: with two projections of one shape (ffn gate, up), also
     * act[r] = silu(out0[r]) * out1[r] (the values qh_swiglu forms), each
     * CTA for the rows it computed; the next phase then quantizes act
     * (QH_STEP_X_QUANT) instead of every CTA forming the SwiGLU row */
    float *d_act_out;
    /* QH_STEP_GDN (sequence 0 of the qh_gdn_fused_y arguments) */
    const float *d_qkv;
    float *d_ring;
    const float *d_conv_w, *d_b, *d_a, *d_dt_bias, *d_ssm_a;
    float *d_state;
    const float *d_z, *d_norm_w;
    float *d_y;
    int32_t heads, head_dim, conv_kernel;
    /* QH_STEP_ATTN (sequence 0 of the qh_attn_pre + qh_attn_decode
     * arguments; head_dim above must be 128; caches [max_pos][n_kv_heads][128]) */
    const float *d_qraw, *d_kin, *d_vin, *d_qnorm_w, *d_knorm_w, *d_rope;
    uint16_t *d_kcache, *d_vcache;
    float *d_ctx;
    int32_t n_heads, n_kv_heads, rope_dim, max_pos;
} qh_step_phase;

typedef struct qh_step_prog qh_step_prog;

/* Validates and uploads the phases (device tables, barrier counters) for the
 * current device. QH_ERR_UNSUPPORTED for weight types other than the K-quants
 * or a device without cooperative launch. */
int qh_step_create(const qh_step_phase *phases, int32_t n_phases, const int32_t *d_pos, qh_step_prog **out);
/* Runs phases [first, first + count) as one launch on `stream`. Launches of
 * one program must not overlap (they share the barrier counters). */
int qh_step_run(qh_step_prog *prog, int32_t first, int32_t count, void *stream);
void qh_step_destroy(qh_step_prog *prog);
/* Measurement hook: with d_stamps non-null (qh_step_phase_count records of
 * 8 + 2G uint64, G = the device's SM count, the launch's CTAs), later
 * launches write %globaltimer (ns) per phase p into record p: [0] CTA 0 at
 * the phase start, [1] input formed, [2] work done, [3] past the grid
 * barrier; [4..7] points inside the phase's work on CTA 0 (DeltaNet: inputs
 * ready, state landed, recurrence done, output written; attention: norms
 * done, scores, softmax, output written; RMSNorm inputs: sums formed, block
 * sum done, weights landed); [8 + c] CTA c's work done; [8 + G + c] CTA c's
 * input formed.
 * Null turns it off. Launches already captured in a CUDA graph keep the
 * setting they were captured with. */
int qh_step_set_stamps(qh_step_prog *prog, uint64_t *d_stamps);
int32_t qh_step_phase_count(const qh_step_prog *prog);
/* Failure-detection test hook (no reference counterpart): the program's next
 * launches leave out the copy of the tile that CTA 0 streams as its number
 * `tile` (counted from 0 over the launch's projection phases; -1: none), and
 * every shared-memory barrier wait polls at most wait_limit times (0: the
 * kernel's default, seconds) -- the path of a lost copy: CTA 0 records the
 * timeout in the device error word and stops, the other CTAs leave at their
 * next grid barrier, every CTA waits (bounded) for its own copies in flight,
 * and qh_check_device_error reports QH_ERR_DEVICE. Nothing faults; the
 * outputs of such a launch are not defined. */
int qh_step_test_timeout(qh_step_prog *prog, int32_t tile, uint32_t wait_limit);

#ifdef __cplusplus
}
#endif

#endif /* QH_KERNELS_H */
