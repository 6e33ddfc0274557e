/* SPDX-License-Identifier: MIT
 *
 * qh_slm.h -- the Qwen3.5-0.8B-shaped hybrid forward pass (Gated DeltaNet
 * + gated attention) on B200, token level.
 *
 * Reference counterparts (qwen.haiku, path:line):
 *   struct slm_config                    slm/model.c:72-98
 *   struct slm_weights / slm_load_weights slm/model.c:154-188, slm/qwen.c:174-252
 *   slm_ctx caches (KV, conv ring, SSM)  slm/model.c:289-391, 488-504
 *   slm_forward_step                     slm/qwen.c:874-981
 *     slm_forward_ssm (GDN layer)        slm/qwen.c:318-611
 *     slm_forward_attn (attention layer) slm/model.c:766-953
 *   sample_argmax (greedy pick)          slm/model.c:401-412
 *   slm_generate_raw (generation loop)   slm/slm.c:237-357
 *   slm_ctx_snapshot / slm_ctx_restore   slm/model.c:1262-1371
 *   JSONL parity tracer (slm_trace_*)    slm/model.c:585-727
 * The reference's text layer (tokenizer, chat template, agent) is not part
 * of this path: these entry points take token ids.
 *
 * One qh_slm holds the weights of one model on one GPU plus the decode
 * state of n_seq independent sequences (the reference's slm_ctx, one per
 * sequence); a step advances every sequence by one token at the same
 * position, i.e. batched decode for data-parallel serving. All calls return
 * QH_OK or a negative QH_ERR_* status (include/qh_backend.h).
 */
#ifndef QH_SLM_H
#define QH_SLM_H

#include <stdint.h>

#include "qh_sampler.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct qh_slm_config {
    int32_t n_layers;           /* 24 */
    int32_t hidden;             /* 1024 */
    int32_t ffn;                /* 3584 */
    int32_t vocab;              /* 151936 */
    int32_t n_heads;            /* attention query heads, 8 */
    int32_t n_kv_heads;         /* 2 */
    int32_t head_dim;           /* 128 */
    int32_t rope_dim;           /* rotated dims per head, 64 */
    float rope_theta;           /* 1e6 */
    int32_t rope_sections[4];   /* interleaved MRoPE sections, {11, 11, 10, 0} */
    float norm_eps;             /* RMSNorm epsilon */
    int32_t gdn_heads;          /* Gated DeltaNet heads, 16 */
    int32_t gdn_head_dim;       /* key = value head dim, 128 */
    int32_t conv_kernel;        /* 4 */
    int32_t full_attn_interval; /* every 4th layer is attention (L % 4 == 3) */
    int32_t max_pos;            /* KV-cache positions per sequence */
} qh_slm_config;

/* BASELINE config 4/5 shape: Qwen3.5-0.8B-like hybrid, vocab 151936. */
void qh_slm_config_default(qh_slm_config *cfg, int32_t max_pos);

/* ------------------------------------------------------------------------
 * Synthetic weights (host). The reference runs on a real GGUF; with none
 * available, a seeded blob of tensors with the GGUF names, types and shapes
 * stands in: matrices N(0, 0.02) quantized with qh_synth_quantize (Q4_K,
 * Q6_K for ffn_down and the tied token embedding / LM head), fp32 norms
 * 1 + N(0, 0.02), ssm_a = -exp(N(0, 0.02)), conv1d N(0, 0.5), dt bias
 * N(0, 0.02). Shapes follow GGUF order: shape[0] = input dim.
 * ---------------------------------------------------------------------- */
typedef struct qh_blob qh_blob;

int qh_blob_synthetic(const qh_slm_config *cfg, uint64_t seed, qh_blob **out);
/* The same model with the weight types of a mix: QH_MIX_BASELINE (the one
 * above), QH_MIX_Q4_K_M (the released Qwen3.5-0.8B Q4_K_M file's types,
 * docs/DESIGN.md:96-119 of the reference: Q5_K attn_q / attn_qkv / ssm_out,
 * Q6_K attn_v / ffn_down / token_embd, Q8_0 ssm_alpha / ssm_beta, Q4_K the
 * rest) or QH_MIX_ALL_TYPES (F32, Q8_0, Q5_K, Q6_K matrices in roles where
 * the released file has none, to exercise every matmul case of the model). */
#define QH_MIX_BASELINE 0
#define QH_MIX_Q4_K_M 1
#define QH_MIX_ALL_TYPES 2
int qh_blob_synthetic_mix(const qh_slm_config *cfg, uint64_t seed, int32_t mix, qh_blob **out);
int qh_blob_count(const qh_blob *blob);
/* Tensor i: GGUF name, GGUF type id, shape (shape[1] = 1 for vectors), host
 * data and byte size. Pointers stay valid until qh_blob_free. */
int qh_blob_tensor(const qh_blob *blob, int i, const char **name, int32_t *type, int64_t shape[2],
                   const void **data, int64_t *nbytes);
/* Index of the tensor named `name`, or -1. */
int qh_blob_find(const qh_blob *blob, const char *name);
void qh_blob_free(qh_blob *blob);

/* A blob built from the caller's tensors (e.g. a GGUF file's, with the GGUF
 * names and shapes, shape[0] = input dim): qh_blob_add copies the bytes.
 * Types F32 (0), Q8_0, Q4_K, Q5_K, Q6_K; nbytes must match the shape. */
int qh_blob_create(qh_blob **out);
int qh_blob_add(qh_blob *blob, const char *name, int32_t type, const int64_t shape[2], const void *data,
                int64_t nbytes);

/* ------------------------------------------------------------------------
 * Device model + n_seq sequences
 * ---------------------------------------------------------------------- */
typedef struct qh_slm qh_slm;

/* Uploads every blob tensor to the current device (weights keep their GGUF
 * block layout) and allocates the caches of n_seq sequences. */
int qh_slm_create(const qh_slm_config *cfg, const qh_blob *blob, int32_t n_seq, qh_slm **out);
void qh_slm_destroy(qh_slm *m);

/* Clears every sequence's KV cache, conv ring and recurrent state. */
int qh_slm_reset(qh_slm *m);

/* slm_forward_step + sample_argmax for all n_seq sequences at position pos
 * (slm/qwen.c:874-981, slm/model.c:401-412): h_tokens[n_seq] in,
 * h_next[n_seq] (greedy argmax) out, optionally the logits
 * h_logits[n_seq][vocab]. Synchronous. The step is one CUDA graph launch
 * (captured on the second call; the first runs the kernels directly). */
int qh_slm_step(qh_slm *m, const int32_t *h_tokens, int32_t pos, int32_t *h_next, float *h_logits);

/* Device-driven decoding, no host round trip per token:
 *   qh_slm_begin   uploads prompt[n_seq][n_prompt], clears the caches
 *                  (qh_slm_reset) and sets position 0;
 *   qh_slm_advance launches n_steps steps (asynchronous on qh_slm_stream):
 *                  step p feeds prompt[s][p] while p < n_prompt, else the
 *                  greedy pick of step p - 1, and records its own pick;
 *   qh_slm_picks   waits, then out[s][i] = pick of step from_pos + i.
 * Positions stay below max_pos. */
int qh_slm_begin(qh_slm *m, const int32_t *prompt, int32_t n_prompt);
int qh_slm_advance(qh_slm *m, int32_t n_steps);
int qh_slm_picks(qh_slm *m, int32_t from_pos, int32_t n, int32_t *out);

/* Prompt in chunks (batched prefill): the same result as qh_slm_begin +
 * qh_slm_advance(n_prompt - 1) -- the same caches, bit for bit -- with the
 * projections of many prompt tokens as tensor-core GEMMs and the recurrence
 * and attention of a chunk in one launch per layer. The last prompt token is
 * left as the input of the next qh_slm_advance step (position n_prompt - 1);
 * the picks of the prompt positions are not computed. Needs head dim 128 and
 * conv kernel 4 (QH_ERR_UNSUPPORTED otherwise). Synchronous. */
int qh_slm_prefill(qh_slm *m, const int32_t *prompt, int32_t n_prompt);

/* qh_slm_prefill for a prompt that continues every sequence at position
 * pos (the caches of positions 0..pos-1 kept; pos == 0 starts afresh):
 * prompt[s][i] is the input of position pos + i, and the last prompt token
 * is left as the input of the next step (position pos + n_prompt - 1). In
 * QH_PREFILL_CHUNKED mode pos must be a multiple of 64 (the chunk grid);
 * QH_ERR_UNSUPPORTED otherwise. Synchronous. */
int qh_slm_prefill_at(qh_slm *m, const int32_t *prompt, int32_t n_prompt, int32_t pos);

/* Position of the next step (its input token is already set). */
int32_t qh_slm_position(const qh_slm *m);

/* Tokens per sequence in one prompt chunk (0 = the default: 8192 rows over
 * all sequences); only before the first qh_slm_prefill. */
int qh_slm_set_prefill_chunk(qh_slm *m, int32_t max_tokens_per_seq);

/* How qh_slm_prefill runs the Gated DeltaNet layers:
 *   QH_PREFILL_STEPWISE (default) -- the per-token recurrence, the same
 *     caches as feeding the prompt one token per step (slm_generate_raw's
 *     default prefill, slm/slm.c:280-287);
 *   QH_PREFILL_CHUNKED -- the reference's batched prefill taken under
 *     LLM_USE_FORWARD_BATCH (slm_forward_batch, slm/qwen.c:1018-1106): the
 *     64-token chunk algebra of chunked_ssm_step_f32 (slm/chunked.c:287),
 *     bit-identical to it, not to the per-token recurrence. Attention and
 *     FFN layers are the same in both. Chunks of 64 tokens count from
 *     position 0, so a prompt chunk (qh_slm_set_prefill_chunk) is rounded
 *     down to a multiple of 64 (at least 64) in this mode.
 * Only before the first qh_slm_prefill. */
#define QH_PREFILL_STEPWISE 0
#define QH_PREFILL_CHUNKED 1
int qh_slm_set_prefill_mode(qh_slm *m, int32_t mode);

/* How a decode step (qh_slm_step, qh_slm_advance, the generation loops)
 * runs, with bit-identical results either way:
 *   QH_DECODE_PERSISTENT (default) -- for one sequence whose projection
 *     weights are all K-quants: the step's operations as a few cooperative
 *     launches of one CTA per SM with grid-wide barriers between phases
 *     (qh_step_run, include/qh_kernels.h), the attention layers' cache
 *     kernels between them; weights stream ahead of the phase that reads
 *     them. Models that do not qualify (more sequences, Q8_0 or F32
 *     projections, an F32 embedding table) run QH_DECODE_LAUNCHES;
 *   QH_DECODE_LAUNCHES -- one launch per operation (norm, projection set,
 *     DeltaNet head update, attention, ...), captured in a CUDA graph.
 * A traced step (qh_slm_trace) always runs QH_DECODE_LAUNCHES. */
#define QH_DECODE_PERSISTENT 0
#define QH_DECODE_LAUNCHES 1
int qh_slm_set_decode_mode(qh_slm *m, int32_t mode);
/* The mode decode steps of m actually run (after the first step: a model
 * that does not qualify for QH_DECODE_PERSISTENT reports QH_DECODE_LAUNCHES). */
int32_t qh_slm_decode_mode(const qh_slm *m);
/* The persistent step's measurement hook (qh_step_set_stamps) for the next
 * steps of m: returns the number of phases P (d_stamps holds P records of
 * 8 + 2 * SM-count uint64), or QH_ERR_UNSUPPORTED when m does not run
 * QH_DECODE_PERSISTENT (after its first step). Replaces the captured step
 * graphs. */
int qh_slm_step_stamps(qh_slm *m, uint64_t *d_stamps);

/* Greedy generation, the per-step prefill path of slm_generate_raw
 * (slm/slm.c:237-357) for every sequence: the prompt runs through
 * qh_slm_prefill (the same caches as feeding one token per step) and the
 * pick of the last prompt step is the first of the n_new generated tokens; out[s][i] is the i-th generated token of sequence s.
 * slm_generate_raw re-feeds the last prompt token once more at position
 * n_prompt before its first sample; callers wanting that schedule pass the
 * prompt with its last token repeated. */
int qh_slm_generate(qh_slm *m, const int32_t *prompt, int32_t n_prompt, int32_t n_new, int32_t *out);

/* Sampled generation, slm_generate_raw (slm/slm.c:237-357) with the sampler
 * chain of qh_sampler.h, for every sequence at once; the whole loop stays on
 * the device (one captured step per token, the sample and the token feed
 * inside it). Starts each sequence afresh at position 0 (like qh_slm_begin):
 * prompt[s][0..n_prompt) at positions 0..n_prompt-1, then the decode loop
 * from position n_prompt, whose first input is the last prompt token again,
 * as in the reference. Per step: logits, eos_id/eot_id masked to -inf while
 * fewer than min_new tokens were generated, sample_with over the history
 * (this call's prompt plus the tokens generated so far) with the sequence's
 * generator. seeds[s] != 0 re-seeds sequence s (rng_seed); 0, or seeds ==
 * NULL, continues its generator (each starts seeded with s + 1). Up to
 * max_new tokens (fewer if the positions run out: the loop runs while the
 * position is below max_pos); a sequence ends at its first eos_id, eot_id
 * or stop_ids token, which is included. out[s][i] (row pitch max_new) for
 * i < n_out[s]; later entries are unspecified. n_prompt < max_pos. */
int qh_slm_generate_sampled(qh_slm *m, const int32_t *prompt, int32_t n_prompt, int32_t max_new, int32_t min_new,
                            const qh_sampler *sp, const uint64_t *seeds, int32_t eos_id, int32_t eot_id,
                            const int32_t *stop_ids, int32_t n_stop, int32_t *out, int32_t *n_out);

/* The sampled decode loop of qh_slm_generate_sampled in pieces, for a
 * caller that inspects every token (stop rules, streaming) and continues
 * sequences across calls as slm_generate_raw does (slm/slm.c:237-361):
 *   qh_slm_sample_setup  sampler, eos/eot masking for the first min_new
 *                        steps from the current position, the history
 *                        hist[s][0..n_hist) every sequence's penalty window
 *                        starts with, and seeds (as qh_slm_generate_sampled);
 *   qh_slm_sample_steps  n_steps sampled steps from the current position,
 *                        each fed the previous step's sample (after the
 *                        pending input); out[s][i] the sample of step i.
 * Synchronous. */
int qh_slm_sample_setup(qh_slm *m, const qh_sampler *sp, const uint64_t *seeds, int32_t eos_id, int32_t eot_id,
                        int32_t min_new, const int32_t *hist, int32_t n_hist);
int qh_slm_sample_steps(qh_slm *m, int32_t n_steps, int32_t *out);

/* Snapshot / restore of every sequence's decode state (slm_ctx_snapshot,
 * slm_ctx_restore, slm_snapshot_free; slm/model.c:1262-1371), held in device
 * memory: the position and pending input tokens, generator words, KV rows
 * 0..pos-1 of every attention layer (sized to the position, as the
 * reference's), the conv rings and recurrent states (full), plus prompts,
 * picks by position and the sampler history. qh_slm_restore puts them back
 * into the model they came from (QH_ERR_INVALID for another one); the next
 * step continues from the snapshot's position. Synchronous. */
typedef struct qh_slm_snap qh_slm_snap;
int qh_slm_snapshot(qh_slm *m, qh_slm_snap **out);
int qh_slm_restore(qh_slm *m, const qh_slm_snap *s);
void qh_slm_snapshot_free(qh_slm_snap *s);
/* Device bytes the snapshot holds; its position. -1 for NULL. */
int64_t qh_slm_snapshot_bytes(const qh_slm_snap *s);
int32_t qh_slm_snapshot_pos(const qh_slm_snap *s);

/* Parity tracer (slm_trace_open / slm_trace_f32, slm/model.c:585-727):
 * the next qh_slm_step writes one JSON line per traced tensor of sequence
 * `seq` to `path` (truncated), in the reference's schema and number
 * formatting (name, op, type, ne, nb, nbytes, fnv64 of the raw bytes, first
 * and last 8 values as %.9g and as fp32 hex, sum, n_nan, n_inf), so a line
 * is textually identical to the reference's line of the same name when the
 * tensor is bit-identical. Names follow the reference's (inp_embd,
 * attn_norm-L, attn_qkv-L, alpha-L, beta-L, V_raw-L, Q_l2norm-L, K_l2norm-L,
 * beta_in-L, attn_output-L, y_norm-L, ssm_out-L, Qfull-L, Kcur-L, Vcur-L,
 * attn_out-L, mix-L, mix_residual-L, ffn_norm-L, ffn_out-L, l_out-L,
 * result_norm, result_output); intermediates that the device never holds
 * (conv_raw, Q_raw, K_raw, a_softplus, g_in, conv_silu) are not written.
 * The traced step runs its kernels one by one (the Gated DeltaNet layers as
 * the unfused pre/recurrence/gated-norm chain, whose results are the same)
 * and synchronizes after each traced tensor; the file is closed when the
 * step ends. */
int qh_slm_trace(qh_slm *m, int32_t seq, const char *path);

/* The model's CUDA stream (cudaStream_t) and the device buffer of the last
 * greedy picks [n_seq], for callers that order their own work (events, a
 * token gather over NCCL) after qh_slm_advance. */
void *qh_slm_stream(const qh_slm *m);
const int32_t *qh_slm_device_next(const qh_slm *m);

/* Device memory held by the model (weights) and by the per-sequence state. */
int qh_slm_memory(const qh_slm *m, int64_t *weight_bytes, int64_t *state_bytes);

#ifdef __cplusplus
}
#endif

#endif /* QH_SLM_H */
