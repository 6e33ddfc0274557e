/* SPDX-License-Identifier: MIT
 *
 * slm.h -- the reference's public C API (slm/slm.h of qwen.haiku) for the
 * parts that drive the model: load a GGUF, create per-conversation contexts,
 * generate over token ids, snapshot / restore, sampler and ctrl defaults,
 * history and timing accessors. Same names, signatures and meaning as the
 * reference's declarations (cited per function); implemented over the
 * device model of qh_slm.h (csrc/slm_api.c), so a caller of these functions
 * relinks against libqh200.so unchanged.
 *
 * Not declared here: the text-level functions (slm_tokenize,
 * slm_ctx_system_prompt, slm_generate with a text prompt, the chat template
 * and message history, slm/slm.h:258-330), which need the reference's
 * tokenizer, chat framing and tool agent -- outside this library. A caller
 * tokenizes and frames the conversation itself and passes token ids to
 * slm_generate_ids, the token-level loop the reference's slm_generate runs
 * internally (slm_generate_raw, slm/slm.c:237-361).
 *
 * Thread-safety as the reference's: one slm_ctx per thread; the model is
 * read-only after load and may be shared by many contexts. Every context
 * holds its own device copy of the weights and its caches on the current
 * CUDA device.
 */
#ifndef SLM_H
#define SLM_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct slm_model;
struct slm_ctx;
struct slm_snapshot;

/* slm/slm.h:59-62. Reads the GGUF (qwen35 architecture; weight types F32,
 * Q8_0, Q4_K, Q5_K, Q6_K). Returns non-NULL even on failure; check
 * slm_model_loaded() / slm_model_error(). */
struct slm_model *slm_model_load(const char *path);
void slm_model_unload(struct slm_model *model);
bool slm_model_loaded(const struct slm_model *model);
const char *slm_model_error(const struct slm_model *model);

/* slm/slm.h:69-70. A fresh context (KV cache, conv ring, recurrent state on
 * the device; position 0). NULL if the model is not loaded or the device
 * model cannot be created. Its generator starts seeded with 1. */
struct slm_ctx *slm_ctx_create(struct slm_model *model);
void slm_ctx_destroy(struct slm_ctx *ctx);

/* slm/slm.h:98-109. The context's mutable state at this moment (position,
 * KV rows 0..pos-1, conv ring, recurrent state, generator, token count),
 * held in device memory. Restore puts it back into the context it came from
 * (a snapshot of another context is ignored); tokens past the saved count
 * are dropped from slm_ctx_tokens. */
struct slm_snapshot *slm_ctx_snapshot(const struct slm_ctx *ctx);
void slm_ctx_restore(struct slm_ctx *ctx, const struct slm_snapshot *snap);
void slm_snapshot_free(struct slm_snapshot *snap);

/* slm/slm.h:117-128. Zero-initialized = greedy. */
struct slm_sampler {
    float temperature;
    int top_k;
    float top_p;
    float min_p;
    float repetition_penalty;
    int repetition_window;
};
/* T=0.7, top_k=40, top_p=0.9, min_p=0.05, rep=1.25, win=64. */
struct slm_sampler slm_sampler_defaults(void);

/* slm/slm.h:135-142, 194-199. tools / think / effort / dump_layer belong to
 * the text layer and are kept only for layout; trace_tokens makes
 * slm_generate_ids print "[tok] <id>" per sampled token to stderr, as the
 * reference's generation loop does. */
struct slm_ctrl {
    bool tools;
    bool think;
    const char *effort;
    int32_t debug;
    bool trace_tokens;
    int32_t dump_layer;
};
struct slm_ctrl slm_ctrl_defaults(void);
struct slm_ctrl *slm_ctx_ctrl(struct slm_ctx *ctx);

/* Per-token callback of slm_generate_ids: the sampled token id (not a stop
 * token); return non-zero to stop. */
typedef int (*slm_token_fn)(int32_t token, void *user);

/* The reference's generation loop over token ids (slm_generate_raw,
 * slm/slm.c:237-361, which slm_generate runs after tokenizing): the prompt
 * ids at the context's positions pos..pos+n-1, then a decode loop that
 * re-feeds the last prompt token (bos when prompt_n == 0) and samples with
 * sample_with over the history (this call's prompt plus the tokens sampled
 * so far), eos/eot masked while fewer than min_new tokens were generated,
 * until max_new tokens, the end of the context, a stop token (eos, eot or
 * the model's end-of-generation set; counted, not passed to cb) or cb
 * returning non-zero. sampler NULL = greedy ({0}); seed != 0 re-seeds the
 * context's generator, 0 continues it. The context continues at the
 * returned position on the next call. Returns the number of tokens
 * generated, or -1 on an error. */
int slm_generate_ids(struct slm_ctx *ctx, const int32_t *prompt_ids, int prompt_n, int max_new, int min_new,
                     const struct slm_sampler *sampler, uint64_t seed, slm_token_fn cb, void *user);

/* slm/slm.h:315. Every token id prefilled or generated since ctx_create. */
const int32_t *slm_ctx_tokens(const struct slm_ctx *ctx, int32_t *out_n);

/* slm/slm.h:331-339. */
int slm_vocab_size(const struct slm_ctx *ctx);
int slm_eos_id(const struct slm_ctx *ctx);
int slm_bos_id(const struct slm_ctx *ctx);
double slm_pp_per_sec(const struct slm_ctx *ctx);
double slm_tg_per_sec(const struct slm_ctx *ctx);
int32_t slm_n_prefill(const struct slm_ctx *ctx);
int32_t slm_n_generated(const struct slm_ctx *ctx);

#ifdef __cplusplus
}
#endif

#endif /* SLM_H */
