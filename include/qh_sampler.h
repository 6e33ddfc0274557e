/* SPDX-License-Identifier: MIT
 *
 * qh_sampler.h -- the reference's sampler chain on B200 (sm_100a), one CTA
 * per sequence, so sampled decoding stays on the device like the greedy
 * pick does.
 *
 * Reference counterparts (qwen.haiku, path:line):
 *   struct slm_sampler                       slm/slm.h:117-124
 *   slm_sampler_defaults                     slm/sampler.c:22-31
 *   struct rng, rng_next, rng_seed,
 *   rng_uniform                              slm/model.c:414-447
 *   sample_with (the chain)                  slm/sampler.c:134-180
 *     apply_rep_penalty                      slm/sampler.c:49-63
 *     topk_collect                           slm/sampler.c:70-93
 *     topk_softmax                           slm/sampler.c:97-112
 *     topk_sort_desc                         slm/sampler.c:117-130
 *   sample_argmax (temperature <= 0)         slm/model.c:401-412
 *
 * The chain is reproduced step for step, so the pick equals the
 * reference's for the same logits, history and generator state: the
 * penalty is applied once per occurrence of a token in the window; the
 * top-k candidates keep the slot order of the reference's replace-the-
 * first-minimum scan (the softmax sum runs over that order); the
 * descending sort is stable; the nucleus, min-p and roulette sums are
 * sequential float sums. The exponential is evaluated in double precision
 * and rounded once to float (a correctly rounded expf).
 */
#ifndef QH_SAMPLER_H
#define QH_SAMPLER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* struct slm_sampler (slm/slm.h:117-124), same fields and meaning. */
typedef struct qh_sampler {
    float temperature;         /* <= 0: greedy argmax of the penalized logits */
    int32_t top_k;             /* <= 0 or > 256: 256 candidates */
    float top_p;               /* nucleus cut, effective in (0, 1) */
    float min_p;               /* > 0: drop candidates below min_p * top probability */
    float repetition_penalty;  /* 1 = off */
    int32_t repetition_window; /* <= 0: the whole history; > 0: its last N tokens */
} qh_sampler;

/* Largest candidate set of the chain (SLM_SAMPLE_TOPK_MAX, slm/sampler.c:68). */
#define QH_SAMPLE_TOPK_MAX 256

/* slm_sampler_defaults (slm/sampler.c:22-31): T 0.7, top-k 40, top-p 0.9,
 * min-p 0.05, penalty 1.25 over the last 64 tokens. */
void qh_sampler_defaults(qh_sampler *s);

/* rng_seed (slm/model.c:431-442): SplitMix64 expansion of a 64-bit seed
 * into the generator's two words. Host-side; the state is what the device
 * generator (rng_next, slm/model.c:420-428) advances. */
void qh_rng_seed(uint64_t seed, uint64_t state[2]);

/* sample_with (slm/sampler.c:134-180) for B rows at once:
 *   d_logits [B][vocab] fp32 -- modified in place by the repetition
 *                               penalty, as the reference does;
 *   d_hist [B][hist_stride], d_hist_n [B] -- each row's token history
 *                               (prompt + generated so far);
 *   d_rng [B][2] u64          -- generator state, advanced by one draw per
 *                               row when temperature > 0;
 *   d_out [B]                 -- the picks.
 * Asynchronous on `stream`. Returns QH_OK or QH_ERR_INVALID. */
int qh_sample(const qh_sampler *sp, float *d_logits, int32_t B, int64_t vocab, const int32_t *d_hist,
              int32_t hist_stride, const int32_t *d_hist_n, uint64_t *d_rng, int32_t *d_out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* QH_SAMPLER_H */
