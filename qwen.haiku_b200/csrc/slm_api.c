// SPDX-License-Identifier: MIT
//
// slm_api.c -- the reference's slm.h entry points (include/slm.h) over the
// device model of qh_slm.h: a model is a GGUF read into a host blob plus its
// special token ids; a context is a one-sequence qh_slm (weights, KV cache,
// conv ring and recurrent state on the current device) with the position,
// token history, ctrl and timing the reference keeps on its slm_ctx
// (slm/model.c:1209-1260, slm/slm.c:237-361, 858-892).

#define _POSIX_C_SOURCE 200809L  // clock_gettime under -std=c17

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "qh_backend.h"
#include "qh_gguf.h"
#include "qh_sampler.h"
#include "qh_slm.h"
#include "slm.h"

struct slm_model {
    int loaded;
    char err[256];
    qh_slm_config cfg;
    qh_blob *blob;
    qh_special_tokens tok;
};

struct slm_ctx {
    struct slm_model *model;
    qh_slm *m;
    int32_t pos;  // position of the next token to process
    struct slm_ctrl ctrl;
    int32_t *ids;
    int32_t n_ids, cap_ids;
    double t_prefill_s, t_gen_s;
    int32_t n_prefill, n_generated;
};

struct slm_snapshot {
    const struct slm_ctx *owner;
    qh_slm_snap *snap;
    int32_t pos, n_ids;
};

static double seconds(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

struct slm_model *slm_model_load(const char *path) {
    struct slm_model *m = (struct slm_model *)calloc(1, sizeof(*m));
    if (!m) return NULL;
    int rc = path ? qh_gguf_load(path, 0, &m->cfg, &m->blob) : QH_ERR_INVALID;
    if (!rc) rc = qh_gguf_special_tokens(path, &m->tok);
    if (rc) {
        snprintf(m->err, sizeof(m->err), "cannot load %s (status %d: %s)", path ? path : "(null)", rc,
                 rc == QH_ERR_UNSUPPORTED ? "unsupported architecture or tensor type" : "malformed or unreadable");
        if (m->blob) qh_blob_free(m->blob);
        m->blob = NULL;
        return m;
    }
    m->loaded = 1;
    return m;
}

void slm_model_unload(struct slm_model *m) {
    if (!m) return;
    if (m->blob) qh_blob_free(m->blob);
    free(m);
}

bool slm_model_loaded(const struct slm_model *m) { return m && m->loaded; }

const char *slm_model_error(const struct slm_model *m) { return !m ? "no model" : m->loaded ? NULL : m->err; }

struct slm_sampler slm_sampler_defaults(void) {
    qh_sampler q;
    qh_sampler_defaults(&q);
    struct slm_sampler s = {q.temperature, q.top_k, q.top_p, q.min_p, q.repetition_penalty, q.repetition_window};
    return s;
}

struct slm_ctrl slm_ctrl_defaults(void) {
    struct slm_ctrl c = {true, false, NULL, 1, false, -1};
    return c;
}

struct slm_ctx *slm_ctx_create(struct slm_model *model) {
    if (!slm_model_loaded(model)) return NULL;
    struct slm_ctx *c = (struct slm_ctx *)calloc(1, sizeof(*c));
    if (!c) return NULL;
    c->model = model;
    c->ctrl = slm_ctrl_defaults();
    if (qh_slm_create(&model->cfg, model->blob, 1, &c->m)) {
        free(c);
        return NULL;
    }
    return c;
}

void slm_ctx_destroy(struct slm_ctx *c) {
    if (!c) return;
    qh_slm_destroy(c->m);
    free(c->ids);
    free(c);
}

struct slm_ctrl *slm_ctx_ctrl(struct slm_ctx *c) { return &c->ctrl; }

static int push_id(struct slm_ctx *c, int32_t id) {
    if (c->n_ids == c->cap_ids) {
        const int32_t cap = c->cap_ids ? 2 * c->cap_ids : 256;
        int32_t *p = (int32_t *)realloc(c->ids, sizeof(int32_t) * (size_t)cap);
        if (!p) return -1;
        c->ids = p;
        c->cap_ids = cap;
    }
    c->ids[c->n_ids++] = id;
    return 0;
}

static int is_stop(const struct slm_model *m, int32_t t) {
    if (t == m->tok.eos_id || t == m->tok.eot_id) return 1;
    for (int32_t i = 0; i < m->tok.n_stop; ++i)
        if (t == m->tok.stop_ids[i]) return 1;
    return 0;
}

int slm_generate_ids(struct slm_ctx *c, const int32_t *prompt_ids, int prompt_n, int max_new, int min_new,
                     const struct slm_sampler *sampler, uint64_t seed, slm_token_fn cb, void *user) {
    if (!c || prompt_n < 0 || (prompt_n > 0 && !prompt_ids) || max_new < 0) return -1;
    const struct slm_model *model = c->model;
    const int32_t P = model->cfg.max_pos, pos = c->pos;
    if (pos + prompt_n > P) return -1;
    qh_sampler sp;
    memset(&sp, 0, sizeof(sp));
    if (sampler) {
        sp.temperature = sampler->temperature;
        sp.top_k = sampler->top_k;
        sp.top_p = sampler->top_p;
        sp.min_p = sampler->min_p;
        sp.repetition_penalty = sampler->repetition_penalty;
        sp.repetition_window = sampler->repetition_window;
    }
    const double t0 = seconds();
    // prefill: the prompt at pos..pos+n-1; the decode loop then feeds the
    // last prompt token (bos without a prompt) once more at pos+n
    const int32_t last = prompt_n > 0 ? prompt_ids[prompt_n - 1] : model->tok.bos_id;
    int32_t *ext = (int32_t *)malloc(sizeof(int32_t) * (size_t)(prompt_n + 1));
    if (!ext) return -1;
    if (prompt_n > 0) memcpy(ext, prompt_ids, sizeof(int32_t) * (size_t)prompt_n);
    ext[prompt_n] = last;
    int rc;
    const int decode = pos + prompt_n < P;  // the loop runs while pos < max_position
    if (decode)
        rc = qh_slm_prefill_at(c->m, ext, prompt_n + 1, pos);
    else  // no room to decode: just the prompt, its last token processed too
        rc = qh_slm_prefill_at(c->m, ext, prompt_n, pos) ? -1 : qh_slm_advance(c->m, 1);
    for (int i = 0; i < prompt_n && !rc; ++i) rc = push_id(c, prompt_ids[i]);
    free(ext);
    if (rc) return -1;
    const double t1 = seconds();
    c->t_prefill_s = t1 - t0;
    c->n_prefill = prompt_n;
    int32_t p = pos + prompt_n, generated = 0;
    if (decode) {
        if (qh_slm_sample_setup(c->m, &sp, seed ? &seed : NULL, model->tok.eos_id, model->tok.eot_id, min_new,
                                prompt_ids, prompt_n))
            return -1;
        int stop = 0;
        while (!stop && generated < max_new && p < P) {
            int32_t next;
            if (qh_slm_sample_steps(c->m, 1, &next)) return -1;
            p++;
            generated++;
            if (push_id(c, next)) return -1;
            if (c->ctrl.trace_tokens) fprintf(stderr, "[tok] %d\n", (int)next);
            if (is_stop(model, next))
                stop = 1;
            else if (cb && cb(next, user) != 0)
                stop = 1;
        }
    }
    c->t_gen_s = seconds() - t1;
    c->n_generated = generated;
    c->pos = p;
    return generated;
}

struct slm_snapshot *slm_ctx_snapshot(const struct slm_ctx *c) {
    if (!c) return NULL;
    struct slm_snapshot *s = (struct slm_snapshot *)calloc(1, sizeof(*s));
    if (!s) return NULL;
    if (qh_slm_snapshot(c->m, &s->snap)) {
        free(s);
        return NULL;
    }
    s->owner = c;
    s->pos = c->pos;
    s->n_ids = c->n_ids;
    return s;
}

void slm_ctx_restore(struct slm_ctx *c, const struct slm_snapshot *s) {
    if (!c || !s || s->owner != c) return;
    if (qh_slm_restore(c->m, s->snap)) return;
    c->pos = s->pos;
    if (s->n_ids < c->n_ids) c->n_ids = s->n_ids;
}

void slm_snapshot_free(struct slm_snapshot *s) {
    if (!s) return;
    qh_slm_snapshot_free(s->snap);
    free(s);
}

const int32_t *slm_ctx_tokens(const struct slm_ctx *c, int32_t *out_n) {
    const int32_t *p = NULL;
    int32_t n = 0;
    if (c && c->n_ids > 0) {
        p = c->ids;
        n = c->n_ids;
    }
    if (out_n) *out_n = n;
    return p;
}

int slm_vocab_size(const struct slm_ctx *c) { return c->model->cfg.vocab; }
int slm_eos_id(const struct slm_ctx *c) { return c->model->tok.eos_id; }
int slm_bos_id(const struct slm_ctx *c) { return c->model->tok.bos_id; }

double slm_pp_per_sec(const struct slm_ctx *c) {
    return c && c->t_prefill_s > 0.0 ? (double)c->n_prefill / c->t_prefill_s : 0.0;
}

double slm_tg_per_sec(const struct slm_ctx *c) {
    return c && c->t_gen_s > 0.0 ? (double)c->n_generated / c->t_gen_s : 0.0;
}

int32_t slm_n_prefill(const struct slm_ctx *c) { return c ? c->n_prefill : 0; }
int32_t slm_n_generated(const struct slm_ctx *c) { return c ? c->n_generated : 0; }
