// SPDX-License-Identifier: MIT
//
// ref_harness.c -- exports the reference's own CPU code for the quantized
// matmul path (and its model forward step) from a shared library.
//
// TEST INFRASTRUCTURE, NOT PRODUCT CODE. oracle/Makefile compiles this file
// with the qwen.haiku sources on the include path (the reference is a
// single-translation-unit C17 program: slm/qwen.c pulls in model.c,
// tensor.c, simd/simd.c, simd/avx.c and simd/quants.h). No reference source
// is copied here; these are thin wrappers that reach the reference's static
// functions through that translation unit. Output: oracle/_ref/libqhref.so.
//
// Wrapped entry points:
//   simd_init / simd_dispatch_label            simd/simd.c:191-234
//   simd_q{4k,5k,6k}_row_dot_q8k, _q8_0_dot    simd/simd.c:236-250
//   q_scalar_*                                 simd/quants.h:244-402
//   quantize_row_q8_K                          slm/tensor.c:683-720
//   tensor_quantize_row_q8_0                   slm/tensor.c:930-950
//   matmul_dispatch                            slm/model.c:220-264
//   q{4k,5k,6k}_dequant_block                  slm/tensor.c:800, 867, 988
//   slm_forward_step + sample_argmax           slm/qwen.c:874-981, slm/model.c:401
//   sample_with, rng_seed, rng_uniform         slm/sampler.c:134, slm/model.c:431-447
//   slm_ctx_snapshot / restore / free           slm/model.c:1262-1371
//   JSONL tracer (g_qh_trace_fp, slm_trace_close) slm/model.c:585-727
//   slm_forward_batch (chunked prefill)          slm/qwen.c:1018-1106
//   chunked_ssm_step_f32                        slm/chunked.c:287-523

#include "slm/qwen.c"
#include "slm/sampler.c"

#include <pthread.h>

void ref_simd_init(void) { simd_init(); }
const char *ref_dispatch_label(void) { return simd_dispatch_label(); }

float ref_q4k_row_dot(int nb, const void *w, const void *y) {
    return simd_q4k_row_dot_q8k(nb, (const q4k_block *)w, (const q8k_block *)y);
}
float ref_q5k_row_dot(int nb, const void *w, const void *y) {
    return simd_q5k_row_dot_q8k(nb, (const q5k_block *)w, (const q8k_block *)y);
}
float ref_q6k_row_dot(int nb, const void *w, const void *y) {
    return simd_q6k_row_dot_q8k(nb, (const q6k_block *)w, (const q8k_block *)y);
}
float ref_q8_0_dot(const void *w, const void *y, int64_t k) {
    return simd_q8_0_dot_q8_0((const q8_0_block *)w, (const q8_0_block *)y, k);
}
float ref_scalar_q4k_row_dot(int nb, const void *w, const void *y) {
    return q_scalar_q4k_row_dot_q8k(nb, (const q4k_block *)w, (const q8k_block *)y);
}
float ref_scalar_q5k_row_dot(int nb, const void *w, const void *y) {
    return q_scalar_q5k_row_dot_q8k(nb, (const q5k_block *)w, (const q8k_block *)y);
}
float ref_scalar_q6k_row_dot(int nb, const void *w, const void *y) {
    return q_scalar_q6k_row_dot_q8k(nb, (const q6k_block *)w, (const q8k_block *)y);
}
float ref_scalar_q8_0_dot(const void *w, const void *y, int64_t k) {
    return q_scalar_q8_0_dot_q8_0((const q8_0_block *)w, (const q8_0_block *)y, k);
}

int ref_sizeof_q8k_block(void) { return (int)sizeof(q8k_block); }

// Activation quantizers exactly as the matmul wrappers call them.
void ref_quantize_row_q8k(const float *x, void *dst, int64_t k) {
    quantize_row_q8_K(x, (q8k_block *)dst, k);
}
void ref_quantize_row_q8_0(const float *x, void *dst, int64_t k) {
    tensor_quantize_row_q8_0(x, (q8_0_block *)dst, k);
}

void ref_dequant_block(int type, const void *blk, float *y) {
    switch (type) {
        case GGUF_TT_Q4_K: q4k_dequant_block((const q4k_block *)blk, y); break;
        case GGUF_TT_Q5_K: q5k_dequant_block((const q5k_block *)blk, y); break;
        case GGUF_TT_Q6_K: q6k_dequant_block((const q6k_block *)blk, y); break;
        default: break;
    }
}

// matmul_dispatch on a weight tensor of GGUF type `type`, shape (k, out_f);
// x is [n][k] fp32, out is [n][out_f] fp32. This is the reference's own
// single-threaded path (LLM_PAR_FOR is a plain loop off Apple).
int ref_matmul(int type, const void *w, int64_t out_f, int64_t k,
               const float *x, int64_t n, float *out) {
    simd_init();
    size_t need = (size_t)(k * n + out_f * n) * sizeof(float) + (size_t)k * 4 + (1u << 20);
    struct arena *a = arena_new(need);
    struct tensor *xt = tensor_new_2d(a, k, n);
    memcpy(xt->data, x, (size_t)(k * n) * sizeof(float));
    struct slm_tensor wt;
    memset(&wt, 0, sizeof(wt));
    wt.data = w;
    wt.type = type;
    wt.n_dims = 2;
    wt.shape[0] = k;
    wt.shape[1] = out_f;
    wt.shape[2] = wt.shape[3] = 1;
    int rc = -1;
    if (type == GGUF_TT_Q4_K || type == GGUF_TT_Q5_K || type == GGUF_TT_Q6_K ||
        type == GGUF_TT_Q8_0 || type == GGUF_TT_F32) {
        struct tensor *r = matmul_dispatch(&wt, xt);
        memcpy(out, r->data, (size_t)(out_f * n) * sizeof(float));
        rc = 0;
    }
    arena_free(a);
    return rc;
}

// ---------------------------------------------------------------------------
// All-cores CPU baseline: the reference's dispatched row dot, with the output
// rows split over `nthreads` pthreads (the reference's LLM_PAR_FOR runs rows
// sequentially on Linux; this harness only spreads the same calls over cores).
// `xq` is ONE pre-quantized activation row (q8k_block[k/256], or
// q8_0_block[k/32] for Q8_0). Rows [0, out_f) of matrix w.
// ---------------------------------------------------------------------------
struct mt_job {
    int type;
    const uint8_t *w;
    int64_t k, r0, r1, row_bytes;
    const void *xq;
    float *out;
};

static void *mt_worker(void *arg) {
    struct mt_job *j = (struct mt_job *)arg;
    const int nb = (int)(j->k / QK_K);
    for (int64_t r = j->r0; r < j->r1; r++) {
        const void *row = j->w + r * j->row_bytes;
        float v = 0.0f;
        switch (j->type) {
            case GGUF_TT_Q4_K: v = simd_q4k_row_dot_q8k(nb, row, j->xq); break;
            case GGUF_TT_Q5_K: v = simd_q5k_row_dot_q8k(nb, row, j->xq); break;
            case GGUF_TT_Q6_K: v = simd_q6k_row_dot_q8k(nb, row, j->xq); break;
            case GGUF_TT_Q8_0: v = simd_q8_0_dot_q8_0(row, j->xq, j->k); break;
            default: break;
        }
        j->out[r] = v;
    }
    return NULL;
}

int ref_matvec_mt(int type, const void *w, int64_t out_f, int64_t k,
                  const void *xq, float *out, int nthreads) {
    simd_init();
    int64_t row_bytes;
    switch (type) {
        case GGUF_TT_Q4_K: row_bytes = (k / QK_K) * 144; break;
        case GGUF_TT_Q5_K: row_bytes = (k / QK_K) * 176; break;
        case GGUF_TT_Q6_K: row_bytes = (k / QK_K) * 210; break;
        case GGUF_TT_Q8_0: row_bytes = (k / 32) * 34; break;
        default: return -1;
    }
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    struct mt_job jobs[256];
    int64_t per = (out_f + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        int64_t r0 = t * per, r1 = r0 + per < out_f ? r0 + per : out_f;
        if (r0 >= r1) break;
        jobs[t] = (struct mt_job){type, (const uint8_t *)w, k, r0, r1, row_bytes, xq, out};
        if (nthreads == 1) { mt_worker(&jobs[t]); started = 0; break; }
        pthread_create(&th[t], NULL, mt_worker, &jobs[t]);
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 0;
}

// Same as ref_matvec_mt over a pool of n_mats matrices (each out_f rows, one
// shared activation row): each thread walks its row range of every matrix,
// so threads are created once per pass instead of once per matrix.
struct pool_job {
    int type;
    const uint8_t *const *ws;
    int n_mats;
    int64_t k, r0, r1, row_bytes;
    const void *xq;
    float *out;
};

static void *pool_worker(void *arg) {
    struct pool_job *p = (struct pool_job *)arg;
    for (int m = 0; m < p->n_mats; m++) {
        struct mt_job j = {p->type, p->ws[m], p->k, p->r0, p->r1, p->row_bytes, p->xq, p->out};
        mt_worker(&j);
    }
    return NULL;
}

int ref_matvec_pool_mt(int type, const void *const *ws, int n_mats, int64_t out_f, int64_t k,
                       const void *xq, float *out, int nthreads) {
    simd_init();
    int64_t row_bytes;
    switch (type) {
        case GGUF_TT_Q4_K: row_bytes = (k / QK_K) * 144; break;
        case GGUF_TT_Q5_K: row_bytes = (k / QK_K) * 176; break;
        case GGUF_TT_Q6_K: row_bytes = (k / QK_K) * 210; break;
        case GGUF_TT_Q8_0: row_bytes = (k / 32) * 34; break;
        default: return -1;
    }
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    struct pool_job jobs[256];
    int64_t per = (out_f + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        int64_t r0 = t * per, r1 = r0 + per < out_f ? r0 + per : out_f;
        if (r0 >= r1) break;
        jobs[t] = (struct pool_job){type, (const uint8_t *const *)ws, n_mats, k, r0, r1, row_bytes, xq, out};
        pthread_create(&th[t], NULL, pool_worker, &jobs[t]);
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 0;
}

// ---------------------------------------------------------------------------
// Model level: the reference's own forward step over caller-provided weights.
// Builds struct slm_model / slm_ctx the way slm_model_load + slm_ctx_create
// do (slm/model.c:1130-1240, slm/qwen.c:59-252), but from an in-memory table
// of named tensors instead of a GGUF file, then runs slm_forward_step
// (slm/qwen.c:874) and sample_argmax (slm/model.c:401).
//
// ic[] = {n_layers, hidden, ffn, vocab, n_heads, n_kv_heads, head_dim,
//         rope_dim, sec0, sec1, sec2, sec3, gdn_heads, gdn_head_dim,
//         conv_kernel, full_attn_interval, max_pos}
// fc[] = {rope_theta, norm_eps}
// ---------------------------------------------------------------------------
struct ref_model {
    struct slm_model m;
    struct slm_ctx c;
};

static int ref_find(int n, const char **names, const char *want) {
    for (int i = 0; i < n; i++)
        if (strcmp(names[i], want) == 0) return i;
    return -1;
}

static void ref_bind(struct slm_tensor *t, int i, const int32_t *types, const int64_t *shapes,
                     const void **datas) {
    memset(t, 0, sizeof(*t));
    if (i < 0) return;
    t->data = datas[i];
    t->type = types[i];
    t->shape[0] = shapes[2 * i];
    t->shape[1] = shapes[2 * i + 1];
    t->shape[2] = t->shape[3] = 1;
    t->n_dims = t->shape[1] > 1 ? 2 : 1;
}

void *ref_model_create(const int32_t *ic, const float *fc, int n, const char **names,
                       const int32_t *types, const int64_t *shapes, const void **datas) {
    simd_init();
    struct ref_model *r = (struct ref_model *)calloc(1, sizeof(*r));
    struct slm_config *cfg = &r->m.cfg;
    cfg->n_layers = ic[0];
    cfg->hidden_dim = ic[1];
    cfg->ffn_dim = ic[2];
    cfg->vocab_size = ic[3];
    cfg->n_heads = ic[4];
    cfg->n_kv_heads = ic[5];
    cfg->head_dim = ic[6];
    cfg->rope_dim = ic[7];
    for (int i = 0; i < 4; i++) cfg->rope_sections[i] = ic[8 + i];
    cfg->linear_n_heads = ic[12];
    cfg->linear_k_head_dim = ic[13];
    cfg->linear_v_head_dim = ic[13];
    cfg->linear_conv_kernel = ic[14];
    cfg->full_attn_interval = ic[15];
    cfg->max_position = ic[16];
    cfg->rope_theta = fc[0];
    cfg->norm_eps = fc[1];
    cfg->is_hybrid = 1;
    cfg->attn_output_gate = 1;
    cfg->eot_id = -1;

    struct slm_weights *W = &r->m.W;
    char nm[96];
    ref_bind(&W->tok_embd, ref_find(n, names, "token_embd.weight"), types, shapes, datas);
    ref_bind(&W->output_norm, ref_find(n, names, "output_norm.weight"), types, shapes, datas);
    int out_i = ref_find(n, names, "output.weight");
    if (out_i >= 0) ref_bind(&W->output, out_i, types, shapes, datas);
    else W->output = W->tok_embd;
    W->layers = (struct slm_layer *)calloc((size_t)cfg->n_layers, sizeof(struct slm_layer));
    for (int L = 0; L < cfg->n_layers; L++) {
        struct slm_layer *Lw = &W->layers[L];
#define BIND(field, fmt) do { snprintf(nm, sizeof(nm), fmt, L); \
        ref_bind(&Lw->field, ref_find(n, names, nm), types, shapes, datas); } while (0)
        snprintf(nm, sizeof(nm), "blk.%d.ssm_a", L);
        Lw->is_ssm = ref_find(n, names, nm) >= 0;
        BIND(attn_norm, "blk.%d.attn_norm.weight");
        BIND(ffn_norm, "blk.%d.post_attention_norm.weight");
        BIND(ffn_gate, "blk.%d.ffn_gate.weight");
        BIND(ffn_up, "blk.%d.ffn_up.weight");
        BIND(ffn_down, "blk.%d.ffn_down.weight");
        if (Lw->is_ssm) {
            BIND(attn_qkv, "blk.%d.attn_qkv.weight");
            BIND(attn_gate, "blk.%d.attn_gate.weight");
            BIND(ssm_a, "blk.%d.ssm_a");
            BIND(ssm_alpha, "blk.%d.ssm_alpha.weight");
            BIND(ssm_beta, "blk.%d.ssm_beta.weight");
            BIND(ssm_conv1d, "blk.%d.ssm_conv1d.weight");
            BIND(ssm_dt_bias, "blk.%d.ssm_dt.bias");
            BIND(ssm_norm, "blk.%d.ssm_norm.weight");
            BIND(ssm_out, "blk.%d.ssm_out.weight");
        } else {
            BIND(attn_q, "blk.%d.attn_q.weight");
            BIND(attn_k, "blk.%d.attn_k.weight");
            BIND(attn_v, "blk.%d.attn_v.weight");
            BIND(attn_q_norm, "blk.%d.attn_q_norm.weight");
            BIND(attn_k_norm, "blk.%d.attn_k_norm.weight");
            BIND(attn_out, "blk.%d.attn_output.weight");
        }
#undef BIND
    }
    r->m.loaded = 1;
    r->c.model = &r->m;
    r->c.ctrl = slm_ctrl_defaults();
    kv_init(&r->c.kv, cfg->n_layers, cfg->n_kv_heads, cfg->head_dim, cfg->max_position);
    ssm_cache_init(&r->c.ssm, cfg);
    r->c.arena = arena_new(64 * 1024 * 1024);
    return r;
}

// One slm_forward_step; copies the logits out (if non-null) and returns
// sample_argmax of them.
int ref_model_step(void *h, int32_t tok, int32_t pos, float *logits) {
    struct ref_model *r = (struct ref_model *)h;
    struct tensor *lg = slm_forward_step(&r->c, tok, pos);
    if (logits) memcpy(logits, lg->data, (size_t)r->m.cfg.vocab_size * sizeof(float));
    return sample_argmax(lg);
}

// The reference's own GGUF path: gguf_open (slm/gguf.c:172), slm_load_config
// (slm/qwen.c:59) and slm_load_weights (slm/qwen.c:174) on a file, then the
// caches as above. ic/fc receive the config in ref_model_create's order.
// NULL if any step fails.
void *ref_model_from_gguf(const char *path, int32_t *ic, float *fc) {
    simd_init();
    struct ref_model *r = (struct ref_model *)calloc(1, sizeof(*r));
    if (gguf_open(&r->m.gguf, path) != 0) { free(r); return NULL; }
    struct slm_config *cfg = &r->m.cfg;
    if (slm_load_config(&r->m.gguf, cfg) != 0 || slm_load_weights(&r->m.gguf, cfg, &r->m.W) != 0) {
        gguf_close(&r->m.gguf);
        free(r->m.W.layers);
        free(r);
        return NULL;
    }
    ic[0] = cfg->n_layers; ic[1] = cfg->hidden_dim; ic[2] = cfg->ffn_dim; ic[3] = cfg->vocab_size;
    ic[4] = cfg->n_heads; ic[5] = cfg->n_kv_heads; ic[6] = cfg->head_dim; ic[7] = cfg->rope_dim;
    for (int i = 0; i < 4; i++) ic[8 + i] = cfg->rope_sections[i];
    ic[12] = cfg->linear_n_heads; ic[13] = cfg->linear_k_head_dim; ic[14] = cfg->linear_conv_kernel;
    ic[15] = cfg->full_attn_interval; ic[16] = cfg->max_position;
    fc[0] = cfg->rope_theta; fc[1] = cfg->norm_eps;
    r->m.loaded = 1;
    r->c.model = &r->m;
    r->c.ctrl = slm_ctrl_defaults();
    kv_init(&r->c.kv, cfg->n_layers, cfg->n_kv_heads, cfg->head_dim, cfg->max_position);
    ssm_cache_init(&r->c.ssm, cfg);
    r->c.arena = arena_new(64 * 1024 * 1024);
    return r;
}

void ref_model_destroy(void *h) {
    struct ref_model *r = (struct ref_model *)h;
    if (!r) return;
    if (r->m.gguf.base) gguf_close(&r->m.gguf);
    ssm_cache_free(&r->c.ssm);
    kv_free(&r->c.kv);
    arena_free(r->c.arena);
    free(r->m.W.layers);
    free(r);
}

// The sampler chain, sample_with (slm/sampler.c:134-180), on caller
// logits (modified in place as the reference does). fp = {temperature,
// top_p, min_p, repetition_penalty}, ip = {top_k, repetition_window}; st =
// the generator's two words, advanced in place.
int32_t ref_sample_with(float *logits, int64_t n, const float *fp, const int32_t *ip, uint64_t *st,
                        const int32_t *hist, int32_t hist_n) {
    struct tensor t;
    memset(&t, 0, sizeof(t));
    t.ne[0] = n;
    t.ne[1] = t.ne[2] = t.ne[3] = 1;
    t.ndim = 1;
    t.data = logits;
    struct slm_sampler sp;
    sp.temperature = fp[0];
    sp.top_p = fp[1];
    sp.min_p = fp[2];
    sp.repetition_penalty = fp[3];
    sp.top_k = ip[0];
    sp.repetition_window = ip[1];
    struct rng r = {st[0], st[1]};
    int32_t pick = sample_with(&t, &sp, &r, hist, hist_n);
    st[0] = r.s0;
    st[1] = r.s1;
    return pick;
}

// rng_seed (slm/model.c:431) into st[2].
void ref_rng_seed(uint64_t seed, uint64_t *st) {
    struct rng r;
    rng_seed(&r, seed);
    st[0] = r.s0;
    st[1] = r.s1;
}

// slm_sampler_defaults (slm/sampler.c:22): fp/ip in ref_sample_with's order.
void ref_sampler_defaults(float *fp, int32_t *ip) {
    struct slm_sampler s = slm_sampler_defaults();
    fp[0] = s.temperature;
    fp[1] = s.top_p;
    fp[2] = s.min_p;
    fp[3] = s.repetition_penalty;
    ip[0] = s.top_k;
    ip[1] = s.repetition_window;
}

// slm_ctx_snapshot / slm_ctx_restore / slm_snapshot_free (slm/model.c:
// 1262-1371) on a ref_model's context; pos = the context's position (the
// number of KV rows written), which ref_model_step does not track itself.
void *ref_model_snapshot(void *h, int32_t pos) {
    struct ref_model *r = (struct ref_model *)h;
    r->c.pos = pos;
    return slm_ctx_snapshot(&r->c);
}
void ref_model_restore(void *h, void *snap) {
    struct ref_model *r = (struct ref_model *)h;
    slm_ctx_restore(&r->c, (const struct slm_snapshot *)snap);
}
void ref_snapshot_free(void *snap) { slm_snapshot_free((struct slm_snapshot *)snap); }

// The reference's JSONL parity tracer (slm/model.c:585-727): records of
// the forward steps run between ref_trace_begin and ref_trace_end go to
// `path` (slm_trace_open reads the path from QH_TRACE_OUT; this sets the
// same file handle directly).
int ref_trace_begin(const char *path) {
    if (g_qh_trace_fp) fclose(g_qh_trace_fp);
    g_qh_trace_fp = fopen(path, "w");
    return g_qh_trace_fp ? 0 : -1;
}
void ref_trace_end(void) { slm_trace_close(); }

// The batched prefill the reference runs under LLM_USE_FORWARD_BATCH
// (slm/slm.c:274-283): slm_forward_batch (slm/qwen.c:1018-1106) over n
// tokens at positions pos_start.. -- chunked Gated DeltaNet layers
// (slm_forward_ssm_batch, slm/qwen.c:627-806) and batched attention
// (slm_forward_attn_batch, slm/model.c:955-1120). Copies the last token's
// logits out (if non-null) and returns their sample_argmax.
int ref_model_forward_batch(void *h, const int32_t *toks, int32_t n, int32_t pos_start, float *logits) {
    struct ref_model *r = (struct ref_model *)h;
    struct tensor *lg = slm_forward_batch(&r->c, toks, n, pos_start);
    if (logits) memcpy(logits, lg->data, (size_t)r->m.cfg.vocab_size * sizeof(float));
    return sample_argmax(lg);
}

// One chunked_ssm_step_f32 (slm/chunked.c:287-523) on caller arrays: n
// (<= 64) tokens of one head, state [k_hd][v_hd] updated in place, out
// [n][v_hd]. The kernel's scratch is allocated here.
int ref_chunked_step(int32_t n, int32_t k_hd, int32_t v_hd, const float *q, const float *k, const float *v,
                     const float *g_log, const float *beta, float *state, float *out) {
    if (n < 1 || n > CHUNK_SIZE) return -1;
    const size_t C = CHUNK_SIZE, kd = (size_t)k_hd, vd = (size_t)v_hd;
    const size_t sizes[19] = {C, C, C * C, C * kd, C * vd, C * C, C * C, C * C, C * vd, C * kd,
                              C * kd, C * C, C * kd, C * vd, C * vd, C * vd, C * vd, C * kd, kd * vd};
    float *s[19];
    int ok = 1;
    for (int i = 0; i < 19; i++) {
        s[i] = (float *)calloc(sizes[i] > C * C ? sizes[i] : C * C, sizeof(float));
        ok &= s[i] != NULL;
    }
    if (ok)
        chunked_ssm_step_f32(n, k_hd, v_hd, q, k, v, g_log, beta, state, out, s[0], s[1], s[2], s[3], s[4], s[5],
                             s[6], s[7], s[8], s[9], s[10], s[11], s[12], s[13], s[14], s[15], s[16], s[17], s[18]);
    for (int i = 0; i < 19; i++) free(s[i]);
    return ok ? 0 : -1;
}

// Accessors for a matmul backend that replaces the reference's
// tensor_matmul_* entry points from another shared library (oracle/
// ref_dropin.c): the fields of a struct tensor it needs, and a new 2-D
// tensor in a given tensor's arena (tensor_new_2d, slm/tensor.c:251), so the
// backend never depends on the struct's layout.
float *ref_tensor_data(const struct tensor *t) { return t->data; }
int64_t ref_tensor_ne(const struct tensor *t, int i) { return t->ne[i]; }
struct tensor *ref_tensor_new_like(const struct tensor *t, int64_t n0, int64_t n1) {
    return tensor_new_2d(t->arena, n0, n1);
}
