// SPDX-License-Identifier: MIT
//
// qh_synth_model.c -- seeded synthetic weights for the Qwen3.5-0.8B-shaped
// hybrid model (include/qh_slm.h), held in a host blob of named tensors.
//
// Tensor names, types and shapes are the GGUF ones the reference resolves in
// slm_load_weights (slm/qwen.c:174-252): GDN layers carry attn_qkv,
// attn_gate, ssm_{a,alpha,beta,conv1d,dt.bias,norm,out}; every
// full_attn_interval-th layer carries attn_{q,k,v,output,q_norm,k_norm};
// all layers carry attn_norm, post_attention_norm and the SwiGLU FFN;
// output.weight is absent, so the LM head is the tied token_embd
// (slm/qwen.c:181-183). Every tensor draws from its own stream (seed mixed
// with a hash of its name), so the bytes do not depend on generation order;
// large matrices are generated and quantized on all host cores.

#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "qh_backend.h"
#include "qh_formats.h"
#include "qh_slm.h"
#include "qh_synth.h"

typedef struct {
    char name[64];
    int32_t type;
    int64_t shape[2];
    int64_t nbytes;
    void *data;
} blob_tensor;

struct qh_blob {
    int count, cap;
    blob_tensor *t;
};

void qh_slm_config_default(qh_slm_config *c, int32_t max_pos) {
    memset(c, 0, sizeof(*c));
    c->n_layers = 24;
    c->hidden = 1024;
    c->ffn = 3584;
    c->vocab = 151936;
    c->n_heads = 8;
    c->n_kv_heads = 2;
    c->head_dim = 128;
    c->rope_dim = 64;
    c->rope_theta = 1e6f;
    c->rope_sections[0] = 11;
    c->rope_sections[1] = 11;
    c->rope_sections[2] = 10;
    c->rope_sections[3] = 0;
    c->norm_eps = 1e-6f;
    c->gdn_heads = 16;
    c->gdn_head_dim = 128;
    c->conv_kernel = 4;
    c->full_attn_interval = 4;
    c->max_pos = max_pos;
}

static uint64_t name_hash(const char *s) {
    uint64_t h = 1469598103934665603ull;  // FNV-1a
    for (; *s; ++s) h = (h ^ (uint8_t)*s) * 1099511628211ull;
    return h;
}

static blob_tensor *blob_add(qh_blob *b, const char *name, int32_t type, int64_t s0, int64_t s1) {
    if (b->count == b->cap) {
        int cap = b->cap ? 2 * b->cap : 64;
        blob_tensor *t = (blob_tensor *)realloc(b->t, sizeof(blob_tensor) * cap);
        if (!t) return NULL;
        b->t = t;
        b->cap = cap;
    }
    blob_tensor *t = &b->t[b->count];
    memset(t, 0, sizeof(*t));
    snprintf(t->name, sizeof(t->name), "%s", name);
    t->type = type;
    t->shape[0] = s0;
    t->shape[1] = s1;
    t->nbytes = type == QH_GGUF_F32 ? s0 * s1 * 4 : qhf_row_bytes(type, s0) * s1;
    t->data = malloc((size_t)t->nbytes);
    if (!t->data) return NULL;
    b->count++;
    return t;
}

// ---- quantized matrices, rows split over threads ----
typedef struct {
    int32_t type;
    int64_t k, r0, r1;
    uint64_t seed;
    float std_dev;
    uint8_t *out;
    int rc;
} qjob;

static void *qjob_run(void *arg) {
    qjob *j = (qjob *)arg;
    const int64_t chunk = 256;
    float *w = (float *)malloc(sizeof(float) * chunk * j->k);
    if (!w) { j->rc = QH_ERR_INVALID; return NULL; }
    const int64_t rb = qhf_row_bytes(j->type, j->k);
    for (int64_t r = j->r0; r < j->r1; r += chunk) {
        const int64_t n = (j->r1 - r) < chunk ? (j->r1 - r) : chunk;
        // row r draws values r*k .. of the tensor's stream
        for (int64_t i = 0; i < n; ++i) {
            int rc = qh_synth_normal(j->seed + (uint64_t)(r + i) * 0x632BE59BD9B4E019ull, j->k, 0.0f,
                                     j->std_dev, w + i * j->k);
            if (rc) { j->rc = rc; free(w); return NULL; }
        }
        int rc = qh_synth_quantize(j->type, w, n, j->k, j->out + r * rb);
        if (rc) { j->rc = rc; free(w); return NULL; }
    }
    free(w);
    return NULL;
}

static int fill_matrix(blob_tensor *t, uint64_t seed, float std_dev) {
    const int64_t rows = t->shape[1], k = t->shape[0];
    long ncpu = sysconf(_SC_NPROCESSORS_ONLN);
    int nth = (int)(ncpu < 1 ? 1 : (ncpu > 64 ? 64 : ncpu));
    if (rows < 512) nth = 1;
    pthread_t th[64];
    qjob jobs[64];
    const int64_t per = (rows + nth - 1) / nth;
    int started = 0;
    for (int i = 0; i < nth; ++i) {
        const int64_t r0 = i * per, r1 = r0 + per < rows ? r0 + per : rows;
        if (r0 >= r1) break;
        jobs[i] = (qjob){t->type, k, r0, r1, seed, std_dev, (uint8_t *)t->data, 0};
        if (nth == 1) {
            qjob_run(&jobs[i]);
            started = 1;
            break;
        }
        pthread_create(&th[i], NULL, qjob_run, &jobs[i]);
        started++;
    }
    int rc = 0;
    for (int i = 0; i < started; ++i) {
        if (nth > 1) pthread_join(th[i], NULL);
        if (jobs[i].rc) rc = jobs[i].rc;
    }
    return rc;
}

static int add_matrix(qh_blob *b, uint64_t seed, const char *name, int32_t type, int64_t k, int64_t n) {
    blob_tensor *t = blob_add(b, name, type, k, n);
    if (!t) return QH_ERR_INVALID;
    return fill_matrix(t, seed ^ name_hash(name), 0.02f);
}

enum vec_kind { VEC_NORM, VEC_NEG_EXP, VEC_NORMAL };

static int add_vector(qh_blob *b, uint64_t seed, const char *name, int64_t s0, int64_t s1, int kind,
                      float std_dev) {
    blob_tensor *t = blob_add(b, name, QH_GGUF_F32, s0, s1);
    if (!t) return QH_ERR_INVALID;
    float *v = (float *)t->data;
    const int64_t n = s0 * s1;
    int rc = qh_synth_normal(seed ^ name_hash(name), n, 0.0f, std_dev, v);
    if (rc) return rc;
    for (int64_t i = 0; i < n; ++i) {
        if (kind == VEC_NORM) v[i] = 1.0f + v[i];
        else if (kind == VEC_NEG_EXP) v[i] = (float)(-exp((double)v[i]));
    }
    return QH_OK;
}

// Weight types of the mixes (roles in the order of the table below).
enum { R_EMBD, R_FFN_GATE, R_FFN_UP, R_FFN_DOWN, R_Q, R_K, R_V, R_O, R_QKV, R_GATE, R_ALPHA, R_BETA, R_SSM_OUT, R_N };
static const int32_t k_mix[3][R_N] = {
    // Q4_K mostly, Q6_K for ffn_down and the tied embedding / head
    {QH_GGUF_Q6_K, QH_GGUF_Q4_K, QH_GGUF_Q4_K, QH_GGUF_Q6_K, QH_GGUF_Q4_K, QH_GGUF_Q4_K, QH_GGUF_Q4_K,
     QH_GGUF_Q4_K, QH_GGUF_Q4_K, QH_GGUF_Q4_K, QH_GGUF_Q4_K, QH_GGUF_Q4_K, QH_GGUF_Q4_K},
    // the released Q4_K_M file's types (Qwen3.5-0.8B): Q5_K attn_q / attn_qkv / ssm_out, Q6_K attn_v,
    // Q8_0 ssm_alpha / ssm_beta
    {QH_GGUF_Q6_K, QH_GGUF_Q4_K, QH_GGUF_Q4_K, QH_GGUF_Q6_K, QH_GGUF_Q5_K, QH_GGUF_Q4_K, QH_GGUF_Q6_K,
     QH_GGUF_Q4_K, QH_GGUF_Q5_K, QH_GGUF_Q4_K, QH_GGUF_Q8_0, QH_GGUF_Q8_0, QH_GGUF_Q5_K},
    // every computed type in some role, including fp32 matrices and Q8_0 outputs
    {QH_GGUF_F32, QH_GGUF_Q5_K, QH_GGUF_Q6_K, QH_GGUF_Q5_K, QH_GGUF_Q6_K, QH_GGUF_F32, QH_GGUF_Q8_0,
     QH_GGUF_Q8_0, QH_GGUF_Q6_K, QH_GGUF_Q5_K, QH_GGUF_F32, QH_GGUF_Q8_0, QH_GGUF_Q8_0},
};

static int add_weight(qh_blob *b, uint64_t seed, const char *name, int32_t type, int64_t k, int64_t n) {
    if (type != QH_GGUF_F32) return add_matrix(b, seed, name, type, k, n);
    blob_tensor *t = blob_add(b, name, QH_GGUF_F32, k, n);
    if (!t) return QH_ERR_INVALID;
    return qh_synth_normal(seed ^ name_hash(name), k * n, 0.0f, 0.02f, (float *)t->data);
}

int qh_blob_synthetic(const qh_slm_config *c, uint64_t seed, qh_blob **out) {
    return qh_blob_synthetic_mix(c, seed, QH_MIX_BASELINE, out);
}

int qh_blob_synthetic_mix(const qh_slm_config *c, uint64_t seed, int32_t mix, qh_blob **out) {
    if (!c || !out || mix < 0 || mix > 2) return QH_ERR_INVALID;
    const int32_t *ty = k_mix[mix];
    *out = NULL;
    if (c->hidden % 256 || c->ffn % 256 || c->n_layers <= 0 || c->vocab <= 0 || c->head_dim <= 0)
        return QH_ERR_INVALID;
    qh_blob *b = (qh_blob *)calloc(1, sizeof(qh_blob));
    if (!b) return QH_ERR_INVALID;
    const int64_t H = c->hidden, F = c->ffn, hd = c->head_dim;
    const int64_t kdim = (int64_t)c->gdn_heads * c->gdn_head_dim, conv_dim = 3 * kdim;
    char nm[64];
    int rc = 0;
#define CHK(x) do { rc = (x); if (rc) goto fail; } while (0)
    CHK(add_weight(b, seed, "token_embd.weight", ty[R_EMBD], H, c->vocab));
    CHK(add_vector(b, seed, "output_norm.weight", H, 1, VEC_NORM, 0.02f));
    for (int L = 0; L < c->n_layers; ++L) {
        const int attn = (L % c->full_attn_interval) == c->full_attn_interval - 1;
#define NAME(s) (snprintf(nm, sizeof(nm), "blk.%d." s, L), nm)
        CHK(add_vector(b, seed, NAME("attn_norm.weight"), H, 1, VEC_NORM, 0.02f));
        CHK(add_vector(b, seed, NAME("post_attention_norm.weight"), H, 1, VEC_NORM, 0.02f));
        CHK(add_weight(b, seed, NAME("ffn_gate.weight"), ty[R_FFN_GATE], H, F));
        CHK(add_weight(b, seed, NAME("ffn_up.weight"), ty[R_FFN_UP], H, F));
        CHK(add_weight(b, seed, NAME("ffn_down.weight"), ty[R_FFN_DOWN], F, H));
        if (attn) {
            CHK(add_weight(b, seed, NAME("attn_q.weight"), ty[R_Q], H, 2 * c->n_heads * hd));
            CHK(add_weight(b, seed, NAME("attn_k.weight"), ty[R_K], H, c->n_kv_heads * hd));
            CHK(add_weight(b, seed, NAME("attn_v.weight"), ty[R_V], H, c->n_kv_heads * hd));
            CHK(add_vector(b, seed, NAME("attn_q_norm.weight"), hd, 1, VEC_NORM, 0.02f));
            CHK(add_vector(b, seed, NAME("attn_k_norm.weight"), hd, 1, VEC_NORM, 0.02f));
            CHK(add_weight(b, seed, NAME("attn_output.weight"), ty[R_O], c->n_heads * hd, H));
        } else {
            CHK(add_weight(b, seed, NAME("attn_qkv.weight"), ty[R_QKV], H, conv_dim));
            CHK(add_weight(b, seed, NAME("attn_gate.weight"), ty[R_GATE], H, kdim));
            CHK(add_vector(b, seed, NAME("ssm_a"), c->gdn_heads, 1, VEC_NEG_EXP, 0.02f));
            CHK(add_weight(b, seed, NAME("ssm_alpha.weight"), ty[R_ALPHA], H, c->gdn_heads));
            CHK(add_weight(b, seed, NAME("ssm_beta.weight"), ty[R_BETA], H, c->gdn_heads));
            CHK(add_vector(b, seed, NAME("ssm_conv1d.weight"), c->conv_kernel, conv_dim, VEC_NORMAL, 0.5f));
            CHK(add_vector(b, seed, NAME("ssm_dt.bias"), c->gdn_heads, 1, VEC_NORMAL, 0.02f));
            CHK(add_vector(b, seed, NAME("ssm_norm.weight"), c->gdn_head_dim, 1, VEC_NORM, 0.02f));
            CHK(add_weight(b, seed, NAME("ssm_out.weight"), ty[R_SSM_OUT], kdim, H));
        }
#undef NAME
    }
#undef CHK
    *out = b;
    return QH_OK;
fail:
    qh_blob_free(b);
    return rc;
}

int qh_blob_create(qh_blob **out) {
    if (!out) return QH_ERR_INVALID;
    *out = (qh_blob *)calloc(1, sizeof(qh_blob));
    return *out ? QH_OK : QH_ERR_INVALID;
}

int qh_blob_add(qh_blob *b, const char *name, int32_t type, const int64_t shape[2], const void *data,
                int64_t nbytes) {
    if (!b || !name || !shape || !data || strlen(name) >= sizeof(((blob_tensor *)0)->name) || shape[0] <= 0 ||
        shape[1] <= 0 || qh_blob_find(b, name) >= 0)
        return QH_ERR_INVALID;
    if (type != QH_GGUF_F32 && (qhf_block_bytes(type) == 0 || shape[0] % qhf_block_weights(type)))
        return QH_ERR_UNSUPPORTED;
    const int64_t want = type == QH_GGUF_F32 ? shape[0] * shape[1] * 4 : qhf_row_bytes(type, shape[0]) * shape[1];
    if (nbytes != want) return QH_ERR_INVALID;
    blob_tensor *t = blob_add(b, name, type, shape[0], shape[1]);
    if (!t) return QH_ERR_INVALID;
    memcpy(t->data, data, (size_t)nbytes);
    return QH_OK;
}

int qh_blob_count(const qh_blob *b) { return b ? b->count : 0; }

int qh_blob_tensor(const qh_blob *b, int i, const char **name, int32_t *type, int64_t shape[2],
                   const void **data, int64_t *nbytes) {
    if (!b || i < 0 || i >= b->count) return QH_ERR_INVALID;
    const blob_tensor *t = &b->t[i];
    if (name) *name = t->name;
    if (type) *type = t->type;
    if (shape) { shape[0] = t->shape[0]; shape[1] = t->shape[1]; }
    if (data) *data = t->data;
    if (nbytes) *nbytes = t->nbytes;
    return QH_OK;
}

int qh_blob_find(const qh_blob *b, const char *name) {
    if (!b || !name) return -1;
    for (int i = 0; i < b->count; ++i)
        if (strcmp(b->t[i].name, name) == 0) return i;
    return -1;
}

void qh_blob_free(qh_blob *b) {
    if (!b) return;
    for (int i = 0; i < b->count; ++i) free(b->t[i].data);
    free(b->t);
    free(b);
}
