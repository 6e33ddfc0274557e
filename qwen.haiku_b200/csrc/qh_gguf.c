// SPDX-License-Identifier: MIT
//
// qh_gguf.c -- GGUF v3 reader and writer for the device model
// (include/qh_gguf.h). The format (little-endian): magic "GGUF", version,
// tensor count, key/value count; key/value pairs (string key, value type,
// value; arrays carry their element type and count); tensor infos (name,
// dims, type, data offset); data at the next multiple of general.alignment
// (32 by default) after the infos. Read the way the reference's gguf_open
// does (slm/gguf.c:172-261), config keys as its slm_load_config
// (slm/qwen.c:59-159).

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qh_backend.h"
#include "qh_formats.h"
#include "qh_gguf.h"

enum { VT_U8, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STR, VT_ARR, VT_U64, VT_I64, VT_F64 };

// ---------------------------------------------------------------------------
// reader over an in-memory copy of the file, with bounds checks
// ---------------------------------------------------------------------------
typedef struct {
    const uint8_t *p;
    size_t n, c;
    int bad;
} rd;

static int need(rd *r, size_t k) {
    if (r->bad || k > r->n - r->c) { r->bad = 1; return 0; }
    return 1;
}
static uint64_t rd_uint(rd *r, int bytes) {
    uint64_t v = 0;
    if (!need(r, (size_t)bytes)) return 0;
    for (int i = 0; i < bytes; ++i) v |= (uint64_t)r->p[r->c + i] << (8 * i);
    r->c += (size_t)bytes;
    return v;
}
static const char *rd_str(rd *r, uint64_t *len) {
    *len = rd_uint(r, 8);
    if (!need(r, (size_t)*len)) return NULL;
    const char *s = (const char *)(r->p + r->c);
    r->c += (size_t)*len;
    return s;
}
static int vt_size(uint32_t t) {
    switch (t) {
        case VT_U8: case VT_I8: case VT_BOOL: return 1;
        case VT_U16: case VT_I16: return 2;
        case VT_U32: case VT_I32: case VT_F32: return 4;
        case VT_U64: case VT_I64: case VT_F64: return 8;
        default: return 0;
    }
}
static void rd_skip_value(rd *r, uint32_t t) {
    if (t == VT_STR) { uint64_t l; rd_str(r, &l); return; }
    if (t == VT_ARR) {
        const uint32_t et = (uint32_t)rd_uint(r, 4);
        const uint64_t n = rd_uint(r, 8);
        if (et == VT_STR || et == VT_ARR) {
            for (uint64_t i = 0; i < n && !r->bad; ++i) rd_skip_value(r, et);
        } else {
            const int sz = vt_size(et);
            if (!sz || n > (r->n - r->c) / (uint64_t)sz) { r->bad = 1; return; }
            r->c += (size_t)(n * (uint64_t)sz);
        }
        return;
    }
    const int sz = vt_size(t);
    if (!sz || !need(r, (size_t)sz)) { r->bad = 1; return; }
    r->c += (size_t)sz;
}

typedef struct {
    const char *key;
    uint64_t klen;
    uint32_t type;
    size_t at;  // offset of the value
} kv_ref;

static const kv_ref *find_kv(const kv_ref *kv, uint64_t n, const char *key) {
    const size_t l = strlen(key);
    for (uint64_t i = 0; i < n; ++i)
        if (kv[i].klen == l && memcmp(kv[i].key, key, l) == 0) return &kv[i];
    return NULL;
}
// Integer-valued key (any integer type), else dflt.
static int64_t kv_int(const rd *file, const kv_ref *kv, uint64_t n, const char *key, int64_t dflt) {
    const kv_ref *k = find_kv(kv, n, key);
    if (!k) return dflt;
    rd r = *file;
    r.c = k->at;
    switch (k->type) {
        case VT_U8: case VT_BOOL: return (int64_t)rd_uint(&r, 1);
        case VT_I8: return (int8_t)rd_uint(&r, 1);
        case VT_U16: return (int64_t)rd_uint(&r, 2);
        case VT_I16: return (int16_t)rd_uint(&r, 2);
        case VT_U32: return (int64_t)rd_uint(&r, 4);
        case VT_I32: return (int32_t)rd_uint(&r, 4);
        case VT_U64: case VT_I64: return (int64_t)rd_uint(&r, 8);
        default: return dflt;
    }
}
static float kv_f32(const rd *file, const kv_ref *kv, uint64_t n, const char *key, float dflt) {
    const kv_ref *k = find_kv(kv, n, key);
    if (!k || k->type != VT_F32) return dflt;
    rd r = *file;
    r.c = k->at;
    const uint32_t bits = (uint32_t)rd_uint(&r, 4);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static int tensor_type_ok(uint32_t t) {
    return t == QH_TYPE_F32 || t == QH_TYPE_Q8_0 || t == QH_TYPE_Q4_K || t == QH_TYPE_Q5_K || t == QH_TYPE_Q6_K;
}

int qh_gguf_load(const char *path, int32_t max_pos_cap, qh_slm_config *cfg, qh_blob **out) {
    if (!path || !cfg || !out) return QH_ERR_INVALID;
    *out = NULL;
    FILE *f = fopen(path, "rb");
    if (!f) return QH_ERR_INVALID;
    uint8_t *buf = NULL;
    long sz = -1;
    if (fseek(f, 0, SEEK_END) == 0) sz = ftell(f);
    if (sz > 0 && fseek(f, 0, SEEK_SET) == 0) {
        buf = (uint8_t *)malloc((size_t)sz);
        if (buf && fread(buf, 1, (size_t)sz, f) != (size_t)sz) { free(buf); buf = NULL; }
    }
    fclose(f);
    if (!buf) return QH_ERR_INVALID;
    int rc = QH_ERR_INVALID;
    kv_ref *kv = NULL;
    qh_blob *blob = NULL;
    rd r = {buf, (size_t)sz, 0, 0};
    const uint32_t magic = (uint32_t)rd_uint(&r, 4), version = (uint32_t)rd_uint(&r, 4);
    const uint64_t n_tensors = rd_uint(&r, 8), n_kv = rd_uint(&r, 8);
    if (r.bad || magic != 0x46554747u || version != 3 || n_kv > (uint64_t)sz || n_tensors > (uint64_t)sz) goto done;
    kv = (kv_ref *)calloc((size_t)n_kv + 1, sizeof(kv_ref));
    if (!kv) goto done;
    for (uint64_t i = 0; i < n_kv && !r.bad; ++i) {
        kv[i].key = rd_str(&r, &kv[i].klen);
        kv[i].type = (uint32_t)rd_uint(&r, 4);
        kv[i].at = r.c;
        rd_skip_value(&r, kv[i].type);
    }
    if (r.bad) goto done;
    {   // architecture
        const kv_ref *a = find_kv(kv, n_kv, "general.architecture");
        if (!a || a->type != VT_STR) goto done;
        rd ar = r;
        ar.c = a->at;
        uint64_t al;
        const char *as = rd_str(&ar, &al);
        if (ar.bad || al != 6 || memcmp(as, "qwen35", 6) != 0) { rc = QH_ERR_UNSUPPORTED; goto done; }
    }
    memset(cfg, 0, sizeof(*cfg));
    cfg->hidden = (int32_t)kv_int(&r, kv, n_kv, "qwen35.embedding_length", 0);
    cfg->n_layers = (int32_t)kv_int(&r, kv, n_kv, "qwen35.block_count", 0);
    cfg->n_heads = (int32_t)kv_int(&r, kv, n_kv, "qwen35.attention.head_count", 0);
    cfg->n_kv_heads = (int32_t)kv_int(&r, kv, n_kv, "qwen35.attention.head_count_kv", cfg->n_heads);
    cfg->ffn = (int32_t)kv_int(&r, kv, n_kv, "qwen35.feed_forward_length", 0);
    {
        const int64_t cl = kv_int(&r, kv, n_kv, "qwen35.context_length", 2048);
        const int64_t cap = max_pos_cap > 0 ? max_pos_cap : 4096;
        cfg->max_pos = (int32_t)(cl < cap ? cl : cap);
    }
    cfg->rope_theta = kv_f32(&r, kv, n_kv, "qwen35.rope.freq_base", 10000.0f);
    cfg->norm_eps = kv_f32(&r, kv, n_kv, "qwen35.attention.layer_norm_rms_epsilon", 1e-5f);
    {
        const int64_t kl = kv_int(&r, kv, n_kv, "qwen35.attention.key_length", 0);
        cfg->head_dim = (int32_t)(kl > 0 ? kl : (cfg->n_heads > 0 ? cfg->hidden / cfg->n_heads : 0));
    }
    cfg->rope_dim = (int32_t)kv_int(&r, kv, n_kv, "qwen35.rope.dimension_count", 0);
    {
        const kv_ref *sec = find_kv(kv, n_kv, "qwen35.rope.dimension_sections");
        if (sec && sec->type == VT_ARR) {
            rd sr = r;
            sr.c = sec->at;
            const uint32_t et = (uint32_t)rd_uint(&sr, 4);
            uint64_t n = rd_uint(&sr, 8);
            if (et == VT_I32 || et == VT_U32)
                for (uint64_t i = 0; i < n && i < 4; ++i) cfg->rope_sections[i] = (int32_t)rd_uint(&sr, 4);
        }
    }
    cfg->full_attn_interval = (int32_t)kv_int(&r, kv, n_kv, "qwen35.full_attention_interval", 4);
    cfg->gdn_heads = (int32_t)kv_int(&r, kv, n_kv, "qwen35.ssm.group_count", 16);
    cfg->gdn_head_dim = (int32_t)kv_int(&r, kv, n_kv, "qwen35.ssm.state_size", 128);
    cfg->conv_kernel = (int32_t)kv_int(&r, kv, n_kv, "qwen35.ssm.conv_kernel", 4);
    {
        const kv_ref *tk = find_kv(kv, n_kv, "tokenizer.ggml.tokens");
        if (tk && tk->type == VT_ARR) {
            rd tr = r;
            tr.c = tk->at;
            rd_uint(&tr, 4);
            cfg->vocab = (int32_t)rd_uint(&tr, 8);
        }
    }
    {
        const int64_t al = kv_int(&r, kv, n_kv, "general.alignment", 32);
        if (al <= 0 || (al & (al - 1))) goto done;
        // tensor infos
        typedef struct { const char *name; uint64_t nlen; uint32_t nd, type; int64_t dims[4]; uint64_t off; } tinfo;
        tinfo *ti = (tinfo *)calloc((size_t)n_tensors + 1, sizeof(tinfo));
        if (!ti) goto done;
        for (uint64_t i = 0; i < n_tensors && !r.bad; ++i) {
            ti[i].name = rd_str(&r, &ti[i].nlen);
            ti[i].nd = (uint32_t)rd_uint(&r, 4);
            if (ti[i].nd < 1 || ti[i].nd > 4) { r.bad = 1; break; }
            for (uint32_t d = 0; d < ti[i].nd; ++d) ti[i].dims[d] = (int64_t)rd_uint(&r, 8);
            ti[i].type = (uint32_t)rd_uint(&r, 4);
            ti[i].off = rd_uint(&r, 8);
        }
        const size_t data0 = (r.c + (size_t)al - 1) & ~((size_t)al - 1);
        if (r.bad || data0 > (size_t)sz || qh_blob_create(&blob)) { free(ti); goto done; }
        rc = QH_OK;
        for (uint64_t i = 0; i < n_tensors; ++i) {
            char name[128];
            if (ti[i].nlen >= sizeof(name)) { rc = QH_ERR_INVALID; break; }
            memcpy(name, ti[i].name, (size_t)ti[i].nlen);
            name[ti[i].nlen] = 0;
            if (!tensor_type_ok(ti[i].type)) { rc = QH_ERR_UNSUPPORTED; break; }
            int64_t shape[2] = {ti[i].dims[0], 1};
            for (uint32_t d = 1; d < ti[i].nd; ++d) shape[1] *= ti[i].dims[d];
            const int64_t nbytes = ti[i].type == QH_TYPE_F32 ? shape[0] * shape[1] * 4
                                                             : qhf_row_bytes((int)ti[i].type, shape[0]) * shape[1];
            if (shape[0] <= 0 || shape[1] <= 0 || ti[i].off > (uint64_t)sz - data0 ||
                (uint64_t)nbytes > (uint64_t)sz - data0 - ti[i].off) { rc = QH_ERR_INVALID; break; }
            rc = qh_blob_add(blob, name, (int32_t)ti[i].type, shape, buf + data0 + ti[i].off, nbytes);
            if (rc) break;
        }
        free(ti);
        if (rc) goto done;
    }
    if (cfg->vocab <= 0) {  // no tokenizer array: the embedding's row count
        int64_t shape[2];
        const int e = qh_blob_find(blob, "token_embd.weight");
        if (e >= 0 && qh_blob_tensor(blob, e, NULL, NULL, shape, NULL, NULL) == QH_OK) cfg->vocab = (int32_t)shape[1];
    }
    if (cfg->hidden <= 0 || cfg->n_layers <= 0 || cfg->n_heads <= 0 || cfg->ffn <= 0 || cfg->vocab <= 0) {
        rc = QH_ERR_INVALID;
        goto done;
    }
    *out = blob;
    blob = NULL;
    rc = QH_OK;
done:
    if (blob) qh_blob_free(blob);
    free(kv);
    free(buf);
    return rc;
}

// The special token ids slm_model_load binds: bos/eos from their keys
// (default 0, slm/qwen.c:150-155), eot = the id of "<|im_end|>" and the
// end-of-generation set from the vocabulary strings (slm/model.c:1153-1178),
// -1 / empty when absent.
int qh_gguf_special_tokens(const char *path, qh_special_tokens *out) {
    if (!path || !out) return QH_ERR_INVALID;
    memset(out, 0, sizeof(*out));
    out->eot_id = -1;
    FILE *f = fopen(path, "rb");
    if (!f) return QH_ERR_INVALID;
    uint8_t *buf = NULL;
    long sz = -1;
    if (fseek(f, 0, SEEK_END) == 0) sz = ftell(f);
    if (sz > 0 && fseek(f, 0, SEEK_SET) == 0) {
        buf = (uint8_t *)malloc((size_t)sz);
        if (buf && fread(buf, 1, (size_t)sz, f) != (size_t)sz) { free(buf); buf = NULL; }
    }
    fclose(f);
    if (!buf) return QH_ERR_INVALID;
    int rc = QH_ERR_INVALID;
    rd r = {buf, (size_t)sz, 0, 0};
    const uint32_t magic = (uint32_t)rd_uint(&r, 4), version = (uint32_t)rd_uint(&r, 4);
    rd_uint(&r, 8);
    const uint64_t n_kv = rd_uint(&r, 8);
    kv_ref *kv = NULL;
    if (r.bad || magic != 0x46554747u || version != 3 || n_kv > (uint64_t)sz) goto done;
    kv = (kv_ref *)calloc((size_t)n_kv + 1, sizeof(kv_ref));
    if (!kv) goto done;
    for (uint64_t i = 0; i < n_kv && !r.bad; ++i) {
        kv[i].key = rd_str(&r, &kv[i].klen);
        kv[i].type = (uint32_t)rd_uint(&r, 4);
        kv[i].at = r.c;
        rd_skip_value(&r, kv[i].type);
    }
    if (r.bad) goto done;
    out->bos_id = (int32_t)kv_int(&r, kv, n_kv, "tokenizer.ggml.bos_token_id", 0);
    out->eos_id = (int32_t)kv_int(&r, kv, n_kv, "tokenizer.ggml.eos_token_id", 0);
    {
        static const char *const stops[] = {"<|endoftext|>", "<|im_end|>", "<|fim_pad|>", "<|repo_name|>",
                                            "<|file_sep|>"};
        int32_t found[5] = {-1, -1, -1, -1, -1};
        const kv_ref *tk = find_kv(kv, n_kv, "tokenizer.ggml.tokens");
        if (tk && tk->type == VT_ARR) {
            rd tr = r;
            tr.c = tk->at;
            const uint32_t et = (uint32_t)rd_uint(&tr, 4);
            const uint64_t n = rd_uint(&tr, 8);
            for (uint64_t i = 0; et == VT_STR && i < n && !tr.bad; ++i) {
                uint64_t l;
                const char *t = rd_str(&tr, &l);
                for (int j = 0; j < 5 && !tr.bad; ++j)
                    if (found[j] < 0 && l == strlen(stops[j]) && memcmp(t, stops[j], (size_t)l) == 0)
                        found[j] = (int32_t)i;
            }
            if (tr.bad) goto done;
        }
        out->eot_id = found[1];
        for (int j = 0; j < 5; ++j)
            if (found[j] >= 0) out->stop_ids[out->n_stop++] = found[j];
    }
    rc = QH_OK;
done:
    free(kv);
    free(buf);
    return rc;
}

// ---------------------------------------------------------------------------
// writer
// ---------------------------------------------------------------------------
typedef struct {
    FILE *f;
    uint64_t pos;
    int bad;
} wr;

static void w_bytes(wr *w, const void *p, size_t n) {
    if (w->bad) return;
    if (n && fwrite(p, 1, n, w->f) != n) w->bad = 1;
    w->pos += n;
}
static void w_uint(wr *w, uint64_t v, int bytes) {
    uint8_t b[8];
    for (int i = 0; i < bytes; ++i) b[i] = (uint8_t)(v >> (8 * i));
    w_bytes(w, b, (size_t)bytes);
}
static void w_str(wr *w, const char *s) {
    const size_t n = strlen(s);
    w_uint(w, n, 8);
    w_bytes(w, s, n);
}
static void w_key(wr *w, const char *k, uint32_t type) {
    w_str(w, k);
    w_uint(w, type, 4);
}
static void kv_u32(wr *w, const char *k, uint32_t v) { w_key(w, k, VT_U32); w_uint(w, v, 4); }
static void kv_f32w(wr *w, const char *k, float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    w_key(w, k, VT_F32);
    w_uint(w, bits, 4);
}

int qh_gguf_write(const char *path, const qh_slm_config *c, const qh_blob *blob) {
    if (!path || !c || !blob || c->vocab <= 0) return QH_ERR_INVALID;
    const int nt = qh_blob_count(blob);
    FILE *f = fopen(path, "wb");
    if (!f) return QH_ERR_INVALID;
    wr w = {f, 0, 0};
    const uint64_t align = 32;
    const int n_kv = 21;
    w_uint(&w, 0x46554747u, 4);
    w_uint(&w, 3, 4);
    w_uint(&w, (uint64_t)nt, 8);
    w_uint(&w, (uint64_t)n_kv, 8);
    w_key(&w, "general.architecture", VT_STR);
    w_str(&w, "qwen35");
    kv_u32(&w, "general.alignment", (uint32_t)align);
    kv_u32(&w, "qwen35.block_count", (uint32_t)c->n_layers);
    kv_u32(&w, "qwen35.context_length", (uint32_t)c->max_pos);
    kv_u32(&w, "qwen35.embedding_length", (uint32_t)c->hidden);
    kv_u32(&w, "qwen35.feed_forward_length", (uint32_t)c->ffn);
    kv_u32(&w, "qwen35.attention.head_count", (uint32_t)c->n_heads);
    kv_u32(&w, "qwen35.attention.head_count_kv", (uint32_t)c->n_kv_heads);
    kv_u32(&w, "qwen35.attention.key_length", (uint32_t)c->head_dim);
    kv_f32w(&w, "qwen35.attention.layer_norm_rms_epsilon", c->norm_eps);
    kv_f32w(&w, "qwen35.rope.freq_base", c->rope_theta);
    kv_u32(&w, "qwen35.rope.dimension_count", (uint32_t)c->rope_dim);
    w_key(&w, "qwen35.rope.dimension_sections", VT_ARR);
    w_uint(&w, VT_I32, 4);
    w_uint(&w, 4, 8);
    for (int i = 0; i < 4; ++i) w_uint(&w, (uint32_t)c->rope_sections[i], 4);
    kv_u32(&w, "qwen35.full_attention_interval", (uint32_t)c->full_attn_interval);
    kv_u32(&w, "qwen35.ssm.group_count", (uint32_t)c->gdn_heads);
    kv_u32(&w, "qwen35.ssm.state_size", (uint32_t)c->gdn_head_dim);
    kv_u32(&w, "qwen35.ssm.conv_kernel", (uint32_t)c->conv_kernel);
    kv_u32(&w, "qwen35.ssm.inner_size", (uint32_t)(c->gdn_heads * c->gdn_head_dim));
    w_key(&w, "tokenizer.ggml.tokens", VT_ARR);  // placeholder vocabulary
    w_uint(&w, VT_STR, 4);
    w_uint(&w, (uint64_t)c->vocab, 8);
    for (int32_t i = 0; i < c->vocab; ++i) {
        char t[24];
        snprintf(t, sizeof(t), "<t%d>", i);
        w_str(&w, t);
    }
    kv_u32(&w, "tokenizer.ggml.bos_token_id", 0);
    kv_u32(&w, "tokenizer.ggml.eos_token_id", 0);
    // tensor infos
    uint64_t off = 0;
    for (int i = 0; i < nt; ++i) {
        const char *name;
        int32_t type;
        int64_t shape[2], nbytes;
        qh_blob_tensor(blob, i, &name, &type, shape, NULL, &nbytes);
        w_str(&w, name);
        const uint32_t nd = shape[1] > 1 ? 2 : 1;
        w_uint(&w, nd, 4);
        w_uint(&w, (uint64_t)shape[0], 8);
        if (nd == 2) w_uint(&w, (uint64_t)shape[1], 8);
        w_uint(&w, (uint32_t)type, 4);
        w_uint(&w, off, 8);
        off = (off + (uint64_t)nbytes + align - 1) & ~(align - 1);
    }
    static const uint8_t zeros[32] = {0};
    w_bytes(&w, zeros, (size_t)(((w.pos + align - 1) & ~(align - 1)) - w.pos));
    for (int i = 0; i < nt; ++i) {
        const void *data;
        int64_t nbytes;
        qh_blob_tensor(blob, i, NULL, NULL, NULL, &data, &nbytes);
        w_bytes(&w, data, (size_t)nbytes);
        w_bytes(&w, zeros, (size_t)((((uint64_t)nbytes + align - 1) & ~(align - 1)) - (uint64_t)nbytes));
    }
    const int bad = w.bad;
    if (fclose(f) != 0 || bad) return QH_ERR_INVALID;
    return QH_OK;
}
