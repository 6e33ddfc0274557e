// SPDX-License-Identifier: MIT
//
// qh_slm.c -- host step driver of the hybrid forward pass (include/qh_slm.h).
//
// C host layer over the backend C-ABI: it uploads the GGUF-layout weights,
// owns the per-sequence caches and chains, per token and for all sequences
// at once, the same operations as the reference's slm_forward_step
// (slm/qwen.c:874-981):
//   embed (Q6_K row) -> for each layer:
//     GDN layer  (slm/qwen.c:318-611): rmsnorm, one grouped matvec launch for
//       attn_qkv/attn_gate/ssm_beta/ssm_alpha, conv+SiLU+L2norm+beta/g,
//       recurrence, gated norm, ssm_out;
//     attention  (slm/model.c:766-953): rmsnorm, grouped q/k/v, q/k norm +
//       MRoPE + fp16 KV append, attention + sigmoid gate, attn_output;
//     residual add, post-attention rmsnorm, grouped ffn_gate/ffn_up, SwiGLU,
//     ffn_down (Q6_K), residual add;
//   output rmsnorm -> tied Q6_K LM head -> argmax.
// Every matmul input is quantized once on the device (Q8_K) and shared by
// the projections that read it, which is what the reference's
// tensor_matmul_* wrappers compute per call.

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "qh_backend.h"
#include "qh_formats.h"
#include "qh_kernels.h"
#include "qh_slm.h"

#define MAX_LAYERS 128

// A weight matrix as the GGUF file stores it: type, shape (k = input dim,
// out_f = output dim) and the device copy of its bytes.
typedef struct {
    const void *d;
    int type;
    int64_t k, out_f;
} wref;

// The projections that read one input (q/k/v; qkv/gate/beta/alpha; gate/up;
// one output projection). Each weight is computed by its own GGUF type, as
// matmul_dispatch does (slm/model.c:220-264):
//   * K-quant weights (Q4_K, Q5_K, Q6_K) read the input's Q8_K rows, which
//     the kernel before the set writes: one grouped matvec plan per type
//     (GEMV kernel; rows <= 8) or one tensor-core GEMM launch per type over
//     expanded weights (more rows);
//   * Q8_0 weights read Q8_0 rows of the fp32 input (tensor_quantize_row_q8_0
//     per token, as tensor_matmul_q8_0_f32), F32 weights the fp32 input
//     itself (tensor_matmul_f32); the step forms that fp32 input (x32) only
//     for sets that hold such weights.
#define PS_MAX 8
typedef struct {
    int n;
    const wref *w[PS_MAX];
    float *out[PS_MAX];
    int64_t k;
    int gemm;
    const void *xq;
    qh_matvec_plan plan[3];
    int nplan;
    struct {
        int type, njobs;
        qh_gemm_job jobs[PS_MAX];
    } gg[3];
    int ngg;
    int n32, has_q8_0;
    const float *x32;
    void *xq80;
} plan_set;

typedef struct {
    int is_attn;
    const float *attn_norm, *ffn_norm;
    wref ffn_gate, ffn_up, ffn_down;
    // GDN
    wref qkv, gate, alpha, beta, ssm_out;
    const float *ssm_a, *conv_w, *dt_bias, *ssm_norm;
    // attention
    wref wq, wk, wv, wo;
    const float *q_norm, *k_norm;
    int gdn_index, attn_index;
    plan_set p_in, p_out, p_ffn, p_down;
} layer;

struct qh_slm {
    qh_slm_config cfg;
    int32_t B;
    int use_gemm;   // B > 8: tensor-core GEMM over tiled weights and activations
    int xq_tile;    // activation layout the fused quantizers write (0 split, 64 tiled)
    void *gemm_scratch;            // split-K terms + counters shared by every GEMM of a step
    int64_t gemm_scratch_bytes;
    cudaStream_t stream;
    void **allocs;
    int nallocs, capallocs;
    int64_t weight_bytes, state_bytes;
    wref tok_embd;
    const float *out_norm;
    layer L[MAX_LAYERS];
    int n_gdn, n_attn;
    // activations [B][...]
    float *h, *h2, *hn, *mix, *qkv, *z, *bt, *at, *gq, *gk, *gv, *gbeta, *gg, *gout, *gy;
    float *qraw, *kb, *vb, *aq, *agate, *actx, *fgate, *fup, *fact, *logits, *rope;
    void *xq_h, *xq_gdn, *xq_ffn;  // split Q8_K activations for K = hidden, gdn width, ffn
    int32_t *d_tok, *d_next;
    int32_t *d_ctl;                // [0] = position, [1] = prompt length
    void *amax_scratch;            // qh_argmax_feed partials + tickets (kept zeroed)
    int32_t *d_prompt, *d_picks;   // [B][max_pos]: prompt tokens, greedy picks by position
    int32_t *h_tok, *h_next, *h_ctl;  // pinned
    int32_t host_pos;              // position of the next step
    int32_t n_prompt;
    // tiled copies of the weights (tensor-core path), by raw pointer
    struct { const void *raw; void *wt; } tiled[4 * MAX_LAYERS * 4 + 8];
    int ntiled;
    // prompt chunks (qh_slm_prefill), allocated on first use
    int32_t pf_chunk, pf_chunk_max;
    int32_t pf_mode;               // QH_PREFILL_STEPWISE or QH_PREFILL_CHUNKED
    float *pf_o;                   // chunked mode: DeltaNet outputs [rows][gdn width]
    float *pf_h, *pf_h2, *pf_mix, *pf_qkv, *pf_z, *pf_bt, *pf_at, *pf_qraw, *pf_kb, *pf_vb, *pf_aq, *pf_agate,
        *pf_actx, *pf_fgate, *pf_fup;
    float *pf_hn, *pf_fact;        // fp32 rows for Q8_0/F32 weights (allocated when a set has them)
    void *pf_xq_h, *pf_xq_gdn, *pf_xq_ffn;
    int32_t *pf_tok, *pf_pos;
    plan_set pf_in[MAX_LAYERS], pf_out[MAX_LAYERS], pf_ffn[MAX_LAYERS], pf_down[MAX_LAYERS];
    // The whole step is captured once in a CUDA graph (after one direct run
    // has set every kernel attribute) and replayed; position and tokens are
    // read from device memory, so one graph serves every position. Two
    // graphs: [0] ends in the greedy pick, [1] in the sampler chain.
    cudaGraph_t graph[2];
    cudaGraphExec_t graph_exec[2];
    int steps_run[2];
    int no_graph[2];               // the step could not be captured: launched directly
    int sampling;                  // the step ends in qh_sample_feed
    // persistent decode (QH_DECODE_PERSISTENT): the step's phases as one
    // program, run as segments separated by the attention layers' cache
    // kernels (qh_attn_pre, qh_attn_decode)
    int32_t decode_mode;           // requested
    int step_state;                // 0 not built, 1 built, -1 the model does not qualify
    qh_step_prog *step_prog;
    int32_t n_seg;
    struct { int32_t first, count, attn_layer; } seg[MAX_LAYERS + 1];
    // sampled decoding (qh_slm_generate_sampled)
    qh_sample_ctl *d_sctl;
    int32_t *d_hist, *d_hist_n;    // [B][max_pos + 1] prompt + generated tokens, lengths
    uint64_t *d_rng;               // [B][2] generator words
    unsigned *d_sticket;
    // parity tracer (qh_slm_trace): armed for the next qh_slm_step
    FILE *trace_fp;
    int32_t trace_seq;
    float *trace_buf;              // host copy of one traced row
    int64_t trace_cap;
    // caches
    float *ring, *state;
    uint16_t *kcache, *vcache;
    plan_set p_head;
};

static int dev_alloc(qh_slm *m, void **p, size_t bytes, int64_t *counter) {
    if (m->nallocs == m->capallocs) {
        int cap = m->capallocs ? 2 * m->capallocs : 256;
        void **a = (void **)realloc(m->allocs, sizeof(void *) * cap);
        if (!a) return QH_ERR_INVALID;
        m->allocs = a;
        m->capallocs = cap;
    }
    int rc = qh_malloc(p, bytes);
    if (rc) return rc;
    m->allocs[m->nallocs++] = *p;
    if (counter) *counter += (int64_t)bytes;
    return QH_OK;
}

#define CK(x) do { int rc_ = (x); if (rc_) return rc_; } while (0)

// Device copy of the blob's matrix `name`, checked against the shape the
// model needs (GGUF order: k = input dim, out_f = output dim): a type the
// matmuls compute -- F32, Q8_0, Q4_K, Q5_K, Q6_K, the cases of
// matmul_dispatch (slm/model.c:220-264) -- else QH_ERR_UNSUPPORTED; a
// different shape, QH_ERR_INVALID. (The reference aborts on an unknown type
// and trusts the shapes; here a file whose tensors do not fit the model is
// refused before any kernel reads past a weight buffer.)
static int upload_w(qh_slm *m, const qh_blob *blob, const char *name, int64_t k, int64_t out_f, wref *out) {
    int i = qh_blob_find(blob, name);
    if (i < 0) return QH_ERR_INVALID;
    const void *data;
    int64_t nbytes, shape[2];
    int32_t type;
    CK(qh_blob_tensor(blob, i, NULL, &type, shape, &data, &nbytes));
    if (type != QH_GGUF_F32 && type != QH_GGUF_Q8_0 && type != QH_GGUF_Q4_K && type != QH_GGUF_Q5_K &&
        type != QH_GGUF_Q6_K)
        return QH_ERR_UNSUPPORTED;
    if (shape[0] != k || shape[1] != out_f) return QH_ERR_INVALID;
    const int64_t want = type == QH_GGUF_F32 ? 4 * k * out_f : qhf_row_bytes(type, k) * out_f;
    if (type != QH_GGUF_F32 && k % qhf_block_weights(type)) return QH_ERR_INVALID;
    if (nbytes != want) return QH_ERR_INVALID;
    void *d;
    CK(dev_alloc(m, &d, (size_t)nbytes, &m->weight_bytes));
    CK(qh_memcpy_h2d(d, data, (size_t)nbytes, m->stream));
    out->d = d;
    out->type = type;
    out->k = k;
    out->out_f = out_f;
    return QH_OK;
}

// Device copy of an fp32 vector of n values (norm weights, conv kernel,
// ssm_a, dt bias).
static int upload_vec(qh_slm *m, const qh_blob *blob, const char *name, int64_t n, const float **out) {
    int i = qh_blob_find(blob, name);
    if (i < 0) return QH_ERR_INVALID;
    const void *data;
    int64_t nbytes;
    int32_t type;
    CK(qh_blob_tensor(blob, i, NULL, &type, NULL, &data, &nbytes));
    if (type != QH_GGUF_F32) return QH_ERR_UNSUPPORTED;
    if (nbytes != 4 * n) return QH_ERR_INVALID;
    void *d;
    CK(dev_alloc(m, &d, (size_t)nbytes, &m->weight_bytes));
    CK(qh_memcpy_h2d(d, data, (size_t)nbytes, m->stream));
    *out = (const float *)d;
    return QH_OK;
}

// Expanded copy of a weight matrix for the tensor-core GEMM (the MMA
// operand image of every 128-row tile and super-block, qh_gemm_expand_weights),
// made on first request through a temporary tiled copy and shared by the
// decode and prompt plans. Each weight is used by few token tiles per
// launch, so streaming the stored operands beats expanding them per launch.
static int get_tiled(qh_slm *m, const void *raw, int type, int64_t k, int64_t out_f, const void **wt) {
    for (int i = 0; i < m->ntiled; ++i)
        if (m->tiled[i].raw == raw) { *wt = m->tiled[i].wt; return QH_OK; }
    if (m->ntiled >= (int)(sizeof(m->tiled) / sizeof(m->tiled[0]))) return QH_ERR_INVALID;
    const int64_t tb = qh_gemm_weight_bytes(type, k, out_f), eb = qh_gemm_expanded_bytes(type, k, out_f);
    if (tb < 0 || eb < 0) return QH_ERR_INVALID;
    void *tiled = NULL, *d;
    CK(dev_alloc(m, &d, (size_t)eb, NULL));
    CK(qh_malloc(&tiled, (size_t)tb));
    int rc = qh_gemm_pack_weights(type, raw, k, out_f, tiled, m->stream);
    if (!rc) rc = qh_gemm_expand_weights(type, tiled, k, out_f, d, m->stream);
    if (!rc) rc = qh_stream_sync(m->stream);
    qh_free(tiled);
    if (rc) return rc;
    m->tiled[m->ntiled].raw = raw;
    m->tiled[m->ntiled].wt = d;
    m->ntiled++;
    *wt = d;
    return QH_OK;
}

static int is_kquant(int type) { return type == QH_GGUF_Q4_K || type == QH_GGUF_Q5_K || type == QH_GGUF_Q6_K; }

// A set over `nm` (<= 8) weights that read one input of k values per row:
// xq its Q8_K rows (split layout for the GEMV at `rows` <= 8, tiled for the
// GEMM), rows the rows per launch. gemm: K-quant weights on the tensor-core
// GEMM (their expanded copies are made here). Q8_0/F32 weights get a Q8_0
// buffer; the caller points x32 at the fp32 input before the set runs.
static int make_set(qh_slm *m, plan_set *ps, int nm, const wref *const *w, float *const *out, const void *xq,
                    int64_t k, int64_t rows, int gemm) {
    if (nm > PS_MAX) return QH_ERR_INVALID;
    memset(ps, 0, sizeof(*ps));
    ps->n = nm;
    ps->k = k;
    ps->gemm = gemm;
    ps->xq = xq;
    static const int kq[3] = {QH_GGUF_Q4_K, QH_GGUF_Q5_K, QH_GGUF_Q6_K};
    for (int i = 0; i < nm; ++i) {
        if (w[i]->k != k) return QH_ERR_INVALID;
        ps->w[i] = w[i];
        ps->out[i] = out[i];
        if (!is_kquant(w[i]->type)) {
            ps->n32++;
            if (w[i]->type == QH_GGUF_Q8_0) ps->has_q8_0 = 1;
        }
    }
    for (int t = 0; t < 3; ++t) {
        qh_matvec_job jobs[PS_MAX];
        int nj = 0;
        memset(jobs, 0, sizeof(jobs));
        for (int i = 0; i < nm; ++i) {
            if (w[i]->type != kq[t]) continue;
            if (gemm) {
                const void *wt;
                CK(get_tiled(m, w[i]->d, kq[t], k, w[i]->out_f, &wt));
                qh_gemm_job *j = &ps->gg[ps->ngg].jobs[nj];
                j->d_wt = wt;
                j->out_f = w[i]->out_f;
                j->d_out = out[i];
                j->ld_out = w[i]->out_f;
            } else {
                jobs[nj].d_w = w[i]->d;
                jobs[nj].d_xq = xq;
                jobs[nj].d_out = out[i];
                jobs[nj].k = k;
                jobs[nj].out_f = w[i]->out_f;
                jobs[nj].xq_rows = rows;
                jobs[nj].xq_row0 = 0;
            }
            nj++;
        }
        if (!nj) continue;
        if (gemm) {
            ps->gg[ps->ngg].type = kq[t];
            ps->gg[ps->ngg].njobs = nj;
            ps->ngg++;
        } else {
            CK(qh_matvec_plan_create(kq[t], jobs, nj, rows, &ps->plan[ps->nplan]));
            ps->nplan++;
        }
    }
    if (ps->has_q8_0) CK(dev_alloc(m, &ps->xq80, (size_t)qh_q8_0_bytes(k, rows), NULL));
    return QH_OK;
}

// Runs a set for `rows` input rows (the fp32 input, when the set needs it,
// at ps->x32); scratch: split-K terms of the GEMM (may be null).
static int run_set(qh_slm *m, plan_set *ps, int64_t rows, void *scratch, int64_t scratch_bytes) {
    for (int g = 0; g < ps->ngg; ++g)  /* expanded weights made at create, then synchronized */
        CK(qh_gemm(ps->gg[g].type, ps->gg[g].jobs, ps->gg[g].njobs, ps->k, ps->xq, rows, scratch, scratch_bytes,
                   QH_GEMM_WEIGHTS_READY | QH_GEMM_EXPANDED, m->stream));
    for (int i = 0; i < ps->nplan; ++i) CK(qh_matvec_plan_run(ps->plan[i], m->stream));
    if (!ps->n32) return QH_OK;
    if (!ps->x32) return QH_ERR_INVALID;
    if (ps->has_q8_0) CK(qh_quantize_q8_0(ps->x32, ps->k, rows, ps->xq80, m->stream));
    for (int i = 0; i < ps->n; ++i) {
        const wref *w = ps->w[i];
        if (w->type == QH_GGUF_Q8_0)
            CK(qh_matmul_preq(QH_GGUF_Q8_0, w->d, ps->k, w->out_f, ps->xq80, rows, ps->out[i], m->stream));
        else if (w->type == QH_GGUF_F32)
            CK(qh_matmul_f32((const float *)w->d, w->out_f, ps->k, ps->x32, rows, ps->out[i], m->stream));
    }
    return QH_OK;
}

static int run_plans(qh_slm *m, plan_set *ps) {
    return run_set(m, ps, m->B, m->gemm_scratch, m->gemm_scratch_bytes);
}

static void free_plans(plan_set *ps) {
    for (int i = 0; i < ps->nplan; ++i) qh_matvec_plan_destroy(ps->plan[i]);
    ps->nplan = 0;
}

// cos/sin of the interleaved-MRoPE angles for text positions, computed with
// the host libm exactly as tensor_rope_mrope_i does (slm/tensor.c:394-437):
// pair i rotates by pos * theta^(-2i/rope_dim) when i % 3 == 0 and
// i < 3*sections[0]; the H/W/E axes are 0 for text, leaving those pairs
// unrotated (cos 1, sin 0).
static void rope_table(const qh_slm_config *c, float *tab) {
    const int half = c->rope_dim / 2;
    for (int p = 0; p < c->max_pos; ++p)
        for (int i = 0; i < half; ++i) {
            float pos_axis = 0.0f;
            if (i % 3 == 0 && i < 3 * c->rope_sections[0]) pos_axis = (float)p;
            const float theta_scale = powf(c->rope_theta, -2.0f * (float)i / (float)c->rope_dim);
            const float theta = pos_axis * theta_scale;
            tab[((size_t)p * half + i) * 2] = cosf(theta);
            tab[((size_t)p * half + i) * 2 + 1] = sinf(theta);
        }
}

static int bind_layers(qh_slm *m, const qh_blob *blob) {
    const qh_slm_config *c = &m->cfg;
    const int64_t H = c->hidden, F = c->ffn, hd = c->head_dim;
    const int64_t kdim = (int64_t)c->gdn_heads * c->gdn_head_dim, conv_dim = 3 * kdim;
    const int64_t qdim = (int64_t)c->n_heads * hd, kvd = (int64_t)c->n_kv_heads * hd;
    char nm[96];
#define W(field, fmt, k_, out_f_) do { snprintf(nm, sizeof(nm), fmt, l); CK(upload_w(m, blob, nm, (k_), (out_f_), &Ly->field)); } while (0)
#define V(field, fmt, n_) do { snprintf(nm, sizeof(nm), fmt, l); CK(upload_vec(m, blob, nm, (n_), &Ly->field)); } while (0)
    for (int l = 0; l < c->n_layers; ++l) {
        layer *Ly = &m->L[l];
        snprintf(nm, sizeof(nm), "blk.%d.ssm_a", l);
        Ly->is_attn = qh_blob_find(blob, nm) < 0;
        V(attn_norm, "blk.%d.attn_norm.weight", H);
        V(ffn_norm, "blk.%d.post_attention_norm.weight", H);
        W(ffn_gate, "blk.%d.ffn_gate.weight", H, F);
        W(ffn_up, "blk.%d.ffn_up.weight", H, F);
        W(ffn_down, "blk.%d.ffn_down.weight", F, H);
        if (Ly->is_attn) {
            W(wq, "blk.%d.attn_q.weight", H, 2 * qdim);
            W(wk, "blk.%d.attn_k.weight", H, kvd);
            W(wv, "blk.%d.attn_v.weight", H, kvd);
            W(wo, "blk.%d.attn_output.weight", qdim, H);
            V(q_norm, "blk.%d.attn_q_norm.weight", hd);
            V(k_norm, "blk.%d.attn_k_norm.weight", hd);
            Ly->attn_index = m->n_attn++;
        } else {
            W(qkv, "blk.%d.attn_qkv.weight", H, conv_dim);
            W(gate, "blk.%d.attn_gate.weight", H, kdim);
            W(alpha, "blk.%d.ssm_alpha.weight", H, c->gdn_heads);
            W(beta, "blk.%d.ssm_beta.weight", H, c->gdn_heads);
            W(ssm_out, "blk.%d.ssm_out.weight", kdim, H);
            V(ssm_a, "blk.%d.ssm_a", c->gdn_heads);
            V(conv_w, "blk.%d.ssm_conv1d.weight", (int64_t)c->conv_kernel * conv_dim);
            V(dt_bias, "blk.%d.ssm_dt.bias", c->gdn_heads);
            V(ssm_norm, "blk.%d.ssm_norm.weight", c->gdn_head_dim);
            Ly->gdn_index = m->n_gdn++;
        }
    }
#undef W
#undef V
    return QH_OK;
}

static int alloc_f(qh_slm *m, float **p, int64_t n) { return dev_alloc(m, (void **)p, (size_t)n * 4, NULL); }

int qh_slm_create(const qh_slm_config *cfg, const qh_blob *blob, int32_t n_seq, qh_slm **out) {
    if (!cfg || !blob || !out || n_seq <= 0 || n_seq > 65535 || cfg->n_layers > MAX_LAYERS ||
        cfg->n_heads % cfg->n_kv_heads || cfg->max_pos <= 0)
        return QH_ERR_INVALID;
    *out = NULL;
    qh_slm *m = (qh_slm *)calloc(1, sizeof(qh_slm));
    if (!m) return QH_ERR_INVALID;
    m->cfg = *cfg;
    m->B = n_seq;
    m->use_gemm = n_seq > 8;
    m->xq_tile = m->use_gemm ? QH_Q8KT_TILE_TOKENS : 0;
    int rc = QH_OK;
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) { rc = QH_ERR_CUDA; goto fail; }
#define TRY(x) do { rc = (x); if (rc) goto fail; } while (0)
    TRY(upload_w(m, blob, "token_embd.weight", cfg->hidden, cfg->vocab, &m->tok_embd));
    // the embedding row reader takes the two types the reference's does (slm/qwen.c:885-907)
    if (m->tok_embd.type != QH_GGUF_Q6_K && m->tok_embd.type != QH_GGUF_F32) { rc = QH_ERR_UNSUPPORTED; goto fail; }
    TRY(upload_vec(m, blob, "output_norm.weight", cfg->hidden, &m->out_norm));
    TRY(bind_layers(m, blob));
    {
        const int64_t B = n_seq, H = cfg->hidden, F = cfg->ffn, hd = cfg->head_dim;
        const int64_t kdim = (int64_t)cfg->gdn_heads * cfg->gdn_head_dim, conv_dim = 3 * kdim;
        const int64_t qdim = (int64_t)cfg->n_heads * hd, kvd = (int64_t)cfg->n_kv_heads * hd;
        TRY(alloc_f(m, &m->h, B * H));
        TRY(alloc_f(m, &m->h2, B * H));
        TRY(alloc_f(m, &m->hn, B * H));
        TRY(alloc_f(m, &m->mix, B * H));
        TRY(alloc_f(m, &m->qkv, B * conv_dim));
        TRY(alloc_f(m, &m->z, B * kdim));
        TRY(alloc_f(m, &m->bt, B * cfg->gdn_heads));
        TRY(alloc_f(m, &m->at, B * cfg->gdn_heads));
        TRY(alloc_f(m, &m->gq, B * kdim));
        TRY(alloc_f(m, &m->gk, B * kdim));
        TRY(alloc_f(m, &m->gv, B * kdim));
        TRY(alloc_f(m, &m->gbeta, B * cfg->gdn_heads));
        TRY(alloc_f(m, &m->gg, B * cfg->gdn_heads));
        TRY(alloc_f(m, &m->gout, B * kdim));
        TRY(alloc_f(m, &m->gy, B * kdim));
        TRY(alloc_f(m, &m->qraw, B * 2 * qdim));
        TRY(alloc_f(m, &m->kb, B * kvd));
        TRY(alloc_f(m, &m->vb, B * kvd));
        TRY(alloc_f(m, &m->aq, B * qdim));
        TRY(alloc_f(m, &m->agate, B * qdim));
        TRY(alloc_f(m, &m->actx, B * qdim));
        TRY(alloc_f(m, &m->fgate, B * F));
        TRY(alloc_f(m, &m->fup, B * F));
        TRY(alloc_f(m, &m->fact, B * F));
        TRY(alloc_f(m, &m->logits, B * cfg->vocab));
        const int64_t max_in = H > qdim ? H : qdim;
        {
            int64_t (*xq_bytes)(int64_t, int64_t) = m->use_gemm ? qh_q8kt_bytes : qh_q8k_bytes;
            TRY(dev_alloc(m, &m->xq_h, (size_t)xq_bytes(max_in, B), NULL));
            TRY(dev_alloc(m, &m->xq_gdn, (size_t)xq_bytes(kdim, B), NULL));
            TRY(dev_alloc(m, &m->xq_ffn, (size_t)xq_bytes(F, B), NULL));
        }
        TRY(dev_alloc(m, (void **)&m->d_tok, (size_t)B * 4, NULL));
        TRY(dev_alloc(m, (void **)&m->d_next, (size_t)B * 4, NULL));
        TRY(dev_alloc(m, (void **)&m->d_ctl, 16, NULL));
        {
            const int64_t ab = qh_argmax_feed_scratch_bytes(n_seq, cfg->vocab);
            if (ab <= 0) { rc = QH_ERR_INVALID; goto fail; }
            TRY(dev_alloc(m, &m->amax_scratch, (size_t)ab, NULL));
            TRY(qh_memset(m->amax_scratch, 0, (size_t)ab, m->stream));
        }
        TRY(dev_alloc(m, (void **)&m->d_prompt, (size_t)B * cfg->max_pos * 4, NULL));
        TRY(dev_alloc(m, (void **)&m->d_picks, (size_t)B * cfg->max_pos * 4, NULL));
        TRY(dev_alloc(m, (void **)&m->d_sctl, sizeof(qh_sample_ctl), NULL));
        TRY(dev_alloc(m, (void **)&m->d_hist, (size_t)B * (cfg->max_pos + 1) * 4, NULL));
        TRY(dev_alloc(m, (void **)&m->d_hist_n, (size_t)B * 4, NULL));
        TRY(dev_alloc(m, (void **)&m->d_rng, (size_t)B * 16, NULL));
        TRY(dev_alloc(m, (void **)&m->d_sticket, 16, NULL));
        TRY(qh_memset(m->d_sticket, 0, 16, m->stream));
        TRY(qh_memset(m->d_hist_n, 0, (size_t)B * 4, m->stream));
        {
            // each sequence's generator starts seeded with its index + 1
            uint64_t *st = (uint64_t *)malloc((size_t)B * 16);
            if (!st) { rc = QH_ERR_INVALID; goto fail; }
            for (int64_t b = 0; b < B; ++b) qh_rng_seed((uint64_t)b + 1, st + 2 * b);
            rc = qh_memcpy_h2d(m->d_rng, st, (size_t)B * 16, m->stream);
            if (!rc) rc = qh_stream_sync(m->stream);
            free(st);
            if (rc) goto fail;
        }
        if (cudaMallocHost((void **)&m->h_tok, (size_t)B * 4) != cudaSuccess ||
            cudaMallocHost((void **)&m->h_next, (size_t)B * 4) != cudaSuccess ||
            cudaMallocHost((void **)&m->h_ctl, 16) != cudaSuccess) { rc = QH_ERR_CUDA; goto fail; }
        // caches
        const int64_t ng = m->n_gdn > 0 ? m->n_gdn : 1, na = m->n_attn > 0 ? m->n_attn : 1;
        TRY(dev_alloc(m, (void **)&m->ring, (size_t)(ng * B * cfg->conv_kernel * conv_dim * 4), &m->state_bytes));
        TRY(dev_alloc(m, (void **)&m->state,
                      (size_t)(ng * B * cfg->gdn_heads * (int64_t)cfg->gdn_head_dim * cfg->gdn_head_dim * 4),
                      &m->state_bytes));
        const size_t kv = (size_t)(na * B * cfg->max_pos * kvd * 2);
        TRY(dev_alloc(m, (void **)&m->kcache, kv, &m->state_bytes));
        TRY(dev_alloc(m, (void **)&m->vcache, kv, &m->state_bytes));
        // rope table
        const size_t rb = (size_t)cfg->max_pos * (cfg->rope_dim / 2) * 2 * sizeof(float);
        float *tab = (float *)malloc(rb);
        if (!tab) { rc = QH_ERR_INVALID; goto fail; }
        rope_table(cfg, tab);
        rc = dev_alloc(m, (void **)&m->rope, rb, NULL);
        if (!rc) rc = qh_memcpy_h2d(m->rope, tab, rb, m->stream);
        if (!rc) rc = qh_stream_sync(m->stream);
        free(tab);
        if (rc) goto fail;
        // projection sets, each weight by its own type
        const int g = m->use_gemm;
        for (int l = 0; l < cfg->n_layers; ++l) {
            layer *Ly = &m->L[l];
            if (Ly->is_attn) {
                const wref *w[3] = {&Ly->wq, &Ly->wk, &Ly->wv};
                float *o[3] = {m->qraw, m->kb, m->vb};
                TRY(make_set(m, &Ly->p_in, 3, w, o, m->xq_h, H, B, g));
                const wref *w2[1] = {&Ly->wo};
                float *o2[1] = {m->mix};
                TRY(make_set(m, &Ly->p_out, 1, w2, o2, m->xq_h, qdim, B, g));
                Ly->p_out.x32 = m->actx;
            } else {
                const wref *w[4] = {&Ly->qkv, &Ly->gate, &Ly->beta, &Ly->alpha};
                float *o[4] = {m->qkv, m->z, m->bt, m->at};
                TRY(make_set(m, &Ly->p_in, 4, w, o, m->xq_h, H, B, g));
                const wref *w2[1] = {&Ly->ssm_out};
                float *o2[1] = {m->mix};
                TRY(make_set(m, &Ly->p_out, 1, w2, o2, m->xq_gdn, kdim, B, g));
                Ly->p_out.x32 = m->gy;
            }
            Ly->p_in.x32 = m->hn;
            const wref *wf[2] = {&Ly->ffn_gate, &Ly->ffn_up};
            float *of_[2] = {m->fgate, m->fup};
            TRY(make_set(m, &Ly->p_ffn, 2, wf, of_, m->xq_h, H, B, g));
            Ly->p_ffn.x32 = m->hn;
            const wref *wd[1] = {&Ly->ffn_down};
            float *od[1] = {m->mix};
            TRY(make_set(m, &Ly->p_down, 1, wd, od, m->xq_ffn, F, B, g));
            Ly->p_down.x32 = m->fact;
        }
        const wref *wh[1] = {&m->tok_embd};
        float *oh[1] = {m->logits};
        TRY(make_set(m, &m->p_head, 1, wh, oh, m->xq_h, H, B, g));
        m->p_head.x32 = m->hn;
        // (Output tails, qh_matvec_plan_fuse_output, could form each next
        // Q8_K input inside the projection before it; measured in the
        // captured step at batch 1 they are slower -- 1.51 against 1.04 ms
        // per step -- because one CTA then runs the norm serially after the
        // grid's arrival counter, where the separate kernel spreads it over
        // the row's blocks and overlaps its launch.)
        if (m->use_gemm) {
            int64_t need = 0;
            plan_set *all[4 * MAX_LAYERS + 1];
            int na_ = 0;
            for (int l = 0; l < cfg->n_layers; ++l) {
                all[na_++] = &m->L[l].p_in;
                all[na_++] = &m->L[l].p_out;
                all[na_++] = &m->L[l].p_ffn;
                all[na_++] = &m->L[l].p_down;
            }
            all[na_++] = &m->p_head;
            for (int i = 0; i < na_; ++i)
                for (int q = 0; q < all[i]->ngg; ++q) {
                    // only launches with few output tiles split K (the LM head never does)
                    int64_t tiles = 0;
                    for (int j = 0; j < all[i]->gg[q].njobs; ++j) tiles += (all[i]->gg[q].jobs[j].out_f + 127) / 128;
                    tiles *= (B + QH_Q8KT_TILE_TOKENS - 1) / QH_Q8KT_TILE_TOKENS;
                    if (tiles >= 148) continue;
                    const int64_t b = qh_gemm_scratch_bytes(all[i]->gg[q].jobs, all[i]->gg[q].njobs, all[i]->k, B);
                    if (b > need) need = b;
                }
            if (need == 0) need = 256;
            TRY(dev_alloc(m, &m->gemm_scratch, (size_t)need, NULL));
            TRY(qh_memset(m->gemm_scratch, 0, (size_t)need, m->stream));
            m->gemm_scratch_bytes = need;
        }
    }
#undef TRY
    rc = qh_slm_reset(m);
    if (rc) goto fail;
    *out = m;
    return QH_OK;
fail:
    qh_slm_destroy(m);
    return rc ? rc : QH_ERR_INVALID;
}

void qh_slm_destroy(qh_slm *m) {
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (int l = 0; l < m->cfg.n_layers && l < MAX_LAYERS; ++l) {
        free_plans(&m->L[l].p_in);
        free_plans(&m->L[l].p_out);
        free_plans(&m->L[l].p_ffn);
        free_plans(&m->L[l].p_down);
    }
    free_plans(&m->p_head);
    qh_step_destroy(m->step_prog);
    for (int i = 0; i < 2; ++i) {
        if (m->graph_exec[i]) cudaGraphExecDestroy(m->graph_exec[i]);
        if (m->graph[i]) cudaGraphDestroy(m->graph[i]);
    }
    for (int i = 0; i < m->nallocs; ++i) qh_free(m->allocs[i]);
    free(m->allocs);
    if (m->trace_fp) fclose(m->trace_fp);
    free(m->trace_buf);
    if (m->h_tok) cudaFreeHost(m->h_tok);
    if (m->h_next) cudaFreeHost(m->h_next);
    if (m->h_ctl) cudaFreeHost(m->h_ctl);
    if (m->stream) cudaStreamDestroy(m->stream);
    free(m);
}

int qh_slm_reset(qh_slm *m) {
    if (!m) return QH_ERR_INVALID;
    const qh_slm_config *c = &m->cfg;
    const int64_t B = m->B, kdim = (int64_t)c->gdn_heads * c->gdn_head_dim;
    const int64_t ng = m->n_gdn > 0 ? m->n_gdn : 1, na = m->n_attn > 0 ? m->n_attn : 1;
    const int64_t kvd = (int64_t)c->n_kv_heads * c->head_dim;
    CK(qh_memset(m->ring, 0, (size_t)(ng * B * c->conv_kernel * 3 * kdim * 4), m->stream));
    CK(qh_memset(m->state, 0, (size_t)(ng * B * c->gdn_heads * (int64_t)c->gdn_head_dim * c->gdn_head_dim * 4), m->stream));
    CK(qh_memset(m->kcache, 0, (size_t)(na * B * c->max_pos * kvd * 2), m->stream));
    CK(qh_memset(m->vcache, 0, (size_t)(na * B * c->max_pos * kvd * 2), m->stream));
    CK(qh_memset(m->d_picks, 0, (size_t)B * c->max_pos * 4, m->stream));
    m->host_pos = 0;
    m->n_prompt = 0;
    return qh_stream_sync(m->stream);
}

// ---------------------------------------------------------------------------
// Parity tracer: one JSONL record per traced tensor, the schema and number
// formatting of the reference's slm_trace_f32 (slm/model.c:585-727) so the
// lines of bit-identical tensors are identical text. Rows of sequence
// m->trace_seq are copied to the host after a stream synchronization.
// ---------------------------------------------------------------------------
static uint64_t fnv1a64(const uint8_t *p, size_t n) {
    uint64_t h = 0xcbf29ce484222325ULL;
    for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 0x100000001b3ULL;
    return h;
}

static void trace_floats(FILE *f, const char *key, const float *v, int n) {
    fprintf(f, ",\"%s\":[", key);
    for (int i = 0; i < n; ++i) {
        if (i) fputc(',', f);
        if (isnan(v[i])) fputs("\"nan\"", f);
        else if (isinf(v[i])) fputs(v[i] < 0.0f ? "\"-inf\"" : "\"inf\"", f);
        else fprintf(f, "%.9g", v[i]);
    }
    fprintf(f, "],\"%s_hex\":[", key);
    for (int i = 0; i < n; ++i) {
        uint32_t u;
        memcpy(&u, &v[i], 4);
        fprintf(f, "%s\"%08x\"", i ? "," : "", u);
    }
    fputc(']', f);
}

static int trace_row(qh_slm *m, const char *op, const float *d_rows, int64_t n, const char *fmt, ...) {
    char name[64];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(name, sizeof(name), fmt, ap);
    va_end(ap);
    if (n > m->trace_cap) return QH_ERR_INVALID;
    CK(qh_stream_sync(m->stream));
    CK(qh_memcpy_d2h(m->trace_buf, d_rows + (int64_t)m->trace_seq * n, (size_t)n * 4, m->stream));
    CK(qh_stream_sync(m->stream));
    const float *v = m->trace_buf;
    FILE *f = m->trace_fp;
    const int k = n < 8 ? (int)n : 8;
    float sum = 0.0f;
    int n_nan = 0, n_inf = 0;
    for (int64_t i = 0; i < n; ++i) {
        if (isnan(v[i])) ++n_nan;
        else if (isinf(v[i])) ++n_inf;
        else sum += v[i];
    }
    fprintf(f,
            "{\"name\":\"%s\",\"op\":\"%s\",\"type\":\"f32\",\"ne\":[%lld,1,1,1],\"nb\":[4,%lld,%lld,%lld],"
            "\"nbytes\":%zu,\"fnv64\":\"%016llx\"",
            name, op, (long long)n, (long long)(n * 4), (long long)(n * 4), (long long)(n * 4), (size_t)n * 4,
            (unsigned long long)fnv1a64((const uint8_t *)v, (size_t)n * 4));
    trace_floats(f, "head", v, k);
    trace_floats(f, "tail", v + (n - k), k);
    fprintf(f, ",\"sum\":%.9g,\"n_nan\":%d,\"n_inf\":%d}\n", sum, n_nan, n_inf);
    return ferror(f) ? QH_ERR_INVALID : QH_OK;
}

int qh_slm_trace(qh_slm *m, int32_t seq, const char *path) {
    if (!m || !path || seq < 0 || seq >= m->B) return QH_ERR_INVALID;
    const qh_slm_config *c = &m->cfg;
    int64_t cap = c->vocab;
    const int64_t conv_dim = 3 * (int64_t)c->gdn_heads * c->gdn_head_dim;
    if (conv_dim > cap) cap = conv_dim;
    if (2 * (int64_t)c->n_heads * c->head_dim > cap) cap = 2 * (int64_t)c->n_heads * c->head_dim;
    if (c->ffn > cap) cap = c->ffn;
    if (cap > m->trace_cap) {
        float *b = (float *)realloc(m->trace_buf, (size_t)cap * 4);
        if (!b) return QH_ERR_INVALID;
        m->trace_buf = b;
        m->trace_cap = cap;
    }
    if (m->trace_fp) fclose(m->trace_fp);
    m->trace_fp = fopen(path, "w");
    if (!m->trace_fp) return QH_ERR_INVALID;
    m->trace_seq = seq;
    return QH_OK;
}

// One step for all sequences: the forward pass of tokens m->d_tok at
// position d_ctl[0], the greedy picks, then the device-side feed of the next
// inputs. Launches only (no allocation, no synchronization), so it is
// captured in a CUDA graph.
static int forward(qh_slm *m) {
    const qh_slm_config *c = &m->cfg;
    const int32_t B = m->B;
    const int64_t H = c->hidden, F = c->ffn, hd = c->head_dim;
    const int64_t kdim = (int64_t)c->gdn_heads * c->gdn_head_dim, conv_dim = 3 * kdim;
    const int64_t qdim = (int64_t)c->n_heads * hd, kvd = (int64_t)c->n_kv_heads * hd;
    void *s = m->stream;
    // tracing (qh_slm_trace) records the reference's named intermediates
    // (slm/qwen.c:318-981, slm/model.c:766-953); the normalized rows, which
    // the fused kernels only quantize, are recomputed with qh_rmsnorm
#define TR(op, ptr, n, ...)                                            \
    do {                                                               \
        if (m->trace_fp) CK(trace_row(m, (op), (ptr), (n), __VA_ARGS__)); \
    } while (0)
    CK(m->tok_embd.type == QH_GGUF_F32 ? qh_embed_f32((const float *)m->tok_embd.d, H, m->d_tok, B, m->h, s)
                                       : qh_embed_q6k(m->tok_embd.d, H, m->d_tok, B, m->h, s));
    TR("GET_ROWS", m->h, H, "inp_embd");
    // The residual stream alternates between two buffers: each add writes
    // h + mix into the other one (the fused kernel reads h from many CTAs).
    float *hc = m->h, *hx = m->h2;
    const float *pending = NULL;  // residual branch output not yet added to hc
    // Residual add + RMSNorm + Q8_K (one fused kernel), then the plan that
    // reads the quantized row. (The GEMV plans can also form this input
    // themselves, qh_matvec_plan_fuse_input; in the captured step that is
    // slower, because two GEMV launches in a row cannot share SMs the way a
    // small norm kernel and a GEMV do under programmatic launch.)
#define NORMED(ps, w, ADD_NAME, ADD_L, NORM_NAME, NORM_L)                                                  \
    do {                                                                                                   \
        const int added_ = pending != NULL;                                                                \
        CK(qh_rmsnorm_q8k(hc, pending, pending ? hx : NULL, (w), H, B, c->norm_eps, m->xq_h, m->xq_tile, s)); \
        if (pending) { float *t_ = hc; hc = hx; hx = t_; }                                               \
        pending = NULL;                                                                                    \
        if ((ps)->n32) CK(qh_rmsnorm(hc, (w), H, B, c->norm_eps, m->hn, s)); /* fp32 rows for Q8_0/F32 */ \
        CK(run_plans(m, (ps)));                                                                            \
        if (m->trace_fp) {                                                                                 \
            if (added_) TR("ADD", hc, H, ADD_NAME, ADD_L);                                                 \
            CK(qh_rmsnorm(hc, (w), H, B, c->norm_eps, m->hn, s));                                          \
            TR("RMS_NORM", m->hn, H, NORM_NAME, NORM_L);                                                   \
        }                                                                                                  \
    } while (0)
    for (int l = 0; l < c->n_layers; ++l) {
        layer *Ly = &m->L[l];
        NORMED(&Ly->p_in, Ly->attn_norm, "l_out-%d", l - 1, "attn_norm-%d", l);
        if (Ly->is_attn) {
            TR("MUL_MAT", m->qraw, 2 * qdim, "Qfull-%d", l);
            TR("MUL_MAT", m->kb, kvd, "Kcur-%d", l);
            TR("MUL_MAT", m->vb, kvd, "Vcur-%d", l);
            const int64_t ai = Ly->attn_index;
            uint16_t *kc = m->kcache + ai * B * c->max_pos * kvd;
            uint16_t *vc = m->vcache + ai * B * c->max_pos * kvd;
            CK(qh_attn_pre(m->qraw, m->kb, m->vb, Ly->q_norm, Ly->k_norm, m->rope, B, c->n_heads, c->n_kv_heads,
                           (int32_t)hd, c->rope_dim, c->norm_eps, m->d_ctl, c->max_pos, m->aq, m->agate, kc, vc,
                           s));
            CK(qh_attn_decode(m->aq, kc, vc, m->agate, B, c->n_heads, c->n_kv_heads, (int32_t)hd, m->d_ctl,
                              c->max_pos, m->actx, s));
            CK(m->use_gemm ? qh_quantize_q8kt(m->actx, qdim, B, m->xq_h, s)
                           : qh_quantize_q8k(m->actx, qdim, B, m->xq_h, s));
        } else {
            TR("MUL_MAT", m->qkv, conv_dim, "attn_qkv-%d", l);
            TR("MUL_MAT", m->at, c->gdn_heads, "alpha-%d", l);
            TR("MUL_MAT", m->bt, c->gdn_heads, "beta-%d", l);
            const int64_t gi = Ly->gdn_index;
            float *ring = m->ring + gi * B * c->conv_kernel * conv_dim;
            float *state = m->state + gi * B * c->gdn_heads * (int64_t)c->gdn_head_dim * c->gdn_head_dim;
            if (m->trace_fp) {  /* the unfused chain, whose intermediates are traced */
                CK(qh_gdn_pre(m->qkv, ring, Ly->conv_w, m->bt, m->at, Ly->dt_bias, Ly->ssm_a, B, c->gdn_heads,
                              c->gdn_head_dim, c->conv_kernel, m->d_ctl, m->gq, m->gk, m->gv, m->gbeta, m->gg, s));
                TR("VIEW", m->gv, kdim, "V_raw-%d", l);
                TR("L2_NORM_SCALE", m->gq, kdim, "Q_l2norm-%d", l);
                TR("L2_NORM", m->gk, kdim, "K_l2norm-%d", l);
                TR("SIGMOID", m->gbeta, c->gdn_heads, "beta_in-%d", l);
                CK(qh_gdn_recurrence(state, m->gq, m->gk, m->gv, m->gbeta, m->gg, B, c->gdn_heads, c->gdn_head_dim,
                                     m->gout, s));
                TR("RECURRENT", m->gout, kdim, "attn_output-%d", l);
                CK(qh_gdn_gated_norm(m->gout, m->z, Ly->ssm_norm, B, c->gdn_heads, c->gdn_head_dim, c->norm_eps,
                                     m->gy, s));
                TR("RMS_NORM_GATED", m->gy, kdim, "y_norm-%d", l);
                CK(m->use_gemm ? qh_quantize_q8kt(m->gy, kdim, B, m->xq_gdn, s)
                               : qh_quantize_q8k(m->gy, kdim, B, m->xq_gdn, s));
            } else if (m->use_gemm || Ly->p_out.n32) {
                /* many sequences: heads as independent CTAs, then the quantizer; also when
                   ssm_out reads the fp32 rows (Q8_0 / F32 weights) */
                CK(qh_gdn_fused_y(m->qkv, ring, Ly->conv_w, m->bt, m->at, Ly->dt_bias, Ly->ssm_a, state, m->z,
                                  Ly->ssm_norm, B, c->gdn_heads, c->gdn_head_dim, c->conv_kernel, c->norm_eps,
                                  m->d_ctl, m->gy, s));
                CK(m->use_gemm ? qh_quantize_q8kt(m->gy, kdim, B, m->xq_gdn, s)
                               : qh_quantize_q8k(m->gy, kdim, B, m->xq_gdn, s));
            } else {
                CK(qh_gdn_fused(m->qkv, ring, Ly->conv_w, m->bt, m->at, Ly->dt_bias, Ly->ssm_a, state, m->z,
                                Ly->ssm_norm, B, c->gdn_heads, c->gdn_head_dim, c->conv_kernel, c->norm_eps,
                                m->d_ctl, m->xq_gdn, m->xq_tile, s));
            }
        }
        CK(run_plans(m, &Ly->p_out));
        if (Ly->is_attn)
            TR("MUL_MAT", m->mix, H, "attn_out-%d", l);
        else
            TR("MUL_MAT", m->mix, H, "ssm_out-%d", l);
        TR(Ly->is_attn ? "ATTN" : "SSM", m->mix, H, "mix-%d", l);
        pending = m->mix;
        NORMED(&Ly->p_ffn, Ly->ffn_norm, "mix_residual-%d", l, "ffn_norm-%d", l);
        CK(qh_swiglu_q8k(m->fgate, m->fup, F, B, m->xq_ffn, m->xq_tile, s));
        if (Ly->p_down.n32) CK(qh_swiglu(m->fgate, m->fup, m->fact, B * F, s));
        CK(run_plans(m, &Ly->p_down));
        TR("MUL_MAT", m->mix, H, "ffn_out-%d", l);
        pending = m->mix;
    }
    NORMED(&m->p_head, m->out_norm, "l_out-%d", c->n_layers - 1, "result_norm", 0);
#undef NORMED
    TR("MUL_MAT", m->logits, c->vocab, "result_output");
#undef TR
    if (m->sampling)
        CK(qh_sample_feed(m->logits, B, c->vocab, m->d_sctl, m->d_hist, c->max_pos + 1, m->d_hist_n, m->d_rng,
                          m->d_next, c->max_pos, m->d_ctl, m->d_tok, m->d_picks, m->d_sticket, s));
    else
        CK(qh_argmax_feed(m->logits, B, c->vocab, m->amax_scratch, m->d_next, m->d_prompt, c->max_pos, m->d_ctl,
                          m->d_tok, m->d_picks, s));
    return QH_OK;
}

// ---------------------------------------------------------------------------
// Persistent decode step (one sequence): the operations of forward() as
// phases of qh_step programs. Every projection phase forms its own Q8_K
// input (the fused norm/SwiGLU/quantize kernels of forward()), a DeltaNet
// layer is one phase, and each attention layer ends a segment: its cache
// kernels run as launches between two segments.
// ---------------------------------------------------------------------------
static void step_mv(qh_step_phase *ph, int32_t xform, int64_t xk, const float *xa, const float *xb, const float *xw,
                    float *xh_out, float eps, const plan_set *ps) {
    memset(ph, 0, sizeof(*ph));
    ph->kind = QH_STEP_MATVEC;
    ph->xform = xform;
    ph->xk = xk;
    ph->eps = eps;
    ph->d_xa = xa;
    ph->d_xb = xb;
    ph->d_xw = xw;
    ph->d_xh_out = xh_out;
    ph->n_proj = ps->n;
    for (int i = 0; i < ps->n; ++i) {
        ph->proj[i].type = ps->w[i]->type;
        ph->proj[i].d_w = ps->w[i]->d;
        ph->proj[i].k = ps->w[i]->k;
        ph->proj[i].out_f = ps->w[i]->out_f;
        ph->proj[i].d_out = ps->out[i];
    }
}

static int step_set_ok(const plan_set *ps) { return ps->n > 0 && ps->n <= QH_STEP_MAX_PROJ && !ps->n32 && !ps->gemm; }

// Builds the program; step_state -1 (and QH_OK) when the model does not qualify.
static int build_step_prog(qh_slm *m) {
    const qh_slm_config *c = &m->cfg;
    m->step_state = -1;
    if (m->B != 1 || !step_set_ok(&m->p_head) || c->gdn_head_dim != 128) return QH_OK;
    for (int l = 0; l < c->n_layers; ++l) {
        const layer *Ly = &m->L[l];
        if (!step_set_ok(&Ly->p_in) || !step_set_ok(&Ly->p_out) || !step_set_ok(&Ly->p_ffn) ||
            !step_set_ok(&Ly->p_down))
            return QH_OK;
    }
    const int64_t H = c->hidden, F = c->ffn, hd = c->head_dim;
    const int64_t kdim = (int64_t)c->gdn_heads * c->gdn_head_dim, conv_dim = 3 * kdim;
    const int64_t qdim = (int64_t)c->n_heads * hd, kvd = (int64_t)c->n_kv_heads * hd;
    // attention inside the program while its scores fit the kernel's shared
    // memory; longer caches split the program at the attention layers
    const int attn_inside = c->max_pos <= QH_STEP_ATTN_MAX_POS;
    // at most 5 phases per layer (DeltaNet: input projections, head update,
    // output projection, FFN up, FFN down) and the head
    const int max_ph = 5 * c->n_layers + 1;
    qh_step_phase *ph = (qh_step_phase *)calloc((size_t)max_ph, sizeof(qh_step_phase));
    if (!ph) return QH_ERR_INVALID;
    int np = 0, first = 0;
    m->n_seg = 0;
    // the residual stream alternates between h and h2, as in forward()
    float *hc = m->h, *hx = m->h2;
    const float *pending = NULL;
    for (int l = 0; l < c->n_layers; ++l) {
        const layer *Ly = &m->L[l];
        step_mv(&ph[np++], QH_STEP_X_RESNORM, H, hc, pending, Ly->attn_norm, pending ? hx : NULL, c->norm_eps,
                &Ly->p_in);
        if (pending) { float *t = hc; hc = hx; hx = t; }
        if (Ly->is_attn) {
            if (attn_inside) {
                const int64_t ai = Ly->attn_index;
                qh_step_phase *a = &ph[np++];
                a->kind = QH_STEP_ATTN;
                a->eps = c->norm_eps;
                a->head_dim = (int32_t)hd;
                a->d_qraw = m->qraw;
                a->d_kin = m->kb;
                a->d_vin = m->vb;
                a->d_qnorm_w = Ly->q_norm;
                a->d_knorm_w = Ly->k_norm;
                a->d_rope = m->rope;
                a->d_kcache = m->kcache + ai * c->max_pos * kvd;
                a->d_vcache = m->vcache + ai * c->max_pos * kvd;
                a->d_ctx = m->actx;
                a->n_heads = c->n_heads;
                a->n_kv_heads = c->n_kv_heads;
                a->rope_dim = c->rope_dim;
                a->max_pos = c->max_pos;
            } else {  // the cache kernels run as launches between two segments
                m->seg[m->n_seg].first = first;
                m->seg[m->n_seg].count = np - first;
                m->seg[m->n_seg].attn_layer = l;
                m->n_seg++;
                first = np;
            }
            step_mv(&ph[np++], QH_STEP_X_QUANT, qdim, m->actx, NULL, NULL, NULL, c->norm_eps, &Ly->p_out);
        } else {
            const int64_t gi = Ly->gdn_index;
            qh_step_phase *g = &ph[np++];
            g->kind = QH_STEP_GDN;
            g->eps = c->norm_eps;
            g->d_qkv = m->qkv;
            g->d_ring = m->ring + gi * c->conv_kernel * conv_dim;
            g->d_conv_w = Ly->conv_w;
            g->d_b = m->bt;
            g->d_a = m->at;
            g->d_dt_bias = Ly->dt_bias;
            g->d_ssm_a = Ly->ssm_a;
            g->d_state = m->state + gi * c->gdn_heads * (int64_t)c->gdn_head_dim * c->gdn_head_dim;
            g->d_z = m->z;
            g->d_norm_w = Ly->ssm_norm;
            g->d_y = m->gy;
            g->heads = c->gdn_heads;
            g->head_dim = c->gdn_head_dim;
            g->conv_kernel = c->conv_kernel;
            step_mv(&ph[np++], QH_STEP_X_QUANT, kdim, m->gy, NULL, NULL, NULL, c->norm_eps, &Ly->p_out);
        }
        pending = m->mix;
        // gate/up also form the SwiGLU row (each CTA its own rows), which the
        // down projection's phase only quantizes
        step_mv(&ph[np], QH_STEP_X_RESNORM, H, hc, pending, Ly->ffn_norm, hx, c->norm_eps, &Ly->p_ffn);
        ph[np++].d_act_out = m->fact;
        { float *t = hc; hc = hx; hx = t; }
        step_mv(&ph[np++], QH_STEP_X_QUANT, F, m->fact, NULL, NULL, NULL, c->norm_eps, &Ly->p_down);
        pending = m->mix;
    }
    step_mv(&ph[np++], QH_STEP_X_RESNORM, H, hc, pending, m->out_norm, hx, c->norm_eps, &m->p_head);
    m->seg[m->n_seg].first = first;
    m->seg[m->n_seg].count = np - first;
    m->seg[m->n_seg].attn_layer = -1;
    m->n_seg++;
    const int rc = qh_step_create(ph, np, m->d_ctl, &m->step_prog);
    free(ph);
    if (rc == QH_ERR_UNSUPPORTED) return QH_OK;
    if (rc) return rc;
    m->step_state = 1;
    return QH_OK;
}

static int forward_persistent(qh_slm *m) {
    const qh_slm_config *c = &m->cfg;
    const int32_t B = m->B;
    const int64_t H = c->hidden, hd = c->head_dim, kvd = (int64_t)c->n_kv_heads * hd;
    void *s = m->stream;
    CK(m->tok_embd.type == QH_GGUF_F32 ? qh_embed_f32((const float *)m->tok_embd.d, H, m->d_tok, B, m->h, s)
                                       : qh_embed_q6k(m->tok_embd.d, H, m->d_tok, B, m->h, s));
    for (int i = 0; i < m->n_seg; ++i) {
        CK(qh_step_run(m->step_prog, m->seg[i].first, m->seg[i].count, s));
        if (m->seg[i].attn_layer < 0) continue;
        const layer *Ly = &m->L[m->seg[i].attn_layer];
        const int64_t ai = Ly->attn_index;
        uint16_t *kc = m->kcache + ai * B * c->max_pos * kvd;
        uint16_t *vc = m->vcache + ai * B * c->max_pos * kvd;
        CK(qh_attn_pre(m->qraw, m->kb, m->vb, Ly->q_norm, Ly->k_norm, m->rope, B, c->n_heads, c->n_kv_heads,
                       (int32_t)hd, c->rope_dim, c->norm_eps, m->d_ctl, c->max_pos, m->aq, m->agate, kc, vc, s));
        CK(qh_attn_decode(m->aq, kc, vc, m->agate, B, c->n_heads, c->n_kv_heads, (int32_t)hd, m->d_ctl, c->max_pos,
                          m->actx, s));
    }
    if (m->sampling)
        CK(qh_sample_feed(m->logits, B, c->vocab, m->d_sctl, m->d_hist, c->max_pos + 1, m->d_hist_n, m->d_rng,
                          m->d_next, c->max_pos, m->d_ctl, m->d_tok, m->d_picks, m->d_sticket, s));
    else
        CK(qh_argmax_feed(m->logits, B, c->vocab, m->amax_scratch, m->d_next, m->d_prompt, c->max_pos, m->d_ctl,
                          m->d_tok, m->d_picks, s));
    return QH_OK;
}

static void drop_graphs(qh_slm *m) {
    for (int i = 0; i < 2; ++i) {
        if (m->graph_exec[i]) cudaGraphExecDestroy(m->graph_exec[i]);
        if (m->graph[i]) cudaGraphDestroy(m->graph[i]);
        m->graph_exec[i] = NULL;
        m->graph[i] = NULL;
        m->steps_run[i] = 0;
        m->no_graph[i] = 0;
    }
}

int qh_slm_set_decode_mode(qh_slm *m, int32_t mode) {
    if (!m || (mode != QH_DECODE_PERSISTENT && mode != QH_DECODE_LAUNCHES)) return QH_ERR_INVALID;
    if (mode == m->decode_mode) return QH_OK;
    if (qh_stream_sync(m->stream)) return QH_ERR_CUDA;
    drop_graphs(m);  // the next step captures the other form
    m->decode_mode = mode;
    return QH_OK;
}

int32_t qh_slm_decode_mode(const qh_slm *m) {
    if (!m) return -1;
    return m->decode_mode == QH_DECODE_PERSISTENT && m->step_state == 1 ? QH_DECODE_PERSISTENT : QH_DECODE_LAUNCHES;
}

int qh_slm_step_stamps(qh_slm *m, uint64_t *d_stamps) {
    if (!m) return QH_ERR_INVALID;
    if (m->decode_mode != QH_DECODE_PERSISTENT || m->step_state != 1) return QH_ERR_UNSUPPORTED;
    if (qh_stream_sync(m->stream)) return QH_ERR_CUDA;
    drop_graphs(m);
    CK(qh_step_set_stamps(m->step_prog, d_stamps));
    return qh_step_phase_count(m->step_prog);
}

// The step's operations, either form (not while tracing).
static int forward_step(qh_slm *m) {
    if (m->decode_mode == QH_DECODE_PERSISTENT && m->step_state == 1) return forward_persistent(m);
    return forward(m);
}

static int launch_step(qh_slm *m) {
    const int gi = m->sampling ? 1 : 0;
    if (m->decode_mode == QH_DECODE_PERSISTENT && m->step_state == 0) CK(build_step_prog(m));
    if (m->graph_exec[gi]) {
        if (cudaGraphLaunch(m->graph_exec[gi], m->stream) != cudaSuccess) return QH_ERR_CUDA;
        return QH_OK;
    }
    // the first run sets kernel attributes (and builds programs) outside a capture
    if (m->steps_run[gi]++ == 0 || m->no_graph[gi]) return forward_step(m);
    // capture the step once, then replay it; a step that cannot be captured
    // runs its launches directly from then on
    if (cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        m->no_graph[gi] = 1;
        return forward_step(m);
    }
    int rc = forward_step(m);
    cudaGraph_t g = NULL;
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rc || e != cudaSuccess || g == NULL) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        m->no_graph[gi] = 1;
        return forward_step(m);
    }
    if (cudaGraphInstantiate(&m->graph_exec[gi], g, 0) != cudaSuccess) {
        cudaGraphDestroy(g);
        m->graph_exec[gi] = NULL;
        cudaGetLastError();
        m->no_graph[gi] = 1;
        return forward_step(m);
    }
    m->graph[gi] = g;
    return cudaGraphLaunch(m->graph_exec[gi], m->stream) == cudaSuccess ? QH_OK : QH_ERR_CUDA;
}

int qh_slm_step(qh_slm *m, const int32_t *h_tokens, int32_t pos, int32_t *h_next, float *h_logits) {
    if (!m || !h_tokens || pos < 0 || pos >= m->cfg.max_pos) return QH_ERR_INVALID;
    memcpy(m->h_tok, h_tokens, sizeof(int32_t) * m->B);
    for (int32_t b = 0; b < m->B; ++b)
        if (m->h_tok[b] < 0 || m->h_tok[b] >= m->cfg.vocab) return QH_ERR_INVALID;
    m->h_ctl[0] = pos;
    m->h_ctl[1] = 0;
    CK(qh_memcpy_h2d(m->d_ctl, m->h_ctl, 2 * sizeof(int32_t), m->stream));
    CK(qh_memcpy_h2d(m->d_tok, m->h_tok, sizeof(int32_t) * m->B, m->stream));
    if (m->trace_fp) {  // a traced step runs its kernels directly
        const int rc = forward(m);
        fclose(m->trace_fp);
        m->trace_fp = NULL;
        CK(rc);
    } else {
        CK(launch_step(m));
    }
    m->host_pos = pos + 1;
    m->n_prompt = 0;
    CK(qh_memcpy_d2h(m->h_next, m->d_next, sizeof(int32_t) * m->B, m->stream));
    if (h_logits)
        CK(qh_memcpy_d2h(h_logits, m->logits, sizeof(float) * (size_t)m->B * m->cfg.vocab, m->stream));
    CK(qh_stream_sync(m->stream));
    CK(qh_check_device_error(NULL));
    if (h_next) memcpy(h_next, m->h_next, sizeof(int32_t) * m->B);
    return QH_OK;
}

// Prompt tokens prompt[s][0..n_prompt) as the inputs of positions
// p0 .. p0 + n_prompt - 1. p0 == 0 starts every sequence afresh (the conv
// ring and recurrent state are read before they are written, so they are
// cleared); p0 > 0 continues the sequences where the last step left them.
static int begin_at(qh_slm *m, const int32_t *prompt, int32_t n_prompt, int32_t p0) {
    if (!m || !prompt || n_prompt <= 0 || p0 < 0 || p0 + n_prompt > m->cfg.max_pos) return QH_ERR_INVALID;
    const int32_t B = m->B, P = m->cfg.max_pos;
    for (int64_t i = 0; i < (int64_t)B * n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->cfg.vocab) return QH_ERR_INVALID;
    if (p0 == 0) CK(qh_slm_reset(m));
    // prompt[s][i] -> d_prompt[s][p0 + i] (row pitch max_pos)
    if (cudaMemcpy2DAsync(m->d_prompt + p0, (size_t)P * 4, prompt, (size_t)n_prompt * 4, (size_t)n_prompt * 4,
                          (size_t)B, cudaMemcpyHostToDevice, m->stream) != cudaSuccess)
        return QH_ERR_CUDA;
    CK(qh_stream_sync(m->stream));  // the pinned staging buffers below are reused
    for (int32_t b = 0; b < B; ++b) m->h_tok[b] = prompt[(int64_t)b * n_prompt];
    m->h_ctl[0] = p0;
    m->h_ctl[1] = p0 + n_prompt;
    CK(qh_memcpy_h2d(m->d_ctl, m->h_ctl, 2 * sizeof(int32_t), m->stream));
    CK(qh_memcpy_h2d(m->d_tok, m->h_tok, sizeof(int32_t) * B, m->stream));
    CK(qh_stream_sync(m->stream));
    m->host_pos = p0;
    m->n_prompt = p0 + n_prompt;
    return QH_OK;
}

int qh_slm_begin(qh_slm *m, const int32_t *prompt, int32_t n_prompt) { return begin_at(m, prompt, n_prompt, 0); }

int32_t qh_slm_position(const qh_slm *m) { return m ? m->host_pos : -1; }

int qh_slm_advance(qh_slm *m, int32_t n_steps) {
    if (!m || n_steps < 0 || m->host_pos + n_steps > m->cfg.max_pos) return QH_ERR_INVALID;
    for (int32_t i = 0; i < n_steps; ++i) CK(launch_step(m));
    m->host_pos += n_steps;
    return QH_OK;
}

int qh_slm_picks(qh_slm *m, int32_t from_pos, int32_t n, int32_t *out) {
    if (!m || !out || from_pos < 0 || n < 0 || from_pos + n > m->host_pos) return QH_ERR_INVALID;
    if (n == 0) return QH_OK;
    const size_t P = (size_t)m->cfg.max_pos;
    if (cudaMemcpy2DAsync(out, (size_t)n * 4, m->d_picks + from_pos, P * 4, (size_t)n * 4, (size_t)m->B,
                          cudaMemcpyDeviceToHost, m->stream) != cudaSuccess)
        return QH_ERR_CUDA;
    CK(qh_stream_sync(m->stream));
    return qh_check_device_error(NULL);
}

// ---------------------------------------------------------------------------
// Prompt chunks: every projection of B x C prompt tokens as one tensor-core
// GEMM, the recurrence and attention per token inside one launch per layer.
// Bit-identical to feeding the prompt one token per step.
// ---------------------------------------------------------------------------
#define PF_MAX_ROWS 8192

static int ensure_prefill(qh_slm *m) {
    if (m->pf_chunk) return QH_OK;
    const qh_slm_config *c = &m->cfg;
    const int64_t B = m->B;
    int64_t C = m->pf_chunk_max > 0 ? m->pf_chunk_max : PF_MAX_ROWS / B;
    if (C < 1) C = 1;
    if (C > c->max_pos) C = c->max_pos;
    if (m->pf_mode == QH_PREFILL_CHUNKED) {
        // launches start on the 64-token chunk grid counted from position 0
        // (slm/qwen.c:777-780); a prompt shorter than max_pos fits one launch
        // when max_pos < 64
        C = C < 64 ? 64 : C / 64 * 64;
        if (C > c->max_pos) C = c->max_pos;
    }
    const int64_t M = B * C, H = c->hidden, F = c->ffn, hd = c->head_dim;
    const int64_t kdim = (int64_t)c->gdn_heads * c->gdn_head_dim, conv_dim = 3 * kdim;
    const int64_t qdim = (int64_t)c->n_heads * hd, kvd = (int64_t)c->n_kv_heads * hd;
    CK(alloc_f(m, &m->pf_h, M * H));
    CK(alloc_f(m, &m->pf_h2, M * H));
    CK(alloc_f(m, &m->pf_mix, M * H));
    CK(alloc_f(m, &m->pf_qkv, M * conv_dim));
    CK(alloc_f(m, &m->pf_z, M * kdim));
    CK(alloc_f(m, &m->pf_bt, M * c->gdn_heads));
    CK(alloc_f(m, &m->pf_at, M * c->gdn_heads));
    CK(alloc_f(m, &m->pf_qraw, M * 2 * qdim));
    CK(alloc_f(m, &m->pf_kb, M * kvd));
    CK(alloc_f(m, &m->pf_vb, M * kvd));
    CK(alloc_f(m, &m->pf_aq, M * qdim));
    CK(alloc_f(m, &m->pf_agate, M * qdim));
    CK(alloc_f(m, &m->pf_actx, M * qdim));
    CK(alloc_f(m, &m->pf_fgate, M * F));
    CK(alloc_f(m, &m->pf_fup, M * F));
    if (m->pf_mode == QH_PREFILL_CHUNKED) CK(alloc_f(m, &m->pf_o, M * kdim));
    const int64_t max_in = H > qdim ? H : qdim;
    CK(dev_alloc(m, &m->pf_xq_h, (size_t)qh_q8kt_bytes(max_in, M), NULL));
    CK(dev_alloc(m, &m->pf_xq_gdn, (size_t)qh_q8kt_bytes(kdim, M), NULL));
    CK(dev_alloc(m, &m->pf_xq_ffn, (size_t)qh_q8kt_bytes(F, M), NULL));
    CK(dev_alloc(m, (void **)&m->pf_tok, (size_t)M * 4, NULL));
    CK(dev_alloc(m, (void **)&m->pf_pos, 16, NULL));
    // Q8_0/F32 weights read fp32 rows: normalized inputs and the SwiGLU output
    int need_hn = m->p_head.n32, need_fact = 0;
    for (int l = 0; l < c->n_layers; ++l) {
        need_hn |= m->L[l].p_in.n32 | m->L[l].p_ffn.n32;
        need_fact |= m->L[l].p_down.n32;
        // the step-wise DeltaNet prompt kernel writes only the Q8_K rows of its output
        if (!m->L[l].is_attn && m->L[l].p_out.n32 && m->pf_mode != QH_PREFILL_CHUNKED) return QH_ERR_UNSUPPORTED;
    }
    if (need_hn) CK(alloc_f(m, &m->pf_hn, M * H));
    if (need_fact) CK(alloc_f(m, &m->pf_fact, M * F));
    for (int l = 0; l < c->n_layers; ++l) {
        layer *Ly = &m->L[l];
        if (Ly->is_attn) {
            const wref *w[3] = {&Ly->wq, &Ly->wk, &Ly->wv};
            float *o[3] = {m->pf_qraw, m->pf_kb, m->pf_vb};
            CK(make_set(m, &m->pf_in[l], 3, w, o, m->pf_xq_h, H, M, 1));
            const wref *w2[1] = {&Ly->wo};
            float *o2[1] = {m->pf_mix};
            CK(make_set(m, &m->pf_out[l], 1, w2, o2, m->pf_xq_h, qdim, M, 1));
            m->pf_out[l].x32 = m->pf_actx;
        } else {
            const wref *w[4] = {&Ly->qkv, &Ly->gate, &Ly->beta, &Ly->alpha};
            float *o[4] = {m->pf_qkv, m->pf_z, m->pf_bt, m->pf_at};
            CK(make_set(m, &m->pf_in[l], 4, w, o, m->pf_xq_h, H, M, 1));
            const wref *w2[1] = {&Ly->ssm_out};
            float *o2[1] = {m->pf_mix};
            CK(make_set(m, &m->pf_out[l], 1, w2, o2, m->pf_xq_gdn, kdim, M, 1));
            m->pf_out[l].x32 = m->pf_o;
        }
        m->pf_in[l].x32 = m->pf_hn;
        const wref *wf[2] = {&Ly->ffn_gate, &Ly->ffn_up};
        float *of_[2] = {m->pf_fgate, m->pf_fup};
        CK(make_set(m, &m->pf_ffn[l], 2, wf, of_, m->pf_xq_h, H, M, 1));
        m->pf_ffn[l].x32 = m->pf_hn;
        const wref *wd[1] = {&Ly->ffn_down};
        float *od[1] = {m->pf_mix};
        CK(make_set(m, &m->pf_down[l], 1, wd, od, m->pf_xq_ffn, F, M, 1));
        m->pf_down[l].x32 = m->pf_fact;
    }
    CK(qh_stream_sync(m->stream));  // tiled weights complete before any early weight stream
    m->pf_chunk = (int32_t)C;
    return QH_OK;
}

static int run_pf(qh_slm *m, plan_set *ps, int64_t rows) { return run_set(m, ps, rows, NULL, 0); }

// One chunk of cn tokens per sequence at positions *pf_pos .. + cn - 1;
// tokens in pf_tok (row = s * cn + j). Leaves caches, ring and state as cn
// decode steps would; computes no logits.
static int forward_prefill(qh_slm *m, int32_t cn) {
    const qh_slm_config *c = &m->cfg;
    const int32_t B = m->B;
    const int64_t M = (int64_t)B * cn, H = c->hidden, F = c->ffn, hd = c->head_dim;
    const int64_t kdim = (int64_t)c->gdn_heads * c->gdn_head_dim, conv_dim = 3 * kdim;
    const int64_t qdim = (int64_t)c->n_heads * hd, kvd = (int64_t)c->n_kv_heads * hd;
    void *s = m->stream;
    const int32_t T = QH_Q8KT_TILE_TOKENS;
    CK(m->tok_embd.type == QH_GGUF_F32
           ? qh_embed_f32((const float *)m->tok_embd.d, H, m->pf_tok, (int32_t)M, m->pf_h, s)
           : qh_embed_q6k(m->tok_embd.d, H, m->pf_tok, (int32_t)M, m->pf_h, s));
    float *hc = m->pf_h, *hx = m->pf_h2;
    const float *pending = NULL;
#define PF_RESNORM(w, xq, ps)                                                                              \
    do {                                                                                                   \
        CK(qh_rmsnorm_q8k(hc, pending, pending ? hx : NULL, (w), H, (int32_t)M, c->norm_eps, (xq), T, s)); \
        if (pending) { float *t_ = hc; hc = hx; hx = t_; }                                               \
        pending = NULL;                                                                                    \
        if ((ps)->n32) CK(qh_rmsnorm(hc, (w), H, M, c->norm_eps, m->pf_hn, s));                          \
    } while (0)
    for (int l = 0; l < c->n_layers; ++l) {
        layer *Ly = &m->L[l];
        PF_RESNORM(Ly->attn_norm, m->pf_xq_h, &m->pf_in[l]);
        CK(run_pf(m, &m->pf_in[l], M));
        if (Ly->is_attn) {
            const int64_t ai = Ly->attn_index;
            uint16_t *kc = m->kcache + ai * B * c->max_pos * kvd;
            uint16_t *vc = m->vcache + ai * B * c->max_pos * kvd;
            CK(qh_attn_prefill_pre(m->pf_qraw, m->pf_kb, m->pf_vb, Ly->q_norm, Ly->k_norm, m->rope, B, cn,
                                   c->n_heads, c->n_kv_heads, (int32_t)hd, c->rope_dim, c->norm_eps, m->pf_pos,
                                   c->max_pos, m->pf_aq, m->pf_agate, kc, vc, s));
            CK(qh_attn_prefill(m->pf_aq, kc, vc, m->pf_agate, B, cn, c->n_heads, c->n_kv_heads, (int32_t)hd,
                               m->pf_pos, c->max_pos, m->pf_actx, s));
            CK(qh_quantize_q8kt(m->pf_actx, qdim, M, m->pf_xq_h, s));
        } else {
            const int64_t gi = Ly->gdn_index;
            float *ring = m->ring + gi * B * c->conv_kernel * conv_dim;
            float *state = m->state + gi * B * c->gdn_heads * (int64_t)c->gdn_head_dim * c->gdn_head_dim;
            if (m->pf_mode == QH_PREFILL_CHUNKED) {
                // slm_forward_ssm_batch (slm/qwen.c:627-806): conv, norms, beta, g_log;
                // the chunk algebra; gated RMSNorm; then Q8_K for ssm_out
                CK(qh_gdn_chunk_prep(m->pf_qkv, ring, Ly->conv_w, m->pf_bt, m->pf_at, Ly->dt_bias, Ly->ssm_a, B, cn,
                                     c->gdn_heads, c->gdn_head_dim, c->conv_kernel, m->pf_pos, s));
                CK(qh_gdn_chunked(m->pf_qkv, m->pf_bt, m->pf_at, state, B, cn, c->gdn_heads, c->gdn_head_dim,
                                  m->pf_o, s));
                CK(qh_gdn_gated_norm(m->pf_o, m->pf_z, Ly->ssm_norm, (int32_t)M, c->gdn_heads, c->gdn_head_dim,
                                     c->norm_eps, m->pf_o, s));
                CK(qh_quantize_q8kt(m->pf_o, kdim, M, m->pf_xq_gdn, s));
            } else {
                CK(qh_gdn_prefill(m->pf_qkv, ring, Ly->conv_w, m->pf_bt, m->pf_at, Ly->dt_bias, Ly->ssm_a, state,
                                  m->pf_z, Ly->ssm_norm, B, cn, c->gdn_heads, c->gdn_head_dim, c->conv_kernel,
                                  c->norm_eps, m->pf_pos, m->pf_xq_gdn, T, s));
            }
        }
        CK(run_pf(m, &m->pf_out[l], M));
        pending = m->pf_mix;
        PF_RESNORM(Ly->ffn_norm, m->pf_xq_h, &m->pf_ffn[l]);
        CK(run_pf(m, &m->pf_ffn[l], M));
        CK(qh_swiglu_q8k(m->pf_fgate, m->pf_fup, F, (int32_t)M, m->pf_xq_ffn, T, s));
        if (m->pf_down[l].n32) CK(qh_swiglu(m->pf_fgate, m->pf_fup, m->pf_fact, M * F, s));
        CK(run_pf(m, &m->pf_down[l], M));
        pending = m->pf_mix;
    }
#undef PF_RESNORM
    return QH_OK;
}

int qh_slm_set_prefill_chunk(qh_slm *m, int32_t max_tokens_per_seq) {
    if (!m || max_tokens_per_seq < 0) return QH_ERR_INVALID;
    if (m->pf_chunk) return max_tokens_per_seq == 0 || max_tokens_per_seq == m->pf_chunk ? QH_OK : QH_ERR_INVALID;
    m->pf_chunk_max = max_tokens_per_seq;
    return QH_OK;
}

int qh_slm_set_prefill_mode(qh_slm *m, int32_t mode) {
    if (!m || (mode != QH_PREFILL_STEPWISE && mode != QH_PREFILL_CHUNKED)) return QH_ERR_INVALID;
    if (m->pf_chunk) return mode == m->pf_mode ? QH_OK : QH_ERR_INVALID;
    m->pf_mode = mode;
    return QH_OK;
}

int qh_slm_prefill_at(qh_slm *m, const int32_t *prompt, int32_t n_prompt, int32_t pos) {
    CK(begin_at(m, prompt, n_prompt, pos));
    const int32_t n_ctx = n_prompt - 1;  // the last prompt token is the next step's input
    if (n_ctx == 0) return QH_OK;
    const qh_slm_config *c = &m->cfg;
    if (c->head_dim != 128 || c->gdn_head_dim != 128 || c->conv_kernel != 4) return QH_ERR_UNSUPPORTED;
    // the chunk algebra counts its 64-token chunks from position 0
    if (m->pf_mode == QH_PREFILL_CHUNKED && pos % 64) return QH_ERR_UNSUPPORTED;
    CK(ensure_prefill(m));
    const int32_t B = m->B, C = m->pf_chunk;
    int32_t *tok = (int32_t *)malloc(sizeof(int32_t) * (size_t)B * C);
    if (!tok) return QH_ERR_INVALID;
    int rc = QH_OK;
    for (int32_t j0 = 0; j0 < n_ctx && !rc; j0 += C) {
        const int32_t cn = n_ctx - j0 < C ? n_ctx - j0 : C, p0 = pos + j0;
        for (int32_t b = 0; b < B; ++b)
            for (int32_t j = 0; j < cn; ++j) tok[(int64_t)b * cn + j] = prompt[(int64_t)b * n_prompt + j0 + j];
        // pageable sources: the copies are staged before these calls return
        rc = qh_memcpy_h2d(m->pf_tok, tok, sizeof(int32_t) * (size_t)B * cn, m->stream);
        if (!rc) rc = qh_memcpy_h2d(m->pf_pos, &p0, sizeof(int32_t), m->stream);
        if (!rc) rc = forward_prefill(m, cn);
    }
    free(tok);
    if (rc) return rc;
    // next step: position pos + n_ctx, input the last prompt token
    for (int32_t b = 0; b < B; ++b) m->h_tok[b] = prompt[(int64_t)b * n_prompt + n_ctx];
    m->h_ctl[0] = pos + n_ctx;
    m->h_ctl[1] = pos + n_prompt;
    CK(qh_memcpy_h2d(m->d_ctl, m->h_ctl, 2 * sizeof(int32_t), m->stream));
    CK(qh_memcpy_h2d(m->d_tok, m->h_tok, sizeof(int32_t) * B, m->stream));
    CK(qh_stream_sync(m->stream));
    CK(qh_check_device_error(NULL));
    m->host_pos = pos + n_ctx;
    return QH_OK;
}

int qh_slm_prefill(qh_slm *m, const int32_t *prompt, int32_t n_prompt) {
    return qh_slm_prefill_at(m, prompt, n_prompt, 0);
}

int qh_slm_generate(qh_slm *m, const int32_t *prompt, int32_t n_prompt, int32_t n_new, int32_t *out) {
    if (!m || !prompt || !out || n_prompt <= 0 || n_new < 0 || n_prompt + n_new - 1 > m->cfg.max_pos)
        return QH_ERR_INVALID;
    // the prompt in chunks (all but its last token), then one step per
    // token: the step at n_prompt - 1 consumes the last prompt token and
    // picks the first generated one
    CK(qh_slm_prefill(m, prompt, n_prompt));
    if (n_new == 0) return QH_OK;
    CK(qh_slm_advance(m, n_new));
    return qh_slm_picks(m, n_prompt - 1, n_new, out);
}

int qh_slm_sample_setup(qh_slm *m, const qh_sampler *sp, const uint64_t *seeds, int32_t eos_id, int32_t eot_id,
                        int32_t min_new, const int32_t *hist, int32_t n_hist) {
    if (!m || !sp || n_hist < 0 || n_hist > m->cfg.max_pos || (n_hist > 0 && !hist)) return QH_ERR_INVALID;
    const int32_t B = m->B, P = m->cfg.max_pos;
    int rc = QH_OK;
    int32_t *hn = (int32_t *)malloc(sizeof(int32_t) * (size_t)B);
    uint64_t *st = (uint64_t *)malloc(16 * (size_t)B);
    if (!hn || !st) rc = QH_ERR_INVALID;
    // the repetition-penalty history (slm/slm.c:257-263)
    if (!rc && n_hist > 0 &&
        cudaMemcpy2DAsync(m->d_hist, (size_t)(P + 1) * 4, hist, (size_t)n_hist * 4, (size_t)n_hist * 4, (size_t)B,
                          cudaMemcpyHostToDevice, m->stream) != cudaSuccess)
        rc = QH_ERR_CUDA;
    for (int32_t b = 0; b < B && !rc; ++b) hn[b] = n_hist;
    if (!rc) rc = qh_memcpy_h2d(m->d_hist_n, hn, sizeof(int32_t) * (size_t)B, m->stream);
    // a non-zero seed re-seeds a sequence's generator; zero continues it
    if (!rc && seeds) {
        rc = qh_memcpy_d2h(st, m->d_rng, 16 * (size_t)B, m->stream);
        if (!rc) rc = qh_stream_sync(m->stream);
        for (int32_t b = 0; b < B && !rc; ++b)
            if (seeds[b] != 0) qh_rng_seed(seeds[b], st + 2 * b);
        if (!rc) rc = qh_memcpy_h2d(m->d_rng, st, 16 * (size_t)B, m->stream);
    }
    if (!rc) {
        qh_sample_ctl sc;
        memset(&sc, 0, sizeof(sc));
        sc.sp = *sp;
        sc.eos_id = eos_id;
        sc.eot_id = eot_id;
        sc.min_new = min_new;
        sc.gen0 = m->host_pos;  // the next step is the first sampled one
        rc = qh_memcpy_h2d(m->d_sctl, &sc, sizeof(sc), m->stream);
        if (!rc) rc = qh_stream_sync(m->stream);
    }
    free(hn);
    free(st);
    return rc;
}

int qh_slm_sample_steps(qh_slm *m, int32_t n_steps, int32_t *out) {
    if (!m || n_steps < 0 || (n_steps > 0 && !out) || m->host_pos + n_steps > m->cfg.max_pos) return QH_ERR_INVALID;
    if (n_steps == 0) return QH_OK;
    const int32_t p0 = m->host_pos;
    m->sampling = 1;
    int rc = qh_slm_advance(m, n_steps);
    m->sampling = 0;
    if (!rc) rc = qh_slm_picks(m, p0, n_steps, out);
    return rc;
}

int qh_slm_generate_sampled(qh_slm *m, const int32_t *prompt, int32_t n_prompt, int32_t max_new, int32_t min_new,
                            const qh_sampler *sp, const uint64_t *seeds, int32_t eos_id, int32_t eot_id,
                            const int32_t *stop_ids, int32_t n_stop, int32_t *out, int32_t *n_out) {
    if (!m || !prompt || !sp || !out || !n_out || n_prompt <= 0 || max_new < 0 || n_stop < 0 ||
        (n_stop > 0 && !stop_ids) || n_prompt >= m->cfg.max_pos)
        return QH_ERR_INVALID;
    const int32_t B = m->B, P = m->cfg.max_pos, n = n_prompt;
    // slm_generate_raw's decode loop runs while pos < max_position
    const int32_t n_gen = max_new < P - n ? max_new : P - n;
    // prompt at positions 0..n-1, then the decode loop re-feeds the last
    // prompt token at position n: a prefill of the prompt plus that token
    // leaves exactly this state with the token pending at position n
    int32_t *ext = (int32_t *)malloc(sizeof(int32_t) * (size_t)B * (n + 1));
    int32_t *picks = (int32_t *)malloc(sizeof(int32_t) * (size_t)B * (n_gen > 0 ? n_gen : 1));
    int rc = (ext && picks) ? QH_OK : QH_ERR_INVALID;
    if (!rc) {
        for (int32_t b = 0; b < B; ++b) {
            memcpy(ext + (int64_t)b * (n + 1), prompt + (int64_t)b * n, sizeof(int32_t) * (size_t)n);
            ext[(int64_t)b * (n + 1) + n] = prompt[(int64_t)b * n + n - 1];
        }
        rc = qh_slm_prefill(m, ext, n + 1);
    }
    // the history starts as this call's prompt (slm/slm.c:257-263)
    if (!rc) rc = qh_slm_sample_setup(m, sp, seeds, eos_id, eot_id, min_new, prompt, n);
    if (!rc) rc = qh_slm_sample_steps(m, n_gen, picks);
    if (!rc) {
        // a sequence ends at its first eos, eot or stop token, which is
        // counted (slm/slm.c:330-341)
        for (int32_t b = 0; b < B; ++b) {
            int32_t cnt = n_gen;
            for (int32_t i = 0; i < n_gen; ++i) {
                const int32_t t = picks[(int64_t)b * n_gen + i];
                int stop = t == eos_id || t == eot_id;
                for (int32_t j = 0; j < n_stop && !stop; ++j) stop = t == stop_ids[j];
                out[(int64_t)b * max_new + i] = t;
                if (stop) { cnt = i + 1; break; }
            }
            n_out[b] = cnt;
        }
    }
    free(ext);
    free(picks);
    return rc;
}

// ---------------------------------------------------------------------------
// Snapshot / restore (slm_ctx_snapshot / slm_ctx_restore, slm/model.c:1262-
// 1371): a device-memory copy of everything a step reads and writes --
// position and feed state, generator words, KV rows 0..pos-1 of every
// attention layer, conv rings and recurrent states, prompts, picks and the
// sampler history.
// ---------------------------------------------------------------------------
struct qh_slm_snap {
    const qh_slm *owner;
    int32_t host_pos, n_prompt, kv_rows;
    int64_t bytes;
    void *ctl, *tok, *next, *rng, *picks, *prompt, *hist, *hist_n, *ring, *state, *k, *v;
};

typedef struct {
    void **snap_field;
    void *model_buf;
    size_t bytes;
} snap_part;

static int snap_parts(const qh_slm *m, qh_slm_snap *s, snap_part *parts) {
    const qh_slm_config *c = &m->cfg;
    const int64_t B = m->B, kdim = (int64_t)c->gdn_heads * c->gdn_head_dim;
    const int64_t ng = m->n_gdn > 0 ? m->n_gdn : 1;
    int n = 0;
#define PART(field, buf, nb) parts[n++] = (snap_part){(void **)&s->field, (void *)(buf), (size_t)(nb)}
    PART(ctl, m->d_ctl, 16);
    PART(tok, m->d_tok, B * 4);
    PART(next, m->d_next, B * 4);
    PART(rng, m->d_rng, B * 16);
    PART(picks, m->d_picks, B * c->max_pos * 4);
    PART(prompt, m->d_prompt, B * c->max_pos * 4);
    PART(hist, m->d_hist, B * (c->max_pos + 1) * 4);
    PART(hist_n, m->d_hist_n, B * 4);
    PART(ring, m->ring, ng * B * c->conv_kernel * 3 * kdim * 4);
    PART(state, m->state, ng * B * c->gdn_heads * (int64_t)c->gdn_head_dim * c->gdn_head_dim * 4);
#undef PART
    return n;
}

int qh_slm_snapshot(qh_slm *m, qh_slm_snap **out) {
    if (!m || !out) return QH_ERR_INVALID;
    *out = NULL;
    const qh_slm_config *c = &m->cfg;
    qh_slm_snap *s = (qh_slm_snap *)calloc(1, sizeof(qh_slm_snap));
    if (!s) return QH_ERR_INVALID;
    s->owner = m;
    s->host_pos = m->host_pos;
    s->n_prompt = m->n_prompt;
    s->kv_rows = m->host_pos;
    snap_part parts[16];
    const int np = snap_parts(m, s, parts);
    int rc = QH_OK;
    for (int i = 0; i < np && !rc; ++i) {
        rc = qh_malloc(parts[i].snap_field, parts[i].bytes);
        if (!rc && cudaMemcpyAsync(*parts[i].snap_field, parts[i].model_buf, parts[i].bytes, cudaMemcpyDeviceToDevice,
                                   m->stream) != cudaSuccess)
            rc = QH_ERR_CUDA;
        s->bytes += (int64_t)parts[i].bytes;
    }
    // KV rows 0..pos-1: the (layer, sequence) rows of a cache share one pitch
    const int64_t kvd = (int64_t)c->n_kv_heads * c->head_dim, rows = (int64_t)m->n_attn * m->B;
    if (!rc && s->kv_rows > 0 && rows > 0) {
        const size_t w = (size_t)s->kv_rows * kvd * 2, pitch = (size_t)c->max_pos * kvd * 2;
        rc = qh_malloc(&s->k, w * rows);
        if (!rc) rc = qh_malloc(&s->v, w * rows);
        if (!rc && (cudaMemcpy2DAsync(s->k, w, m->kcache, pitch, w, (size_t)rows, cudaMemcpyDeviceToDevice,
                                      m->stream) != cudaSuccess ||
                    cudaMemcpy2DAsync(s->v, w, m->vcache, pitch, w, (size_t)rows, cudaMemcpyDeviceToDevice,
                                      m->stream) != cudaSuccess))
            rc = QH_ERR_CUDA;
        s->bytes += 2 * (int64_t)(w * rows);
    }
    if (!rc) rc = qh_stream_sync(m->stream);
    if (rc) {
        qh_slm_snapshot_free(s);
        return rc;
    }
    *out = s;
    return QH_OK;
}

int qh_slm_restore(qh_slm *m, const qh_slm_snap *s) {
    if (!m || !s || s->owner != m) return QH_ERR_INVALID;
    const qh_slm_config *c = &m->cfg;
    qh_slm_snap view = *s;
    snap_part parts[16];
    const int np = snap_parts(m, &view, parts);
    for (int i = 0; i < np; ++i)
        if (cudaMemcpyAsync(parts[i].model_buf, *parts[i].snap_field, parts[i].bytes, cudaMemcpyDeviceToDevice,
                            m->stream) != cudaSuccess)
            return QH_ERR_CUDA;
    const int64_t kvd = (int64_t)c->n_kv_heads * c->head_dim, rows = (int64_t)m->n_attn * m->B;
    if (s->kv_rows > 0 && rows > 0) {
        const size_t w = (size_t)s->kv_rows * kvd * 2, pitch = (size_t)c->max_pos * kvd * 2;
        if (cudaMemcpy2DAsync(m->kcache, pitch, s->k, w, w, (size_t)rows, cudaMemcpyDeviceToDevice, m->stream) !=
                cudaSuccess ||
            cudaMemcpy2DAsync(m->vcache, pitch, s->v, w, w, (size_t)rows, cudaMemcpyDeviceToDevice, m->stream) !=
                cudaSuccess)
            return QH_ERR_CUDA;
    }
    CK(qh_stream_sync(m->stream));
    m->host_pos = s->host_pos;
    m->n_prompt = s->n_prompt;
    return QH_OK;
}

void qh_slm_snapshot_free(qh_slm_snap *s) {
    if (!s) return;
    void *bufs[] = {s->ctl, s->tok, s->next, s->rng, s->picks, s->prompt, s->hist, s->hist_n, s->ring, s->state,
                    s->k, s->v};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); ++i)
        if (bufs[i]) qh_free(bufs[i]);
    free(s);
}

int64_t qh_slm_snapshot_bytes(const qh_slm_snap *s) { return s ? s->bytes : -1; }

int32_t qh_slm_snapshot_pos(const qh_slm_snap *s) { return s ? s->host_pos : -1; }

void *qh_slm_stream(const qh_slm *m) { return m ? (void *)m->stream : NULL; }

const int32_t *qh_slm_device_next(const qh_slm *m) { return m ? m->d_next : NULL; }

int qh_slm_memory(const qh_slm *m, int64_t *weight_bytes, int64_t *state_bytes) {
    if (!m) return QH_ERR_INVALID;
    if (weight_bytes) *weight_bytes = m->weight_bytes;
    if (state_bytes) *state_bytes = m->state_bytes;
    return QH_OK;
}
