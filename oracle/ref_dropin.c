// SPDX-License-Identifier: MIT
//
// ref_dropin.c -- the reference's matmul entry points (tensor_matmul_q4k_f32,
// _q5k_, _q6k_, _q8_0_ and tensor_matmul_f32; slm/tensor.c:517, 827, 898,
// 952, 1012) implemented on the GPU through this repository's C-ABI
// (include/qh_backend.h): the host activations are copied to the device,
// qh_matmul computes the product there, and the result lands in a new
// tensor of the caller's arena, as the reference's functions return it.
//
// TEST INFRASTRUCTURE, NOT PRODUCT CODE: it shows the drop-in boundary at
// work. Loaded into a process with RTLD_GLOBAL before the reference's own
// library (oracle/_ref/libqhref.so), its definitions take the place of the
// reference's: matmul_dispatch (slm/model.c:220-264) reaches the
// tensor_matmul_* functions through the dynamic linker, so the reference's
// unmodified forward pass (slm_forward_step, slm/qwen.c:874-981) then runs
// every projection on the GPU. The reference's struct tensor stays opaque:
// its fields are read through the accessors oracle/ref_harness.c exports.
//
// Weights are copied to the device once per host pointer (the reference's
// weights are immutable after load) and kept until the process exits.
// Not thread-safe, like a reference context. libqh200.so is opened with
// RTLD_LOCAL, so its own symbols (it exports the slm.h names too) never
// shadow the reference's.

#include <dlfcn.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../include/qh_backend.h"

struct tensor;  // the reference's, opaque here

// the C-ABI entry points used, bound from libqh200.so by dropin_init
#define QH_FNS(X)                                                                                         \
    X(int, qh_malloc, (void **, size_t))                                                                  \
    X(int, qh_free, (void *))                                                                             \
    X(int, qh_memcpy_h2d, (void *, const void *, size_t, void *))                                         \
    X(int, qh_memcpy_d2h, (void *, const void *, size_t, void *))                                         \
    X(int, qh_stream_sync, (void *))                                                                      \
    X(const char *, qh_last_error, (void))                                                                \
    X(int64_t, qh_matmul_workspace_bytes, (int, int64_t, int64_t))                                        \
    X(int, qh_matmul, (int, const void *, int64_t, int64_t, const float *, int64_t, float *, void *, int64_t, void *))
#define DECL(ret, name, args) static ret(*p_##name) args;
QH_FNS(DECL)
#undef DECL

static float *(*t_data)(const struct tensor *);
static int64_t (*t_ne)(const struct tensor *, int);
static struct tensor *(*t_new_like)(const struct tensor *, int64_t, int64_t);

static struct {
    const void *host;
    void *dev;
} g_w[4096];
static int g_nw;
static void *g_x, *g_out, *g_work;
static int64_t g_x_cap, g_out_cap, g_work_cap;
static int64_t g_calls[16];  // by GGUF type id

// Binds the accessors of the reference library at `ref_path` (already
// loaded) and the C-ABI of libqh200.so at `qh_path`. Returns 0 on success.
int dropin_init(const char *ref_path, const char *qh_path) {
    void *q = dlopen(qh_path, RTLD_NOW | RTLD_LOCAL);
    if (!q) return -1;
#define BIND(ret, name, args) p_##name = (ret(*) args)dlsym(q, #name); if (!p_##name) return -1;
    QH_FNS(BIND)
#undef BIND
    void *h = dlopen(ref_path, RTLD_LAZY | RTLD_NOLOAD);
    if (!h) return -1;
    t_data = (float *(*)(const struct tensor *))dlsym(h, "ref_tensor_data");
    t_ne = (int64_t(*)(const struct tensor *, int))dlsym(h, "ref_tensor_ne");
    t_new_like = (struct tensor * (*)(const struct tensor *, int64_t, int64_t)) dlsym(h, "ref_tensor_new_like");
    return t_data && t_ne && t_new_like ? 0 : -1;
}

// Calls of each weight type served on the GPU so far.
int64_t dropin_calls(int type) { return type >= 0 && type < 16 ? g_calls[type] : -1; }

static void die(const char *what) {
    fprintf(stderr, "ref_dropin: %s: %s\n", what, p_qh_last_error());
    abort();  // where the reference itself aborts (slm/model.c:259-261)
}

static void *grow(void **p, int64_t *cap, int64_t bytes) {
    if (bytes > *cap) {
        if (*p) p_qh_free(*p);
        if (p_qh_malloc(p, (size_t)bytes)) die("qh_malloc");
        *cap = bytes;
    }
    return *p;
}

static const void *device_weights(const void *host, int64_t bytes) {
    for (int i = 0; i < g_nw; ++i)
        if (g_w[i].host == host) return g_w[i].dev;
    if (g_nw == (int)(sizeof(g_w) / sizeof(g_w[0]))) die("too many weight tensors");
    void *d = NULL;
    if (p_qh_malloc(&d, (size_t)bytes) || p_qh_memcpy_h2d(d, host, (size_t)bytes, NULL) || p_qh_stream_sync(NULL))
        die("weight upload");
    g_w[g_nw].host = host;
    g_w[g_nw].dev = d;
    g_nw++;
    return d;
}

// out[t][j] for the n tokens of x (x->ne[0] == k, ne[1] == n), on the GPU.
static struct tensor *gpu_matmul(int type, const void *w, int64_t w_bytes, int64_t out_f, int64_t k,
                                 struct tensor *x) {
    if (!t_data) die("dropin_init was not called");
    const int64_t n = t_ne(x, 1);
    struct tensor *out = t_new_like(x, out_f, n);
    const void *dw = device_weights(w, w_bytes);
    const int64_t wb = p_qh_matmul_workspace_bytes(type, k, n);
    if (wb < 0) die("unsupported type");
    float *dx = (float *)grow(&g_x, &g_x_cap, 4 * k * n);
    float *dout = (float *)grow(&g_out, &g_out_cap, 4 * out_f * n);
    void *work = wb > 0 ? grow(&g_work, &g_work_cap, wb) : NULL;
    if (p_qh_memcpy_h2d(dx, t_data(x), (size_t)(4 * k * n), NULL)) die("activations");
    if (p_qh_matmul(type, dw, k, out_f, dx, n, dout, work, wb, NULL)) die("qh_matmul");
    if (p_qh_memcpy_d2h(t_data(out), dout, (size_t)(4 * out_f * n), NULL) || p_qh_stream_sync(NULL)) die("result");
    g_calls[type]++;
    return out;
}

struct tensor *tensor_matmul_q4k_f32(const void *w, int64_t out_f, int64_t k, struct tensor *x) {
    return gpu_matmul(QH_TYPE_Q4_K, w, out_f * (k / 256) * 144, out_f, k, x);
}
struct tensor *tensor_matmul_q5k_f32(const void *w, int64_t out_f, int64_t k, struct tensor *x) {
    return gpu_matmul(QH_TYPE_Q5_K, w, out_f * (k / 256) * 176, out_f, k, x);
}
struct tensor *tensor_matmul_q6k_f32(const void *w, int64_t out_f, int64_t k, struct tensor *x) {
    return gpu_matmul(QH_TYPE_Q6_K, w, out_f * (k / 256) * 210, out_f, k, x);
}
struct tensor *tensor_matmul_q8_0_f32(const void *w, int64_t out_f, int64_t k, struct tensor *x) {
    return gpu_matmul(QH_TYPE_Q8_0, w, out_f * (k / 32) * 34, out_f, k, x);
}
// w: the fp32 view of shape (k, out_f) matmul_dispatch builds (slm/model.c:226-240)
struct tensor *tensor_matmul_f32(struct tensor *w, struct tensor *x) {
    const int64_t k = t_ne(w, 0), out_f = t_ne(w, 1);
    return gpu_matmul(QH_TYPE_F32, t_data(w), 4 * k * out_f, out_f, k, x);
}
