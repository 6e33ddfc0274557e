// SPDX-License-Identifier: MIT
//
// qh_api.cu -- the extern "C" entry points of include/qh_backend.h:
// argument checking, status codes, workspace layout and kernel launches.

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "../../include/qh_backend.h"
#include "qh_internal.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    cudaGetLastError();  // clear a sticky launch error so later calls start clean
    return fail(QH_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
int *g_err_words[kMaxDevices] = {nullptr};
int g_sm_count[kMaxDevices] = {0};

int current_device(int *dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (*dev < 0 || *dev >= kMaxDevices) return fail(QH_ERR_INVALID, "device id %d out of range", *dev);
    return QH_OK;
}

// Per-device state: SM count and the device error word (allocated once).
int device_state(int *sm_count, int **err_word) {
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_dev_mu);
    if (g_sm_count[dev] == 0) {
        int sms = 0;
        cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        int *w = nullptr;
        e = cudaMalloc(&w, sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(error word)");
        e = cudaMemset(w, 0, sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error word)");
        g_err_words[dev] = w;
        g_sm_count[dev] = sms;
    }
    if (sm_count) *sm_count = g_sm_count[dev];
    if (err_word) *err_word = g_err_words[dev];
    return QH_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_shape(int type, int64_t k, int64_t out_f, int64_t n_tok) {
    if (qhf_block_bytes(type) == 0)
        return fail(QH_ERR_UNSUPPORTED, "matmul: unsupported weight type %d", type);
    const int64_t bw = qhf_block_weights(type);
    if (k <= 0 || k % bw) return fail(QH_ERR_INVALID, "matmul: k=%lld not a multiple of %lld",
                                      (long long)k, (long long)bw);
    if (out_f <= 0 || out_f > (1ll << 30)) return fail(QH_ERR_INVALID, "matmul: bad out_f %lld", (long long)out_f);
    if (n_tok <= 0 || n_tok > 65535) return fail(QH_ERR_INVALID, "matmul: bad n_tok %lld", (long long)n_tok);
    if (qhf_row_bytes(type, k) > (1ll << 30)) return fail(QH_ERR_INVALID, "matmul: row too long");
    return QH_OK;
}

int64_t act_bytes(int type, int64_t k, int64_t n_tok) {
    return type == QH_GGUF_Q8_0 ? qhf_q8_0_total_bytes(k, n_tok) : qhf_q8k_total_bytes(k, n_tok);
}

// Fills a GemvJob for tokens [t0, t0 + nt) of a matmul whose activations are
// in split buffer `xq` quantized for n_tok rows.
qh::GemvJob make_job(int type, const void *w, int64_t k, int64_t out_f, const void *xq,
                     int64_t n_tok, int64_t t0, float *out) {
    const uint8_t *base = static_cast<const uint8_t *>(xq);
    qh::GemvJob j{};
    j.w = static_cast<const uint8_t *>(w);
    j.k = static_cast<int32_t>(k);
    j.nb = static_cast<int32_t>(k / qhf_block_weights(type));
    j.row_bytes = static_cast<int32_t>(qhf_row_bytes(type, k));
    j.n_rows = static_cast<int32_t>(out_f);
    j.xqs = reinterpret_cast<const int8_t *>(base) + t0 * k;
    if (type == QH_GGUF_Q8_0) {
        j.d_stride = static_cast<int32_t>(qhf_q8_0_d_stride(k));
        j.xd = base + qhf_q8_0_d_offset(k, n_tok) + t0 * j.d_stride * 2;
        j.xbs = nullptr;
    } else {
        j.d_stride = static_cast<int32_t>(qhf_q8k_d_stride(k));
        j.xd = base + qhf_q8k_d_offset(k, n_tok) + t0 * j.d_stride * 4;
        j.xbs = reinterpret_cast<const int16_t *>(base + qhf_q8k_bsums_offset(k, n_tok)) + t0 * j.nb * 16;
    }
    j.out = out + t0 * out_f;
    return j;
}

int run_preq(int type, const void *d_w, int64_t k, int64_t out_f, const void *d_xq, int64_t n_tok,
             float *d_out, cudaStream_t s) {
    int sms;
    int *err;
    int rc = device_state(&sms, &err);
    if (rc) return rc;
    return qh::matmul_preq_launch(type, d_w, k, out_f, d_xq, n_tok, d_out, s, sms, err);
}

int matmul_f32_impl(const float *d_w, int64_t k, int64_t out_f, const float *d_x, int64_t n_tok, float *d_out,
                    void *stream) {
    if (k <= 0 || out_f <= 0 || out_f > (1ll << 30) || n_tok <= 0 || n_tok > 65535 || k > (1ll << 28))
        return fail(QH_ERR_INVALID, "matmul f32: bad shape k=%lld out_f=%lld n_tok=%lld", (long long)k,
                    (long long)out_f, (long long)n_tok);
    if (!d_w || !d_x || !d_out) return fail(QH_ERR_INVALID, "matmul f32: null pointer");
    cudaError_t e = qh::matmul_f32_launch(d_w, k, out_f, d_x, n_tok, d_out, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "matmul f32 launch");
    return QH_OK;
}

int matmul_impl(int type, const void *d_w, int64_t k, int64_t out_f, const float *d_x,
                int64_t n_tok, float *d_out, void *d_work, int64_t work_bytes, void *stream) {
    if (type == QH_GGUF_F32)  // no quantization, no workspace
        return matmul_f32_impl(static_cast<const float *>(d_w), k, out_f, d_x, n_tok, d_out, stream);
    int rc = check_shape(type, k, out_f, n_tok);
    if (rc) return rc;
    if (!d_w || !d_x || !d_out) return fail(QH_ERR_INVALID, "matmul: null pointer");
    if (!aligned16(d_w)) return fail(QH_ERR_ALIGN, "matmul: weight pointer not 16-byte aligned");
    if (!d_work || !aligned16(d_work)) return fail(QH_ERR_WORKSPACE, "matmul: workspace missing or not 16-byte aligned");
    if (work_bytes < act_bytes(type, k, n_tok))
        return fail(QH_ERR_WORKSPACE, "matmul: workspace %lld bytes < %lld needed",
                    (long long)work_bytes, (long long)act_bytes(type, k, n_tok));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = type == QH_GGUF_Q8_0 ? qh::quantize_q8_0_launch(d_x, k, n_tok, d_work, s)
                                         : qh::quantize_q8k_launch(d_x, k, n_tok, d_work, s);
    if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
    return run_preq(type, d_w, k, out_f, d_work, n_tok, d_out, s);
}

}  // namespace

namespace qh {
void set_last_error_message(const char *msg) { snprintf(g_err, sizeof(g_err), "%s", msg); }

int *device_error_word() {
    int *w = nullptr;
    device_state(nullptr, &w);
    return w;
}

int matmul_preq_launch(int type, const void *d_w, int64_t k, int64_t out_f, const void *d_xq, int64_t n_tok,
                       float *d_out, cudaStream_t s, int sm_count, int *err_word) {
    if (type == QH_GGUF_Q8_0 && n_tok > 8) {  // one launch over all tokens (same lane arithmetic)
        cudaError_t e = matmul_q8_0_many_launch(d_w, k, out_f, d_xq, n_tok, 0, n_tok, d_out, s);
        return e == cudaSuccess ? QH_OK : cuda_fail(e, "q8_0 matmul launch");
    }
    int chunk = 8;  // tokens per launch; halved while a stage cannot hold them
    for (int64_t t0 = 0; t0 < n_tok; t0 += chunk) {
        GemvParams p{};
        GemvGeometry g{};
        cudaError_t e;
        for (;;) {
            const int nt = static_cast<int>(n_tok - t0 < chunk ? n_tok - t0 : chunk);
            GemvJob job = make_job(type, d_w, k, out_f, d_xq, n_tok, t0, d_out);
            e = gemv_plan(type, &job, 1, nt, sm_count, &p, &g);
            if (e == cudaSuccess || chunk == 1) break;
            chunk >>= 1;
        }
        if (e != cudaSuccess) return fail(QH_ERR_INVALID, "matmul: cannot tile rows of %lld bytes (%s)",
                                          (long long)qhf_row_bytes(type, k), cudaGetErrorString(e));
        p.err_flag = err_word;
        p.table = nullptr;
        e = gemv_launch(type, p, g, s);
        if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
    }
    return QH_OK;
}
}  // namespace qh

struct qh_matvec_plan_s {
    int type;
    int device;
    int n_tok, sms;
    std::vector<qh::GemvJob> jobs;  // as planned (for re-planning with a fused input)
    qh::GemvParams params;
    qh::GemvGeometry geom;
    qh::GemvJob *d_table;
    unsigned *d_ticket;             // output tail's arrival counter (qh_matvec_plan_fuse_output)
};

extern "C" {

// For the library's C sources (not in a public header).
void qh_internal_set_error(const char *msg) { snprintf(g_err, sizeof(g_err), "%s", msg); }

const char *qh_version(void) { return "qh200 0.1.0 (sm_100a)"; }
const char *qh_last_error(void) { return g_err; }

int qh_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int qh_set_device(int device) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    return device_state(nullptr, nullptr);
}

int qh_malloc(void **d_ptr, size_t bytes) {
    if (!d_ptr) return fail(QH_ERR_INVALID, "qh_malloc: null out pointer");
    *d_ptr = nullptr;
    // Round up so 16-byte vector/bulk reads of the last bytes stay inside.
    cudaError_t e = cudaMalloc(d_ptr, (bytes + 255) & ~size_t(255));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    return QH_OK;
}

int qh_free(void *d_ptr) {
    cudaError_t e = cudaFree(d_ptr);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFree");
    return QH_OK;
}

int qh_memcpy_h2d(void *d_dst, const void *h_src, size_t bytes, void *stream) {
    cudaError_t e = cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice,
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(H2D)");
    return QH_OK;
}

int qh_memcpy_d2h(void *h_dst, const void *d_src, size_t bytes, void *stream) {
    cudaError_t e = cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost,
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(D2H)");
    return QH_OK;
}

int qh_memset(void *d_dst, int value, size_t bytes, void *stream) {
    cudaError_t e = cudaMemsetAsync(d_dst, value, bytes, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    return QH_OK;
}

int qh_stream_sync(void *stream) {
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    return QH_OK;
}

int qh_check_device_error(int *code) {
    // Reads (and clears) the words the kernels report to on the current
    // device: the library's own, and the no-allocation entry point's. Only
    // words that already exist are read, so this call allocates nothing.
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    int *words[2];
    {
        std::lock_guard<std::mutex> lock(g_dev_mu);
        words[0] = g_err_words[dev];
    }
    words[1] = qh::noalloc_error_word(dev);
    int first = 0;
    for (int *w : words) {
        if (!w) continue;
        int v = 0;
        cudaError_t e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return cuda_fail(e, "read device error word");
        if (v != 0) {
            e = cudaMemset(w, 0, sizeof(int));
            if (e != cudaSuccess) return cuda_fail(e, "clear device error word");
            if (!first) first = v;
        }
    }
    if (code) *code = first;
    if (first != 0) return fail(QH_ERR_DEVICE, "device error %d (a bounded wait timed out)", first);
    return QH_OK;
}

int64_t qh_q8k_bytes(int64_t k, int64_t n_tok) { return qhf_q8k_total_bytes(k, n_tok); }
int64_t qh_q8_0_bytes(int64_t k, int64_t n_tok) { return qhf_q8_0_total_bytes(k, n_tok); }
int64_t qh_q8k_d_offset(int64_t k, int64_t n_tok) { return qhf_q8k_d_offset(k, n_tok); }
int64_t qh_q8k_bsums_offset(int64_t k, int64_t n_tok) { return qhf_q8k_bsums_offset(k, n_tok); }
int64_t qh_q8_0_d_offset(int64_t k, int64_t n_tok) { return qhf_q8_0_d_offset(k, n_tok); }

int qh_quantize_q8k(const float *d_x, int64_t k, int64_t n_tok, void *d_q8k, void *stream) {
    if (!d_x || !d_q8k) return fail(QH_ERR_INVALID, "quantize_q8k: null pointer");
    if (k <= 0 || k % 256 || n_tok <= 0 || n_tok > 65535)
        return fail(QH_ERR_INVALID, "quantize_q8k: k=%lld n_tok=%lld", (long long)k, (long long)n_tok);
    if (!aligned16(d_q8k)) return fail(QH_ERR_ALIGN, "quantize_q8k: output not 16-byte aligned");
    cudaError_t e = qh::quantize_q8k_launch(d_x, k, n_tok, d_q8k, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "quantize_q8k launch");
    return QH_OK;
}

int qh_quantize_q8_0(const float *d_x, int64_t k, int64_t n_tok, void *d_q8_0, void *stream) {
    if (!d_x || !d_q8_0) return fail(QH_ERR_INVALID, "quantize_q8_0: null pointer");
    if (k <= 0 || k % 32 || n_tok <= 0)
        return fail(QH_ERR_INVALID, "quantize_q8_0: k=%lld n_tok=%lld", (long long)k, (long long)n_tok);
    if (!aligned16(d_q8_0)) return fail(QH_ERR_ALIGN, "quantize_q8_0: output not 16-byte aligned");
    cudaError_t e = qh::quantize_q8_0_launch(d_x, k, n_tok, d_q8_0, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "quantize_q8_0 launch");
    return QH_OK;
}

int64_t qh_matmul_workspace_bytes(int type, int64_t k, int64_t n_tok) {
    if (type == QH_GGUF_F32 && k > 0 && n_tok > 0) return 0;
    if (qhf_block_bytes(type) == 0 || k <= 0 || n_tok <= 0) return -1;
    return act_bytes(type, k, n_tok);
}

int qh_matmul(int type, const void *d_w, int64_t k, int64_t out_f, const float *d_x,
              int64_t n_tok, float *d_out, void *d_work, int64_t work_bytes, void *stream) {
    return matmul_impl(type, d_w, k, out_f, d_x, n_tok, d_out, d_work, work_bytes, stream);
}

int qh_matmul_q4k_f32(const void *d_w, int64_t out_f, int64_t k, const float *d_x, int64_t n_tok,
                      float *d_out, void *d_work, int64_t work_bytes, void *stream) {
    return matmul_impl(QH_GGUF_Q4_K, d_w, k, out_f, d_x, n_tok, d_out, d_work, work_bytes, stream);
}
int qh_matmul_q5k_f32(const void *d_w, int64_t out_f, int64_t k, const float *d_x, int64_t n_tok,
                      float *d_out, void *d_work, int64_t work_bytes, void *stream) {
    return matmul_impl(QH_GGUF_Q5_K, d_w, k, out_f, d_x, n_tok, d_out, d_work, work_bytes, stream);
}
int qh_matmul_q6k_f32(const void *d_w, int64_t out_f, int64_t k, const float *d_x, int64_t n_tok,
                      float *d_out, void *d_work, int64_t work_bytes, void *stream) {
    return matmul_impl(QH_GGUF_Q6_K, d_w, k, out_f, d_x, n_tok, d_out, d_work, work_bytes, stream);
}
int qh_matmul_q8_0_f32(const void *d_w, int64_t out_f, int64_t k, const float *d_x, int64_t n_tok,
                       float *d_out, void *d_work, int64_t work_bytes, void *stream) {
    return matmul_impl(QH_GGUF_Q8_0, d_w, k, out_f, d_x, n_tok, d_out, d_work, work_bytes, stream);
}

int qh_matmul_f32(const float *d_w, int64_t out_f, int64_t k, const float *d_x, int64_t n_tok, float *d_out,
                  void *stream) {
    return matmul_f32_impl(d_w, k, out_f, d_x, n_tok, d_out, stream);
}

int qh_matmul_preq(int type, const void *d_w, int64_t k, int64_t out_f, const void *d_xq,
                   int64_t n_tok, float *d_out, void *stream) {
    int rc = check_shape(type, k, out_f, n_tok);
    if (rc) return rc;
    if (!d_w || !d_xq || !d_out) return fail(QH_ERR_INVALID, "matmul_preq: null pointer");
    if (!aligned16(d_w) || !aligned16(d_xq)) return fail(QH_ERR_ALIGN, "matmul_preq: pointer not 16-byte aligned");
    return run_preq(type, d_w, k, out_f, d_xq, n_tok, d_out, static_cast<cudaStream_t>(stream));
}

int qh_matvec_plan_create(int type, const qh_matvec_job *h_jobs, int n_jobs, int64_t n_tok,
                          qh_matvec_plan *out_plan) {
    if (!out_plan) return fail(QH_ERR_INVALID, "plan_create: null out pointer");
    *out_plan = nullptr;
    if (!h_jobs || n_jobs <= 0) return fail(QH_ERR_INVALID, "plan_create: no jobs");
    if (n_tok < 1 || n_tok > 8) return fail(QH_ERR_INVALID, "plan_create: n_tok %lld not in [1,8]", (long long)n_tok);
    int sms;
    int *err;
    int rc = device_state(&sms, &err);
    if (rc) return rc;
    std::vector<qh::GemvJob> jobs(n_jobs);
    for (int i = 0; i < n_jobs; ++i) {
        const qh_matvec_job &j = h_jobs[i];
        rc = check_shape(type, j.k, j.out_f, n_tok);
        if (rc) return rc;
        const int64_t rows = j.xq_rows > 0 ? j.xq_rows : n_tok;
        if (j.xq_row0 < 0 || j.xq_row0 + n_tok > rows)
            return fail(QH_ERR_INVALID, "plan_create: job %d rows [%lld, %lld) outside its %lld-row activation buffer",
                        i, (long long)j.xq_row0, (long long)(j.xq_row0 + n_tok), (long long)rows);
        if (!j.d_w || !j.d_xq || !j.d_out) return fail(QH_ERR_INVALID, "plan_create: job %d has a null pointer", i);
        if (!aligned16(j.d_w) || !aligned16(j.d_xq))
            return fail(QH_ERR_ALIGN, "plan_create: job %d pointer not 16-byte aligned", i);
        jobs[i] = make_job(type, j.d_w, j.k, j.out_f, j.d_xq, rows, j.xq_row0, j.d_out);
        jobs[i].out = j.d_out;
    }
    qh_matvec_plan p = new qh_matvec_plan_s{};
    p->type = type;
    p->n_tok = static_cast<int>(n_tok);
    p->sms = sms;
    p->jobs = jobs;
    cudaGetDevice(&p->device);
    cudaError_t e = qh::gemv_plan(type, jobs.data(), n_jobs, static_cast<int>(n_tok), sms, &p->params, &p->geom);
    if (e != cudaSuccess) {
        delete p;
        return fail(QH_ERR_INVALID, "plan_create: cannot tile these rows (%s)", cudaGetErrorString(e));
    }
    p->params.err_flag = err;
    p->params.table = nullptr;
    p->d_table = nullptr;
    if (n_jobs > qh::kGemvInlineJobs) {
        e = cudaMalloc(&p->d_table, sizeof(qh::GemvJob) * n_jobs);
        if (e == cudaSuccess)
            e = cudaMemcpy(p->d_table, jobs.data(), sizeof(qh::GemvJob) * n_jobs, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            if (p->d_table) cudaFree(p->d_table);
            delete p;
            return cuda_fail(e, "plan_create: job table");
        }
        p->params.table = p->d_table;
    }
    *out_plan = p;
    return QH_OK;
}

int qh_matvec_plan_fuse_input(qh_matvec_plan plan, int mode, const float *d_a, const float *d_b, const float *d_w,
                              float eps, float *d_h_out) {
    if (!plan) return fail(QH_ERR_INVALID, "plan_fuse_input: null plan");
    if (mode < 0 || mode > QH_FUSE_QUANT) return fail(QH_ERR_INVALID, "plan_fuse_input: unknown mode %d", mode);
    if (mode != 0 && plan->type == QH_GGUF_Q8_0)
        return fail(QH_ERR_UNSUPPORTED, "plan_fuse_input: Q8_0 weights take Q8_0 activations");
    const int64_t k = plan->jobs[0].k;
    for (const qh::GemvJob &j : plan->jobs)
        if (j.k != k) return fail(QH_ERR_INVALID, "plan_fuse_input: the jobs read inputs of different sizes");
    if (mode != 0 && !d_a) return fail(QH_ERR_INVALID, "plan_fuse_input: null input");
    if (mode == QH_FUSE_SWIGLU && !d_b) return fail(QH_ERR_INVALID, "plan_fuse_input: SwiGLU needs gate and up");
    if (mode == QH_FUSE_RMSNORM && (!d_w || (d_b && !d_h_out) || (d_h_out && (d_h_out == d_a || d_h_out == d_b))))
        return fail(QH_ERR_INVALID, "plan_fuse_input: RMSNorm needs a weight, and h_out (not an input) with a residual");
    if (mode == QH_FUSE_RMSNORM && k > 16 * QH_QK)
        return fail(QH_ERR_UNSUPPORTED, "plan_fuse_input: RMSNorm rows longer than 4096");
    std::vector<qh::GemvJob> jobs = plan->jobs;
    qh::GemvParams p{};
    qh::GemvGeometry g{};
    cudaError_t e = qh::gemv_plan(plan->type, jobs.data(), static_cast<int>(jobs.size()), plan->n_tok, plan->sms, &p, &g,
                                  mode);
    if (e != cudaSuccess) return fail(QH_ERR_INVALID, "plan_fuse_input: cannot tile these rows (%s)", cudaGetErrorString(e));
    p.err_flag = plan->params.err_flag;
    p.table = plan->params.table;
    // an output tail set earlier stays
    p.tform = plan->params.tform;
    p.tk = plan->params.tk;
    p.teps = plan->params.teps;
    p.ta = plan->params.ta;
    p.tb = plan->params.tb;
    p.tw = plan->params.tw;
    p.th_out = plan->params.th_out;
    p.txq = plan->params.txq;
    p.ticket = plan->params.ticket;
    if (mode) {
        p.xa = d_a;
        p.xb = d_b;
        p.xw = d_w;
        p.eps = eps;
        p.xh_out = mode == QH_FUSE_RMSNORM ? d_h_out : nullptr;
    }
    if (plan->d_table) {  // tile ranges of the table follow the new tiling
        e = cudaMemcpy(plan->d_table, jobs.data(), sizeof(qh::GemvJob) * jobs.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_fail(e, "plan_fuse_input: job table");
    }
    plan->params = p;
    plan->geom = g;
    return QH_OK;
}

int qh_matvec_plan_fuse_output(qh_matvec_plan plan, int mode, int64_t k, const float *d_a, const float *d_b,
                               const float *d_w, float eps, float *d_h_out, void *d_xq) {
    if (!plan) return fail(QH_ERR_INVALID, "plan_fuse_output: null plan");
    if (mode < 0 || mode > QH_FUSE_QUANT) return fail(QH_ERR_INVALID, "plan_fuse_output: unknown mode %d", mode);
    if (mode == 0) {
        plan->params.tform = 0;
        return QH_OK;
    }
    if (k <= 0 || k % QH_QK) return fail(QH_ERR_INVALID, "plan_fuse_output: k=%lld", (long long)k);
    if (!d_a || !d_xq) return fail(QH_ERR_INVALID, "plan_fuse_output: null input or output");
    if (!aligned16(d_xq)) return fail(QH_ERR_ALIGN, "plan_fuse_output: output not 16-byte aligned");
    if (mode == QH_FUSE_SWIGLU && !d_b) return fail(QH_ERR_INVALID, "plan_fuse_output: SwiGLU needs gate and up");
    if (mode == QH_FUSE_RMSNORM && (!d_w || (d_b && !d_h_out) || (d_h_out && (d_h_out == d_a || d_h_out == d_b))))
        return fail(QH_ERR_INVALID, "plan_fuse_output: RMSNorm needs a weight, and h_out (not an input) with a residual");
    if (mode == QH_FUSE_RMSNORM && k > 16 * QH_QK)
        return fail(QH_ERR_UNSUPPORTED, "plan_fuse_output: RMSNorm rows longer than 4096");
    if (!plan->d_ticket) {
        cudaError_t e = cudaMalloc(&plan->d_ticket, sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemset(plan->d_ticket, 0, sizeof(unsigned));
        if (e != cudaSuccess) {
            if (plan->d_ticket) cudaFree(plan->d_ticket);
            plan->d_ticket = nullptr;
            return cuda_fail(e, "plan_fuse_output: ticket");
        }
    }
    qh::GemvParams &p = plan->params;
    p.tform = mode;
    p.tk = static_cast<int32_t>(k);
    p.teps = eps;
    p.ta = d_a;
    p.tb = mode == QH_FUSE_QUANT ? nullptr : d_b;
    p.tw = mode == QH_FUSE_RMSNORM ? d_w : nullptr;
    p.th_out = mode == QH_FUSE_RMSNORM ? d_h_out : nullptr;
    p.txq = static_cast<uint8_t *>(d_xq);
    p.ticket = plan->d_ticket;
    return QH_OK;
}

int qh_matvec_plan_run(qh_matvec_plan plan, void *stream) {
    if (!plan) return fail(QH_ERR_INVALID, "plan_run: null plan");
    cudaError_t e = qh::gemv_launch(plan->type, plan->params, plan->geom, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "plan_run launch");
    return QH_OK;
}

int qh_matvec_plan_test_timeout(qh_matvec_plan plan, int32_t tile, uint32_t wait_limit) {
    if (!plan) return fail(QH_ERR_INVALID, "plan_test_timeout: null plan");
    if (tile < -1 || tile >= plan->params.total_tiles)
        return fail(QH_ERR_INVALID, "plan_test_timeout: tile %d outside [-1, %d)", tile, plan->params.total_tiles);
    plan->params.test_withhold = tile + 1;
    plan->params.wait_limit = wait_limit;
    return QH_OK;
}

int qh_matvec_plan_info(qh_matvec_plan plan, int *rows_per_tile, int *n_stages, int *grid, int *smem_bytes) {
    if (!plan) return fail(QH_ERR_INVALID, "plan_info: null plan");
    if (rows_per_tile) *rows_per_tile = plan->params.rows_per_tile;
    if (n_stages) *n_stages = plan->params.n_stages;
    if (grid) *grid = plan->geom.grid;
    if (smem_bytes) *smem_bytes = plan->geom.smem_bytes;
    return QH_OK;
}

int qh_matvec_plan_destroy(qh_matvec_plan plan) {
    if (!plan) return QH_OK;
    if (plan->d_table) cudaFree(plan->d_table);
    if (plan->d_ticket) cudaFree(plan->d_ticket);
    delete plan;
    return QH_OK;
}

}  // extern "C"
