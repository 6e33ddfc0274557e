// SPDX-License-Identifier: MIT
//
// qh_noalloc.cu -- qh_matmul_q4k_f32_noalloc: the Q4_K matmul (activation
// quantization + grouped matvec kernel) for callers that may not allocate
// device memory.
//
// Who needs it: some host programs own every byte of device memory
// themselves -- an application that carves all buffers out of one pool it
// reserved at start-up, or a latency-critical service that forbids any
// cudaMalloc after initialization because an allocation can synchronize
// the device and stall its other streams. Such a caller can hand us its
// weights, input and output buffers, but it cannot give us (or let us
// create) the extra device buffer that holds the quantized activation rows.
// This entry point keeps that buffer in a fixed, file-scope device array
// instead, so it allocates nothing.
//
// Costs and rules of the fixed array:
//   * Every GPU that loads this library holds kNoallocScratchBytes of it
//     until the process exits, whether or not this entry point is called.
//   * All calls share it and it keeps the last call's contents, so two calls
//     whose work overlaps on the GPU (different streams, or different host
//     threads on one device) race on it. Serialize them on one stream.
//   * The quantized rows are rewritten completely by every call. The only
//     part that must start at zero is the kernel error word in the first
//     256 bytes: it is zero when the library loads, a kernel whose bounded
//     wait runs out sets it (first error wins), and qh_check_device_error
//     reads and clears it together with the library's other error word, so
//     a timeout in this path reaches the caller like one anywhere else.
//   * Host code cannot use the array's name as a device address, so the
//     first call on each device (with that device current) looks the
//     address up with cudaGetSymbolAddress and caches it. Make that first
//     call before starting any stream capture on that device.

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "../../include/qh_backend.h"
#include "qh_internal.h"

namespace {

// 256 bytes of control (the error word) followed by the quantized activation
// rows. 128 KiB holds e.g. 112 rows of k = 1024 or 35 rows of k = 3584.
constexpr int64_t kNoallocScratchBytes = 128 * 1024;
constexpr int64_t kNoallocControlBytes = 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {nullptr};
int g_sms[kMaxDevices] = {0};

thread_local char g_msg[256];

int noalloc_fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    qh::set_last_error_message(g_msg);
    return code;
}

// Once per device, with that device current: resolve the array's device
// address and read the SM count. Allocates nothing.
int noalloc_setup(void **scratch, int *sms) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return noalloc_fail(QH_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return noalloc_fail(QH_ERR_INVALID, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return noalloc_fail(QH_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        int n = 0;
        e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return noalloc_fail(QH_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
        g_sms[dev] = n;
        g_scratch_addr[dev] = p;
    }
    *scratch = g_scratch_addr[dev];
    *sms = g_sms[dev];
    return QH_OK;
}

}  // namespace

extern "C" int qh_matmul_q4k_f32_noalloc(const void *d_w, int64_t out_f, int64_t k, const float *d_x,
                                         int64_t n_tok, float *d_out, void *stream) {
    if (!d_w || !d_x || !d_out) return noalloc_fail(QH_ERR_INVALID, "null pointer");
    if (k <= 0 || k % QH_QK || out_f <= 0 || out_f > (1ll << 30) || n_tok <= 0)
        return noalloc_fail(QH_ERR_INVALID, "bad shape k=%lld out_f=%lld n_tok=%lld", (long long)k,
                            (long long)out_f, (long long)n_tok);
    if (reinterpret_cast<uintptr_t>(d_w) & 15) return noalloc_fail(QH_ERR_ALIGN, "weights not 16-byte aligned");
    const int64_t need = qhf_q8k_total_bytes(k, n_tok);
    if (need > kNoallocScratchBytes - kNoallocControlBytes)
        return noalloc_fail(QH_ERR_WORKSPACE,
                            "k=%lld x n_tok=%lld needs %lld bytes of activation scratch; the fixed "
                            "array holds %lld (use qh_matmul_q4k_f32 with a workspace)",
                            (long long)k, (long long)n_tok, (long long)need,
                            (long long)(kNoallocScratchBytes - kNoallocControlBytes));
    void *base = nullptr;
    int sms = 0;
    int rc = noalloc_setup(&base, &sms);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int *err_word = static_cast<int *>(base);
    uint8_t *xq = static_cast<uint8_t *>(base) + kNoallocControlBytes;
    cudaError_t e = qh::quantize_q8k_launch(d_x, k, n_tok, xq, s);
    if (e != cudaSuccess) return noalloc_fail(QH_ERR_CUDA, "quantize launch: %s", cudaGetErrorString(e));
    // the same launches (and token chunking) as qh_matmul_q4k_f32
    return qh::matmul_preq_launch(QH_GGUF_Q4_K, d_w, k, out_f, xq, n_tok, d_out, s, sms, err_word);
}

namespace qh {
int *noalloc_error_word(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_mu);
    return static_cast<int *>(g_scratch_addr[dev]);
}
}  // namespace qh
