// SPDX-License-Identifier: MIT
//
// qh_libm.cu -- qh_libm_eval: the device expf/logf (qh_libm.cuh) over a
// range of float bit patterns, so they can be compared with the host C
// library on every input.

#include <cuda_runtime.h>

#include "../../include/qh_backend.h"
#include "../../include/qh_kernels.h"
#include "qh_common.cuh"
#include "qh_internal.h"

namespace {

__global__ void libm_eval_kernel(int fn, uint32_t first, int64_t n, float *out) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += stride) {
        const float x = __uint_as_float(first + static_cast<uint32_t>(j));
        out[j] = fn == 0 ? qh::expf_ref(x) : qh::logf_ref(x);
    }
}

}  // namespace

extern "C" int qh_libm_eval(int fn, uint32_t first, int64_t n, float *d_out, void *stream) {
    if ((fn != 0 && fn != 1) || n <= 0 || n > (int64_t(1) << 32) || !d_out) {
        qh::set_last_error_message("qh_libm_eval: fn must be 0 (expf) or 1 (logf), 0 < n <= 2^32, output set");
        return QH_ERR_INVALID;
    }
    const int64_t blocks = (n + 255) / 256;
    libm_eval_kernel<<<static_cast<unsigned>(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0,
                       static_cast<cudaStream_t>(stream)>>>(fn, first, n, d_out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        qh::set_last_error_message(cudaGetErrorString(e));
        return QH_ERR_CUDA;
    }
    return QH_OK;
}
