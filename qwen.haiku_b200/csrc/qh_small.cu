// SPDX-License-Identifier: MIT
//
// qh_small.cu -- the matmuls of the two weight types the K-quant GEMV and
// tensor-core GEMM do not cover:
//
//   * F32 weights (tensor_matmul_f32, slm/tensor.c:517-535): out[t][j] =
//     sum_i w[j][i] * x[t][i], one float product and one float add per i in
//     index order -- the reference's plain loop, which its C17 build neither
//     contracts nor reorders. One thread per (row, token); rows and inputs
//     staged through shared memory in 64-value slices so the global loads
//     are coalesced.
//   * Q8_0 weights against Q8_0 activations for any number of tokens
//     (tensor_matmul_q8_0_f32, slm/tensor.c:952-981, through
//     q8_0_dot_q8_0_avxvnni, simd/avx.c:65-88): the lane arithmetic of the
//     grouped GEMV (qh_gemv.cu) -- lane jj of 8 owns bytes 4jj..4jj+3 of
//     every 32-block and accumulates one fma per block, the 8 lanes are
//     added as ((l0+l4)+(l1+l5))+((l2+l6)+(l3+l7)) -- over a grid of (row
//     groups, token groups), so a many-token Q8_0 projection is one launch
//     instead of one GEMV launch per 8 tokens. Q8_0 matrices of the model are
//     small (the real Q4_K_M mix has them only for ssm_alpha/ssm_beta,
//     1024 -> 16), so weights are read from L2 directly.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "qh_common.cuh"
#include "qh_internal.h"

namespace qh {
namespace {

constexpr int kF32Rows = 32, kF32Toks = 8, kF32Slice = 64;

__global__ void __launch_bounds__(kF32Rows *kF32Toks) matmul_f32_kernel(const float *__restrict__ w, int64_t k,
                                                                        int64_t out_f, const float *__restrict__ x,
                                                                        int64_t n_tok, float *__restrict__ out) {
    pdl_launch_dependents();
    __shared__ float ws[kF32Rows][kF32Slice + 1];
    __shared__ float xs[kF32Toks][kF32Slice + 1];
    const int tid = threadIdx.x;
    const int jr = tid % kF32Rows, tt = tid / kF32Rows;
    const int64_t j0 = static_cast<int64_t>(blockIdx.x) * kF32Rows, t0 = static_cast<int64_t>(blockIdx.y) * kF32Toks;
    pdl_wait();
    float acc = 0.0f;
    for (int64_t i0 = 0; i0 < k; i0 += kF32Slice) {
        const int len = static_cast<int>(k - i0 < kF32Slice ? k - i0 : kF32Slice);
        for (int e = tid; e < kF32Rows * kF32Slice; e += blockDim.x) {
            const int r = e / kF32Slice, c = e % kF32Slice;
            ws[r][c] = (j0 + r < out_f && c < len) ? w[(j0 + r) * k + i0 + c] : 0.0f;
        }
        for (int e = tid; e < kF32Toks * kF32Slice; e += blockDim.x) {
            const int r = e / kF32Slice, c = e % kF32Slice;
            xs[r][c] = (t0 + r < n_tok && c < len) ? x[(t0 + r) * k + i0 + c] : 0.0f;
        }
        __syncthreads();
        for (int c = 0; c < len; ++c) acc = __fadd_rn(acc, __fmul_rn(ws[jr][c], xs[tt][c]));
        __syncthreads();
    }
    if (j0 + jr < out_f && t0 + tt < n_tok) out[(t0 + tt) * out_f + j0 + jr] = acc;
}

// 8 warps; warp w covers rows 4w..4w+3 of the CTA's 32-row group (lane >> 3)
// and the CTA's 8 tokens.
__global__ void __launch_bounds__(256) matmul_q8_0_many_kernel(const uint8_t *__restrict__ w, int64_t k, int64_t out_f,
                                                               const int8_t *__restrict__ xqs,
                                                               const uint16_t *__restrict__ xd, int64_t d_stride,
                                                               int64_t n_tok, float *__restrict__ out) {
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rr = lane >> 3, jj = lane & 7;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 32 + warp * 4 + rr;
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * 8;
    const int64_t nb = k / QH_QK8_0;
    const bool row_ok = row < out_f;
    const uint8_t *wr = w + (row_ok ? row : 0) * nb * QH_Q8_0_BYTES;
    pdl_wait();
    float acc[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *blk = wr + b * QH_Q8_0_BYTES;
        const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);  // blocks are 2-byte aligned
        const float dw = h2f_bits(h[0]);
        const int wq = static_cast<int>(static_cast<uint32_t>(h[1 + 2 * jj]) | (static_cast<uint32_t>(h[2 + 2 * jj]) << 16));
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            if (t0 + t < n_tok) {
                const int xw = *reinterpret_cast<const int *>(xqs + (t0 + t) * k + b * QH_QK8_0 + 4 * jj);
                const float dx = h2f_bits(xd[(t0 + t) * d_stride + b]);
                acc[t] = __fmaf_rn(static_cast<float>(__dp4a(wq, xw, 0)), __fmul_rn(dw, dx), acc[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        float v = acc[t];
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
        if (jj == 0 && row_ok && t0 + t < n_tok) out[(t0 + t) * out_f + row] = v;
    }
}

}  // namespace

cudaError_t matmul_f32_launch(const float *w, int64_t k, int64_t out_f, const float *x, int64_t n_tok, float *out,
                              cudaStream_t s) {
    const dim3 grid(static_cast<unsigned>((out_f + kF32Rows - 1) / kF32Rows),
                    static_cast<unsigned>((n_tok + kF32Toks - 1) / kF32Toks));
    return launch_pdl(matmul_f32_kernel, grid, dim3(kF32Rows * kF32Toks), 0, s, w, k, out_f, x, n_tok, out);
}

cudaError_t matmul_q8_0_many_launch(const void *w, int64_t k, int64_t out_f, const void *xq, int64_t xq_rows,
                                    int64_t row0, int64_t n_tok, float *out, cudaStream_t s) {
    const uint8_t *base = static_cast<const uint8_t *>(xq);
    const int64_t d_stride = qhf_q8_0_d_stride(k);
    const int8_t *qs = reinterpret_cast<const int8_t *>(base) + row0 * k;
    const uint16_t *d = reinterpret_cast<const uint16_t *>(base + qhf_q8_0_d_offset(k, xq_rows)) + row0 * d_stride;
    const dim3 grid(static_cast<unsigned>((out_f + 31) / 32), static_cast<unsigned>((n_tok + 7) / 8));
    return launch_pdl(matmul_q8_0_many_kernel, grid, dim3(256), 0, s, static_cast<const uint8_t *>(w), k, out_f, qs,
                      d, d_stride, n_tok, out);
}

}  // namespace qh
