// SPDX-License-Identifier: MIT
//
// qh_quant.cu -- activation quantizers on sm_100a, bit-exact with the
// reference's CPU quantizers.
//
//   Q8_K (K-quant weights), slm/tensor.c:683-720 (+ nearest_int 673-678):
//     per 256-block: xmax = the value of largest magnitude (first index wins
//     on ties), iscale = -127/xmax, q = clamp(round_half_even(iscale*x)),
//     d = 1/iscale, bsums = sums of 16-element groups.
//   Q8_0 (Q8_0 weights), slm/tensor.c:930-950:
//     per 32-block: d = amax/127 (kept as fp16, round to nearest even),
//     q = clamp(roundf(x * (1/d))) -- half away from zero, unrounded d.
//
// Divisions use __fdiv_rn (IEEE round-to-nearest), products __fmul_rn, so
// the device never substitutes approximate or fused arithmetic.

#include "qh_common.cuh"
#include "qh_internal.h"

namespace qh {

// One 256-thread CTA per (block, token): thread i owns element i.
__global__ void __launch_bounds__(256) quantize_q8k_kernel(const float *__restrict__ x, int64_t k,
                                                           int8_t *__restrict__ qs,
                                                           float *__restrict__ dv,
                                                           int16_t *__restrict__ bsums) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float s_abs[8];
    __shared__ int s_idx[8];
    __shared__ float s_xmax;
    const int nb = static_cast<int>(k / QH_QK);
    const int blk = blockIdx.x, tok = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t base = static_cast<int64_t>(tok) * k + static_cast<int64_t>(blk) * QH_QK;
    const float v = x[base + tid];
    // NaN never wins (the reference's `fabsf(x) > amax` is false for NaN).
    float a = (v == v) ? fabsf(v) : -1.0f;
    int idx = tid;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_down_sync(0xffffffffu, a, off);
        const int oi = __shfl_down_sync(0xffffffffu, idx, off);
        if (oa > a || (oa == a && oi < idx)) { a = oa; idx = oi; }
    }
    if (lane == 0) { s_abs[warp] = a; s_idx[warp] = idx; }
    __syncthreads();
    if (tid == 0) {
        float ba = s_abs[0];
        int bi = s_idx[0];
        for (int w = 1; w < 8; ++w)
            if (s_abs[w] > ba || (s_abs[w] == ba && s_idx[w] < bi)) { ba = s_abs[w]; bi = s_idx[w]; }
        s_xmax = (ba > 0.0f) ? x[base + bi] : 0.0f;
    }
    __syncthreads();
    const float xmax = s_xmax;
    int q = 0;
    if (xmax != 0.0f) {
        const float iscale = __fdiv_rn(-127.0f, xmax);
        const float f = __fmul_rn(iscale, v);
        // round half to even through the 1.5*2^23 bias, as the reference does
        const float biased = __fadd_rn(f, 12582912.0f);
        q = (__float_as_int(biased) & 0x007fffff) - 0x00400000;
        if (f != f) q = 0;  // x86 default NaN (0xffc00000) decodes to 0 there
        q = q > 127 ? 127 : (q < -128 ? -128 : q);
        if (tid == 0) dv[static_cast<int64_t>(tok) * qhf_q8k_d_stride(k) + blk] = __fdiv_rn(1.0f, iscale);
    } else if (tid == 0) {
        dv[static_cast<int64_t>(tok) * qhf_q8k_d_stride(k) + blk] = 0.0f;
    }
    qs[base + tid] = static_cast<int8_t>(q);
    // 16-element group sums: each half-warp is one group.
    int s = q;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((lane & 15) == 0)
        bsums[(static_cast<int64_t>(tok) * nb + blk) * 16 + warp * 2 + (lane >> 4)] = static_cast<int16_t>(s);
}

// One warp per 32-block; 8 warps per CTA.
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float *__restrict__ x, int64_t k,
                                                            int64_t n_blocks,
                                                            int8_t *__restrict__ qs,
                                                            uint16_t *__restrict__ dbits) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t b = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (b >= n_blocks) return;
    const float v = x[b * QH_QK8_0 + lane];
    float amax = fabsf(v);
    if (!(amax == amax)) amax = 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    int q = static_cast<int>(roundf(__fmul_rn(v, id)));
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    qs[b * QH_QK8_0 + lane] = static_cast<int8_t>(q);
    if (lane == 0) {
        const int64_t nb0 = k / QH_QK8_0;
        dbits[(b / nb0) * qhf_q8_0_d_stride(k) + b % nb0] = __half_as_ushort(__float2half_rn(d));
    }
}

cudaError_t quantize_q8k_launch(const float *x, int64_t k, int64_t n_tok, void *q8k,
                                cudaStream_t stream) {
    if (k <= 0 || k % QH_QK || n_tok <= 0 || n_tok > 65535) return cudaErrorInvalidValue;
    uint8_t *base = static_cast<uint8_t *>(q8k);
    dim3 grid(static_cast<unsigned>(k / QH_QK), static_cast<unsigned>(n_tok));
    const cudaError_t le = launch_pdl(quantize_q8k_kernel, dim3(grid), dim3(256), 0, stream, 
        x, k, reinterpret_cast<int8_t *>(base),
        reinterpret_cast<float *>(base + qhf_q8k_d_offset(k, n_tok)),
        reinterpret_cast<int16_t *>(base + qhf_q8k_bsums_offset(k, n_tok)));
    return le != cudaSuccess ? le : cudaGetLastError();
}

cudaError_t quantize_q8_0_launch(const float *x, int64_t k, int64_t n_tok, void *q8_0,
                                 cudaStream_t stream) {
    if (k <= 0 || k % QH_QK8_0 || n_tok <= 0) return cudaErrorInvalidValue;
    uint8_t *base = static_cast<uint8_t *>(q8_0);
    const int64_t n_blocks = (k / QH_QK8_0) * n_tok;
    const int64_t grid = (n_blocks + 7) / 8;
    if (grid > 0x7fffffff) return cudaErrorInvalidValue;
    const cudaError_t le = launch_pdl(quantize_q8_0_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, stream, 
        x, k, n_blocks, reinterpret_cast<int8_t *>(base),
        reinterpret_cast<uint16_t *>(base + qhf_q8_0_d_offset(k, n_tok)));
    return le != cudaSuccess ? le : cudaGetLastError();
}

}  // namespace qh
