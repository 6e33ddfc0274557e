// SPDX-License-Identifier: MIT
//
// qh_q8k.cuh -- device-side Q8_K activation quantization shared by the
// fused kernels (qh_model.cu) and the tensor-core path (qh_gemm.cu):
// quantize_row_q8_K (slm/tensor.c:673-720) for one 256-value block held by a
// CTA, writing either the split layout the GEMV reads or the tiled layout
// the tcgen05 GEMM reads.

#ifndef QH_Q8K_CUH
#define QH_Q8K_CUH

#include <stdint.h>

#include "qh_common.cuh"

namespace qh {

// Candidate for the Q8_K block maximum: |x| (NaN never wins), its index in
// the block and its signed value; ties go to the smaller index, as the
// reference's first-strictly-greater scan does.
__device__ __forceinline__ void best_merge(float &a, int &i, float &v, float oa, int oi, float ov) {
    if (oa > a || (oa == a && oi < i)) { a = oa; i = oi; v = ov; }
}

__device__ __forceinline__ void warp_best(float &a, int &i, float &v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, a, off);
        const int oi = __shfl_xor_sync(0xffffffffu, i, off);
        const float ov = __shfl_xor_sync(0xffffffffu, v, off);
        best_merge(a, i, v, oa, oi, ov);
    }
}

// q = clamp(round_half_even(iscale * v)) through the 1.5*2^23 bias, as
// quantize_q8k_kernel does (slm/tensor.c:673-678, 683-720).
__device__ __forceinline__ int q8k_value(float v, float iscale) {
    const float f = __fmul_rn(iscale, v);
    const float biased = __fadd_rn(f, 12582912.0f);
    int q = (__float_as_int(biased) & 0x007fffff) - 0x00400000;
    if (f != f) q = 0;
    return q > 127 ? 127 : (q < -128 ? -128 : q);
}

// Destination of the Q8_K quantization of row `tok` in either activation
// layout (qh_formats.h):
//   split  (tile == 0):  qs [n_tok][K], d [n_tok][d_stride], bsums;
//   tiled  (tile == QH_Q8KT_TILE): per (64-token tile, block) the operand
//          quants, the scales and the min operand rows.
// Element p (0..255) of block b sits at qs + b * bstride + (p / 16) * cstride
// + p % 16; its scale at d + b * dstride.
struct Q8KRow {
    int8_t *qs;
    int32_t bstride, cstride;
    float *d;
    int32_t dstride;
    int16_t *bs;      // split layout only
    int8_t *mins;     // tiled layout only: min-operand row of this token (block 0)
};
__device__ __forceinline__ Q8KRow q8k_row(uint8_t *base, int64_t k, int64_t n_tok, int64_t tok, int tile = 0) {
    Q8KRow r;
    if (tile == 0) {
        r.qs = reinterpret_cast<int8_t *>(base) + tok * k;
        r.bstride = QH_QK;
        r.cstride = 16;
        r.d = reinterpret_cast<float *>(base + qhf_q8k_d_offset(k, n_tok)) + tok * qhf_q8k_d_stride(k);
        r.dstride = 1;
        r.bs = reinterpret_cast<int16_t *>(base + qhf_q8k_bsums_offset(k, n_tok)) + tok * (k / QH_QK) * 16;
        r.mins = nullptr;
    } else {
        const int64_t nb = k / QH_QK, tl = tok % QH_Q8KT_TILE;
        uint8_t *tb = base + (tok / QH_Q8KT_TILE) * nb * QH_Q8KT_BLOCK_BYTES;
        r.qs = reinterpret_cast<int8_t *>(tb) + tl * 16;
        r.bstride = QH_Q8KT_BLOCK_BYTES;
        r.cstride = QH_Q8KT_TILE * 16;
        r.d = reinterpret_cast<float *>(tb + QH_Q8KT_D_OFF) + tl;
        r.dstride = QH_Q8KT_BLOCK_BYTES / 4;
        r.bs = nullptr;
        r.mins = reinterpret_cast<int8_t *>(tb + QH_Q8KT_MIN_OFF) + tl * 16;
    }
    return r;
}
__device__ __forceinline__ int8_t *q8k_elem(const Q8KRow &r, int b, int p) {
    return r.qs + static_cast<int64_t>(b) * r.bstride + (p >> 4) * r.cstride + (p & 15);
}
__device__ __forceinline__ float *q8k_scale(const Q8KRow &r, int b) { return r.d + static_cast<int64_t>(b) * r.dstride; }

// Tiled layout: the min operand entries of sub-block j (the 32 quants of
// one warp-aligned group), given their sum S; bytes 8..15 of both rows are
// zeroed by the caller for j == 0.
__device__ __forceinline__ void q8k_put_min(const Q8KRow &r, int b, int j, int S) {
    int8_t *m = r.mins + static_cast<int64_t>(b) * r.bstride;
    m[j] = static_cast<int8_t>(S & 127);
    m[QH_Q8KT_TILE * 16 + j] = static_cast<int8_t>(S >> 7);
    if (j == 0) {
        *reinterpret_cast<uint2 *>(m + 8) = make_uint2(0u, 0u);
        *reinterpret_cast<uint2 *>(m + QH_Q8KT_TILE * 16 + 8) = make_uint2(0u, 0u);
    }
}

struct Q8KScratch {
    float a[8], v[8];
    int i[8];
};

// Barrier over the threads of a q8k_block256 call: the whole CTA, or (NAMED)
// threads 0..255 of a larger CTA on named barrier 1.
template <bool NAMED>
__device__ __forceinline__ void q8k_sync() {
    if constexpr (NAMED) asm volatile("bar.sync 1, 256;" ::: "memory");
    else __syncthreads();
}

// Q8_K quantization of block b of row r held one value per thread by 256
// threads (thread t holds element t): a 256-thread CTA, or with NAMED
// threads 0..255 of a larger one. Ends with a barrier, so the scratch can be
// reused by the next block.
template <bool NAMED = false>
__device__ __forceinline__ void q8k_block256(float v, Q8KScratch &sc, const Q8KRow &r, int b) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float a = (v == v) ? fabsf(v) : -1.0f, bv = v;
    int bi = tid;
    warp_best(a, bi, bv);
    if (lane == 0) { sc.a[warp] = a; sc.i[warp] = bi; sc.v[warp] = bv; }
    q8k_sync<NAMED>();
    float ba = sc.a[0], xv = sc.v[0];
    int ii = sc.i[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) best_merge(ba, ii, xv, sc.a[w], sc.i[w], sc.v[w]);
    const float xmax = ba > 0.0f ? xv : 0.0f;
    int q = 0;
    if (xmax != 0.0f) {
        const float iscale = __fdiv_rn(-127.0f, xmax);
        q = q8k_value(v, iscale);
        if (tid == 0) *q8k_scale(r, b) = __fdiv_rn(1.0f, iscale);
    } else if (tid == 0) {
        *q8k_scale(r, b) = 0.0f;
    }
    *q8k_elem(r, b, tid) = static_cast<int8_t>(q);
    int s = q;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (r.bs) {
        if ((lane & 15) == 0) r.bs[b * 16 + warp * 2 + (lane >> 4)] = static_cast<int16_t>(s);
    } else {
        s += __shfl_xor_sync(0xffffffffu, s, 16);  // sub-block (warp) sum
        if (lane == 0) q8k_put_min(r, b, warp, s);
    }
    q8k_sync<NAMED>();
}

}  // namespace qh

#endif  // QH_Q8K_CUH
