// SPDX-License-Identifier: MIT
//
// qh_model.cu -- the non-matmul kernels of the hybrid forward pass
// (include/qh_kernels.h) on sm_100a.
//
// Every kernel reproduces the reference's operation order where that order
// is cheap to keep: float products and sums use explicitly rounded
// __fmul_rn/__fadd_rn (never contracted into FMAs), sequential reductions
// the reference does in float over a short axis stay sequential in one
// thread (attention dot products, softmax sum, value accumulation), and its
// double-precision sums stay double (norms, the DeltaNet kv/out products).
// Transcendentals are the host C library's expf/logf, reproduced bit for
// bit (expf_ref/logf_ref, qh_libm.cuh): the device's own single-precision
// expf/logf differ from them by an ulp often enough that the next layer's
// Q8_K quantization flips int8 values and the token streams drift. RoPE
// cos/sin come from a host-computed table so they match the reference's
// libm bit for bit.

#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>

#include "../../include/qh_backend.h"
#include "../../include/qh_kernels.h"
#include "qh_common.cuh"
#include "qh_internal.h"
#include "qh_gdn.cuh"
#include "qh_q8k.cuh"

namespace qh {


// Block-wide double sum (blockDim.x multiple of 32, <= 1024); all threads
// get the result.
__device__ double block_sum_d(double v, double *scratch) {
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < nw; ++w) t += scratch[w];
    return t;
}

// Two block-wide double sums at once, each with block_sum_d's order (warp
// tree, then the warps in order); scratch holds 2 * 32 doubles.
__device__ double2 block_sum_d2(double a, double b, double *scratch) {
    for (int off = 16; off > 0; off >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, off);
        b += __shfl_xor_sync(0xffffffffu, b, off);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) {
        scratch[warp] = a;
        scratch[32 + warp] = b;
    }
    __syncthreads();
    double ta = 0.0, tb = 0.0;
    for (int w = 0; w < nw; ++w) {
        ta += scratch[w];
        tb += scratch[32 + w];
    }
    return make_double2(ta, tb);
}

__device__ float block_max_f(float v, float *scratch) {
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = scratch[0];
    for (int w = 1; w < nw; ++w) t = fmaxf(t, scratch[w]);
    return t;
}

// ---------------------------------------------------------------------------
// Embedding: one CTA of 256 threads per (token, super-block).
// ---------------------------------------------------------------------------
__global__ void embed_q6k_kernel(const uint8_t *__restrict__ table, int64_t hidden,
                                 const int32_t *__restrict__ tokens, float *__restrict__ h) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.y, sb = blockIdx.x, p = threadIdx.x;
    const int64_t nb = hidden / QH_QK;
    const uint8_t *blk = table + (static_cast<int64_t>(tokens[b]) * nb + sb) * QH_Q6K_BYTES;
    const int half = p >> 7, r = (p >> 5) & 3, l = p & 31;
    const uint8_t lo_byte = blk[64 * half + 32 * (r & 1) + l];
    const int lo = (r >> 1) ? (lo_byte >> 4) : (lo_byte & 0x0f);
    const int hi2 = (blk[128 + 32 * half + l] >> (2 * r)) & 3;
    const int q = (lo | (hi2 << 4)) - 32;
    const float d = h2f_bits(static_cast<uint32_t>(blk[208]) | (static_cast<uint32_t>(blk[209]) << 8));
    const float sc = static_cast<float>(static_cast<int8_t>(blk[192 + (p >> 4)]));
    h[static_cast<int64_t>(b) * hidden + sb * QH_QK + p] = __fmul_rn(__fmul_rn(d, sc), static_cast<float>(q));
}

// F32 table (tensor_get_rows on the fp32 view, slm/qwen.c:885-889).
__global__ void embed_f32_kernel(const float *__restrict__ table, int64_t hidden, const int32_t *__restrict__ tokens,
                                 float *__restrict__ h) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.y;
    const float *row = table + static_cast<int64_t>(tokens[b]) * hidden;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < hidden;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        h[static_cast<int64_t>(b) * hidden + i] = row[i];
}

// ---------------------------------------------------------------------------
// RMSNorm: one CTA per row.
// ---------------------------------------------------------------------------
__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w, int64_t dim,
                               float eps, float *__restrict__ y) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double scratch[32];
    const float *xr = x + blockIdx.x * dim;
    float *yr = y + blockIdx.x * dim;
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
        const float v = xr[i];
        s += static_cast<double>(__fmul_rn(v, v));
    }
    const double ssq = block_sum_d(s, scratch);
    const float rscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ssq / static_cast<double>(dim)), eps)));
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], rscale), w[i]);
}

__global__ void add_kernel(float *__restrict__ h, const float *__restrict__ mix, int64_t n) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) h[i] = __fadd_rn(h[i], mix[i]);
}

__global__ void swiglu_kernel(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ o,
                              int64_t n) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) o[i] = __fmul_rn(silu_f(g[i]), u[i]);
}

// ---------------------------------------------------------------------------
// Gated DeltaNet pre-processing: one CTA (hd threads) per (sequence, head).
// Thread t owns the Q, K and V channels t of its head.
// ---------------------------------------------------------------------------
__global__ void gdn_pre_kernel(const float *__restrict__ qkv, float *__restrict__ ring,
                               const float *__restrict__ conv_w, const float *__restrict__ bb,
                               const float *__restrict__ aa, const float *__restrict__ dt_bias,
                               const float *__restrict__ ssm_a, int heads, int hd, int kk,
                               const int32_t *__restrict__ pos_ptr, float *__restrict__ qo, float *__restrict__ ko, float *__restrict__ vo,
                               float *__restrict__ beta, float *__restrict__ gout) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double scratch[32];
    const int b = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
    const int kdim = heads * hd, conv_dim = 3 * kdim;
    const int pos = max(*pos_ptr, 0);
    const int slot = pos % kk, head_after = (pos + 1) % kk;
    const float *src = qkv + static_cast<int64_t>(b) * conv_dim;
    float *rg = ring + static_cast<int64_t>(b) * kk * conv_dim;
    float mixed[3];
#pragma unroll
    for (int part = 0; part < 3; ++part) {
        const int ch = part * kdim + h * hd + t;
        rg[static_cast<int64_t>(slot) * conv_dim + ch] = src[ch];
        float acc = 0.0f;
        for (int k = 0; k < kk; ++k) {
            const int sl = (head_after + k) % kk;
            acc = __fadd_rn(acc, __fmul_rn(rg[static_cast<int64_t>(sl) * conv_dim + ch], conv_w[ch * kk + k]));
        }
        mixed[part] = silu_f(acc);
    }
    // per-head L2 norms (double sums of float squares), eps applied via fmaxf
    const double qss = block_sum_d(static_cast<double>(__fmul_rn(mixed[0], mixed[0])), scratch);
    const double kss = block_sum_d(static_cast<double>(__fmul_rn(mixed[1], mixed[1])), scratch);
    const float qrs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(qss)), 1e-6f));
    const float krs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(kss)), 1e-6f));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));
    const int64_t o = static_cast<int64_t>(b) * kdim + h * hd + t;
    qo[o] = __fmul_rn(__fmul_rn(mixed[0], qrs), scale);
    ko[o] = __fmul_rn(mixed[1], krs);
    vo[o] = mixed[2];
    if (t == 0) {
        const int i = b * heads + h;
        beta[i] = sigmoid_f(bb[i]);
        const float a = __fadd_rn(aa[i], dt_bias[h]);
        const float sp = a > 20.0f ? a : logf_ref(__fadd_rn(1.0f, expf_ref(a)));
        gout[i] = expf_ref(__fmul_rn(ssm_a[h], sp));
    }
}

// ---------------------------------------------------------------------------
// Gated DeltaNet recurrence: one CTA per (sequence, head); thread v owns
// state column v (hd values in registers), so both reductions over k are
// sequential in k exactly as in the reference.
// ---------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(HD) gdn_recurrence_kernel(float *__restrict__ state,
                                                            const float *__restrict__ q,
                                                            const float *__restrict__ kv,
                                                            const float *__restrict__ vv,
                                                            const float *__restrict__ beta,
                                                            const float *__restrict__ g, int heads,
                                                            float *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float Ks[HD], Qs[HD];
    const int b = blockIdx.x, h = blockIdx.y, v = threadIdx.x;
    const int64_t vec = (static_cast<int64_t>(b) * heads + h) * HD;
    Ks[v] = kv[vec + v];
    Qs[v] = q[vec + v];
    __syncthreads();
    float *st = state + (static_cast<int64_t>(b) * heads + h) * HD * HD;
    const float gh = g[b * heads + h], bh = beta[b * heads + h];
    float s[HD];
    double acc = 0.0;
#pragma unroll
    for (int k = 0; k < HD; ++k) {
        s[k] = __fmul_rn(st[k * HD + v], gh);
        acc += static_cast<double>(__fmul_rn(s[k], Ks[k]));
    }
    const float delta = __fmul_rn(__fsub_rn(vv[vec + v], static_cast<float>(acc)), bh);
    double acc2 = 0.0;
#pragma unroll
    for (int k = 0; k < HD; ++k) {
        s[k] = __fadd_rn(s[k], __fmul_rn(Ks[k], delta));
        st[k * HD + v] = s[k];
        acc2 += static_cast<double>(__fmul_rn(s[k], Qs[k]));
    }
    out[vec + v] = static_cast<float>(acc2);
}

// Gated RMSNorm: one CTA (hd threads) per (sequence, head).
__global__ void gdn_gated_norm_kernel(const float *__restrict__ x, const float *__restrict__ z,
                                      const float *__restrict__ w, int hd, float eps, float *__restrict__ y) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double scratch[32];
    const int64_t base = (static_cast<int64_t>(blockIdx.x) * gridDim.y + blockIdx.y) * hd;
    const int t = threadIdx.x;
    const float v = x[base + t];
    const double ssq = block_sum_d(static_cast<double>(__fmul_rn(v, v)), scratch);
    const float mean = static_cast<float>(ssq / static_cast<double>(hd));
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    y[base + t] = __fmul_rn(__fmul_rn(__fmul_rn(v, rs), w[t]), silu_f(z[base + t]));
}

// ---------------------------------------------------------------------------
// Attention pre-processing: CTA (b, j), hd threads; j < nh is query head j
// (also emits its gate), j >= nh is KV head j - nh (appends K and V).
// ---------------------------------------------------------------------------
__global__ void attn_pre_kernel(const float *__restrict__ qraw, const float *__restrict__ kin,
                                const float *__restrict__ vin, const float *__restrict__ qn_w,
                                const float *__restrict__ kn_w, const float *__restrict__ rope, int nh,
                                int kvh, int hd, int rope_dim, float eps,
                                const int32_t *__restrict__ pos_ptr, int max_pos,
                                float *__restrict__ qout, float *__restrict__ gate,
                                __half *__restrict__ kcache, __half *__restrict__ vcache, int rows_per_seq) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double scratch[32];
    __shared__ float xs[512];
    // row b holds token (b % rows_per_seq) of sequence b / rows_per_seq, at
    // position *pos_ptr + b % rows_per_seq (decode: one row per sequence)
    const int b = blockIdx.x, j = blockIdx.y, t = threadIdx.x;
    const int seq = b / rows_per_seq;
    const int pos = min(max(*pos_ptr + b % rows_per_seq, 0), max_pos - 1);
    const bool is_q = j < nh;
    float x;
    if (is_q) {
        const float *src = qraw + static_cast<int64_t>(b) * 2 * nh * hd + static_cast<int64_t>(j) * 2 * hd;
        x = src[t];
        gate[static_cast<int64_t>(b) * nh * hd + j * hd + t] = src[hd + t];
    } else {
        x = kin[static_cast<int64_t>(b) * kvh * hd + (j - nh) * hd + t];
    }
    const double ssq = block_sum_d(static_cast<double>(__fmul_rn(x, x)), scratch);
    const float rscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ssq / static_cast<double>(hd)), eps)));
    const float xn = __fmul_rn(__fmul_rn(x, rscale), (is_q ? qn_w : kn_w)[t]);
    xs[t] = xn;
    __syncthreads();
    const int half = rope_dim / 2;
    float y = xn;
    if (t < rope_dim) {
        const int i = t < half ? t : t - half;
        const float c = rope[(static_cast<int64_t>(pos) * half + i) * 2];
        const float sn = rope[(static_cast<int64_t>(pos) * half + i) * 2 + 1];
        const float x0 = xs[i], x1 = xs[i + half];
        y = t < half ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn))
                     : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    if (is_q) {
        qout[(static_cast<int64_t>(b) * nh + j) * hd + t] = y;
    } else {
        const int kh = j - nh;
        const int64_t row = ((static_cast<int64_t>(seq) * max_pos + pos) * kvh + kh) * hd + t;
        kcache[row] = __float2half_rn(y);
        vcache[row] = __float2half_rn(vin[static_cast<int64_t>(b) * kvh * hd + kh * hd + t]);
    }
}

// ---------------------------------------------------------------------------
// Attention over the cache: one CTA (hd threads) per (sequence, query head).
// ---------------------------------------------------------------------------
__global__ void attn_decode_kernel(const float *__restrict__ q, const __half *__restrict__ kcache,
                                   const __half *__restrict__ vcache, const float *__restrict__ gate,
                                   int nh, int kvh, int hd, const int32_t *__restrict__ pos_ptr,
                                   int max_pos, float *__restrict__ ctx) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float sh[];  // [hd] query, [max_pos] scores, [32] scratch
    float *qs = sh;
    float *sc = sh + hd;
    float *scratch = sc + max_pos;
    const int pos = min(max(*pos_ptr, 0), max_pos - 1);
    __shared__ float total;
    const int b = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
    const int kh = h / (nh / kvh);
    const int n = pos + 1;
    qs[t] = q[(static_cast<int64_t>(b) * nh + h) * hd + t];
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));
    const __half *kb = kcache + (static_cast<int64_t>(b) * max_pos * kvh + kh) * hd;
    const __half *vb = vcache + (static_cast<int64_t>(b) * max_pos * kvh + kh) * hd;
    const int64_t rstride = static_cast<int64_t>(kvh) * hd;
    float lmax = -INFINITY;
    for (int i = t; i < n; i += blockDim.x) {
        const __half *kr = kb + i * rstride;
        float dot = 0.0f;
        for (int d = 0; d < hd; ++d) dot = __fadd_rn(dot, __fmul_rn(qs[d], __half2float(kr[d])));
        const float s = __fmul_rn(dot, scale);
        sc[i] = s;
        lmax = fmaxf(lmax, s);
    }
    const float m = block_max_f(lmax, scratch);
    for (int i = t; i < n; i += blockDim.x) sc[i] = expf_ref(__fsub_rn(sc[i], m));
    __syncthreads();
    if (t == 0) {
        float s = 0.0f;
        for (int i = 0; i < n; ++i) s = __fadd_rn(s, sc[i]);
        total = s;
    }
    __syncthreads();
    const float inv = __fdiv_rn(1.0f, total);
    for (int i = t; i < n; i += blockDim.x) sc[i] = __fmul_rn(sc[i], inv);
    __syncthreads();
    float o = 0.0f;
    for (int i = 0; i < n; ++i) o = __fadd_rn(o, __fmul_rn(sc[i], __half2float(vb[i * rstride + t])));
    const int64_t oi = static_cast<int64_t>(b) * nh * hd + h * hd + t;
    ctx[oi] = __fmul_rn(o, sigmoid_f(gate[oi]));
}

// Attention over the cache for G query heads of one GQA group: CTA
// (sequence, G heads) of HD threads serves G heads sharing a KV head (the
// whole group, or fewer so that the CTAs fill the GPU in one wave), so every
// cache row is read once for G heads. Per head the arithmetic and its order
// are those of attn_decode_kernel (tensor_attention, slm/tensor.c:1049-1102):
// sequential dot per position, max, exp, sequential sum, scaling, and a
// sequential weighted sum of V rows per dimension.
constexpr int kAttnVChunk = 32;  // V rows per bulk-copied chunk
constexpr int kAttnVBufs = 4;    // chunk buffers: up to kAttnVBufs - 1 chunks in flight ahead
template <int G>
__global__ void __launch_bounds__(128) attn_decode_gqa_kernel(const float *__restrict__ q, const __half *__restrict__ kcache,
                                                              const __half *__restrict__ vcache,
                                                              const float *__restrict__ gate, int nh, int kvh,
                                                              const int32_t *__restrict__ pos_ptr, int max_pos,
                                                              float *__restrict__ ctx, int rows_per_seq, int qgroup) {
    constexpr int HD = 128;
    pdl_launch_dependents();
    pdl_wait();
    // [G][HD] queries, [G][max_pos] scores, then kAttnVBufs V chunks of
    // kAttnVChunk rows (16-byte aligned: max_pos rounded up to 4)
    extern __shared__ __align__(16) float sh[];
    float *qs = sh;
    float *sc = sh + G * HD;
    __half *vbuf = reinterpret_cast<__half *>(sc + G * ((max_pos + 3) & ~3));
    __shared__ float red[G][32];
    __shared__ float s_inv[G];
    // CTA (sequence b, query heads q0 .. q0 + G - 1, query j): the query row
    // b * rows_per_seq + j at position *pos_ptr + j (decode: j = 0, one row per
    // sequence); the heads share KV head q0 / qgroup (G == qgroup: one CTA per
    // KV head, every cache row read once for its G heads; G == 1: one CTA per
    // query head, each reading the rows again -- more CTAs for many sequences)
    const int b = blockIdx.x, q0 = blockIdx.y * G, kh = q0 / qgroup, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t qrow = static_cast<int64_t>(b) * rows_per_seq + blockIdx.z;
    const int pos = min(max(*pos_ptr + static_cast<int>(blockIdx.z), 0), max_pos - 1);
    const int n = pos + 1;
    const int64_t rstride = static_cast<int64_t>(kvh) * HD;
    const __half *kb = kcache + (static_cast<int64_t>(b) * max_pos * kvh + kh) * HD;
    const __half *vb = vcache + (static_cast<int64_t>(b) * max_pos * kvh + kh) * HD;
    const int n_chunks = (n + kAttnVChunk - 1) / kAttnVChunk;
    // V rows of chunk c into buffer c % kAttnVBufs: every thread copies 16-byte
    // pieces with cp.async (16 pieces per 256-byte row), one commit group per
    // chunk (an empty group past the last chunk keeps the group count fixed)
    auto issue_v = [&](int c) {
        if (c < n_chunks) {
            const int r0 = c * kAttnVChunk, rows = min(kAttnVChunk, n - r0);
            __half *dst = vbuf + (c % kAttnVBufs) * kAttnVChunk * HD;
            for (int piece = t; piece < rows * (HD / 8); piece += blockDim.x) {
                const int j = piece / (HD / 8), q16 = piece % (HD / 8);
                const uint32_t sa = smem_addr(dst + j * HD + q16 * 8);
                const __half *ga = vb + (r0 + j) * rstride + q16 * 8;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(ga) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // the first V chunks stream in while the scores are formed
    for (int c = 0; c < kAttnVBufs - 1; ++c) issue_v(c);
#pragma unroll
    for (int g = 0; g < G; ++g) qs[g * HD + t] = q[(qrow * nh + q0 + g) * HD + t];
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HD)));
    float lmax[G];
#pragma unroll
    for (int g = 0; g < G; ++g) lmax[g] = -INFINITY;
    // scores: thread t takes positions t, t + 128, ...; the next row's 256
    // bytes are loaded while the current one is summed
    auto load_row = [&](int i, uint4 (&row)[HD / 8]) {
        const uint4 *kr = reinterpret_cast<const uint4 *>(kb + i * rstride);
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) row[c] = __ldg(kr + c);
    };
    auto score = [&](int i, const uint4 (&row)[HD / 8]) {
        float dot[G];
#pragma unroll
        for (int g = 0; g < G; ++g) dot[g] = 0.0f;
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
            const __half2 *hp = reinterpret_cast<const __half2 *>(&row[c]);
            float kf[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(hp[e]);
                kf[2 * e] = f.x;
                kf[2 * e + 1] = f.y;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e)
#pragma unroll
                for (int g = 0; g < G; ++g) dot[g] = __fadd_rn(dot[g], __fmul_rn(qs[g * HD + 8 * c + e], kf[e]));
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float s = __fmul_rn(dot[g], scale);
            sc[g * max_pos + i] = s;
            lmax[g] = fmaxf(lmax[g], s);
        }
    };
    {
        uint4 ra[HD / 8], rb[HD / 8];
        int i = t;
        if (i < n) load_row(i, ra);
        for (; i < n; i += 2 * blockDim.x) {
            if (i + blockDim.x < n) load_row(i + blockDim.x, rb);
            score(i, ra);
            if (i + blockDim.x >= n) break;
            if (i + 2 * blockDim.x < n) load_row(i + 2 * blockDim.x, ra);
            score(i + blockDim.x, rb);
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float v = lmax[g];
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) red[g][warp] = v;
    }
    __syncthreads();
    float m[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = red[g][0];
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m[g] = fmaxf(m[g], red[g][w]);
    }
    for (int i = t; i < n; i += blockDim.x)
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g * max_pos + i] = expf_ref(__fsub_rn(sc[g * max_pos + i], m[g]));
    __syncthreads();
    if (t < G) {  // sequential sums, one head per thread
        const float *st = sc + t * max_pos;
        float s = 0.0f;
        int i = 0;
        for (; i + 8 <= n; i += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = st[i + j];
#pragma unroll
            for (int j = 0; j < 8; ++j) s = __fadd_rn(s, v[j]);
        }
        for (; i < n; ++i) s = __fadd_rn(s, st[i]);
        s_inv[t] = __fdiv_rn(1.0f, s);
    }
    __syncthreads();
    for (int i = t; i < n; i += blockDim.x)
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g * max_pos + i] = __fmul_rn(sc[g * max_pos + i], s_inv[g]);
    __syncthreads();
    // weighted V sum: chunks of V rows arrive in shared memory by bulk copies
    // (the next chunk in flight while this one is summed); per dimension the
    // sum stays sequential in position order
    float o[G];
#pragma unroll
    for (int g = 0; g < G; ++g) o[g] = 0.0f;
    for (int c = 0; c < n_chunks; ++c) {
        issue_v(c + kAttnVBufs - 1);
        // this thread's pieces of chunk c have landed; the barrier makes
        // every thread's pieces visible
        asm volatile("cp.async.wait_group %0;" ::"n"(kAttnVBufs - 1) : "memory");
        __syncthreads();
        const __half *vc = vbuf + (c % kAttnVBufs) * kAttnVChunk * HD;
        const int r0 = c * kAttnVChunk, rows = min(kAttnVChunk, n - r0);
        for (int j = 0; j < rows; ++j) {
            const float v = __half2float(vc[j * HD + t]);
#pragma unroll
            for (int g = 0; g < G; ++g) o[g] = __fadd_rn(o[g], __fmul_rn(sc[g * max_pos + r0 + j], v));
        }
        __syncthreads();  // this buffer is refilled by the issue of chunk c + kAttnVBufs
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int64_t oi = qrow * nh * HD + (q0 + g) * HD + t;
        ctx[oi] = __fmul_rn(o[g], sigmoid_f(gate[oi]));
    }
}

// Greedy argmax: one CTA per row; ties keep the smaller index.
__global__ void argmax_kernel(const float *__restrict__ logits, int64_t vocab, int32_t *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *row = logits + static_cast<int64_t>(blockIdx.x) * vocab;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float v = row[i];
        if (v > best) { best = v; bi = static_cast<int>(i); }
    }
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = sv[0];
        int i = si[0];
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
            if (sv[w] > b || (sv[w] == b && si[w] < i)) { b = sv[w]; i = si[w]; }
        out[blockIdx.x] = i == 0x7fffffff ? 0 : i;
    }
}

// End of a decode step on the device: record the picks, choose the next
// input (the prompt while inside it, else the pick) and advance the position.
__global__ void feed_next_kernel(const int32_t *__restrict__ next, const int32_t *__restrict__ prompt, int32_t B,
                                 int32_t stride, int32_t *__restrict__ ctl, int32_t *__restrict__ tokens,
                                 int32_t *__restrict__ picks) {
    pdl_launch_dependents();
    pdl_wait();
    const int pos = ctl[0], n_prompt = ctl[1];
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        const int32_t nx = next[b];
        if (pos >= 0 && pos < stride) picks[static_cast<int64_t>(b) * stride + pos] = nx;
        tokens[b] = (pos + 1 < n_prompt && pos + 1 < stride) ? prompt[static_cast<int64_t>(b) * stride + pos + 1] : nx;
    }
    __syncthreads();
    if (threadIdx.x == 0) ctl[0] = pos + 1;
}

}  // namespace qh

// ---------------------------------------------------------------------------
// C-ABI launchers
// ---------------------------------------------------------------------------
namespace {
int launch_status(cudaError_t e, const char *what) {
    const cudaError_t last = cudaGetLastError();
    if (e == cudaSuccess) e = last;
    if (e == cudaSuccess) return QH_OK;
    char msg[256];
    snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
    qh::set_last_error_message(msg);
    return QH_ERR_CUDA;
}
int bad(const char *what) {
    qh::set_last_error_message(what);
    return QH_ERR_INVALID;
}
}  // namespace

extern "C" {

int qh_embed_q6k(const void *d_table, int64_t hidden, const int32_t *d_tokens, int32_t B, float *d_h,
                 void *stream) {
    if (!d_table || !d_tokens || !d_h || hidden % 256 || B <= 0) return bad("qh_embed_q6k: bad arguments");
    dim3 grid(static_cast<unsigned>(hidden / 256), static_cast<unsigned>(B));
    const cudaError_t le = qh::launch_pdl(qh::embed_q6k_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), 
        static_cast<const uint8_t *>(d_table), hidden, d_tokens, d_h);
    return launch_status(le, "qh_embed_q6k");
}

int qh_embed_f32(const float *d_table, int64_t hidden, const int32_t *d_tokens, int32_t B, float *d_h,
                 void *stream) {
    if (!d_table || !d_tokens || !d_h || hidden <= 0 || B <= 0) return bad("qh_embed_f32: bad arguments");
    dim3 grid(static_cast<unsigned>((hidden + 255) / 256 < 8 ? (hidden + 255) / 256 : 8), static_cast<unsigned>(B));
    const cudaError_t le = qh::launch_pdl(qh::embed_f32_kernel, grid, dim3(256), 0, static_cast<cudaStream_t>(stream),
                                          d_table, hidden, d_tokens, d_h);
    return launch_status(le, "qh_embed_f32");
}

int qh_rmsnorm(const float *d_x, const float *d_w, int64_t dim, int64_t rows, float eps, float *d_y,
               void *stream) {
    if (!d_x || !d_w || !d_y || dim <= 0 || rows <= 0 || rows > 0x7fffffff) return bad("qh_rmsnorm: bad arguments");
    const int threads = dim >= 256 ? 256 : 128;
    const cudaError_t le = qh::launch_pdl(qh::rmsnorm_kernel, dim3(static_cast<unsigned>(rows)), dim3(threads), 0, static_cast<cudaStream_t>(stream), 
        d_x, d_w, dim, eps, d_y);
    return launch_status(le, "qh_rmsnorm");
}

int qh_add(float *d_h, const float *d_mix, int64_t n, void *stream) {
    if (!d_h || !d_mix || n <= 0) return bad("qh_add: bad arguments");
    const cudaError_t le = qh::launch_pdl(qh::add_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), d_h, d_mix, n);
    return launch_status(le, "qh_add");
}

int qh_swiglu(const float *d_gate, const float *d_up, float *d_out, int64_t n, void *stream) {
    if (!d_gate || !d_up || !d_out || n <= 0) return bad("qh_swiglu: bad arguments");
    const cudaError_t le = qh::launch_pdl(qh::swiglu_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), 
        d_gate, d_up, d_out, n);
    return launch_status(le, "qh_swiglu");
}

int qh_gdn_pre(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b,
               const float *d_a, const float *d_dt_bias, const float *d_ssm_a, int32_t B,
               int32_t heads, int32_t hd, int32_t kk, const int32_t *d_pos, float *d_q, float *d_k,
               float *d_v, float *d_beta, float *d_g, void *stream) {
    if (B <= 0 || heads <= 0 || hd <= 0 || hd % 32 || hd > 1024 || kk <= 0 || !d_pos)
        return bad("qh_gdn_pre: bad arguments");
    dim3 grid(static_cast<unsigned>(B), static_cast<unsigned>(heads));
    const cudaError_t le = qh::launch_pdl(qh::gdn_pre_kernel, dim3(grid), dim3(hd), 0, static_cast<cudaStream_t>(stream), 
        d_qkv, d_ring, d_conv_w, d_b, d_a, d_dt_bias, d_ssm_a, heads, hd, kk, d_pos, d_q, d_k, d_v, d_beta, d_g);
    return launch_status(le, "qh_gdn_pre");
}

int qh_gdn_recurrence(float *d_state, const float *d_q, const float *d_k, const float *d_v,
                      const float *d_beta, const float *d_g, int32_t B, int32_t heads, int32_t hd,
                      float *d_out, void *stream) {
    if (B <= 0 || heads <= 0) return bad("qh_gdn_recurrence: bad arguments");
    if (hd != 128) {
        qh::set_last_error_message("qh_gdn_recurrence: head dim must be 128");
        return QH_ERR_UNSUPPORTED;
    }
    dim3 grid(static_cast<unsigned>(B), static_cast<unsigned>(heads));
    const cudaError_t le = qh::launch_pdl(qh::gdn_recurrence_kernel<128>, dim3(grid), dim3(128), 0, static_cast<cudaStream_t>(stream), 
        d_state, d_q, d_k, d_v, d_beta, d_g, heads, d_out);
    return launch_status(le, "qh_gdn_recurrence");
}

int qh_gdn_gated_norm(const float *d_x, const float *d_z, const float *d_w, int32_t B, int32_t heads,
                      int32_t hd, float eps, float *d_y, void *stream) {
    if (B <= 0 || heads <= 0 || hd <= 0 || hd % 32 || hd > 1024) return bad("qh_gdn_gated_norm: bad arguments");
    dim3 grid(static_cast<unsigned>(B), static_cast<unsigned>(heads));
    const cudaError_t le = qh::launch_pdl(qh::gdn_gated_norm_kernel, dim3(grid), dim3(hd), 0, static_cast<cudaStream_t>(stream), d_x, d_z, d_w, hd, eps, d_y);
    return launch_status(le, "qh_gdn_gated_norm");
}

}  // extern "C"

namespace {
// rows = n_seq * rows_per_seq query rows (sequence-major), positions
// *d_pos + (row % rows_per_seq).
int attn_pre_impl(const float *d_qraw, const float *d_k, const float *d_v, const float *d_qnorm_w,
                  const float *d_knorm_w, const float *d_rope, int32_t rows, int32_t rows_per_seq, int32_t nh,
                  int32_t kvh, int32_t hd, int32_t rope_dim, float eps, const int32_t *d_pos, int32_t max_pos,
                  float *d_q, float *d_gate, uint16_t *d_kcache, uint16_t *d_vcache, void *stream, const char *what) {
    if (rows <= 0 || rows_per_seq <= 0 || rows % rows_per_seq || nh <= 0 || kvh <= 0 || nh % kvh || hd % 32 ||
        hd > 512 || rope_dim > hd || rope_dim % 2 || !d_pos || max_pos <= 0)
        return bad(what);
    dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>(nh + kvh));
    const cudaError_t le = qh::launch_pdl(qh::attn_pre_kernel, dim3(grid), dim3(hd), 0, static_cast<cudaStream_t>(stream),
        d_qraw, d_k, d_v, d_qnorm_w, d_knorm_w, d_rope, nh, kvh, hd, rope_dim, eps, d_pos, max_pos, d_q, d_gate,
        reinterpret_cast<__half *>(d_kcache), reinterpret_cast<__half *>(d_vcache), rows_per_seq);
    return launch_status(le, what);
}

bool gqa_ok(int32_t nh, int32_t kvh, int32_t hd, const void *kc) {
    const int G = nh / kvh;
    return hd == 128 && (G == 1 || G == 2 || G == 4 || G == 8) && (reinterpret_cast<uintptr_t>(kc) & 15) == 0;
}

int attn_gqa_impl(const float *d_q, const uint16_t *d_kcache, const uint16_t *d_vcache, const float *d_gate,
                  int32_t n_seq, int32_t rows_per_seq, int32_t nh, int32_t kvh, const int32_t *d_pos,
                  int32_t max_pos, float *d_ctx, void *stream, const char *what) {
    const int qgroup = nh / kvh;
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // Query heads per CTA: the whole group (each cache row read once for all
    // of them) when that already fills the GPU twice over, else the fewest
    // whose CTAs still run in one wave (three resident per SM): more CTAs,
    // each reading the rows again, for decode at up to ~100 sequences
    const int64_t group_ctas = static_cast<int64_t>(n_seq) * rows_per_seq * kvh;
    int G = qgroup;
    if (group_ctas < 2 * static_cast<int64_t>(sms)) {
        G = 1;
        while (G < qgroup && group_ctas * (qgroup / G) > 3 * static_cast<int64_t>(sms)) G *= 2;
    }
    const size_t smem = sizeof(float) * static_cast<size_t>(G) * (128 + ((static_cast<size_t>(max_pos) + 3) & ~size_t(3))) +
                        qh::kAttnVBufs * qh::kAttnVChunk * 128 * sizeof(__half);
    if (smem > 200 * 1024) return bad("attention: context too long");
    if (rows_per_seq > 65535) return bad(what);
    static bool gattr[64][4] = {};
    const int gi = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
    void (*kern)(const float *, const __half *, const __half *, const float *, int, int, const int32_t *, int, float *,
                 int, int) = G == 1   ? qh::attn_decode_gqa_kernel<1>
                             : G == 2 ? qh::attn_decode_gqa_kernel<2>
                             : G == 4 ? qh::attn_decode_gqa_kernel<4>
                                      : qh::attn_decode_gqa_kernel<8>;
    if (dev >= 0 && dev < 64 && !gattr[dev][gi]) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        gattr[dev][gi] = true;
    }
    const cudaError_t le = qh::launch_pdl(kern, dim3(static_cast<unsigned>(n_seq), nh / G, rows_per_seq), dim3(128),
                                          smem, static_cast<cudaStream_t>(stream), d_q,
                                          reinterpret_cast<const __half *>(d_kcache),
                                          reinterpret_cast<const __half *>(d_vcache), d_gate, nh, kvh, d_pos, max_pos,
                                          d_ctx, rows_per_seq, qgroup);
    return launch_status(le, what);
}
}  // namespace

extern "C" {

int qh_attn_pre(const float *d_qraw, const float *d_k, const float *d_v, const float *d_qnorm_w,
                const float *d_knorm_w, const float *d_rope, int32_t B, int32_t nh, int32_t kvh,
                int32_t hd, int32_t rope_dim, float eps, const int32_t *d_pos, int32_t max_pos,
                float *d_q, float *d_gate, uint16_t *d_kcache, uint16_t *d_vcache, void *stream) {
    return attn_pre_impl(d_qraw, d_k, d_v, d_qnorm_w, d_knorm_w, d_rope, B, 1, nh, kvh, hd, rope_dim, eps, d_pos,
                         max_pos, d_q, d_gate, d_kcache, d_vcache, stream, "qh_attn_pre: bad arguments");
}

int qh_attn_prefill_pre(const float *d_qraw, const float *d_k, const float *d_v, const float *d_qnorm_w,
                        const float *d_knorm_w, const float *d_rope, int32_t n_seq, int32_t n_tok, int32_t nh,
                        int32_t kvh, int32_t hd, int32_t rope_dim, float eps, const int32_t *d_pos, int32_t max_pos,
                        float *d_q, float *d_gate, uint16_t *d_kcache, uint16_t *d_vcache, void *stream) {
    if (n_seq <= 0 || n_tok <= 0 || static_cast<int64_t>(n_seq) * n_tok > 0x7fffffff)
        return bad("qh_attn_prefill_pre: bad arguments");
    return attn_pre_impl(d_qraw, d_k, d_v, d_qnorm_w, d_knorm_w, d_rope, n_seq * n_tok, n_tok, nh, kvh, hd, rope_dim,
                         eps, d_pos, max_pos, d_q, d_gate, d_kcache, d_vcache, stream,
                         "qh_attn_prefill_pre: bad arguments");
}

int qh_attn_prefill(const float *d_q, const uint16_t *d_kcache, const uint16_t *d_vcache, const float *d_gate,
                    int32_t n_seq, int32_t n_tok, int32_t nh, int32_t kvh, int32_t hd, const int32_t *d_pos,
                    int32_t max_pos, float *d_ctx, void *stream) {
    if (n_seq <= 0 || n_tok <= 0 || nh <= 0 || kvh <= 0 || nh % kvh || !d_pos || max_pos <= 0 || !d_q ||
        !d_kcache || !d_vcache || !d_gate || !d_ctx)
        return bad("qh_attn_prefill: bad arguments");
    if (!gqa_ok(nh, kvh, hd, d_kcache)) {
        qh::set_last_error_message("qh_attn_prefill: needs head dim 128 and a query group of 1, 2, 4 or 8");
        return QH_ERR_UNSUPPORTED;
    }
    return attn_gqa_impl(d_q, d_kcache, d_vcache, d_gate, n_seq, n_tok, nh, kvh, d_pos, max_pos, d_ctx, stream,
                         "qh_attn_prefill");
}

int qh_attn_decode(const float *d_q, const uint16_t *d_kcache, const uint16_t *d_vcache,
                   const float *d_gate, int32_t B, int32_t nh, int32_t kvh, int32_t hd,
                   const int32_t *d_pos, int32_t max_pos, float *d_ctx, void *stream) {
    if (B <= 0 || nh <= 0 || kvh <= 0 || nh % kvh || hd % 32 || hd > 1024 || !d_pos || max_pos <= 0)
        return bad("qh_attn_decode: bad arguments");
    if (gqa_ok(nh, kvh, hd, d_kcache))  // CTAs of one or more query heads sharing a KV head
        return attn_gqa_impl(d_q, d_kcache, d_vcache, d_gate, B, 1, nh, kvh, d_pos, max_pos, d_ctx, stream,
                             "qh_attn_decode");
    const size_t smem = sizeof(float) * (static_cast<size_t>(hd) + max_pos + 32);
    if (smem > 200 * 1024) return bad("qh_attn_decode: context too long");
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaFuncSetAttribute(qh::attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_done[dev] = true;
    }
    dim3 grid(static_cast<unsigned>(B), static_cast<unsigned>(nh));
    const cudaError_t le = qh::launch_pdl(qh::attn_decode_kernel, dim3(grid), dim3(hd), smem, static_cast<cudaStream_t>(stream), 
        d_q, reinterpret_cast<const __half *>(d_kcache), reinterpret_cast<const __half *>(d_vcache), d_gate, nh,
        kvh, hd, d_pos, max_pos, d_ctx);
    return launch_status(le, "qh_attn_decode");
}

int qh_argmax(const float *d_logits, int32_t B, int64_t vocab, int32_t *d_out, void *stream) {
    if (!d_logits || !d_out || B <= 0 || vocab <= 0) return bad("qh_argmax: bad arguments");
    const cudaError_t le = qh::launch_pdl(qh::argmax_kernel, dim3(static_cast<unsigned>(B)), dim3(1024), 0, static_cast<cudaStream_t>(stream), d_logits, vocab, d_out);
    return launch_status(le, "qh_argmax");
}

int qh_feed_next(const int32_t *d_next, const int32_t *d_prompt, int32_t B, int32_t stride, int32_t *d_ctl,
                 int32_t *d_tokens, int32_t *d_picks, void *stream) {
    if (!d_next || !d_prompt || !d_ctl || !d_tokens || !d_picks || B <= 0 || stride <= 0)
        return bad("qh_feed_next: bad arguments");
    const cudaError_t le = qh::launch_pdl(qh::feed_next_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream), d_next, d_prompt, B, stride, d_ctl,
                                                                          d_tokens, d_picks);
    return launch_status(le, "qh_feed_next");
}

}  // extern "C"

// ===========================================================================
// Fused kernels of the decode step. Each one replaces a chain of the kernels
// above with identical arithmetic (same operations, same order, same
// rounding), so results are bit-identical to the unfused chain; they exist
// to cut launches and round trips through HBM per token.
// ===========================================================================
namespace qh {

// (optional residual add) + RMSNorm + Q8_K. CTA (block j, row), 256
// threads: every CTA of a row forms the row's sum of squares in the same
// order (thread t sums elements t, t+256, ... in double, then the block
// reduction of rmsnorm_kernel with 256 threads), then quantizes its own
// block; with a residual, CTA j writes h_out's block j (h_out != h, so no
// CTA reads a value another one has updated).
// NB: the most blocks a row may have (4: hidden sizes up to 1024, held to
// 32 registers so that eight CTAs fit an SM for many-row prompt launches).
constexpr int kResNormMaxBlocks = 16;
template <int NB>
__global__ void __launch_bounds__(256, NB <= 4 ? 8 : 1) resnorm_q8k_kernel(const float *__restrict__ h, const float *__restrict__ mix,
                                                          float *__restrict__ h_out, const float *__restrict__ w,
                                                          int dim, float eps, uint8_t *__restrict__ xq, int n_tok,
                                                          int tile) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double scratch[32];
    __shared__ Q8KScratch sc;
    const int jb = blockIdx.x, row = blockIdx.y, tid = threadIdx.x, nb = dim / QH_QK;
    // every load of the thread (row values, residual branch, norm weight)
    // goes out before the first add: one memory round trip
    const int64_t r0 = static_cast<int64_t>(row) * dim + tid;
    float hv[NB], mv[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        hv[j] = j < nb ? h[r0 + j * QH_QK] : 0.0f;
        mv[j] = (mix && j < nb) ? mix[r0 + j * QH_QK] : 0.0f;
    }
    const float wv = w[jb * QH_QK + tid];
    float mine = 0.0f;
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        if (j < nb) {
            float x = hv[j];
            if (mix) x = __fadd_rn(x, mv[j]);
            if (j == jb) {
                mine = x;
                if (mix) h_out[r0 + j * QH_QK] = x;
            }
            s += static_cast<double>(__fmul_rn(x, x));
        }
    }
    const double ssq = block_sum_d(s, scratch);
    const float rscale =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ssq / static_cast<double>(dim)), eps)));
    const Q8KRow r = q8k_row(xq, dim, n_tok, row, tile);
    q8k_block256(__fmul_rn(__fmul_rn(mine, rscale), wv), sc, r, jb);
}

// SwiGLU + Q8_K: CTA (block, row), 256 threads.
__global__ void __launch_bounds__(256) swiglu_q8k_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                                         int ffn, uint8_t *__restrict__ xq, int n_tok, int tile) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ Q8KScratch sc;
    const int blk = blockIdx.x, row = blockIdx.y, tid = threadIdx.x;
    const int64_t i = static_cast<int64_t>(row) * ffn + blk * QH_QK + tid;
    const float v = __fmul_rn(silu_f(g[i]), u[i]);
    const Q8KRow r = q8k_row(xq, ffn, n_tok, row, tile);
    q8k_block256(v, sc, r, blk);
}

// Whole Gated DeltaNet head for one token: CTA (sequence, head) of HD
// threads runs gdn_pre_kernel, gdn_recurrence_kernel and
// gdn_gated_norm_kernel in registers and shared memory, then quantizes the
// gated-norm output to Q8_K. A Q8_K block (256) spans two heads, so CTAs
// come in clusters of two along the head axis and agree on the block
// maximum through distributed shared memory.
constexpr int kMaxConvTaps = 8;

// QUANT = false: no cluster; the gated-norm output goes to y_out (fp32
// [B][heads*HD]) for a separate quantizer -- more heads per SM when many
// sequences run (cluster pairs limit how many CTAs are resident).
template <int HD, bool QUANT>
__global__ void __launch_bounds__(HD)
    gdn_fused_kernel(const float *__restrict__ qkv, float *__restrict__ ring, const float *__restrict__ conv_w,
                     const float *__restrict__ bb, const float *__restrict__ aa, const float *__restrict__ dt_bias,
                     const float *__restrict__ ssm_a, float *__restrict__ state, const float *__restrict__ z,
                     const float *__restrict__ norm_w, int heads, int kk, float eps,
                     const int32_t *__restrict__ pos_ptr, uint8_t *__restrict__ xq, int n_tok, int tile,
                     int *__restrict__ err_flag, float *__restrict__ y_out) {
    static_assert(HD == 128, "a cluster pair of heads must form one 256-value Q8_K block");
    pdl_launch_dependents();
    // the conv taps' weights are constant: loaded while the previous kernel finishes
    float cw[3][kMaxConvTaps];
    {
        const int ch0 = blockIdx.y * HD + threadIdx.x, kd = heads * HD;
#pragma unroll
        for (int part = 0; part < 3; ++part)
#pragma unroll
            for (int k = 0; k < kMaxConvTaps; ++k)
                if (k < kk) cw[part][k] = conv_w[(part * kd + ch0) * kk + k];
    }
    pdl_wait();
    // The head's 64 KB state arrives by one bulk copy while the conv and
    // norms run, is updated in shared memory and leaves by one bulk store.
    extern __shared__ __align__(128) float st_s[];  // [HD k][HD v]
    __shared__ uint64_t st_bar;
    __shared__ double scratch[64];
    __shared__ float Ks[HD], Qs[HD];
    __shared__ float s_beta, s_g;
    __shared__ float wa[HD / 32], wv[HD / 32];
    __shared__ int wi[HD / 32];
    __shared__ float c_a, c_v;
    __shared__ int c_i;
    const int b = blockIdx.x, h = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int kdim = heads * HD, conv_dim = 3 * kdim;
    float *st = state + (static_cast<int64_t>(b) * heads + h) * HD * HD;
    if (t == 0) {
        mbar_init(&st_bar, 1);
        mbar_fence_init();
        mbar_arrive_expect_tx(&st_bar, HD * HD * 4);
        bulk_copy_g2s(st_s, st, HD * HD * 4, &st_bar);
    }
    // ---- conv ring + SiLU + L2 norms + beta/g (gdn_pre_kernel) ----
    // Every load is issued before the position arrives: the new input and
    // all kk rows of the ring (the taps are picked once the position is known).
    const float *src = qkv + static_cast<int64_t>(b) * conv_dim;
    float *rg = ring + static_cast<int64_t>(b) * kk * conv_dim;
    float xin[3], rows[3][kMaxConvTaps];
#pragma unroll
    for (int part = 0; part < 3; ++part) {
        const int ch = part * kdim + h * HD + t;
        xin[part] = src[ch];
#pragma unroll
        for (int r = 0; r < kMaxConvTaps; ++r)
            if (r < kk) rows[part][r] = rg[static_cast<int64_t>(r) * conv_dim + ch];
    }
    const int pos = max(*pos_ptr, 0);
    const int slot = pos % kk, head_after = (pos + 1) % kk;
    // beta and g on another warp while the conv runs
    if (t == 32) {
        const int i = b * heads + h;
        s_beta = sigmoid_f(bb[i]);
        const float a = __fadd_rn(aa[i], dt_bias[h]);
        const float sp = a > 20.0f ? a : logf_ref(__fadd_rn(1.0f, expf_ref(a)));
        s_g = expf_ref(__fmul_rn(ssm_a[h], sp));
    }
    // The kk - 1 older taps from the ring (the newest tap is the new input
    // itself), then the ring update, then the sums in tap order -- the same
    // values and order as writing the slot and reading every tap back.
    float taps[3][kMaxConvTaps - 1];
#pragma unroll
    for (int part = 0; part < 3; ++part)
#pragma unroll
        for (int k = 0; k < kMaxConvTaps - 1; ++k) {
            const int rsel = (head_after + k) % kk;
            float v = 0.0f;
#pragma unroll
            for (int r = 0; r < kMaxConvTaps; ++r)
                if (r == rsel) v = rows[part][r];
            taps[part][k] = v;
        }
    float mixed[3];
#pragma unroll
    for (int part = 0; part < 3; ++part) {
        const int ch = part * kdim + h * HD + t;
        rg[static_cast<int64_t>(slot) * conv_dim + ch] = xin[part];
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < kMaxConvTaps; ++k)
            if (k < kk) acc = __fadd_rn(acc, __fmul_rn(k < kk - 1 ? taps[part][k] : xin[part], cw[part][k]));
        mixed[part] = silu_f(acc);
    }
    const double2 qkss = block_sum_d2(static_cast<double>(__fmul_rn(mixed[0], mixed[0])),
                                      static_cast<double>(__fmul_rn(mixed[1], mixed[1])), scratch);
    const double qss = qkss.x, kss = qkss.y;
    const float qrs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(qss)), 1e-6f));
    const float krs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(kss)), 1e-6f));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HD)));
    Qs[t] = __fmul_rn(__fmul_rn(mixed[0], qrs), scale);
    Ks[t] = __fmul_rn(mixed[1], krs);
    const float vt = mixed[2];
    __syncthreads();
    // ---- recurrence (gdn_recurrence_kernel): thread v owns state column v ----
    if (!mbar_wait(&st_bar, 0)) report_error(err_flag, kDevWaitTimeout);
    const float gh = s_g, bh = s_beta;
    // The column is read from shared memory in both passes (the decayed
    // value recomputed), which keeps registers low enough for several
    // heads per SM.
    // both chains over the column, and its update in the same pass as the
    // output sum, in k order as in the reference (qh_gdn.cuh)
    const float o = gdn_recur_column<HD>(st_s + t, Ks, Qs, gh, bh, vt);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (t == 0) {
        bulk_copy_s2g(st, st_s, HD * HD * 4);
        bulk_commit_group();
    }
    // ---- gated RMSNorm (gdn_gated_norm_kernel) ----
    const double ssq = block_sum_d(static_cast<double>(__fmul_rn(o, o)), scratch);
    const float mean = static_cast<float>(ssq / static_cast<double>(HD));
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    const int64_t zi = static_cast<int64_t>(b) * kdim + h * HD + t;
    const float y = __fmul_rn(__fmul_rn(__fmul_rn(o, rs), norm_w[t]), silu_f(z[zi]));
    if constexpr (!QUANT) {
        y_out[zi] = y;
    } else {
        // ---- Q8_K over the head pair (quantize_q8k_kernel) ----
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        const int half = static_cast<int>(cluster.block_rank());  // == h & 1
        float a = (y == y) ? fabsf(y) : -1.0f, bv = y;
        int bi = half * HD + t;
        warp_best(a, bi, bv);
        if (lane == 0) { wa[warp] = a; wi[warp] = bi; wv[warp] = bv; }
        __syncthreads();
        if (t == 0) {
            float ca = wa[0], cv = wv[0];
            int ci = wi[0];
            for (int w = 1; w < HD / 32; ++w) best_merge(ca, ci, cv, wa[w], wi[w], wv[w]);
            c_a = ca; c_i = ci; c_v = cv;
        }
        cluster.sync();
        float ba = c_a, xv = c_v;
        int ii = c_i;
        {
            const float *pa = cluster.map_shared_rank(&c_a, half ^ 1);
            const int *pi = cluster.map_shared_rank(&c_i, half ^ 1);
            const float *pv = cluster.map_shared_rank(&c_v, half ^ 1);
            best_merge(ba, ii, xv, *pa, *pi, *pv);
        }
        cluster.sync();  // the partner has read this CTA's candidate
        const float xmax = ba > 0.0f ? xv : 0.0f;
        const Q8KRow r = q8k_row(xq, kdim, n_tok, b, tile);
        const int blk = h >> 1;
        int q = 0;
        if (xmax != 0.0f) {
            const float iscale = __fdiv_rn(-127.0f, xmax);
            q = q8k_value(y, iscale);
            if (half == 0 && t == 0) *q8k_scale(r, blk) = __fdiv_rn(1.0f, iscale);
        } else if (half == 0 && t == 0) {
            *q8k_scale(r, blk) = 0.0f;
        }
        *q8k_elem(r, blk, half * HD + t) = static_cast<int8_t>(q);
        int sum = q;
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        if (r.bs) {
            if ((lane & 15) == 0)
                r.bs[blk * 16 + half * (HD / 16) + warp * 2 + (lane >> 4)] = static_cast<int16_t>(sum);
        } else {
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            if (lane == 0) q8k_put_min(r, blk, half * (HD / 32) + warp, sum);
        }
    }
    if (t == 0) bulk_wait_all();  // the state store has completed before the CTA exits
}

// Gated DeltaNet token update for many (sequence, head) pairs, persistent
// and pipelined: CTA c (128 threads, three per SM) takes pairs c,
// c + gridDim.x, ...; thread t holds state column t in registers while it is
// updated, and the next pair's 64 KB state is copied into shared memory (one
// bulk copy) while the current pair computes -- so the state stream and the
// double-precision chains overlap instead of taking turns wave by wave.
// The next pair's per-thread inputs (its conv rows, new qkv values, conv
// weights, z) are copied into shared memory by cp.async at the start of the
// current pair, so the pair starts without a global-memory round trip; the
// gates (beta, g) of up to 128 of the CTA's pairs are formed at once, one
// pair per thread, instead of by one thread inside every pair. Per pair the
// operations and orders of gdn_fused_kernel<128, false>.
template <int KK>
__global__ void __launch_bounds__(128, 2)
    gdn_stream_kernel(const float *__restrict__ qkv, float *__restrict__ ring, const float *__restrict__ conv_w,
                      const float *__restrict__ bb, const float *__restrict__ aa, const float *__restrict__ dt_bias,
                      const float *__restrict__ ssm_a, float *__restrict__ state, const float *__restrict__ z,
                      const float *__restrict__ norm_w, int heads, float eps, const int32_t *__restrict__ pos_ptr,
                      int n_pairs, int *__restrict__ err_flag, float *__restrict__ y_out) {
    constexpr int HD = 128;
    pdl_launch_dependents();
    extern __shared__ __align__(128) float st_s[];  // [HD k][HD v]: the next pair's state
    __shared__ uint64_t st_bar;
    __shared__ double scratch[64];
    __shared__ float Ks[HD], Qs[HD];
    __shared__ float s_beta[HD], s_g[HD];  // gates of the CTA's pairs pi0 .. pi0 + HD - 1
    // per-thread inputs of the next pair: [part] new value, [part][r] conv
    // ring rows, [part][k] conv weights, z
    constexpr int kPreX = 0, kPreRows = 3, kPreW = 3 + 3 * KK, kPreZ = 3 + 6 * KK, kPre = 4 + 6 * KK;
    __shared__ float pre[kPre][HD];
    const int t = threadIdx.x;
    const int kdim = heads * HD, conv_dim = 3 * kdim;
    auto cp4 = [](float *dst, const float *src) {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
    };
    // every thread its own elements: the conv weights (constants, so the
    // first pair's may be copied before the launch wait), then the rest and
    // one commit group
    auto prefetch_w = [&](int pr) {
        const int ph = pr % heads;
#pragma unroll
        for (int part = 0; part < 3; ++part) {
            const int ch = part * kdim + ph * HD + t;
#pragma unroll
            for (int q = 0; q < KK; ++q) cp4(&pre[kPreW + part * KK + q][t], conv_w + static_cast<int64_t>(ch) * KK + q);
        }
    };
    auto prefetch_x = [&](int pr) {
        const int pb = pr / heads, ph = pr % heads;
        const float *src = qkv + static_cast<int64_t>(pb) * conv_dim;
        const float *rg = ring + static_cast<int64_t>(pb) * KK * conv_dim;
#pragma unroll
        for (int part = 0; part < 3; ++part) {
            const int ch = part * kdim + ph * HD + t;
            cp4(&pre[kPreX + part][t], src + ch);
#pragma unroll
            for (int r = 0; r < KK; ++r) cp4(&pre[kPreRows + part * KK + r][t], rg + static_cast<int64_t>(r) * conv_dim + ch);
        }
        cp4(&pre[kPreZ][t], z + static_cast<int64_t>(pb) * kdim + ph * HD + t);
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // thread t: the gates of the CTA's pair pi0 + t (pair index = sequence * heads + head)
    auto form_gates = [&](int pi0) {
        const int pr = blockIdx.x + (pi0 + t) * static_cast<int>(gridDim.x);
        if (pr < n_pairs) {
            const int ph = pr % heads;
            s_beta[t] = sigmoid_f(bb[pr]);
            const float a = __fadd_rn(aa[pr], dt_bias[ph]);
            const float sp = a > 20.0f ? a : logf_ref(__fadd_rn(1.0f, expf_ref(a)));
            s_g[t] = expf_ref(__fmul_rn(ssm_a[ph], sp));
        }
    };
    if (t == 0) {
        mbar_init(&st_bar, 1);
        mbar_fence_init();
    }
    int pair = blockIdx.x;
    if (t < 32) libm_prefetch_l1(t);
    if (t == 32) asm volatile("prefetch.global.L1 [%0];" ::"l"(dt_bias));
    if (t == 33) asm volatile("prefetch.global.L1 [%0];" ::"l"(ssm_a));
    if (pair < n_pairs) prefetch_w(pair);
    __syncthreads();
    pdl_wait();
    if (pair < n_pairs) prefetch_x(pair);
    auto issue = [&](int pr) {  // thread 0
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the column reads come first
        mbar_arrive_expect_tx(&st_bar, HD * HD * 4);
        bulk_copy_g2s(st_s, state + static_cast<int64_t>(pr) * HD * HD, HD * HD * 4, &st_bar);
    };
    // the gates' loads go out before the state copies of every CTA fill the
    // memory queues; the first state copy follows them
    form_gates(0);  // published by the barrier after the first pair's column reads
    if (t == 0 && pair < n_pairs) issue(pair);
    const float nw = norm_w[t];
    const int pos = max(*pos_ptr, 0);
    const int slot = pos % KK, head_after = (pos + 1) % KK;
    uint32_t parity = 0;
    for (int pi = 0; pair < n_pairs; pair += gridDim.x, ++pi) {
        if (pi > 0 && pi % HD == 0) form_gates(pi);  // the previous pair's gate reads precede its last barrier
        const int b = pair / heads, h = pair % heads;
        // ---- conv ring + SiLU + L2 norms + beta/g (gdn_fused_kernel's order) ----
        asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's prefetched inputs
        float cw[3][KK], xin[3], rows[3][KK];
#pragma unroll
        for (int part = 0; part < 3; ++part) {
            xin[part] = pre[kPreX + part][t];
#pragma unroll
            for (int r = 0; r < KK; ++r) rows[part][r] = pre[kPreRows + part * KK + r][t];
#pragma unroll
            for (int q = 0; q < KK; ++q) cw[part][q] = pre[kPreW + part * KK + q][t];
        }
        const float zs = silu_f(pre[kPreZ][t]);
        // the buffer is this thread's alone: the next pair's inputs go in now
        if (pair + static_cast<int>(gridDim.x) < n_pairs) {
            prefetch_w(pair + gridDim.x);
            prefetch_x(pair + gridDim.x);
        }
        float *rg = ring + static_cast<int64_t>(b) * KK * conv_dim;
        float mixed[3];
#pragma unroll
        for (int part = 0; part < 3; ++part) {
            const int ch = part * kdim + h * HD + t;
            float taps[KK - 1];
#pragma unroll
            for (int k = 0; k < KK - 1; ++k) {
                const int rsel = (head_after + k) % KK;
                float v = 0.0f;
#pragma unroll
                for (int r = 0; r < KK; ++r)
                    if (r == rsel) v = rows[part][r];
                taps[k] = v;
            }
            rg[static_cast<int64_t>(slot) * conv_dim + ch] = xin[part];
            float acc = 0.0f;
#pragma unroll
            for (int k = 0; k < KK; ++k) acc = __fadd_rn(acc, __fmul_rn(k < KK - 1 ? taps[k] : xin[part], cw[part][k]));
            mixed[part] = silu_f(acc);
        }
        const double2 qkss = block_sum_d2(static_cast<double>(__fmul_rn(mixed[0], mixed[0])),
                                          static_cast<double>(__fmul_rn(mixed[1], mixed[1])), scratch);
        const float qrs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(qkss.x)), 1e-6f));
        const float krs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(qkss.y)), 1e-6f));
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HD)));
        Qs[t] = __fmul_rn(__fmul_rn(mixed[0], qrs), scale);
        Ks[t] = __fmul_rn(mixed[1], krs);
        const float vt = mixed[2];
        const int64_t zi = static_cast<int64_t>(b) * kdim + h * HD + t;
        // ---- the state column into registers; the buffer then takes the next pair ----
        if (!mbar_wait(&st_bar, parity)) report_error(err_flag, kDevWaitTimeout);
        parity ^= 1u;
        float S[HD];
#pragma unroll
        for (int k = 0; k < HD; ++k) S[k] = st_s[k * HD + t];
        __syncthreads();  // every column read (and Ks, Qs, s_g, s_beta written)
        if (t == 0 && pair + static_cast<int>(gridDim.x) < n_pairs) issue(pair + gridDim.x);
        // ---- recurrence (gdn_fused_kernel's two chains) ----
        const float gh = s_g[pi % HD], bh = s_beta[pi % HD];
        double acc = 0.0;
#pragma unroll
        for (int k = 0; k < HD; ++k) acc += static_cast<double>(__fmul_rn(__fmul_rn(S[k], gh), Ks[k]));
        const float delta = __fmul_rn(__fsub_rn(vt, static_cast<float>(acc)), bh);
        double acc2 = 0.0;
#pragma unroll
        for (int k = 0; k < HD; ++k) {
            S[k] = __fadd_rn(__fmul_rn(S[k], gh), __fmul_rn(Ks[k], delta));
            acc2 += static_cast<double>(__fmul_rn(S[k], Qs[k]));
        }
        const float o = static_cast<float>(acc2);
        float *st = state + static_cast<int64_t>(pair) * HD * HD;
#pragma unroll
        for (int k = 0; k < HD; ++k) st[k * HD + t] = S[k];
        // ---- gated RMSNorm ----
        const double ssq = block_sum_d(static_cast<double>(__fmul_rn(o, o)), scratch);
        const float mean = static_cast<float>(ssq / static_cast<double>(HD));
        const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        y_out[zi] = __fmul_rn(__fmul_rn(__fmul_rn(o, rs), nw), zs);
        __syncthreads();  // Ks, Qs and the scratch are rewritten by the next pair
    }
}

// Gated DeltaNet over a chunk of n_tok prompt tokens per sequence: CTA
// (sequence, head) runs, token after token, exactly the per-token work of
// gdn_fused_kernel (same operations and order), with the head's state in
// shared memory for the whole chunk and the conv history in registers, so
// a prompt costs one launch per layer and chunk instead of one per token.
// Rows are sequence-major: row = sequence * n_tok + j at position *pos_ptr + j.
template <int HD, int KK>
__global__ void __cluster_dims__(1, 2, 1) __launch_bounds__(HD)
    gdn_prefill_kernel(const float *__restrict__ qkv, float *__restrict__ ring, const float *__restrict__ conv_w,
                       const float *__restrict__ bb, const float *__restrict__ aa, const float *__restrict__ dt_bias,
                       const float *__restrict__ ssm_a, float *__restrict__ state, const float *__restrict__ z,
                       const float *__restrict__ norm_w, int heads, float eps, const int32_t *__restrict__ pos_ptr,
                       int n_tok, uint8_t *__restrict__ xq, int n_rows, int tile, int *__restrict__ err_flag) {
    static_assert(HD == 128, "a cluster pair of heads must form one 256-value Q8_K block");
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ __align__(128) float st_s[];  // [HD k][HD v]
    __shared__ uint64_t st_bar;
    __shared__ double scratch[32];
    __shared__ float Ks[HD], Qs[HD];
    __shared__ float s_beta, s_g;
    __shared__ float wa[HD / 32], wv[HD / 32];
    __shared__ int wi[HD / 32];
    __shared__ float c_a, c_v;
    __shared__ int c_i;
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int b = blockIdx.x, h = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int half = static_cast<int>(cluster.block_rank());
    const int kdim = heads * HD, conv_dim = 3 * kdim;
    float *st = state + (static_cast<int64_t>(b) * heads + h) * HD * HD;
    if (t == 0) {
        mbar_init(&st_bar, 1);
        mbar_fence_init();
        mbar_arrive_expect_tx(&st_bar, HD * HD * 4);
        bulk_copy_g2s(st_s, st, HD * HD * 4, &st_bar);
    }
    const int pos0 = max(*pos_ptr, 0);
    float *rg = ring + static_cast<int64_t>(b) * KK * conv_dim;
    // conv history of this thread's 3 channels, oldest first: positions
    // pos0-(KK-1) .. pos0-1, which the ring holds in slots (pos0+1+k) % KK
    float hist[3][KK - 1], cw[3][KK];
#pragma unroll
    for (int part = 0; part < 3; ++part) {
        const int ch = part * kdim + h * HD + t;
#pragma unroll
        for (int k = 0; k < KK; ++k) cw[part][k] = conv_w[ch * KK + k];
#pragma unroll
        for (int k = 0; k < KK - 1; ++k) hist[part][k] = rg[static_cast<int64_t>((pos0 + 1 + k) % KK) * conv_dim + ch];
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HD)));
    bool have_state = false;
    for (int j = 0; j < n_tok; ++j) {
        const int64_t row = static_cast<int64_t>(b) * n_tok + j;
        if (t == 32) {
            const int64_t i = row * heads + h;
            s_beta = sigmoid_f(bb[i]);
            const float a = __fadd_rn(aa[i], dt_bias[h]);
            const float sp = a > 20.0f ? a : logf_ref(__fadd_rn(1.0f, expf_ref(a)));
            s_g = expf_ref(__fmul_rn(ssm_a[h], sp));
        }
        float mixed[3];
#pragma unroll
        for (int part = 0; part < 3; ++part) {
            const float x = qkv[row * conv_dim + part * kdim + h * HD + t];
            float acc = 0.0f;
#pragma unroll
            for (int k = 0; k < KK; ++k)
                acc = __fadd_rn(acc, __fmul_rn(k < KK - 1 ? hist[part][k] : x, cw[part][k]));
#pragma unroll
            for (int k = 0; k < KK - 2; ++k) hist[part][k] = hist[part][k + 1];
            hist[part][KK - 2] = x;
            mixed[part] = silu_f(acc);
        }
        const double qss = block_sum_d(static_cast<double>(__fmul_rn(mixed[0], mixed[0])), scratch);
        const double kss = block_sum_d(static_cast<double>(__fmul_rn(mixed[1], mixed[1])), scratch);
        const float qrs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(qss)), 1e-6f));
        const float krs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(kss)), 1e-6f));
        Qs[t] = __fmul_rn(__fmul_rn(mixed[0], qrs), scale);
        Ks[t] = __fmul_rn(mixed[1], krs);
        const float vt = mixed[2];
        __syncthreads();
        if (!have_state) {
            if (!mbar_wait(&st_bar, 0)) report_error(err_flag, kDevWaitTimeout);
            have_state = true;
        }
        const float gh = s_g, bh = s_beta;
        const float o = gdn_recur_column<HD>(st_s + t, Ks, Qs, gh, bh, vt);  // as gdn_fused_kernel
        const double ssq = block_sum_d(static_cast<double>(__fmul_rn(o, o)), scratch);
        const float mean = static_cast<float>(ssq / static_cast<double>(HD));
        const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        const float y = __fmul_rn(__fmul_rn(__fmul_rn(o, rs), norm_w[t]), silu_f(z[row * kdim + h * HD + t]));
        float a = (y == y) ? fabsf(y) : -1.0f, bv = y;
        int bi = half * HD + t;
        warp_best(a, bi, bv);
        if (lane == 0) { wa[warp] = a; wi[warp] = bi; wv[warp] = bv; }
        __syncthreads();
        if (t == 0) {
            float ca = wa[0], cv = wv[0];
            int ci = wi[0];
            for (int w = 1; w < HD / 32; ++w) best_merge(ca, ci, cv, wa[w], wi[w], wv[w]);
            c_a = ca; c_i = ci; c_v = cv;
        }
        cluster.sync();
        float ba = c_a, xv = c_v;
        int ii = c_i;
        best_merge(ba, ii, xv, *cluster.map_shared_rank(&c_a, half ^ 1), *cluster.map_shared_rank(&c_i, half ^ 1),
                   *cluster.map_shared_rank(&c_v, half ^ 1));
        cluster.sync();  // the partner has read this CTA's candidate; Ks/Qs/scales free for the next token
        const float xmax = ba > 0.0f ? xv : 0.0f;
        const Q8KRow r = q8k_row(xq, kdim, n_rows, row, tile);
        const int blk = h >> 1;
        int q = 0;
        if (xmax != 0.0f) {
            const float iscale = __fdiv_rn(-127.0f, xmax);
            q = q8k_value(y, iscale);
            if (half == 0 && t == 0) *q8k_scale(r, blk) = __fdiv_rn(1.0f, iscale);
        } else if (half == 0 && t == 0) {
            *q8k_scale(r, blk) = 0.0f;
        }
        *q8k_elem(r, blk, half * HD + t) = static_cast<int8_t>(q);
        int sum = q;
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        if (r.bs) {
            if ((lane & 15) == 0)
                r.bs[blk * 16 + half * (HD / 16) + warp * 2 + (lane >> 4)] = static_cast<int16_t>(sum);
        } else {
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            if (lane == 0) q8k_put_min(r, blk, half * (HD / 32) + warp, sum);
        }
    }
    if (!have_state && t == 0 && !mbar_wait(&st_bar, 0)) report_error(err_flag, kDevWaitTimeout);
    // conv history back to the ring slots of the last KK-1 positions
    const int last = pos0 + n_tok - 1;
#pragma unroll
    for (int part = 0; part < 3; ++part) {
        const int ch = part * kdim + h * HD + t;
#pragma unroll
        for (int k = 0; k < KK - 1; ++k)
            rg[static_cast<int64_t>(((last - (KK - 2) + k) % KK + KK) % KK) * conv_dim + ch] = hist[part][k];
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (t == 0) {
        bulk_copy_s2g(st, st_s, HD * HD * 4);
        bulk_commit_group();
        bulk_wait_all();
    }
}

// Greedy pick + device-side feed (argmax_kernel + feed_next_kernel) over a
// grid of (parts, rows): each CTA scans one slice of the row, the last CTA
// of a row (ticket counter) merges the slices in order, records the pick
// and feeds the next input; the last row advances the position. Counters
// are left at zero for the next launch.
constexpr int kArgmaxThreads = 512;
__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_feed_kernel(const float *__restrict__ logits, int64_t vocab, float *__restrict__ part_v,
                       int *__restrict__ part_i, unsigned *__restrict__ tickets, int32_t *__restrict__ next,
                       const int32_t *__restrict__ prompt, int B, int stride, int32_t *__restrict__ ctl,
                       int32_t *__restrict__ tokens, int32_t *__restrict__ picks) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ int si[kArgmaxThreads / 32];
    __shared__ bool last;
    const int part = blockIdx.x, P = gridDim.x, row = blockIdx.y;
    // slices of a multiple of 4 logits: with 16-byte aligned rows each
    // thread reads float4s, its indices still in increasing order
    const int64_t chunk = (((vocab + P - 1) / P) + 3) & ~int64_t(3);
    const int64_t lo = part * chunk, hi = min(vocab, lo + chunk);
    const float *lr = logits + static_cast<int64_t>(row) * vocab;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    if ((vocab & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0) {
        const float4 *l4 = reinterpret_cast<const float4 *>(lr);
#pragma unroll 4
        for (int64_t q = lo / 4 + threadIdx.x; q < hi / 4; q += blockDim.x) {
            const float4 v = l4[q];
            const int i = static_cast<int>(4 * q);
            if (v.x > best) { best = v.x; bi = i; }
            if (v.y > best) { best = v.y; bi = i + 1; }
            if (v.z > best) { best = v.z; bi = i + 2; }
            if (v.w > best) { best = v.w; bi = i + 3; }
        }
    } else {
        for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const float v = lr[i];
            if (v > best) { best = v; bi = static_cast<int>(i); }
        }
    }
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
        part_v[row * P + part] = best;
        part_i[row * P + part] = bi;
        __threadfence();
        last = atomicAdd(&tickets[row], 1u) == static_cast<unsigned>(P - 1);
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    float bv = -INFINITY;
    int bidx = 0x7fffffff;
    for (int p = 0; p < P; ++p) {
        const float v = __ldcg(part_v + row * P + p);
        const int i = __ldcg(part_i + row * P + p);
        if (v > bv || (v == bv && i < bidx)) { bv = v; bidx = i; }
    }
    // sample_argmax starts from element 0: a NaN there is never replaced
    const float first = lr[0];
    const int32_t nx = (first != first || bidx == 0x7fffffff) ? 0 : bidx;
    next[row] = nx;
    const int pos = ctl[0], n_prompt = ctl[1];
    if (pos >= 0 && pos < stride) picks[static_cast<int64_t>(row) * stride + pos] = nx;
    tokens[row] = (pos + 1 < n_prompt && pos + 1 < stride) ? prompt[static_cast<int64_t>(row) * stride + pos + 1] : nx;
    tickets[row] = 0u;
    __threadfence();
    if (atomicAdd(&tickets[B], 1u) == static_cast<unsigned>(B - 1)) {
        ctl[0] = pos + 1;
        tickets[B] = 0u;
    }
}

}  // namespace qh

// ---------------------------------------------------------------------------
// C-ABI launchers of the fused kernels
// ---------------------------------------------------------------------------
extern "C" {

static bool tile_ok(int32_t t) { return t == 0 || t == QH_Q8KT_TILE; }

int qh_rmsnorm_q8k(const float *d_h, const float *d_mix, float *d_h_out, const float *d_w, int64_t dim, int32_t B,
                   float eps, void *d_xq, int32_t layout_tile, void *stream) {
    if (!d_h || !d_w || !d_xq || dim <= 0 || dim % QH_QK || dim > qh::kResNormMaxBlocks * QH_QK || B <= 0 ||
        B > 65535 || !tile_ok(layout_tile) || (d_mix && (!d_h_out || d_h_out == d_h)))
        return bad("qh_rmsnorm_q8k: bad arguments");
    auto kern = dim <= 4 * QH_QK ? qh::resnorm_q8k_kernel<4> : qh::resnorm_q8k_kernel<qh::kResNormMaxBlocks>;
    const cudaError_t le = qh::launch_pdl(kern, dim3(static_cast<unsigned>(dim / QH_QK), B),
                                          dim3(256), 0, static_cast<cudaStream_t>(stream), d_h, d_mix, d_h_out, d_w,
                                          static_cast<int>(dim), eps, static_cast<uint8_t *>(d_xq), B, layout_tile);
    return launch_status(le, "qh_rmsnorm_q8k");
}

int qh_swiglu_q8k(const float *d_gate, const float *d_up, int64_t ffn, int32_t B, void *d_xq, int32_t layout_tile,
                  void *stream) {
    if (!d_gate || !d_up || !d_xq || ffn <= 0 || ffn % QH_QK || B <= 0 || B > 65535 || !tile_ok(layout_tile))
        return bad("qh_swiglu_q8k: bad arguments");
    const cudaError_t le = qh::launch_pdl(qh::swiglu_q8k_kernel, dim3(static_cast<unsigned>(ffn / QH_QK), B),
                                          dim3(256), 0, static_cast<cudaStream_t>(stream), d_gate, d_up,
                                          static_cast<int>(ffn), static_cast<uint8_t *>(d_xq), B, layout_tile);
    return launch_status(le, "qh_swiglu_q8k");
}

static int gdn_fused_impl(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b,
                          const float *d_a, const float *d_dt_bias, const float *d_ssm_a, float *d_state,
                          const float *d_z, const float *d_norm_w, int32_t B, int32_t heads, int32_t hd, int32_t kk,
                          float eps, const int32_t *d_pos, void *d_xq, int32_t layout_tile, float *d_y, void *stream,
                          const char *what) {
    if (!d_qkv || !d_ring || !d_conv_w || !d_b || !d_a || !d_dt_bias || !d_ssm_a || !d_state || !d_z ||
        !d_norm_w || !d_pos || (!d_xq && !d_y) || B <= 0 || heads <= 0 || heads % 2 || kk <= 0 ||
        kk > qh::kMaxConvTaps || !tile_ok(layout_tile))
        return bad(what);
    if (hd != 128) {
        qh::set_last_error_message("gdn: head dim must be 128");
        return QH_ERR_UNSUPPORTED;
    }
    if (reinterpret_cast<uintptr_t>(d_state) & 15) return bad(what);
    static bool attr_done[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev][d_y != nullptr]) {
        if (d_y)
            cudaFuncSetAttribute(qh::gdn_fused_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 128 * 4);
        else
            cudaFuncSetAttribute(qh::gdn_fused_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 128 * 4);
        attr_done[dev][d_y != nullptr] = true;
    }
    int *err = qh::device_error_word();
    if (!err) return bad("gdn: no device error word");
    const dim3 grid(static_cast<unsigned>(B), heads);
    cudaError_t le;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t pairs = static_cast<int64_t>(B) * heads;
    if (d_y && kk == 4 && pairs > 2 * static_cast<int64_t>(sms)) {
        // many (sequence, head) pairs: the persistent pipelined form
        static bool sattr[64] = {};
        if (dev >= 0 && dev < 64 && !sattr[dev]) {
            cudaFuncSetAttribute(qh::gdn_stream_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 128 * 4);
            sattr[dev] = true;
        }
        le = qh::launch_pdl(qh::gdn_stream_kernel<4>, dim3(static_cast<unsigned>(2 * sms)), dim3(128), 128 * 128 * 4,
                            static_cast<cudaStream_t>(stream), d_qkv, d_ring, d_conv_w, d_b, d_a, d_dt_bias, d_ssm_a,
                            d_state, d_z, d_norm_w, heads, eps, d_pos, static_cast<int>(pairs), err, d_y);
        return launch_status(le, what);
    }
    if (d_y)
        le = qh::launch_pdl(qh::gdn_fused_kernel<128, false>, grid, dim3(128), 128 * 128 * 4,
                            static_cast<cudaStream_t>(stream), d_qkv, d_ring, d_conv_w, d_b, d_a, d_dt_bias, d_ssm_a,
                            d_state, d_z, d_norm_w, heads, kk, eps, d_pos, static_cast<uint8_t *>(nullptr), B, 0, err,
                            d_y);
    else
        le = qh::launch_pdl_cluster(qh::gdn_fused_kernel<128, true>, grid, dim3(128), 128 * 128 * 4,
                                    static_cast<cudaStream_t>(stream), dim3(1, 2, 1), d_qkv, d_ring, d_conv_w, d_b, d_a,
                                    d_dt_bias, d_ssm_a, d_state, d_z, d_norm_w, heads, kk, eps, d_pos,
                                    static_cast<uint8_t *>(d_xq), B, layout_tile, err, static_cast<float *>(nullptr));
    return launch_status(le, what);
}

int qh_gdn_fused(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b, const float *d_a,
                 const float *d_dt_bias, const float *d_ssm_a, float *d_state, const float *d_z,
                 const float *d_norm_w, int32_t B, int32_t heads, int32_t hd, int32_t kk, float eps,
                 const int32_t *d_pos, void *d_xq, int32_t layout_tile, void *stream) {
    if (!d_xq) return bad("qh_gdn_fused: bad arguments");
    return gdn_fused_impl(d_qkv, d_ring, d_conv_w, d_b, d_a, d_dt_bias, d_ssm_a, d_state, d_z, d_norm_w, B, heads, hd,
                          kk, eps, d_pos, d_xq, layout_tile, nullptr, stream, "qh_gdn_fused: bad arguments");
}

int qh_gdn_fused_y(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b, const float *d_a,
                   const float *d_dt_bias, const float *d_ssm_a, float *d_state, const float *d_z,
                   const float *d_norm_w, int32_t B, int32_t heads, int32_t hd, int32_t kk, float eps,
                   const int32_t *d_pos, float *d_y, void *stream) {
    if (!d_y) return bad("qh_gdn_fused_y: bad arguments");
    return gdn_fused_impl(d_qkv, d_ring, d_conv_w, d_b, d_a, d_dt_bias, d_ssm_a, d_state, d_z, d_norm_w, B, heads, hd,
                          kk, eps, d_pos, nullptr, 0, d_y, stream, "qh_gdn_fused_y: bad arguments");
}

int qh_gdn_prefill(const float *d_qkv, float *d_ring, const float *d_conv_w, const float *d_b, const float *d_a,
                   const float *d_dt_bias, const float *d_ssm_a, float *d_state, const float *d_z,
                   const float *d_norm_w, int32_t n_seq, int32_t n_tok, int32_t heads, int32_t hd, int32_t kk,
                   float eps, const int32_t *d_pos, void *d_xq, int32_t layout_tile, void *stream) {
    if (!d_qkv || !d_ring || !d_conv_w || !d_b || !d_a || !d_dt_bias || !d_ssm_a || !d_state || !d_z ||
        !d_norm_w || !d_pos || !d_xq || n_seq <= 0 || n_tok <= 0 || static_cast<int64_t>(n_seq) * n_tok > 0x7fffffff ||
        heads <= 0 || heads % 2 || !tile_ok(layout_tile))
        return bad("qh_gdn_prefill: bad arguments");
    if (hd != 128 || kk != 4) {
        qh::set_last_error_message("qh_gdn_prefill: head dim must be 128 and the conv kernel 4");
        return QH_ERR_UNSUPPORTED;
    }
    if (reinterpret_cast<uintptr_t>(d_state) & 15) return bad("qh_gdn_prefill: state not 16-byte aligned");
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaFuncSetAttribute(qh::gdn_prefill_kernel<128, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 128 * 4);
        attr_done[dev] = true;
    }
    int *err = qh::device_error_word();
    if (!err) return bad("qh_gdn_prefill: no device error word");
    const cudaError_t le = qh::launch_pdl(qh::gdn_prefill_kernel<128, 4>, dim3(static_cast<unsigned>(n_seq), heads),
                                          dim3(128), 128 * 128 * 4, static_cast<cudaStream_t>(stream), d_qkv, d_ring,
                                          d_conv_w, d_b, d_a, d_dt_bias, d_ssm_a, d_state, d_z, d_norm_w, heads, eps,
                                          d_pos, n_tok, static_cast<uint8_t *>(d_xq), n_seq * n_tok, layout_tile, err);
    return launch_status(le, "qh_gdn_prefill");
}

// Slices per row: at most one per 1024 logits and 64 in all (the scratch is
// sized for that); for many rows fewer, so that the grid stays near 600
// CTAs of 512 threads (about one wave at four per SM).
static int argmax_parts_max(int64_t vocab) {
    const int64_t p = (vocab + 1023) / 1024;
    return static_cast<int>(p < 1 ? 1 : (p > 64 ? 64 : p));
}
static int argmax_parts(int64_t vocab, int32_t B) {
    const int pmax = argmax_parts_max(vocab);
    const int p = (600 + B - 1) / B;
    return p < 1 ? 1 : (p > pmax ? pmax : p);
}

int64_t qh_argmax_feed_scratch_bytes(int32_t B, int64_t vocab) {
    if (B <= 0 || vocab <= 0) return -1;
    const int64_t P = argmax_parts_max(vocab);
    return (static_cast<int64_t>(B) * P * 8 + (static_cast<int64_t>(B) + 1) * 4 + 255) & ~int64_t(255);
}

int qh_argmax_feed(const float *d_logits, int32_t B, int64_t vocab, void *d_scratch, int32_t *d_next,
                   const int32_t *d_prompt, int32_t stride, int32_t *d_ctl, int32_t *d_tokens, int32_t *d_picks,
                   void *stream) {
    if (!d_logits || !d_scratch || !d_next || !d_prompt || !d_ctl || !d_tokens || !d_picks || B <= 0 ||
        B > 65535 || vocab <= 0 || vocab > 0x7ffffffe || stride <= 0)
        return bad("qh_argmax_feed: bad arguments");
    const int P = argmax_parts(vocab, B), Pmax = argmax_parts_max(vocab);
    uint8_t *base = static_cast<uint8_t *>(d_scratch);
    float *pv = reinterpret_cast<float *>(base);
    int *pi = reinterpret_cast<int *>(base + static_cast<int64_t>(B) * Pmax * 4);
    unsigned *tickets = reinterpret_cast<unsigned *>(base + static_cast<int64_t>(B) * Pmax * 8);
    const cudaError_t le = qh::launch_pdl(qh::argmax_feed_kernel, dim3(P, B), dim3(qh::kArgmaxThreads), 0,
                                          static_cast<cudaStream_t>(stream), d_logits, vocab, pv, pi, tickets,
                                          d_next, d_prompt, B, stride, d_ctl, d_tokens, d_picks);
    return launch_status(le, "qh_argmax_feed");
}

}  // extern "C"
