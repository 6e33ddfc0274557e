// SPDX-License-Identifier: MIT
//
// qh_gemv_dev.cuh -- the device side of the quantized matvec shared by the
// grouped GEMV kernel (qh_gemv.cu) and the persistent decode-step kernel
// (qh_step.cu): per-type consumers of one 8-row group of GGUF blocks staged
// in shared memory against Q8_K (or Q8_0) activation planes, and the
// one-warp Q8_K block quantizer. Replaces the reference's per-row SIMD dots
// (simd/quants.h:244-402, simd/avx.c:420-591) and quantize_row_q8_K
// (slm/tensor.c:673-720).

#ifndef QH_GEMV_DEV_CUH
#define QH_GEMV_DEV_CUH

#include "qh_common.cuh"
#include "qh_internal.h"
#include "qh_q8k.cuh"

namespace qh {

constexpr int kConsumerWarps = 8;
// ---------------------------------------------------------------------------
// Per-type consumers. A call handles one 8-row group whose rows start at
// `grp` in shared memory (row stride = job.row_bytes). Lanes: r = lane/4 is
// the row, q = lane%4 a quarter of every super-block.
// ---------------------------------------------------------------------------

__device__ __forceinline__ int dot16(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                     const int4 &x, int acc) {
    acc = __dp4a(static_cast<int>(w0), x.x, acc);
    acc = __dp4a(static_cast<int>(w1), x.y, acc);
    acc = __dp4a(static_cast<int>(w2), x.z, acc);
    acc = __dp4a(static_cast<int>(w3), x.w, acc);
    return acc;
}

// Same with unsigned weight bytes (dp4a.u32.s32): the Q4_K high nibbles are
// used in place (16 * w, masked, not shifted) and the sum divided by 16 after
// -- an exact shift, the sum being a multiple of 16.
__device__ __forceinline__ int dot16_u(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, const int4 &x, int acc) {
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(w0), "r"(x.x));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(w1), "r"(x.y));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(w2), "r"(x.z));
    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(w3), "r"(x.w));
    return acc;
}

// The job's activation planes as staged in shared memory next to the
// weight tile (same split layout as in global memory, rows [t0, t0+n_tok)).
struct XView {
    const int8_t *qs;   // [n_tok][k]
    const int16_t *bs;  // [n_tok][nb][16]   (Q8_K only)
    const uint8_t *d;   // [n_tok][d_stride] f32 (Q8_K) or fp16 bits (Q8_0)
};

__device__ __forceinline__ int4 lds128i(const int8_t *p) {
    return *reinterpret_cast<const int4 *>(p);
}

// Unpacked 6-bit scales/mins of the four sub-blocks a lane covers in a
// Q4_K/Q5_K super-block (simd/quants.h:215-224). With j0 = q/2 the lane
// covers sub-blocks 2j0, 2j0+1 (stored in scale bytes 0..7) and 2j0+4,
// 2j0+5 (stored across bytes 8..11 plus the top bits of bytes 0..7).
struct KScales {
    int sc_a, sc_b, sc_c, sc_d;
    int mins_ab, mins_cd;  // bytes {m_a, m_a, m_b, m_b} for dp2a against bsum pairs
};

__device__ __forceinline__ KScales unpack_kscales(const uint4 &h, uint32_t sh) {
    const uint32_t L = (h.y >> sh) & 0xffffu;  // scales[2j0], scales[2j0+1]
    const uint32_t M = (h.z >> sh) & 0xffffu;  // scales[2j0+4], scales[2j0+5]
    const uint32_t H = (h.w >> sh) & 0xffffu;  // scales[2j0+8], scales[2j0+9]
    const uint32_t sc_ab = L & 0x3f3fu;
    const uint32_t m_ab = M & 0x3f3fu;
    const uint32_t sc_cd = (H & 0x0f0fu) | ((L >> 2) & 0x3030u);
    const uint32_t m_cd = ((H >> 4) & 0x0f0fu) | ((M >> 2) & 0x3030u);
    KScales s;
    s.sc_a = static_cast<int>(sc_ab & 0xffu);
    s.sc_b = static_cast<int>(sc_ab >> 8);
    s.sc_c = static_cast<int>(sc_cd & 0xffu);
    s.sc_d = static_cast<int>(sc_cd >> 8);
    s.mins_ab = static_cast<int>(__byte_perm(m_ab, 0u, 0x1100u));
    s.mins_cd = static_cast<int>(__byte_perm(m_cd, 0u, 0x1100u));
    return s;
}

// Where a group's per-block fp32 terms go. Whole rows: added in block order
// into registers (the reference's sequential row sum). Split tiles (the
// blocks of a row spread over several warps): stored to shared memory
// terms[t][row][block] (by the lane of quarter 0, which holds the 4-lane
// total), summed in block order once every warp is done.
template <int NT>
struct Sink {
    float acc[NT];
    float *terms;  // nullptr: accumulate
    int nb;
    __device__ __forceinline__ void init(float *t, int n) {
#pragma unroll
        for (int i = 0; i < NT; ++i) acc[i] = 0.0f;
        terms = t;
        nb = n;
    }
    __device__ __forceinline__ void put(int t, int r, int b, bool writer, float term) {
        if (terms) {
            if (writer) terms[(t * 8 + r) * nb + b] = term;
        } else {
            acc[t] = __fadd_rn(acc[t], term);
        }
    }
};

// Shared tail of Q4_K/Q5_K: integer dots with the four activation slices,
// scale, mins via dp2a, 4-lane reduction, fp32 combination.
// HI16: wb and wd hold the high-nibble sub-blocks as 16 * w (Q4_K).
template <int NT, bool HI16 = false>
__device__ __forceinline__ void kquant_accumulate(const uint32_t (&wa)[4], const uint32_t (&wb)[4],
                                                  const uint32_t (&wc)[4], const uint32_t (&wd)[4],
                                                  const KScales &s, float dw, float dmw,
                                                  const GemvJob &job, const XView &x, int b, int j0,
                                                  int r0, int n_tok, Sink<NT> &acc, int r, bool writer) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (t < n_tok) {
            const int8_t *xq = x.qs + t * job.k + b * QH_QK + 64 * j0 + r0;
            const int4 xa = lds128i(xq);
            const int4 xb = lds128i(xq + 32);
            const int4 xc = lds128i(xq + 128);
            const int4 xd = lds128i(xq + 160);
            const int da = dot16(wa[0], wa[1], wa[2], wa[3], xa, 0);
            const int dc = dot16(wc[0], wc[1], wc[2], wc[3], xc, 0);
            int db, dd;
            if constexpr (HI16) {
                db = dot16_u(wb[0], wb[1], wb[2], wb[3], xb, 0) >> 4;
                dd = dot16_u(wd[0], wd[1], wd[2], wd[3], xd, 0) >> 4;
            } else {
                db = dot16(wb[0], wb[1], wb[2], wb[3], xb, 0);
                dd = dot16(wd[0], wd[1], wd[2], wd[3], xd, 0);
            }
            int isum = da * s.sc_a + db * s.sc_b + dc * s.sc_c + dd * s.sc_d;
            // Lanes q and q^1 share the four sub-blocks (each holds 16 of their
            // 32 weights), so the min terms are split between them: the lane
            // with r0 == 0 takes sub-blocks 2j0, 2j0+1 (bsum pairs at 4j0),
            // the other 2j0+4, 2j0+5 (bsum pairs at 4j0+8).
            const int hi = r0 >> 4;
            const int2 bp = *reinterpret_cast<const int2 *>(x.bs + (t * job.nb + b) * 16 + 4 * j0 + 8 * hi);
            const int msel = hi ? s.mins_cd : s.mins_ab;
            int mins = __dp2a_lo(bp.x, msel, 0);
            mins = __dp2a_hi(bp.y, msel, mins);
            isum += __shfl_xor_sync(0xffffffffu, isum, 1);
            mins += __shfl_xor_sync(0xffffffffu, mins, 1);
            isum += __shfl_xor_sync(0xffffffffu, isum, 2);
            mins += __shfl_xor_sync(0xffffffffu, mins, 2);
            const float yd = reinterpret_cast<const float *>(x.d)[t * job.d_stride + b];
            const float d = __fmul_rn(yd, dw);
            const float dmin = __fmul_rn(yd, dmw);
            acc.put(t, r, b, writer,
                    __fsub_rn(__fmul_rn(d, static_cast<float>(isum)), __fmul_rn(dmin, static_cast<float>(mins))));
        }
    }
}

// Sum over the 4 lanes of a row of four per-block partials p0..p3 (blocks
// b..b+3), transposed: lane q of the row ends with the total of block b + q
// (3 shuffles for the four blocks instead of 2 per block). Integer sums:
// the order of the additions does not matter.
__device__ __forceinline__ int quad_transpose_sum(int p0, int p1, int p2, int p3, int q) {
    const bool up = (q & 2) != 0;
    int k0 = up ? p2 : p0, k1 = up ? p3 : p1;
    const int s0 = up ? p0 : p2, s1 = up ? p1 : p3;
    k0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    k1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    const bool odd = (q & 1) != 0;
    return (odd ? k1 : k0) + __shfl_xor_sync(0xffffffffu, odd ? k0 : k1, 1);
}

// Q4_K, whole rows, four blocks at a time: each lane forms its partial
// integer sums of the four blocks, the transposed reduction gives lane q the
// totals of block b + q, lane q alone forms that block's fp32 term, and the
// four terms are added to the row sum in block order -- the same operations
// on the same values as one block at a time, with a quarter of the
// reductions and of the fp32 work.
template <int NT>
__device__ __forceinline__ void q4k_quad(const uint8_t *row, const GemvJob &job, const XView &x, int b, int q,
                                         float (&acc)[NT], int n_tok) {
    const int j0 = q >> 1, r0 = (q & 1) << 4, hi = r0 >> 4;
    const uint32_t sh = 16u * static_cast<uint32_t>(j0);
    int is[4][NT], mn[4][NT];
    uint32_t hx[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const uint8_t *blk = row + (b + u) * QH_Q4K_BYTES;
        const uint4 h = lds128(blk);
        const uint4 qa = lds128(blk + 16 + 16 * q);
        const uint4 qc = lds128(blk + 80 + 16 * q);
        const KScales s = unpack_kscales(h, sh);
        hx[u] = h.x;
        const uint32_t m4 = 0x0f0f0f0fu, h4 = 0xf0f0f0f0u;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            is[u][t] = 0;
            mn[u][t] = 0;
            if (t < n_tok) {
                const int8_t *xq = x.qs + t * job.k + (b + u) * QH_QK + 64 * j0 + r0;
                const int4 xa = lds128i(xq), xb = lds128i(xq + 32), xc = lds128i(xq + 128), xd = lds128i(xq + 160);
                const int da = dot16(qa.x & m4, qa.y & m4, qa.z & m4, qa.w & m4, xa, 0);
                const int db = dot16_u(qa.x & h4, qa.y & h4, qa.z & h4, qa.w & h4, xb, 0) >> 4;
                const int dc = dot16(qc.x & m4, qc.y & m4, qc.z & m4, qc.w & m4, xc, 0);
                const int dd = dot16_u(qc.x & h4, qc.y & h4, qc.z & h4, qc.w & h4, xd, 0) >> 4;
                is[u][t] = da * s.sc_a + db * s.sc_b + dc * s.sc_c + dd * s.sc_d;
                const int2 bp = *reinterpret_cast<const int2 *>(x.bs + (t * job.nb + b + u) * 16 + 4 * j0 + 8 * hi);
                const int msel = hi ? s.mins_cd : s.mins_ab;
                mn[u][t] = __dp2a_hi(bp.y, msel, __dp2a_lo(bp.x, msel, 0));
            }
        }
    }
    const uint32_t hq = q == 0 ? hx[0] : q == 1 ? hx[1] : q == 2 ? hx[2] : hx[3];
    const float dw = h2f_bits(hq), dmw = h2f_bits(hq >> 16);
    const int base = (threadIdx.x & 31) & ~3;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (t < n_tok) {
            const int isum = quad_transpose_sum(is[0][t], is[1][t], is[2][t], is[3][t], q);
            const int mins = quad_transpose_sum(mn[0][t], mn[1][t], mn[2][t], mn[3][t], q);
            const float yd = reinterpret_cast<const float *>(x.d)[t * job.d_stride + b + q];
            const float term = __fsub_rn(__fmul_rn(__fmul_rn(yd, dw), static_cast<float>(isum)),
                                         __fmul_rn(__fmul_rn(yd, dmw), static_cast<float>(mins)));
            float a = acc[t];
#pragma unroll
            for (int u = 0; u < 4; ++u) a = __fadd_rn(a, __shfl_sync(0xffffffffu, term, base + u));
            acc[t] = a;
        }
    }
}

template <int NT>
__device__ __forceinline__ void group_q4k(const uint8_t *grp, const GemvJob &job, const XView &x, int row0,
                                          int nvalid, int n_tok, int b_first, int b_step, float *terms) {
    const int lane = threadIdx.x & 31;
    const int r = lane >> 2, q = lane & 3, j0 = q >> 1, r0 = (q & 1) << 4;
    const uint8_t *row = grp + r * job.box_pitch;
    const uint32_t sh = 16u * static_cast<uint32_t>(j0);
    Sink<NT> acc;
    acc.init(terms, job.nb);
    int b = b_first;
    if constexpr (NT == 1) {
        if (!terms)  // whole rows: four blocks at a time, then the rest one by one
            for (; b + 4 <= job.nb; b += 4) q4k_quad<NT>(row, job, x, b, q, acc.acc, n_tok);
    }
    // unrolled: the loads and integer work of neighbouring blocks overlap
    // (the row sum still adds the blocks' terms in order)
#pragma unroll 4
    for (; b < job.nb; b += b_step) {
        const uint8_t *blk = row + b * QH_Q4K_BYTES;
        const uint4 h = lds128(blk);
        const uint4 qa = lds128(blk + 16 + 16 * q);  // qs[32*j0 + r0 .. +16]
        const uint4 qc = lds128(blk + 80 + 16 * q);  // qs[32*(j0+2) + r0 .. +16]
        const KScales s = unpack_kscales(h, sh);
        const uint32_t m4 = 0x0f0f0f0fu, h4 = 0xf0f0f0f0u;
        const uint32_t wa[4] = {qa.x & m4, qa.y & m4, qa.z & m4, qa.w & m4};
        const uint32_t wb[4] = {qa.x & h4, qa.y & h4, qa.z & h4, qa.w & h4};  // 16 * w
        const uint32_t wc[4] = {qc.x & m4, qc.y & m4, qc.z & m4, qc.w & m4};
        const uint32_t wd[4] = {qc.x & h4, qc.y & h4, qc.z & h4, qc.w & h4};  // 16 * w
        kquant_accumulate<NT, true>(wa, wb, wc, wd, s, h2f_bits(h.x), h2f_bits(h.x >> 16), job, x, b, j0,
                                    r0, n_tok, acc, r, q == 0);
    }
    if (!terms && q == 0 && r < nvalid) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (t < n_tok) job.out[static_cast<int64_t>(t) * job.n_rows + row0 + r] = acc.acc[t];
    }
}

template <int NT>
__device__ __forceinline__ void group_q5k(const uint8_t *grp, const GemvJob &job, const XView &x, int row0,
                                          int nvalid, int n_tok, int b_first, int b_step, float *terms) {
    const int lane = threadIdx.x & 31;
    const int r = lane >> 2, q = lane & 3, j0 = q >> 1, r0 = (q & 1) << 4;
    const uint8_t *row = grp + r * job.box_pitch;
    const uint32_t sh = 16u * static_cast<uint32_t>(j0);
    // 5th bit of sub-block s sits in bit s of qh[l]; move it to bit 4.
    const uint32_t up_a = 4u - 2u * j0, up_b = 3u - 2u * j0;  // s = 2j0, 2j0+1
    const uint32_t dn_c = 2u * j0, dn_d = 2u * j0 + 1u;       // s = 2j0+4, 2j0+5
    Sink<NT> acc;
    acc.init(terms, job.nb);
    for (int b = b_first; b < job.nb; b += b_step) {
        const uint8_t *blk = row + b * QH_Q5K_BYTES;
        const uint4 h = lds128(blk);
        const uint4 hv = lds128(blk + 16 + r0);       // qh[r0 .. r0+16)
        const uint4 qa = lds128(blk + 48 + 16 * q);   // qs[32*j0 + r0 ..]
        const uint4 qc = lds128(blk + 112 + 16 * q);  // qs[32*(j0+2) + r0 ..]
        const KScales s = unpack_kscales(h, sh);
        const uint32_t m4 = 0x0f0f0f0fu, b4 = 0x10101010u;
        const uint32_t qh[4] = {hv.x, hv.y, hv.z, hv.w};
        const uint32_t la[4] = {qa.x, qa.y, qa.z, qa.w};
        const uint32_t lc[4] = {qc.x, qc.y, qc.z, qc.w};
        uint32_t wa[4], wb[4], wc[4], wd[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wa[i] = (la[i] & m4) | ((qh[i] << up_a) & b4);
            wb[i] = ((la[i] >> 4) & m4) | ((qh[i] << up_b) & b4);
            wc[i] = (lc[i] & m4) | ((qh[i] >> dn_c) & b4);
            wd[i] = ((lc[i] >> 4) & m4) | ((qh[i] >> dn_d) & b4);
        }
        kquant_accumulate<NT>(wa, wb, wc, wd, s, h2f_bits(h.x), h2f_bits(h.x >> 16), job, x, b, j0,
                              r0, n_tok, acc, r, q == 0);
    }
    if (!terms && q == 0 && r < nvalid) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (t < n_tok) job.out[static_cast<int64_t>(t) * job.n_rows + row0 + r] = acc.acc[t];
    }
}

template <int NT>
__device__ __forceinline__ void group_q6k(const uint8_t *grp, const GemvJob &job, const XView &x, int row0,
                                          int nvalid, int n_tok, int b_first, int b_step, float *terms) {
    const int lane = threadIdx.x & 31;
    const int r = lane >> 2, q = lane & 3, n = q >> 1, l0 = (q & 1) << 4;
    const uint8_t *row = grp + r * job.box_pitch;
    const uint32_t bs_shift = 16u * static_cast<uint32_t>(q & 1);
    Sink<NT> acc;
    acc.init(terms, job.nb);
    for (int b = b_first; b < job.nb; b += b_step) {
        const uint8_t *blk = row + b * QH_Q6K_BYTES;
        const uint4 qa = lds128_a2(blk + 64 * n + l0);        // ql, quarters 0 (low) / 2 (high)
        const uint4 qb = lds128_a2(blk + 64 * n + 32 + l0);   // ql, quarters 1 (low) / 3 (high)
        const uint4 hv = lds128_a2(blk + 128 + 32 * n + l0);  // qh, 2 bits per quarter
        const int8_t *scp = reinterpret_cast<const int8_t *>(blk + 192 + 8 * n + (q & 1));
        const int s0 = scp[0], s1 = scp[2], s2 = scp[4], s3 = scp[6];
        const float dw = h2f_bits(*reinterpret_cast<const uint16_t *>(blk + 208));
        const uint32_t m4 = 0x0f0f0f0fu, m2 = 0x30303030u;
        const uint32_t la[4] = {qa.x, qa.y, qa.z, qa.w};
        const uint32_t lb[4] = {qb.x, qb.y, qb.z, qb.w};
        const uint32_t qh[4] = {hv.x, hv.y, hv.z, hv.w};
        uint32_t wa[4], wb[4], wc[4], wd[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wa[i] = (la[i] & m4) | ((qh[i] << 4) & m2);
            wb[i] = (lb[i] & m4) | ((qh[i] << 2) & m2);
            wc[i] = ((la[i] >> 4) & m4) | (qh[i] & m2);
            wd[i] = ((lb[i] >> 4) & m4) | ((qh[i] >> 2) & m2);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < n_tok) {
                const int8_t *xq = x.qs + t * job.k + b * QH_QK + 128 * n + l0;
                const int da = dot16(wa[0], wa[1], wa[2], wa[3], lds128i(xq), 0);
                const int db = dot16(wb[0], wb[1], wb[2], wb[3], lds128i(xq + 32), 0);
                const int dc = dot16(wc[0], wc[1], wc[2], wc[3], lds128i(xq + 64), 0);
                const int dd = dot16(wd[0], wd[1], wd[2], wd[3], lds128i(xq + 96), 0);
                const int4 bv = *reinterpret_cast<const int4 *>(x.bs + (t * job.nb + b) * 16 + 8 * n);
                const int b0 = static_cast<int16_t>(static_cast<uint32_t>(bv.x) >> bs_shift);
                const int b1 = static_cast<int16_t>(static_cast<uint32_t>(bv.y) >> bs_shift);
                const int b2 = static_cast<int16_t>(static_cast<uint32_t>(bv.z) >> bs_shift);
                const int b3 = static_cast<int16_t>(static_cast<uint32_t>(bv.w) >> bs_shift);
                // sum of scale * (dot - 32 * bsum) == isum - 32 * isum_mins
                int tot = s0 * (da - 32 * b0) + s1 * (db - 32 * b1) + s2 * (dc - 32 * b2) +
                          s3 * (dd - 32 * b3);
                tot += __shfl_xor_sync(0xffffffffu, tot, 1);
                tot += __shfl_xor_sync(0xffffffffu, tot, 2);
                const float yd = reinterpret_cast<const float *>(x.d)[t * job.d_stride + b];
                acc.put(t, r, b, q == 0, __fmul_rn(__fmul_rn(dw, yd), static_cast<float>(tot)));
            }
        }
    }
    if (!terms && q == 0 && r < nvalid) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (t < n_tok) job.out[static_cast<int64_t>(t) * job.n_rows + row0 + r] = acc.acc[t];
    }
}

// Q8_0 (against Q8_0 activations): 8 lanes per row, lane jj owns bytes
// 4jj..4jj+3 of every 32-block -- the lane layout of the reference's AVX
// tiers -- and accumulates with one FMA per block; 4 rows per pass.
template <int NT>
__device__ __forceinline__ void group_q8_0(const uint8_t *grp, const GemvJob &job, const XView &x, int row0,
                                           int nvalid, int n_tok) {
    const int lane = threadIdx.x & 31;
    const int rr = lane >> 3, jj = lane & 7;
    const uint16_t *xd = reinterpret_cast<const uint16_t *>(x.d);
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
        const int r = pass * 4 + rr;
        const uint8_t *row = grp + r * job.box_pitch;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        for (int b = 0; b < job.nb; ++b) {
            const uint8_t *blk = row + b * QH_Q8_0_BYTES;
            const int wq = static_cast<int>(lds32_a2(blk + 2 + 4 * jj));
            const float dw = h2f_bits(*reinterpret_cast<const uint16_t *>(blk));
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t < n_tok) {
                    const int xw = *reinterpret_cast<const int *>(x.qs + t * job.k + b * QH_QK8_0 + 4 * jj);
                    const float dx = h2f_bits(xd[t * job.d_stride + b]);
                    const int s = __dp4a(wq, xw, 0);
                    acc[t] = __fmaf_rn(static_cast<float>(s), __fmul_rn(dw, dx), acc[t]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < n_tok) {
                float v = acc[t];
                v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
                v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
                v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
                if (jj == 0 && r < nvalid)
                    job.out[static_cast<int64_t>(t) * job.n_rows + row0 + r] = v;
            }
        }
    }
}

// One 8-row group: blocks b_first, b_first + b_step, ... of its rows; with
// terms == nullptr whole rows (b_first 0, b_step 1) summed and stored.
template <int TYPE, int NT>
__device__ __forceinline__ void process_group(const uint8_t *wbase, int tile_rows, int trow,
                                              const GemvJob &job, const XView &x, int row0, int nvalid,
                                              int n_tok, int b_first = 0, int b_step = 1, float *terms = nullptr) {
    const uint8_t *grp = wbase + trow * job.box_pitch;
    if constexpr (TYPE == QH_GGUF_Q4_K) group_q4k<NT>(grp, job, x, row0, nvalid, n_tok, b_first, b_step, terms);
    else if constexpr (TYPE == QH_GGUF_Q5_K) group_q5k<NT>(grp, job, x, row0, nvalid, n_tok, b_first, b_step, terms);
    else if constexpr (TYPE == QH_GGUF_Q6_K) group_q6k<NT>(grp, job, x, row0, nvalid, n_tok, b_first, b_step, terms);
    else group_q8_0<NT>(grp, job, x, row0, nvalid, n_tok);
}

// Rows per consumer work unit: 8 rows of 4 lanes each.
constexpr int kGroupRows = 8;

// Bytes of the staged activation planes of one job (n_tok rows).
__host__ __device__ __forceinline__ void x_plane_bytes(int type, const GemvJob &job, int n_tok,
                                                       uint32_t *qs, uint32_t *bs, uint32_t *d) {
    *qs = static_cast<uint32_t>(n_tok) * static_cast<uint32_t>(job.k);
    *bs = type == QH_GGUF_Q8_0 ? 0u : static_cast<uint32_t>(n_tok * job.nb * 32);
    *d = static_cast<uint32_t>(n_tok * job.d_stride * (type == QH_GGUF_Q8_0 ? 2 : 4));
}

// ---------------------------------------------------------------------------
// Fused input: the 256 consumer threads form the jobs' shared Q8_K
// activation in the CTA's fixed planes ([qs][bsums][d], as staged ones),
// with the operations and order of resnorm_q8k_kernel (double sum of
// squares: thread t over elements t, t+256, ..., then the warp tree and the
// warps in order), swiglu_q8k_kernel or quantize_q8k_kernel.
// ---------------------------------------------------------------------------
constexpr int kFuseMaxBlocks = 16;  // residual + RMSNorm rows up to 4096

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ double consumers_sum_d(double v, double *scratch) {
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    consumers_sync();
    if (lane == 0) scratch[warp] = v;
    consumers_sync();
    double t = 0.0;
    for (int w = 0; w < kConsumerWarps; ++w) t += scratch[w];
    return t;
}

// One Q8_K block quantized by one warp (quantize_row_q8_K, slm/tensor.c:
// 673-720): lane l holds elements 8l..8l+7; the maximum magnitude with the
// first-index tie rule, the round-half-even quants, 1 / iscale and the 16
// sums of 16 quants -- the bytes q8k_block256 writes, without CTA barriers.
__device__ __forceinline__ void q8k_block_warp(const float (&v)[8], int8_t *qs, int16_t *bsums, float *d) {
    const int lane = threadIdx.x & 31;
    float a = -1.0f, bv = 0.0f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float ax = (v[e] == v[e]) ? fabsf(v[e]) : -1.0f;
        if (ax > a) { a = ax; bv = v[e]; bi = 8 * lane + e; }
    }
    warp_best(a, bi, bv);
    const float xmax = a > 0.0f ? bv : 0.0f;
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (xmax != 0.0f) {
        const float iscale = __fdiv_rn(-127.0f, xmax);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = q8k_value(v[e], iscale);
        if (lane == 0) *d = __fdiv_rn(1.0f, iscale);
    } else if (lane == 0) {
        *d = 0.0f;
    }
    uint32_t lo = 0u, hi = 0u;
    int sum = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        lo |= (static_cast<uint32_t>(q[e]) & 0xffu) << (8 * e);
        hi |= (static_cast<uint32_t>(q[e + 4]) & 0xffu) << (8 * e);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) sum += q[e];
    *reinterpret_cast<uint2 *>(qs + 8 * lane) = make_uint2(lo, hi);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    if ((lane & 1) == 0) bsums[lane >> 1] = static_cast<int16_t>(sum);
}

}  // namespace qh

#endif  // QH_GEMV_DEV_CUH
