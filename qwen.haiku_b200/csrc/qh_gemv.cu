// SPDX-License-Identifier: MIT
//
// qh_gemv.cu -- decode-time quantized matvec (and small-n matmul) for the
// GGUF K-quant / Q8_0 weight formats on sm_100a.
//
// Replaces the reference's per-row SIMD dots (simd/quants.h:244-402,
// simd/avx.c:420-591) as driven by tensor_matmul_{q4k,q5k,q6k,q8_0}_f32
// (slm/tensor.c:827-1033): out[t][j] = row_dot(W row j, Q8 activation row t).
//
// Design (memory-bound stream):
//   * Persistent grouped kernel: the launch walks a list of independent jobs
//     (weight matrix, activation, output) of one weight type; each job is
//     cut into tiles of R consecutive rows (a contiguous byte range).
//   * Warp 8 (one elected lane) is the producer: it streams each tile into a
//     ring of shared-memory stages with a 1-D bulk copy on the TMA engine
//     (cp.async.bulk + mbarrier complete_tx). Ranges are copied from their
//     16-byte-aligned start; the <16-byte tail of a range is fetched with
//     plain loads so the copy never reads past the matrix.
//   * Warps 0..7 consume: every warp owns whole 8-row groups (round-robin
//     across tiles, so short tiles still spread over all warps) and keeps
//     the tile's rows in shared memory while it walks their blocks.
//   * Integer block sums use dp4a/dp2a; the fp32 combination of each block
//     and the block-sequential row sum are done with explicitly rounded
//     __fmul_rn/__fsub_rn/__fadd_rn (no FMA contraction) in exactly the
//     reference's order, so the outputs are bit-identical to the reference's
//     scalar/AVX-VNNI/AVX2 results. Q8_0 reproduces the AVX tiers' 8-lane
//     fused-multiply-add accumulation and their horizontal-sum order.
//   * Every mbarrier wait is bounded; a timeout records an error in the
//     device error word and the CTA drains its own copies and returns.

#include <algorithm>

#include "qh_common.cuh"
#include "qh_internal.h"
#include "qh_q8k.cuh"
#include "qh_tc.cuh"

namespace qh {

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = 32 * (kConsumerWarps + 1);
// Shared memory per CTA: 2 KiB of barriers/stage metadata + the stage ring.
// Two CTAs fit on one SM (228 KiB per SM, 1 KiB reserved per CTA).
constexpr int kSmemHeader = 2048;
constexpr int kSmemDataBudget = 110 * 1024;  // per CTA at 2 CTAs/SM
// Per-block terms of split tiles (two buffers), after the stage ring and
// inside the data budget.
constexpr int kTermsBytes = 4096;
constexpr int kTermsFloats = kTermsBytes / 8;  // per buffer

// Per-stage metadata written by the producer: the tile's job descriptor
// (so consumers never touch the global job table) and its row range.
struct StageMeta {
    GemvJob job;
    int32_t row0, nrows, offset, pad;
};
static_assert(sizeof(StageMeta) <= 96, "stage metadata slot");

__device__ __forceinline__ GemvJob load_job(const GemvParams &p, int j) {
    return p.n_jobs <= kGemvInlineJobs ? p.jobs[j] : p.table[j];
}

// Largest job index whose tile_begin <= tile.
__device__ __forceinline__ int find_job(const GemvParams &p, int tile) {
    if (p.n_jobs <= kGemvInlineJobs) {
        int j = 0;
        for (int i = 1; i < p.n_jobs; ++i)
            if (p.jobs[i].tile_begin <= tile) j = i;
        return j;
    }
    int lo = 0, hi = p.n_jobs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(&p.table[mid].tile_begin) <= tile) lo = mid; else hi = mid - 1;
    }
    return lo;
}

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

// Fused input into the CTA's planes. RMSNorm first forms the row's double
// sum of squares over the 256 consumer threads (thread t: elements t,
// t + 256, ...); then every consumer warp quantizes whole Q8_K blocks (warp
// w: blocks w, w + 8, ...), re-reading its elements (cache hits).
__device__ __noinline__ void fuse_input(const GemvParams &p, uint8_t *xs, double *dscr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = p.xk, nb = K / QH_QK, nt = p.n_tok;
    const int dstride = static_cast<int>(qhf_q8k_d_stride(K));
    for (int t = 0; t < nt; ++t) {
        int8_t *qs = reinterpret_cast<int8_t *>(xs) + t * K;
        int16_t *bs = reinterpret_cast<int16_t *>(xs + nt * K) + t * nb * 16;
        float *dd = reinterpret_cast<float *>(xs + nt * K + nt * nb * 32) + t * dstride;
        const int64_t row = static_cast<int64_t>(t) * K;
        float rscale = 0.0f;
        if (p.xform == 1) {
            double s = 0.0;
#pragma unroll
            for (int j = 0; j < kFuseMaxBlocks; ++j) {
                if (j < nb) {
                    const int64_t i = row + j * QH_QK + tid;
                    float x = p.xa[i];
                    if (p.xb) x = __fadd_rn(x, p.xb[i]);
                    if (p.xh_out && blockIdx.x == 0) p.xh_out[i] = x;
                    s += static_cast<double>(__fmul_rn(x, x));
                }
            }
            const double ssq = consumers_sum_d(s, dscr);
            rscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ssq / static_cast<double>(K)), p.eps)));
        }
        for (int b = warp; b < nb; b += kConsumerWarps) {
            const int64_t e0 = row + b * QH_QK + 8 * lane;
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int64_t i = e0 + e;
                if (p.xform == 1) {
                    float x = p.xa[i];
                    if (p.xb) x = __fadd_rn(x, p.xb[i]);
                    v[e] = __fmul_rn(__fmul_rn(x, rscale), p.xw[b * QH_QK + 8 * lane + e]);
                } else if (p.xform == 2) {
                    v[e] = __fmul_rn(silu_f(p.xa[i]), p.xb[i]);
                } else {
                    v[e] = p.xa[i];
                }
            }
            q8k_block_warp(v, qs + b * QH_QK, bs + b * 16, dd + b);
        }
    }
}

// Output tail: every consumer thread fences its outputs, the CTA takes a
// ticket, and the last CTA of the launch forms the next Q8_K input -- the
// operations and order of fuse_input (and so of resnorm_q8k_kernel,
// swiglu_q8k_kernel, quantize_q8k_kernel), reading the other CTAs' outputs
// from L2 and writing the split layout to global memory. The ticket is left
// at zero for the next launch.
__device__ __noinline__ void gemv_tail(const GemvParams &p) {
    __shared__ double tscr[kConsumerWarps];
    __shared__ int t_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __threadfence();
    consumers_sync();
    if (tid == 0) t_last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
    consumers_sync();
    if (!t_last) return;
    __threadfence();
    pdl_wait();  // a CTA without tiles has not waited for the previous kernel yet
    const int K = p.tk, nb = K / QH_QK, nt = p.n_tok;
    const int64_t d_off = qhf_q8k_d_offset(K, nt), b_off = qhf_q8k_bsums_offset(K, nt);
    const int dstride = static_cast<int>(qhf_q8k_d_stride(K));
    for (int t = 0; t < nt; ++t) {
        int8_t *qs = reinterpret_cast<int8_t *>(p.txq) + static_cast<int64_t>(t) * K;
        float *dd = reinterpret_cast<float *>(p.txq + d_off) + t * dstride;
        int16_t *bs = reinterpret_cast<int16_t *>(p.txq + b_off) + t * nb * 16;
        const int64_t row = static_cast<int64_t>(t) * K;
        float rscale = 0.0f;
        if (p.tform == 1) {
            double s = 0.0;
#pragma unroll
            for (int j = 0; j < kFuseMaxBlocks; ++j) {
                if (j < nb) {
                    const int64_t i = row + j * QH_QK + tid;
                    float x = __ldcg(p.ta + i);
                    if (p.tb) x = __fadd_rn(x, __ldcg(p.tb + i));
                    if (p.th_out) p.th_out[i] = x;
                    s += static_cast<double>(__fmul_rn(x, x));
                }
            }
            const double ssq = consumers_sum_d(s, tscr);
            rscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ssq / static_cast<double>(K)), p.teps)));
        }
        for (int b = warp; b < nb; b += kConsumerWarps) {
            const int64_t e0 = row + b * QH_QK + 8 * lane;
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int64_t i = e0 + e;
                if (p.tform == 1) {
                    float x = __ldcg(p.ta + i);
                    if (p.tb) x = __fadd_rn(x, __ldcg(p.tb + i));
                    v[e] = __fmul_rn(__fmul_rn(x, rscale), p.tw[b * QH_QK + 8 * lane + e]);
                } else if (p.tform == 2) {
                    v[e] = __fmul_rn(silu_f(__ldcg(p.ta + i)), __ldcg(p.tb + i));
                } else {
                    v[e] = __ldcg(p.ta + i);
                }
            }
            q8k_block_warp(v, qs + b * QH_QK, bs + b * 16, dd + b);
        }
    }
    if (tid == 0) *p.ticket = 0u;
}

// ---------------------------------------------------------------------------
// The kernel: producer lane + 8 consumer warps over a ring of stages.
// ---------------------------------------------------------------------------
template <int TYPE, int NT>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kGemvMaxStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 256);
    StageMeta *meta = reinterpret_cast<StageMeta *>(smem + 384);  // kGemvMaxStages x 96 B
    uint8_t *data = smem + kSmemHeader;
    constexpr int GR = kGroupRows;

    const int S = p.n_stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t lim = p.wait_limit ? p.wait_limit : kWaitLimit;
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    // Each CTA streams one contiguous range of tiles (sequential addresses,
    // jobs visited in order).
    const int t_begin = static_cast<int>(static_cast<int64_t>(p.total_tiles) * blockIdx.x / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(p.total_tiles) * (blockIdx.x + 1) / gridDim.x);
    const int n_my = t_end - t_begin;

    if (warp == kConsumerWarps) {
        // ----- producer warp (uniform control flow; lane 0 owns the barriers) -----
        // The weight bytes of the first ring's worth of tiles are requested
        // before pdl_wait() -- they do not depend on earlier kernels, so under
        // programmatic launch they stream in while the previous kernel (the
        // activation quantizer) finishes; the activation planes follow the wait.
        const int n_pre = min(n_my, S);
        // test hook: the tile whose copies are left out (its stage never fills)
        auto withheld = [&](int i) { return p.test_withhold != 0 && t_begin + i == p.test_withhold - 1; };
        auto issue_x = [&](int i, int s) {  // tile i of this CTA in stage s
            if (lane == 0 && !p.xform && !withheld(i)) {
                const GemvJob &jb = meta[s].job;
                uint32_t xq_b, xb_b, xd_b;
                x_plane_bytes(TYPE, jb, p.n_tok, &xq_b, &xb_b, &xd_b);
                uint8_t *xdst = data + static_cast<int64_t>(s) * p.stage_bytes + p.x_offset;
                bulk_copy_g2s(xdst, jb.xqs, xq_b, &full[s]);
                if (xb_b) bulk_copy_g2s(xdst + xq_b, jb.xbs, xb_b, &full[s]);
                bulk_copy_g2s(xdst + xq_b + xb_b, jb.xd, xd_b, &full[s]);
            }
        };
        int issued = 0;
        int j = n_my > 0 ? find_job(p, t_begin) : 0;
        GemvJob job = load_job(p, j);
        for (int i = 0; i < n_my; ++i) {
            if (i == n_pre && !p.xform) {
                pdl_wait();
                for (int t = 0; t < n_pre; ++t) issue_x(t, t);
            }
            // Every decision that ends the loop is made warp-uniform, so the
            // __syncwarp below never waits for a lane that has left.
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            const int s = i % S;
            const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
            const bool ok = __all_sync(0xffffffffu, i < S || mbar_wait_n(&empty[s], ph ^ 1u, lim));
            if (!ok) {
                if (lane == 0) {
                    report_error(p.err_flag, kDevWaitTimeout);
                    *abort_flag = 1;
                }
                break;
            }
            const int tile = t_begin + i;
            while (tile >= job.tile_begin + job.n_tiles && j + 1 < p.n_jobs) job = load_job(p, ++j);
            const int row0 = (tile - job.tile_begin) * p.rows_per_tile;
            const int nrows = min(p.rows_per_tile, job.n_rows - row0);
            const uint8_t *g0 = job.w + static_cast<int64_t>(row0) * job.row_bytes;
            uint8_t *dst = data + static_cast<int64_t>(s) * p.stage_bytes;
            uint32_t xq_b = 0, xb_b = 0, xd_b = 0;
            if (!p.xform) x_plane_bytes(TYPE, job, p.n_tok, &xq_b, &xb_b, &xd_b);
            const uint8_t *g1 = g0 + static_cast<int64_t>(nrows) * job.row_bytes;
            const uint8_t *a0 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(g0) & ~uintptr_t(15));
            const uint8_t *a1 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(g1) & ~uintptr_t(15));
            const uint32_t wbytes = static_cast<uint32_t>(a1 - a0);
            const int offset = static_cast<int>(g0 - a0);
            if (lane == 0)
                for (int t = 0; t < static_cast<int>(g1 - a1); ++t) dst[wbytes + t] = __ldg(a1 + t);
            if (lane == 0) {
                meta[s].job = job;
                meta[s].row0 = row0;
                meta[s].nrows = nrows;
                meta[s].offset = offset;
                // Order this thread's generic-proxy shared writes before the
                // async-proxy bulk copies that later reuse the stage.
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                if (!withheld(i)) mbar_arrive_expect_tx(&full[s], wbytes + xq_b + xb_b + xd_b);
            }
            __syncwarp();
            if (lane == 0 && wbytes && !withheld(i)) bulk_copy_g2s(dst, a0, wbytes, &full[s]);
            if (i >= n_pre) issue_x(i, s);
            ++issued;
        }
        if (issued == n_pre && n_pre > 0 && !p.xform) {  // the loop ended inside the first ring
            pdl_wait();
            for (int t = 0; t < n_pre; ++t) issue_x(t, t);
        }
        // Drain: wait for this CTA's copies in flight before exiting.
        for (int i = max(0, issued - S); i < issued; ++i)
            if (!mbar_wait_n(&full[i % S], static_cast<uint32_t>(i / S) & 1u, lim) && lane == 0)
                report_error(p.err_flag, kDevWaitTimeout);
        return;
    }

    // ----- consumers -----
    // The activation planes: per stage, or (fused input) formed here once.
    uint8_t *xfix = data + p.x_fixed;
    if (p.xform) {
        __shared__ double fscr[kConsumerWarps];
        pdl_wait();
        fuse_input(p, xfix, fscr);
        consumers_sync();
    }
    auto xview = [&](const uint8_t *stage, const GemvJob &job) {
        const uint8_t *xb = p.xform ? xfix : stage + p.x_offset;
        XView x;
        x.qs = reinterpret_cast<const int8_t *>(xb);
        x.bs = reinterpret_cast<const int16_t *>(xb + p.n_tok * job.k);
        x.d = xb + p.n_tok * job.k + (TYPE == QH_GGUF_Q8_0 ? 0 : p.n_tok * job.nb * 32);
        return x;
    };
    if (p.split) {
        // One 8-row group per tile (the planner's condition), its blocks
        // spread over the 8 warps: warp w takes blocks w, w + 8, ...; the
        // terms meet in shared memory and warp 0 adds them in block order.
        // Every wait outcome is agreed on by all consumer warps first, so
        // the named barriers never wait for a warp that has left.
        float *terms = reinterpret_cast<float *>(data + p.terms_off);
        for (int i = 0; i < n_my; ++i) {
            const int s = i % S;
            const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
            const bool ok = !*abort_flag && mbar_wait_n(&full[s], ph, lim);
            if (bar_any(1, 32 * kConsumerWarps, !ok)) {
                if (!ok) {
                    report_error(p.err_flag, kDevWaitTimeout);
                    *abort_flag = 1;
                }
                break;
            }
            const GemvJob job = meta[s].job;
            const int row0 = meta[s].row0, nrows = meta[s].nrows;
            const uint8_t *stage = data + static_cast<int64_t>(s) * p.stage_bytes;
            const XView x = xview(stage, job);
            float *tb = terms + (i & 1) * kTermsFloats;
            const int nvalid = min(GR, nrows);
            if (warp < job.nb)
                process_group<TYPE, NT>(stage + meta[s].offset, p.rows_per_tile, 0, job, x, row0, nvalid, p.n_tok,
                                        warp, kConsumerWarps, tb);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumerWarps) : "memory");
            if (warp == 0 && (lane & 3) == 0 && (lane >> 2) < nvalid) {
                const int r = lane >> 2;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t < p.n_tok) {
                        float acc = 0.0f;
                        for (int b = 0; b < job.nb; ++b) acc = __fadd_rn(acc, tb[(t * GR + r) * job.nb + b]);
                        job.out[static_cast<int64_t>(t) * job.n_rows + row0 + r] = acc;
                    }
                }
            }
        }
        if (p.tform) gemv_tail(p);
        return;
    }
    int group_base = 0;
    for (int i = 0; i < n_my; ++i) {
        const int s = i % S;
        const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
        if (!mbar_wait_n(&full[s], ph, lim)) {
            report_error(p.err_flag, kDevWaitTimeout);
            *abort_flag = 1;
            break;
        }
        const GemvJob job = meta[s].job;
        const int row0 = meta[s].row0, nrows = meta[s].nrows;
        const int ngroups = (nrows + GR - 1) / GR;
        int g = warp - group_base % kConsumerWarps;
        if (g < 0) g += kConsumerWarps;
        const uint8_t *stage = data + static_cast<int64_t>(s) * p.stage_bytes;
        const uint8_t *base = stage + meta[s].offset;
        const XView x = xview(stage, job);
        for (; g < ngroups; g += kConsumerWarps)
            process_group<TYPE, NT>(base, p.rows_per_tile, GR * g, job, x, row0 + GR * g,
                                    min(GR, nrows - GR * g), p.n_tok);
        group_base += ngroups;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (*abort_flag) break;
    }
    if (p.tform) gemv_tail(p);
}

// ---------------------------------------------------------------------------
// Host side: planning and launch.
// ---------------------------------------------------------------------------

cudaError_t gemv_plan(int type, GemvJob *jobs, int n_jobs, int n_tok, int sm_count,
                      GemvParams *p, GemvGeometry *g, int xform) {
    if (n_jobs <= 0 || n_tok < 1 || n_tok > 8 || qhf_block_bytes(type) == 0)
        return cudaErrorInvalidValue;
    if (xform && type == QH_GGUF_Q8_0) return cudaErrorInvalidValue;
    const int GR = kGroupRows;
    int64_t max_pitch = 0, total_rows = 0, max_x = 0;
    for (int j = 0; j < n_jobs; ++j) {
        if (jobs[j].n_rows <= 0 || jobs[j].row_bytes <= 0) return cudaErrorInvalidValue;
        if (xform && jobs[j].k != jobs[0].k) return cudaErrorInvalidValue;
        jobs[j].box_blocks = jobs[j].nb;
        jobs[j].box_pitch = jobs[j].row_bytes;
        max_pitch = std::max<int64_t>(max_pitch, jobs[j].row_bytes);
        total_rows += jobs[j].n_rows;
        uint32_t a, b, c;
        x_plane_bytes(type, jobs[j], n_tok, &a, &b, &c);
        max_x = std::max<int64_t>(max_x, static_cast<int64_t>(a) + b + c);
    }
    const int64_t x_bytes = (max_x + 127) / 128 * 128;
    // With a fused input the activation planes live once per CTA, not per stage.
    const int64_t x_stage = xform ? 0 : x_bytes, x_fixed = xform ? x_bytes : 0;
    const int64_t budget = kSmemDataBudget - x_fixed;
    if (budget <= 0) return cudaErrorInvalidValue;
    // Small launches (the decode step's projections, a few MB each) take one
    // CTA per SM, not two: their time is latency, and with half the
    // registers and shared memory of an SM free, the next launch's CTAs are
    // resident early and stream their weights while this one finishes
    // (programmatic launch). Batch-1 decode step: 1.127 -> 1.036 ms.
    int64_t wtot = 0;
    for (int j = 0; j < n_jobs; ++j) wtot += static_cast<int64_t>(jobs[j].n_rows) * jobs[j].row_bytes;
    const int max_ctas = wtot <= (16ll << 20) ? sm_count : 2 * sm_count;
    // Rows per tile: a multiple of the group size, at most 64, small enough
    // that the launch has ~2 tiles per CTA, and shrunk until the ring holds
    // at least 3 stages (2 at the very least).
    const int64_t r_max = 64;
    const int64_t r_bal = (total_rows / (2 * static_cast<int64_t>(max_ctas))) / GR * GR;
    int64_t R = std::max<int64_t>(GR, std::min<int64_t>(r_bal, r_max));
    auto stage_of = [&](int64_t r) { return (r * max_pitch + 32 + 127) / 128 * 128 + x_stage; };
    while (R > GR && budget / stage_of(R) < 3) R -= GR;
    const int64_t w_bytes = (R * max_pitch + 32 + 127) / 128 * 128;
    const int64_t stage_bytes = w_bytes + x_stage;
    const int64_t stages = std::min<int64_t>(kGemvMaxStages, budget / stage_bytes);
    if (stages < 2) return cudaErrorInvalidValue;  // a row (+ activations) too long to stage
    int64_t tiles = 0;
    for (int j = 0; j < n_jobs; ++j) {
        jobs[j].tile_begin = static_cast<int32_t>(tiles);
        jobs[j].n_tiles = static_cast<int32_t>((jobs[j].n_rows + R - 1) / R);
        tiles += jobs[j].n_tiles;
    }
    if (tiles > (1ll << 30)) return cudaErrorInvalidValue;
    p->n_jobs = n_jobs;
    p->total_tiles = static_cast<int32_t>(tiles);
    p->rows_per_tile = static_cast<int32_t>(R);
    p->n_stages = static_cast<int32_t>(stages);
    p->stage_bytes = static_cast<int32_t>(stage_bytes);
    p->n_tok = n_tok;
    p->x_offset = static_cast<int32_t>(w_bytes);
    p->xform = xform;
    p->xk = xform ? jobs[0].k : 0;
    for (int j = 0; j < kGemvInlineJobs; ++j) p->jobs[j] = j < n_jobs ? jobs[j] : GemvJob{};
    g->grid = static_cast<int>(std::min<int64_t>(tiles, max_ctas));
    // Split tiles: when every CTA holds at most one 8-row tile, one warp per
    // tile would walk all blocks of its rows alone; spread them instead
    // (needs the terms area next to at least two stages).
    int64_t max_nb = 0;
    for (int j = 0; j < n_jobs; ++j) max_nb = std::max<int64_t>(max_nb, jobs[j].nb);
    const int64_t split_stages = std::min<int64_t>(stages, (budget - kTermsBytes) / stage_bytes);
    p->split = (type != QH_GGUF_Q8_0 && R == GR && tiles <= g->grid && max_nb > 1 && split_stages >= 2 &&
                static_cast<int64_t>(n_tok) * GR * max_nb <= kTermsFloats)
                   ? 1
                   : 0;
    if (p->split) p->n_stages = static_cast<int32_t>(split_stages);
    p->x_fixed = static_cast<int32_t>(p->n_stages * stage_bytes);
    p->terms_off = static_cast<int32_t>(p->x_fixed + x_fixed);
    g->smem_bytes = static_cast<int>(kSmemHeader + p->terms_off + (p->split ? kTermsBytes : 0));
    return cudaSuccess;
}

template <int TYPE, int NT>
static cudaError_t launch_one(const GemvParams &p, const GemvGeometry &g, cudaStream_t stream) {
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<TYPE, NT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemHeader + kSmemDataBudget);
        if (e != cudaSuccess) return e;
        attr_done[dev] = true;
    }
    return launch_pdl(gemv_kernel<TYPE, NT>, dim3(g.grid), dim3(kGemvThreads), g.smem_bytes, stream, p);
}

template <int TYPE>
static cudaError_t launch_type(const GemvParams &p, const GemvGeometry &g, cudaStream_t stream) {
    if (p.n_tok <= 1) return launch_one<TYPE, 1>(p, g, stream);
    if (p.n_tok <= 2) return launch_one<TYPE, 2>(p, g, stream);
    if (p.n_tok <= 4) return launch_one<TYPE, 4>(p, g, stream);
    return launch_one<TYPE, 8>(p, g, stream);
}

cudaError_t gemv_launch(int type, const GemvParams &p, const GemvGeometry &g, cudaStream_t stream) {
    if (g.grid <= 0) return cudaSuccess;
    switch (type) {
        case QH_GGUF_Q4_K: return launch_type<QH_GGUF_Q4_K>(p, g, stream);
        case QH_GGUF_Q5_K: return launch_type<QH_GGUF_Q5_K>(p, g, stream);
        case QH_GGUF_Q6_K: return launch_type<QH_GGUF_Q6_K>(p, g, stream);
        case QH_GGUF_Q8_0: return launch_type<QH_GGUF_Q8_0>(p, g, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace qh
