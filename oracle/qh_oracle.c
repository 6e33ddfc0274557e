// SPDX-License-Identifier: MIT
//
// qh_oracle.c -- CPU restatement of qwen.haiku's quantized matmul path.
//
// TEST INFRASTRUCTURE, NOT PRODUCT CODE. Only tests/, the smoke check in
// __graft_entry__.py and bench.py's cpu_baseline leg load this library, and
// only as the checker. Nothing in the qwen.haiku_b200 package links it.
//
// Every function restates one piece of the reference (path:line within the
// qwen.haiku project), written against raw block bytes with explicit field
// offsets instead of the reference's structs:
//
//   GGUF block byte layouts (simd/quants.h:94-130):
//     Q4_K 144 B  [0]fp16 d [2]fp16 dmin [4]u8 scales[12] [16]u8 qs[128]
//     Q5_K 176 B  [0]fp16 d [2]fp16 dmin [4]u8 scales[12] [16]u8 qh[32] [48]u8 qs[128]
//     Q6_K 210 B  [0]u8 ql[128] [128]u8 qh[64] [192]i8 scales[16] [208]fp16 d
//     Q8_0  34 B  [0]fp16 d [2]i8 qs[32]
//   Sampler chain sample_with (slm/sampler.c:134-180), generator
//   (slm/model.c:414-447): orc_sample_with at the end of this file.
//   Activation rows are handed over split into planes (qs int8[K], d float[K/256],
//   bsums int16[K/16]) -- the same numbers as the reference's q8k_block array.
//
// Parity is pinned against the reference compiled from its own sources
// (oracle/ref_harness.c -> oracle/_ref/libqhref.so) by tests/test_oracle.py.
//
// Build: gcc -O2 -std=c17 -ffp-contract=off (the reference's C17 build does
// not contract a*b-c*d into an FMA; neither may this file).

#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>
#include <unistd.h>

#define QK 256

static inline float f16_bits_to_f32(const uint8_t *p) {
    _Float16 h;
    memcpy(&h, p, 2);
    return (float)h;
}

// ---------------------------------------------------------------------------
// Activation quantizers
// ---------------------------------------------------------------------------

// Q8_K row quantizer, slm/tensor.c:683-720 (rounding helper slm/tensor.c:673-678).
// Per 256-block: the value of largest magnitude (first one wins ties) sets
// iscale = -127/xmax; qs = clamp(round-half-even(iscale*x)); d = 1/iscale;
// bsums = sums of 16-element groups. All-zero block -> d=0, qs=0, bsums=0.
void orc_quantize_row_q8k(const float *x, int64_t k, float *d_out,
                          int8_t *qs_out, int16_t *bsums_out) {
    for (int64_t b = 0; b < k / QK; b++) {
        const float *src = x + b * QK;
        int8_t *q = qs_out + b * QK;
        int16_t *bs = bsums_out + b * (QK / 16);
        float best_abs = 0.0f, best_val = 0.0f;
        for (int i = 0; i < QK; i++) {
            float a = fabsf(src[i]);
            if (a > best_abs) { best_abs = a; best_val = src[i]; }
        }
        if (best_abs == 0.0f) {
            d_out[b] = 0.0f;
            memset(q, 0, QK);
            memset(bs, 0, sizeof(int16_t) * (QK / 16));
            continue;
        }
        const float iscale = -127.0f / best_val;
        d_out[b] = 1.0f / iscale;
        for (int i = 0; i < QK; i++) {
            // round-half-even: adding 1.5*2^23 leaves the rounded integer in
            // the low mantissa bits (valid for |v| < 2^22).
            float shifted = iscale * src[i] + 12582912.0f;
            int32_t bits;
            memcpy(&bits, &shifted, 4);
            int32_t v = (bits & 0x007fffff) - 0x00400000;
            q[i] = (int8_t)(v > 127 ? 127 : (v < -128 ? -128 : v));
        }
        for (int g = 0; g < QK / 16; g++) {
            int32_t s = 0;
            for (int i = 0; i < 16; i++) s += q[g * 16 + i];
            bs[g] = (int16_t)s;
        }
    }
}

// Q8_0 activation quantizer used for Q8_0 weights, slm/tensor.c:930-950.
// d = amax/127 stored as fp16 (round to nearest even); qs = roundf(x * (1/d))
// with the UNROUNDED d (half away from zero, unlike the Q8_K path).
void orc_quantize_row_q8_0(const float *x, int64_t k, uint16_t *d_bits_out,
                           int8_t *qs_out) {
    for (int64_t b = 0; b < k / 32; b++) {
        const float *src = x + b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(src[i]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        _Float16 h = (_Float16)d;
        memcpy(&d_bits_out[b], &h, 2);
        for (int i = 0; i < 32; i++) {
            int32_t v = (int32_t)roundf(src[i] * id);
            qs_out[b * 32 + i] = (int8_t)(v > 127 ? 127 : (v < -128 ? -128 : v));
        }
    }
}

// ---------------------------------------------------------------------------
// 6-bit scale/min unpack of the 12-byte K-quant scale field,
// simd/quants.h:215-224. Sub-blocks 0..3 keep their low 6 bits in bytes
// 0..3 (scale) / 4..7 (min); sub-blocks 4..7 take a nibble from bytes 8..11
// and the two spare top bits of bytes 0..7.
// ---------------------------------------------------------------------------
static void unpack_scale_min(const uint8_t *s12, int sb, int *sc, int *mn) {
    if (sb < 4) {
        *sc = s12[sb] & 0x3f;
        *mn = s12[sb + 4] & 0x3f;
    } else {
        *sc = (s12[sb + 4] & 0x0f) | ((s12[sb - 4] >> 6) << 4);
        *mn = (s12[sb + 4] >> 4) | ((s12[sb] >> 6) << 4);
    }
}

// ---------------------------------------------------------------------------
// Per-super-block integer sums (bit-exact quantities)
// ---------------------------------------------------------------------------

// Q4_K, simd/quants.h:267-306. Weight w = nibble; 64-weight chunk c uses
// qs[32c..32c+31]: low nibbles are weights 64c+l (sub-block 2c), high nibbles
// weights 64c+32+l (sub-block 2c+1).
//   isum      = sum_sb scale[sb] * sum_{i in sb} w_i * q8_i
//   isum_mins = sum_sb min[sb] * (bsums[2sb] + bsums[2sb+1])
void orc_q4k_block_ints(const uint8_t *blk, const int8_t *q8,
                        const int16_t *bs, int32_t *isum, int32_t *isum_mins) {
    const uint8_t *qs = blk + 16;
    int32_t acc = 0, accm = 0;
    for (int sb = 0; sb < 8; sb++) {
        int sc, mn;
        unpack_scale_min(blk + 4, sb, &sc, &mn);
        accm += mn * ((int32_t)bs[2 * sb] + (int32_t)bs[2 * sb + 1]);
        const int c = sb / 2, hi = sb & 1;
        int32_t dot = 0;
        for (int l = 0; l < 32; l++) {
            int w = hi ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 0x0f);
            dot += w * q8[64 * c + 32 * hi + l];
        }
        acc += sc * dot;
    }
    *isum = acc;
    *isum_mins = accm;
}

// Q5_K, simd/quants.h:310-351: as Q4_K plus a fifth bit; weight 64c+l takes
// bit 2c of qh[l], weight 64c+32+l takes bit 2c+1 of qh[l].
void orc_q5k_block_ints(const uint8_t *blk, const int8_t *q8,
                        const int16_t *bs, int32_t *isum, int32_t *isum_mins) {
    const uint8_t *qh = blk + 16;
    const uint8_t *qs = blk + 48;
    int32_t acc = 0, accm = 0;
    for (int sb = 0; sb < 8; sb++) {
        int sc, mn;
        unpack_scale_min(blk + 4, sb, &sc, &mn);
        accm += mn * ((int32_t)bs[2 * sb] + (int32_t)bs[2 * sb + 1]);
        const int c = sb / 2, hi = sb & 1;
        int32_t dot = 0;
        for (int l = 0; l < 32; l++) {
            int w = hi ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 0x0f);
            w += ((qh[l] >> sb) & 1) << 4;
            dot += w * q8[64 * c + 32 * hi + l];
        }
        acc += sc * dot;
    }
    *isum = acc;
    *isum_mins = accm;
}

// Q6_K, simd/quants.h:356-402. Unsigned 6-bit w in [0,63]; weight position
// p = 128h + 32r + l (h half, r quarter, l < 32):
//   low 4 bits: ql[64h + 32(r&1) + l] nibble (r>>1: 0 low, 1 high)
//   high 2 bits: qh[32h + l] >> 2r
// 16-wide sub-block sb = p/16 uses signed scale scales[sb].
//   isum      = sum_sb scale[sb] * sum_{i in sb} w_i * q8_i
//   isum_mins = sum_sb scale[sb] * bsums[sb]       (the -32 offset term)
void orc_q6k_block_ints(const uint8_t *blk, const int8_t *q8,
                        const int16_t *bs, int32_t *isum, int32_t *isum_mins) {
    const uint8_t *ql = blk;
    const uint8_t *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    int32_t acc = 0, accm = 0;
    for (int sb = 0; sb < 16; sb++) accm += (int32_t)sc[sb] * (int32_t)bs[sb];
    for (int p = 0; p < QK; p++) {
        const int h = p / 128, r = (p / 32) & 3, l = p & 31;
        const uint8_t lo_byte = ql[64 * h + 32 * (r & 1) + l];
        const int lo = (r >> 1) ? (lo_byte >> 4) : (lo_byte & 0x0f);
        const int hi2 = (qh[32 * h + l] >> (2 * r)) & 3;
        acc += (int32_t)sc[p / 16] * (lo | (hi2 << 4)) * (int32_t)q8[p];
    }
    *isum = acc;
    *isum_mins = accm;
}

// ---------------------------------------------------------------------------
// fp32 row dots. The per-block fp32 combination and the sequential block sum
// follow the scalar reference (simd/quants.h:303, 348, 399), which the
// reference's AVX-VNNI/AVX2 tiers reproduce exactly on x86 (they broadcast
// each block value into 8 lanes and divide the lane sum by 8,
// simd/avx.c:459-467, 515-523, 583-591).
// ---------------------------------------------------------------------------

float orc_q4k_row_dot(int nb, const uint8_t *row, const float *yd,
                      const int8_t *yqs, const int16_t *ybs) {
    float sumf = 0.0f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = row + 144 * b;
        int32_t isum, isum_mins;
        orc_q4k_block_ints(blk, yqs + QK * b, ybs + 16 * b, &isum, &isum_mins);
        const float d = yd[b] * f16_bits_to_f32(blk);
        const float dmin = yd[b] * f16_bits_to_f32(blk + 2);
        sumf += d * (float)isum - dmin * (float)isum_mins;
    }
    return sumf;
}

float orc_q5k_row_dot(int nb, const uint8_t *row, const float *yd,
                      const int8_t *yqs, const int16_t *ybs) {
    float sumf = 0.0f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = row + 176 * b;
        int32_t isum, isum_mins;
        orc_q5k_block_ints(blk, yqs + QK * b, ybs + 16 * b, &isum, &isum_mins);
        const float d = yd[b] * f16_bits_to_f32(blk);
        const float dmin = yd[b] * f16_bits_to_f32(blk + 2);
        sumf += d * (float)isum - dmin * (float)isum_mins;
    }
    return sumf;
}

float orc_q6k_row_dot(int nb, const uint8_t *row, const float *yd,
                      const int8_t *yqs, const int16_t *ybs) {
    float sumf = 0.0f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = row + 210 * b;
        int32_t isum, isum_mins;
        orc_q6k_block_ints(blk, yqs + QK * b, ybs + 16 * b, &isum, &isum_mins);
        sumf += f16_bits_to_f32(blk + 208) * yd[b] * (float)(isum - 32 * isum_mins);
    }
    return sumf;
}

// Q8_0 x Q8_0 row dot as the reference's AVX-VNNI/AVX2 tier computes it
// (simd/avx.c:65-88, 99-124): lane j (0..7) holds the int32 dot of bytes
// 4j..4j+3 of every 32-block and accumulates it with one fused multiply-add
// per block (scale = fp16(w.d) * fp16(x.d)); the 8 lanes are then summed as
// ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)).
float orc_q8_0_row_dot(int64_t k, const uint8_t *row, const uint16_t *yd_bits,
                       const int8_t *yqs) {
    float lane[8] = {0};
    for (int64_t b = 0; b < k / 32; b++) {
        const uint8_t *blk = row + 34 * b;
        const int8_t *wq = (const int8_t *)(blk + 2);
        const float scale = f16_bits_to_f32(blk) *
                            f16_bits_to_f32((const uint8_t *)&yd_bits[b]);
        for (int j = 0; j < 8; j++) {
            int32_t s = 0;
            for (int i = 0; i < 4; i++)
                s += (int32_t)wq[4 * j + i] * (int32_t)yqs[b * 32 + 4 * j + i];
            lane[j] = fmaf((float)s, scale, lane[j]);
        }
    }
    return ((lane[0] + lane[4]) + (lane[1] + lane[5])) +
           ((lane[2] + lane[6]) + (lane[3] + lane[7]));
}

// Q8_0 x Q8_0 row dot in the scalar reference's order (simd/quants.h:244-256):
// sequential per-block sumf += sumi * (fp16(w.d) * fp16(x.d)).
float orc_q8_0_row_dot_scalar(int64_t k, const uint8_t *row,
                              const uint16_t *yd_bits, const int8_t *yqs) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < k / 32; b++) {
        const uint8_t *blk = row + 34 * b;
        const int8_t *wq = (const int8_t *)(blk + 2);
        int32_t s = 0;
        for (int i = 0; i < 32; i++) s += (int32_t)wq[i] * (int32_t)yqs[b * 32 + i];
        sumf += (float)s * (f16_bits_to_f32(blk) *
                            f16_bits_to_f32((const uint8_t *)&yd_bits[b]));
    }
    return sumf;
}

// ---------------------------------------------------------------------------
// Block dequantization, slm/tensor.c:800-820 (Q4_K), 867-896 (Q5_K),
// 988-1010 (Q6_K): 256 fp32 weights of one super-block.
// ---------------------------------------------------------------------------
void orc_dequant_block(int type, const uint8_t *blk, float *y) {
    if (type == 12 || type == 13) {        // Q4_K / Q5_K
        const float d = f16_bits_to_f32(blk), dmin = f16_bits_to_f32(blk + 2);
        const uint8_t *qs = blk + (type == 12 ? 16 : 48);
        for (int p = 0; p < QK; p++) {
            const int c = p / 64, hi = (p / 32) & 1, l = p & 31;
            int sc, mn;
            unpack_scale_min(blk + 4, 2 * c + hi, &sc, &mn);
            int w = hi ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 0x0f);
            if (type == 13) w += ((blk[16 + l] >> (2 * c + hi)) & 1) << 4;
            const float dd = d * (float)sc, mm = dmin * (float)mn;
            y[p] = dd * (float)w - mm;
        }
    } else if (type == 14) {               // Q6_K
        const float d = f16_bits_to_f32(blk + 208);
        const int8_t *sc = (const int8_t *)(blk + 192);
        for (int p = 0; p < QK; p++) {
            const int h = p / 128, r = (p / 32) & 3, l = p & 31;
            const uint8_t lo_byte = blk[64 * h + 32 * (r & 1) + l];
            const int lo = (r >> 1) ? (lo_byte >> 4) : (lo_byte & 0x0f);
            const int hi2 = (blk[128 + 32 * h + l] >> (2 * r)) & 3;
            const int q = (lo | (hi2 << 4)) - 32;
            y[p] = d * (float)sc[p / 16] * (float)q;
        }
    }
}

// ---------------------------------------------------------------------------
// Matmul wrappers: tensor_matmul_{q4k,q5k,q8_0,q6k}_f32, slm/tensor.c:827-853,
// 898-919, 952-981, 1012-1033. For each of n tokens (x is [n][k] fp32):
// quantize the row, then out[t*out_f + j] = row_dot(weight row j).
// type follows the GGUF enum (slm/gguf.c:52-59): 0 F32 (tensor_matmul_f32,
// slm/tensor.c:517), 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K. Scratch comes from the caller (q8 buffers sized for k).
// Returns 0, or -1 for an unsupported type / k.
// ---------------------------------------------------------------------------
int orc_matmul(int type, const uint8_t *w, int64_t out_f, int64_t k,
               const float *x, int64_t n, float *out,
               int8_t *scratch_qs, float *scratch_d, int16_t *scratch_bs) {
    if (type == 0) {  // F32: tensor_matmul_f32, slm/tensor.c:517-535
        const float *wf = (const float *)w;
        for (int64_t t = 0; t < n; t++)
            for (int64_t j = 0; j < out_f; j++) {
                float acc = 0.0f;
                for (int64_t i = 0; i < k; i++) acc += wf[j * k + i] * x[t * k + i];
                out[t * out_f + j] = acc;
            }
        return 0;
    }
    if (type == 8) {
        if (k % 32) return -1;
        uint16_t *dbits = (uint16_t *)scratch_d;
        const int64_t row_bytes = 34 * (k / 32);
        for (int64_t t = 0; t < n; t++) {
            orc_quantize_row_q8_0(x + t * k, k, dbits, scratch_qs);
            for (int64_t j = 0; j < out_f; j++)
                out[t * out_f + j] = orc_q8_0_row_dot(k, w + j * row_bytes,
                                                      dbits, scratch_qs);
        }
        return 0;
    }
    if (k % QK) return -1;
    const int nb = (int)(k / QK);
    int64_t bb;
    float (*dot)(int, const uint8_t *, const float *, const int8_t *, const int16_t *);
    switch (type) {
        case 12: bb = 144; dot = orc_q4k_row_dot; break;
        case 13: bb = 176; dot = orc_q5k_row_dot; break;
        case 14: bb = 210; dot = orc_q6k_row_dot; break;
        default: return -1;
    }
    for (int64_t t = 0; t < n; t++) {
        orc_quantize_row_q8k(x + t * k, k, scratch_d, scratch_qs, scratch_bs);
        for (int64_t j = 0; j < out_f; j++)
            out[t * out_f + j] = dot(nb, w + j * nb * bb, scratch_d, scratch_qs,
                                     scratch_bs);
    }
    return 0;
}

// ---------------------------------------------------------------------------
// Sampler chain: sample_with (slm/sampler.c:134-180) with the generator of
// slm/model.c:414-447. fp = {temperature, top_p, min_p, repetition_penalty},
// ip = {top_k, repetition_window}, st = generator words (advanced in place).
// Logits are penalized in place. The exponential is the host C library's
// expf, as the reference's (and the device kernel's, bit for bit).
// ---------------------------------------------------------------------------

static uint64_t orc_rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

// rng_next + rng_uniform (slm/model.c:420-428, 444-447)
static float orc_uniform(uint64_t *st) {
    const uint64_t a = st[0];
    uint64_t b = st[1];
    const uint64_t out = orc_rotl64(a * 5u, 7) * 9u;
    b ^= a;
    st[0] = orc_rotl64(a, 24) ^ b ^ (b << 16);
    st[1] = orc_rotl64(b, 37);
    return (float)(uint32_t)(out >> 40) / 16777216.0f;
}

#define ORC_TOPK_MAX 256

// First slot holding the smallest value among slot[0..k).
static int orc_first_min(const float *val, int k) {
    int w = 0;
    for (int j = 1; j < k; j++)
        if (val[j] < val[w]) w = j;
    return w;
}

int32_t orc_sample_with(float *lg, int64_t n, const float *fp, const int32_t *ip, uint64_t *st,
                        const int32_t *hist, int32_t hn) {
    const float temp = fp[0], top_p = fp[1], min_p = fp[2], pen = fp[3];
    // repetition penalty: each occurrence in the window scales its logit
    // once more (slm/sampler.c:49-63)
    if (pen != 1.0f && hn != 0) {
        const int32_t win = ip[1];
        for (int32_t i = (win > 0 && win < hn) ? hn - win : 0; i < hn; i++) {
            const int32_t t = hist[i];
            if (t < 0 || (int64_t)t >= n) continue;
            lg[t] = lg[t] > 0.0f ? lg[t] / pen : lg[t] * pen;
        }
    }
    if (temp <= 0.0f) {  // sample_argmax (slm/model.c:401-412)
        int32_t best = 0;
        for (int64_t i = 1; i < n; i++)
            if (lg[i] > lg[best]) best = (int32_t)i;
        return best;
    }
    int k = ip[0] > 0 ? ip[0] : ORC_TOPK_MAX;
    if (k > ORC_TOPK_MAX) k = ORC_TOPK_MAX;
    // top-k slots: fill the first k, then each logit above the current
    // first minimum takes that slot (slm/sampler.c:70-93)
    float val[ORC_TOPK_MAX];
    int32_t idx[ORC_TOPK_MAX];
    int filled = 0;
    int w = 0;
    for (int64_t i = 0; i < n; i++) {
        if (filled < k) {
            val[filled] = lg[i];
            idx[filled] = (int32_t)i;
            if (++filled == k) w = orc_first_min(val, k);
        } else if (lg[i] > val[w]) {
            val[w] = lg[i];
            idx[w] = (int32_t)i;
            w = orc_first_min(val, k);
        }
    }
    // softmax over the slots in slot order (slm/sampler.c:97-112)
    float m = val[0];
    for (int j = 1; j < filled; j++)
        if (val[j] > m) m = val[j];
    float sum = 0.0f;
    for (int j = 0; j < filled; j++) {
        val[j] = expf((val[j] - m) / temp);
        sum += val[j];
    }
    if (sum > 0.0f)
        for (int j = 0; j < filled; j++) val[j] /= sum;
    // stable descending order (slm/sampler.c:117-130)
    float sv[ORC_TOPK_MAX];
    int32_t si[ORC_TOPK_MAX];
    for (int j = 0; j < filled; j++) {
        int r = 0;
        for (int i = 0; i < filled; i++) r += (val[i] > val[j]) || (val[i] == val[j] && i < j);
        sv[r] = val[j];
        si[r] = idx[j];
    }
    int cutoff = filled;
    if (top_p > 0.0f && top_p < 1.0f) {
        float acc = 0.0f;
        for (int j = 0; j < filled; j++) {
            acc += sv[j];
            if (acc >= top_p) { cutoff = j + 1; break; }
        }
    }
    if (min_p > 0.0f) {
        const float thresh = min_p * sv[0];
        int j = 1;
        while (j < cutoff && sv[j] >= thresh) j++;
        cutoff = j;
    }
    float tot = 0.0f;
    for (int j = 0; j < cutoff; j++) tot += sv[j];
    const float u = orc_uniform(st) * tot;
    float c = 0.0f;
    int picked = 0;
    for (int j = 0; j < cutoff; j++) {
        c += sv[j];
        if (u <= c) { picked = j; break; }
    }
    return si[picked];
}

// ---------------------------------------------------------------------------
// Chunked Gated DeltaNet step (slm/chunked.c:287-523, chunked_ssm_step_f32),
// the prompt path of slm_forward_ssm_batch (slm/qwen.c:772-806): one head,
// n <= 64 tokens, state [hd k][hd v] carried in place, out [n][hd v].
//
// Written as the device kernel computes it: every matrix entry is a single
// float chain, terms added in the reference's index order, products and
// sums rounded separately (no FMA). Terms the reference adds that are
// products with an exact zero (the masked upper triangles, the zero rows of
// the forward substitution) leave a finite running sum unchanged and are
// skipped. K*beta, V*beta, K*beta*gexp and Q*gexp are recomputed where used
// (the same rounded products the reference stores).
// expf is the host C library's, as the reference's.
// ---------------------------------------------------------------------------
#define ORC_CH 64
#define ORC_HD 128

int orc_chunked_step(int n, int hd, const float *q, const float *k, const float *v, const float *g_log,
                     const float *beta, float *state, float *out) {
    if (n < 1 || n > ORC_CH || hd < 1 || hd > ORC_HD) return -1;
    static float gcs[ORC_CH], gexp[ORC_CH], diff[ORC_CH];
    static float kk[ORC_CH][ORC_CH], A[ORC_CH][ORC_CH], kq[ORC_CH][ORC_CH];
    static float veff[ORC_CH][ORC_HD], kcd[ORC_CH][ORC_HD], vnew[ORC_CH][ORC_HD];
    static float inter[ORC_CH][ORC_HD], kgd[ORC_HD][ORC_HD];
    // running log-decay and its exponentials (chunked.c:311-320)
    float acc = 0.0f;
    for (int t = 0; t < n; t++) {
        acc += g_log[t];
        gcs[t] = acc;
        gexp[t] = expf(acc);
    }
    // kk[i][j] = (K_j . (K_i*beta_i)) * exp(gcs_i - gcs_j), j < i (chunked.c:340-358)
    for (int i = 0; i < n; i++)
        for (int j = 0; j < i; j++) {
            float s = 0.0f;
            for (int d = 0; d < hd; d++) s += k[j * hd + d] * (k[i * hd + d] * beta[i]);
            kk[i][j] = s * expf(gcs[i] - gcs[j]);
        }
    // forward substitution (I + kk) X = -kk, then A = X + I on and below the
    // diagonal (chunked.c:224-238, 364-386): column j, rows i > j, terms
    // t = j+1 .. i-1 in order
    for (int j = 0; j < n; j++) {
        A[j][j] = 1.0f;
        for (int i = j + 1; i < n; i++) {
            float s = 0.0f;
            for (int t = j + 1; t < i; t++) s += kk[i][t] * A[t][j];
            A[i][j] = -kk[i][j] - s;
        }
    }
    // V_eff = A (V*beta); k_cumdecay = A (K*beta*gexp) (chunked.c:391-426)
    for (int i = 0; i < n; i++)
        for (int e = 0; e < hd; e++) {
            float s = 0.0f, c = 0.0f;
            for (int j = 0; j <= i; j++) {
                if (A[i][j] != 0.0f) {
                    s += A[i][j] * (v[j * hd + e] * beta[j]);
                    c += A[i][j] * ((k[j * hd + e] * beta[j]) * gexp[j]);
                }
            }
            veff[i][e] = s;
            kcd[i][e] = c;
        }
    // kq[i][j] = (K_j . Q_i) * decay, j <= i, decay 1 on the diagonal (chunked.c:430-443)
    for (int i = 0; i < n; i++)
        for (int j = 0; j <= i; j++) {
            float s = 0.0f;
            for (int d = 0; d < hd; d++) s += k[j * hd + d] * q[i * hd + d];
            kq[i][j] = s * (i == j ? 1.0f : expf(gcs[i] - gcs[j]));
        }
    // attn_inter = (Q*gexp) S; v_new = V_eff - k_cumdecay S (chunked.c:445-484)
    for (int t = 0; t < n; t++)
        for (int e = 0; e < hd; e++) {
            float si = 0.0f, sp = 0.0f;
            for (int d = 0; d < hd; d++) {
                const float qg = q[t * hd + d] * gexp[t];
                if (qg != 0.0f) si += qg * state[d * hd + e];
                if (kcd[t][d] != 0.0f) sp += kcd[t][d] * state[d * hd + e];
            }
            inter[t][e] = si;
            vnew[t][e] = veff[t][e] - sp;
        }
    // out = attn_inter + kq v_new (chunked.c:486-501)
    for (int t = 0; t < n; t++)
        for (int e = 0; e < hd; e++) {
            float s = 0.0f;
            for (int u = 0; u <= t; u++) s += kq[t][u] * vnew[u][e];
            out[t * hd + e] = inter[t][e] + s;
        }
    // S = S * exp(gcs_last) + (K * exp(gcs_last - gcs))^T v_new (chunked.c:503-522)
    const float gl = gcs[n - 1], gle = expf(gl);
    for (int t = 0; t < n; t++) diff[t] = expf(gl - gcs[t]);
    for (int d = 0; d < hd; d++)
        for (int e = 0; e < hd; e++) {
            float s = 0.0f;
            for (int t = 0; t < n; t++) s += (k[t * hd + d] * diff[t]) * vnew[t][e];
            kgd[d][e] = s;
        }
    for (int d = 0; d < hd; d++)
        for (int e = 0; e < hd; e++) state[d * hd + e] = state[d * hd + e] * gle + kgd[d][e];
    return 0;
}

// ---- host C library expf / logf --------------------------------------------
// The reference evaluates expf/logf with the host C library (slm/qwen.c:464-470,
// slm/model.c:943, slm/tensor.c:315/491/1086, simd/simd.c:264-277,
// slm/sampler.c:105). Counts how many of vals[j] (a device evaluation of
// expf (fn 0) or logf (fn 1) at the float with bit pattern first + j) differ
// from the host's value; NaN results compare equal to any NaN. *first_bad
// gets the first differing bit pattern (unchanged if none).
static int orc_same_f32(float a, float b) {
    uint32_t ua, ub;
    memcpy(&ua, &a, 4);
    memcpy(&ub, &b, 4);
    return ua == ub || (a != a && b != b);
}

typedef struct {
    int fn;
    uint32_t first;
    int64_t j0, j1;
    const float *vals;
    int64_t mis, bad_j;
} orc_libm_part;

static void *orc_libm_worker(void *arg) {
    orc_libm_part *p = (orc_libm_part *)arg;
    p->mis = 0;
    p->bad_j = -1;
    for (int64_t j = p->j0; j < p->j1; j++) {
        uint32_t u = p->first + (uint32_t)j;
        float x;
        memcpy(&x, &u, 4);
        float want = p->fn == 0 ? expf(x) : logf(x);
        if (!orc_same_f32(want, p->vals[j])) {
            if (p->bad_j < 0) p->bad_j = j;
            p->mis++;
        }
    }
    return NULL;
}

int64_t orc_libm_mismatches(int fn, uint32_t first, int64_t n, const float *vals, uint32_t *first_bad) {
    enum { kMaxThreads = 64 };
    long nc = sysconf(_SC_NPROCESSORS_ONLN);
    int nt = nc < 1 ? 1 : nc > kMaxThreads ? kMaxThreads : (int)nc;
    if (n < 1 << 20) nt = 1;
    orc_libm_part parts[kMaxThreads];
    pthread_t th[kMaxThreads];
    for (int t = 0; t < nt; t++) {
        parts[t] = (orc_libm_part){fn, first, n * t / nt, n * (t + 1) / nt, vals, 0, -1};
        if (t > 0 && pthread_create(&th[t], NULL, orc_libm_worker, &parts[t]) != 0) orc_libm_worker(&parts[t]), th[t] = 0;
    }
    orc_libm_worker(&parts[0]);
    int64_t mis = 0, bad_j = -1;
    for (int t = 0; t < nt; t++) {
        if (t > 0 && th[t]) pthread_join(th[t], NULL);
        mis += parts[t].mis;
        if (bad_j < 0 && parts[t].bad_j >= 0) bad_j = parts[t].bad_j;
    }
    if (mis && first_bad) *first_bad = first + (uint32_t)bad_j;
    return mis;
}
