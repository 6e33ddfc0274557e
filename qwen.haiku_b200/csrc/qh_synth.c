// SPDX-License-Identifier: MIT
//
// qh_synth.c -- seeded synthetic inputs (see include/qh_synth.h) and a
// simple deterministic K-quant weight quantizer for the synthetic model.
//
// The quantizer is this library's own and is only required to emit valid
// blocks: the reference ships no K-quant quantizer (it only dequantizes and
// dots, slm/tensor.c:800-1010), so parity needs identical bytes on both
// sides, not a particular quantization quality. Layout rules it writes are
// the inverse of the unpacking in simd/quants.h:215-224 and
// slm/tensor.c:800-1010.

#include <math.h>
#include <stdint.h>
#include <string.h>

#include "qh_backend.h"
#include "qh_formats.h"
#include "qh_synth.h"

uint64_t qh_synth_u64(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

int qh_synth_normal(uint64_t seed, int64_t n, float mean, float std_dev, float *out) {
    if (n < 0 || (n > 0 && !out)) return QH_ERR_INVALID;
    for (int64_t i = 0; i < n; i++) {
        // twelve 24-bit uniforms from four 64-bit draws (three per draw)
        int64_t s = 0;
        for (int d = 0; d < 4; d++) {
            uint64_t u = qh_synth_u64(seed, (uint64_t)i * 4 + (uint64_t)d);
            s += (int64_t)(u & 0xffffff) + (int64_t)((u >> 24) & 0xffffff) + (int64_t)(u >> 40);
        }
        const double z = (double)(s - 6 * (int64_t)(1 << 24)) / (double)(1 << 24);
        out[i] = (float)((double)mean + (double)std_dev * z);
    }
    return QH_OK;
}

static void put_f16(uint8_t *p, double v) {
    _Float16 h = (_Float16)(float)v;
    memcpy(p, &h, 2);
}

static float get_f16(const uint8_t *p) {
    _Float16 h;
    memcpy(&h, p, 2);
    return (float)h;
}

// Uniform in [1e-3, 1e-2] from one draw (53 random bits).
static double scale_draw(uint64_t seed, uint64_t i) {
    const double u = (double)(qh_synth_u64(seed ^ 0x5ca1ab1eull, i) >> 11) * (1.0 / 9007199254740992.0);
    return 1e-3 + u * 9e-3;
}

int qh_synth_blocks(int type, int64_t n_blocks, uint64_t seed, void *out) {
    const int64_t bb = qhf_block_bytes(type);
    if (bb == 0 || n_blocks < 0 || (n_blocks > 0 && !out)) return QH_ERR_INVALID;
    uint8_t *o = (uint8_t *)out;
    const int64_t total = n_blocks * bb;
    for (int64_t i = 0; i < total; i += 8) {
        uint64_t u = qh_synth_u64(seed, (uint64_t)(i / 8));
        for (int64_t b = 0; b < 8 && i + b < total; b++) o[i + b] = (uint8_t)(u >> (8 * b));
    }
    for (int64_t blk = 0; blk < n_blocks; blk++) {
        uint8_t *p = o + blk * bb;
        switch (type) {
            case QH_GGUF_Q4_K:
            case QH_GGUF_Q5_K:
                put_f16(p, scale_draw(seed, (uint64_t)blk * 2));
                put_f16(p + 2, scale_draw(seed, (uint64_t)blk * 2 + 1));
                break;
            case QH_GGUF_Q6_K: put_f16(p + 208, scale_draw(seed, (uint64_t)blk)); break;
            case QH_GGUF_Q8_0: put_f16(p, scale_draw(seed, (uint64_t)blk)); break;
            default: break;
        }
    }
    return QH_OK;
}

// ---------------------------------------------------------------------------
// Weight quantizer (synthetic model only)
// ---------------------------------------------------------------------------

static int clampi(long v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : (int)v); }

// Q4_K / Q5_K: asymmetric 32-wide sub-blocks, w ~ d*sc*q - dmin*m.
static void quant_kq_asym(const float *w, uint8_t *blk, int nbits) {
    const int qmax = (1 << nbits) - 1;
    double scale[8], mn[8];
    double max_scale = 0.0, max_mn = 0.0;
    for (int j = 0; j < 8; j++) {
        double lo = 0.0, hi = 0.0;
        for (int l = 0; l < 32; l++) {
            const double v = w[32 * j + l];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        scale[j] = (hi - lo) / qmax;
        mn[j] = -lo;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (mn[j] > max_mn) max_mn = mn[j];
    }
    put_f16(blk, max_scale / 63.0);
    put_f16(blk + 2, max_mn / 63.0);
    const double d = get_f16(blk), dmin = get_f16(blk + 2);
    int sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = d > 0 ? clampi(lround(scale[j] / d), 0, 63) : 0;
        m[j] = dmin > 0 ? clampi(lround(mn[j] / dmin), 0, 63) : 0;
    }
    uint8_t *s12 = blk + 4;
    for (int j = 0; j < 4; j++) {
        s12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s12[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s12[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
        const double ds = d * sc[j], dm = dmin * m[j];
        for (int l = 0; l < 32; l++)
            q[32 * j + l] = (uint8_t)(ds > 0 ? clampi(lround((w[32 * j + l] + dm) / ds), 0, qmax) : 0);
    }
    uint8_t *qs = blk + (nbits == 4 ? 16 : 48);
    if (nbits == 5) memset(blk + 16, 0, 32);
    for (int c = 0; c < 4; c++) {
        for (int l = 0; l < 32; l++) {
            const uint8_t lo = q[64 * c + l], hi = q[64 * c + 32 + l];
            qs[32 * c + l] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            if (nbits == 5) {
                blk[16 + l] |= (uint8_t)(((lo >> 4) & 1) << (2 * c));
                blk[16 + l] |= (uint8_t)(((hi >> 4) & 1) << (2 * c + 1));
            }
        }
    }
}

// Q6_K: symmetric 16-wide sub-blocks, w ~ d*sc*(q-32), sc int8.
static void quant_q6k(const float *w, uint8_t *blk) {
    double scale[16], max_scale = 0.0;
    for (int j = 0; j < 16; j++) {
        double amax = 0.0;
        for (int l = 0; l < 16; l++) {
            const double a = fabs((double)w[16 * j + l]);
            if (a > amax) amax = a;
        }
        scale[j] = amax / 31.0;
        if (scale[j] > max_scale) max_scale = scale[j];
    }
    put_f16(blk + 208, max_scale / 127.0);
    const double d = get_f16(blk + 208);
    int8_t *sc = (int8_t *)(blk + 192);
    int q[256];
    for (int j = 0; j < 16; j++) {
        sc[j] = (int8_t)(d > 0 ? clampi(lround(scale[j] / d), 0, 127) : 0);
        const double ds = d * sc[j];
        for (int l = 0; l < 16; l++)
            q[16 * j + l] = ds > 0 ? clampi(lround(w[16 * j + l] / ds), -32, 31) + 32 : 32;
    }
    memset(blk, 0, 192);
    for (int p = 0; p < 256; p++) {
        const int h = p / 128, r = (p / 32) & 3, l = p & 31;
        uint8_t *lo = &blk[64 * h + 32 * (r & 1) + l];
        *lo |= (uint8_t)((r >> 1) ? ((q[p] & 15) << 4) : (q[p] & 15));
        blk[128 + 32 * h + l] |= (uint8_t)(((q[p] >> 4) & 3) << (2 * r));
    }
}

static void quant_q8_0(const float *w, uint8_t *blk) {
    double amax = 0.0;
    for (int l = 0; l < 32; l++) {
        const double a = fabs((double)w[l]);
        if (a > amax) amax = a;
    }
    put_f16(blk, amax / 127.0);
    const double d = get_f16(blk);
    for (int l = 0; l < 32; l++)
        blk[2 + l] = (uint8_t)(int8_t)(d > 0 ? clampi(lround(w[l] / d), -127, 127) : 0);
}

int qh_synth_quantize(int type, const float *w, int64_t rows, int64_t k, void *out) {
    const int64_t bb = qhf_block_bytes(type), bw = qhf_block_weights(type);
    if (bb == 0 || !w || !out || rows < 0 || k <= 0 || k % bw) return QH_ERR_INVALID;
    uint8_t *o = (uint8_t *)out;
    const int64_t nb = k / bw;
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t b = 0; b < nb; b++) {
            const float *src = w + r * k + b * bw;
            uint8_t *blk = o + (r * nb + b) * bb;
            switch (type) {
                case QH_GGUF_Q4_K: quant_kq_asym(src, blk, 4); break;
                case QH_GGUF_Q5_K: quant_kq_asym(src, blk, 5); break;
                case QH_GGUF_Q6_K: quant_q6k(src, blk); break;
                default: quant_q8_0(src, blk); break;
            }
        }
    }
    return QH_OK;
}
