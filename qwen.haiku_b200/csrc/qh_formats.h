// SPDX-License-Identifier: MIT
//
// qh_formats.h -- GGUF quantized block layouts and the device-side activation
// layouts, shared by the CUDA kernels and the C host layer.
//
// Weight blocks keep the GGUF byte layouts bit-for-bit so a GGUF tensor (or
// the reference's mmapped weights) can be uploaded unchanged
// (reference: simd/quants.h:94-130, slm/gguf.c:52-59). Offsets are spelled
// out as constants; no packed structs are used on the device.
//
//   Q4_K  144 B / 256 weights: [0] fp16 d  [2] fp16 dmin  [4] u8 scales[12]
//                              [16] u8 qs[128]   (two 4-bit weights per byte)
//   Q5_K  176 B / 256 weights: [0] fp16 d  [2] fp16 dmin  [4] u8 scales[12]
//                              [16] u8 qh[32] (5th bits)  [48] u8 qs[128]
//   Q6_K  210 B / 256 weights: [0] u8 ql[128]  [128] u8 qh[64]
//                              [192] i8 scales[16]  [208] fp16 d
//   Q8_0   34 B /  32 weights: [0] fp16 d  [2] i8 qs[32]
//
// A weight matrix of shape (K in, N out) is N rows; row j is K/256 (K/32
// for Q8_0) consecutive blocks, rows back to back (slm/tensor.c:846-850).
//
// Activations are quantized on the device into "split" planes instead of the
// reference's 292-byte q8k_block array (which is internal arena scratch in
// the reference, slm/tensor.c:836-839): the same numbers, laid out so that
// int8 quants are 16-byte aligned for vector loads and directly usable as a
// K-major int8 GEMM operand.
//
//   Q8_K split, n_tok rows of K (nb = K/256 blocks per row):
//     qs    int8  [n_tok][K]          at offset 0
//     d     f32   [n_tok][nb]         at qhf_q8k_d_offset(K, n_tok)
//     bsums int16 [n_tok][nb][16]     at qhf_q8k_bsums_offset(K, n_tok)
//   Q8_0 split (for Q8_0 weights), nb0 = K/32:
//     qs    int8  [n_tok][K]          at offset 0
//     d     fp16  [n_tok][nb0]        at qhf_q8_0_d_offset(K, n_tok)

#ifndef QH_FORMATS_H
#define QH_FORMATS_H

#include <stdint.h>
#include <stddef.h>

#define QH_QK 256
#define QH_QK8_0 32

#define QH_Q4K_BYTES 144
#define QH_Q5K_BYTES 176
#define QH_Q6K_BYTES 210
#define QH_Q8_0_BYTES 34

// GGUF tensor type ids (slm/gguf.c:52-59).
#define QH_GGUF_F32 0
#define QH_GGUF_F16 1
#define QH_GGUF_Q8_0 8
#define QH_GGUF_Q4_K 12
#define QH_GGUF_Q5_K 13
#define QH_GGUF_Q6_K 14

#ifdef __CUDACC__
#define QH_HD __host__ __device__
#else
#define QH_HD
#endif

static inline QH_HD int64_t qhf_align16(int64_t v) { return (v + 15) & ~(int64_t)15; }

// Bytes of one weight block and weights per block for a GGUF type; 0 if the
// type has no quantized block layout here.
static inline QH_HD int64_t qhf_block_bytes(int type) {
    return type == QH_GGUF_Q4_K ? QH_Q4K_BYTES
         : type == QH_GGUF_Q5_K ? QH_Q5K_BYTES
         : type == QH_GGUF_Q6_K ? QH_Q6K_BYTES
         : type == QH_GGUF_Q8_0 ? QH_Q8_0_BYTES : 0;
}
static inline QH_HD int64_t qhf_block_weights(int type) {
    return type == QH_GGUF_Q8_0 ? QH_QK8_0 : QH_QK;
}
static inline QH_HD int64_t qhf_row_bytes(int type, int64_t k) {
    return (k / qhf_block_weights(type)) * qhf_block_bytes(type);
}

// Q8_K split activation layout. The per-token scale row is padded to a
// multiple of 4 floats (16 bytes) so every plane of a row range is a
// 16-byte-aligned contiguous span (bulk-copyable).
static inline QH_HD int64_t qhf_q8k_d_stride(int64_t k) { return ((k / QH_QK) + 3) & ~(int64_t)3; }
static inline QH_HD int64_t qhf_q8k_d_offset(int64_t k, int64_t n_tok) {
    return qhf_align16(k * n_tok);
}
static inline QH_HD int64_t qhf_q8k_bsums_offset(int64_t k, int64_t n_tok) {
    return qhf_align16(qhf_q8k_d_offset(k, n_tok) + qhf_q8k_d_stride(k) * n_tok * 4);
}
static inline QH_HD int64_t qhf_q8k_total_bytes(int64_t k, int64_t n_tok) {
    return qhf_align16(qhf_q8k_bsums_offset(k, n_tok) + (k / 16) * n_tok * 2);
}

// Q8_0 split activation layout; fp16 scale rows padded to 8 halves (16 bytes).
static inline QH_HD int64_t qhf_q8_0_d_stride(int64_t k) { return ((k / QH_QK8_0) + 7) & ~(int64_t)7; }
static inline QH_HD int64_t qhf_q8_0_d_offset(int64_t k, int64_t n_tok) {
    return qhf_align16(k * n_tok);
}
static inline QH_HD int64_t qhf_q8_0_total_bytes(int64_t k, int64_t n_tok) {
    return qhf_align16(qhf_q8_0_d_offset(k, n_tok) + qhf_q8_0_d_stride(k) * n_tok * 2);
}

// Q8_K tiled activation layout read by the tensor-core GEMM. Per 64-token
// tile and 256-value block, one contiguous "tile block" of
// QH_Q8KT_BLOCK_BYTES:
//   [16384] quants in the no-swizzle K-major operand layout
//           [16 chunks of 16 values][64 tokens][16 bytes];
//   [  256] the 64 tokens' fp32 scales d;
//   [ 2048] the min operand: 128 rows x 16 bytes; row t < 64 holds, for
//           sub-blocks j = 0..7, S_j(t) mod 128 and row 64 + t holds
//           floor(S_j(t) / 128), where S_j = bsums[2j] + bsums[2j+1] (the
//           sum of the 32 quants of sub-block j); bytes 8..15 are zero.
// Tokens past n_tok in the last tile are padding (never read as results).
#define QH_Q8KT_TILE 64
#define QH_Q8KT_QS_BYTES (QH_Q8KT_TILE * QH_QK)
#define QH_Q8KT_D_OFF QH_Q8KT_QS_BYTES
#define QH_Q8KT_MIN_OFF (QH_Q8KT_QS_BYTES + QH_Q8KT_TILE * 4)
#define QH_Q8KT_BLOCK_BYTES (QH_Q8KT_MIN_OFF + 2 * QH_Q8KT_TILE * 16)
static inline QH_HD int64_t qhf_q8kt_tiles(int64_t n_tok) { return (n_tok + QH_Q8KT_TILE - 1) / QH_Q8KT_TILE; }
static inline QH_HD int64_t qhf_q8kt_total_bytes(int64_t k, int64_t n_tok) {
    return qhf_q8kt_tiles(n_tok) * (k / QH_QK) * QH_Q8KT_BLOCK_BYTES;
}

#endif  // QH_FORMATS_H
