/* SPDX-License-Identifier: MIT
 *
 * qh_synth.h -- seeded synthetic inputs for the quantized matmul path.
 *
 * No reference counterpart: the reference runs on a real GGUF file. These
 * generators produce the seeded stand-ins its benchmark shapes call for
 * (random K-quant blocks, N(0,1)-shaped activations, N(0, s) weights), with
 * integer-only randomness so every machine produces identical bytes:
 *   - value i of stream `seed` is splitmix64 finalization of
 *     seed + (i+1) * 0x9E3779B97F4A7C15 (counter based, no state);
 *   - "normal" values are Irwin-Hall sums of twelve 24-bit uniforms minus
 *     6, exact in double precision, then scaled (variance 1, support +-6).
 * All functions are host-only, need no GPU and return 0 or QH_ERR_INVALID.
 */
#ifndef QH_SYNTH_H
#define QH_SYNTH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Value i of the counter-based stream `seed`. */
uint64_t qh_synth_u64(uint64_t seed, uint64_t i);

/* n fp32 values mean + std * z, z ~ Irwin-Hall(12) - 6. */
int qh_synth_normal(uint64_t seed, int64_t n, float mean, float std_dev, float *out);

/* n_blocks random blocks of GGUF type (Q4_K 12, Q5_K 13, Q6_K 14,
 * Q8_0 8): every byte uniform, then the fp16 scale fields (d, and dmin for
 * Q4_K/Q5_K) replaced by fp16 values uniform in [1e-3, 1e-2]. */
int qh_synth_blocks(int type, int64_t n_blocks, uint64_t seed, void *out);

/* Quantize fp32 weights [rows][k] into GGUF blocks of `type` (Q4_K, Q5_K,
 * Q6_K, Q8_0) with this library's own simple quantizer (the reference has
 * none; any bytes are valid blocks). Deterministic, host only. */
int qh_synth_quantize(int type, const float *w, int64_t rows, int64_t k, void *out);

#ifdef __cplusplus
}
#endif

#endif /* QH_SYNTH_H */
