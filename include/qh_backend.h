/* SPDX-License-Identifier: MIT
 *
 * qh_backend.h -- C-ABI of the B200 (sm_100a) backend for qwen.haiku's
 * quantized matmul path.
 *
 * This header is the drop-in boundary. The reference computes every
 * projection of the model through
 *     matmul_dispatch(w, x)                       slm/model.c:220-264
 * which switches on the GGUF type of `w` and calls one of
 *     tensor_matmul_q4k_f32(w_blocks, out_f, k, x)  slm/tensor.c:827-853
 *     tensor_matmul_q5k_f32(...)                    slm/tensor.c:898-919
 *     tensor_matmul_q8_0_f32(...)                   slm/tensor.c:952-981
 *     tensor_matmul_q6k_f32(...)                    slm/tensor.c:1012-1033
 * each of which quantizes every activation row to Q8_K (Q8_0 for Q8_0
 * weights) and takes one SIMD row dot per output feature
 *     simd_q{4k,5k,6k}_row_dot_q8k / simd_q8_0_dot_q8_0   simd/simd.c:236-250.
 * The entry points below replace those calls one for one on device memory.
 *
 * Conventions
 *   - Plain C types only. Pointers named d_* are device pointers (any
 *     allocation visible to the current CUDA device); h_* are host pointers.
 *   - `stream` is a cudaStream_t passed as void*; NULL is the legacy default
 *     stream. Every compute call is asynchronous on that stream.
 *   - Weights stay in their GGUF block layout (simd/quants.h:94-130): a
 *     (k, out_f) weight is out_f rows of k/256 (Q8_0: k/32) blocks, rows
 *     back to back. The weight pointer must be 16-byte aligned.
 *   - x is fp32 [n_tok][k] (the reference's x->ne[0] == k), out is fp32
 *     [n_tok][out_f]; both caller-allocated.
 *   - Every call returns QH_OK (0) or a negative QH_ERR_* status and never
 *     aborts (the reference abort()s on an unsupported type,
 *     slm/model.c:259-261; here that is QH_ERR_UNSUPPORTED). The message of
 *     the last failure on the calling thread is qh_last_error().
 *   - Results are bit-identical to the reference's CPU path built with gcc
 *     -std=c17 (scalar / AVX2 / AVX-VNNI tiers agree on these formats).
 */
#ifndef QH_BACKEND_H
#define QH_BACKEND_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define QH_OK               0
#define QH_ERR_INVALID     -1  /* bad argument (null pointer, size, shape) */
#define QH_ERR_UNSUPPORTED -2  /* weight type without a kernel here */
#define QH_ERR_CUDA        -3  /* CUDA runtime error (see qh_last_error) */
#define QH_ERR_ALIGN       -4  /* pointer alignment requirement not met */
#define QH_ERR_WORKSPACE   -5  /* workspace missing or too small */
#define QH_ERR_DEVICE      -6  /* a kernel reported a device-side error */

/* GGUF tensor type ids (slm/gguf.c:52-59). */
#define QH_TYPE_F32   0
#define QH_TYPE_Q8_0  8
#define QH_TYPE_Q4_K 12
#define QH_TYPE_Q5_K 13
#define QH_TYPE_Q6_K 14

/* ------------------------------------------------------------------------
 * Runtime plumbing
 * ---------------------------------------------------------------------- */

/* Library version string. */
const char *qh_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char *qh_last_error(void);

/* Number of visible CUDA devices (0 when none); never fails. */
int qh_device_count(void);

/* Make `device` current for the calling thread. */
int qh_set_device(int device);

/* Device memory and copies (thin wrappers over the CUDA runtime). */
int qh_malloc(void **d_ptr, size_t bytes);
int qh_free(void *d_ptr);
int qh_memcpy_h2d(void *d_dst, const void *h_src, size_t bytes, void *stream);
int qh_memcpy_d2h(void *h_dst, const void *d_src, size_t bytes, void *stream);
int qh_memset(void *d_dst, int value, size_t bytes, void *stream);
int qh_stream_sync(void *stream);

/* Reads and clears the device error word of the current device (set by a
 * kernel whose bounded wait ran out). QH_OK when clear, QH_ERR_DEVICE when
 * a kernel reported an error (the code is returned in *code if non-null). */
int qh_check_device_error(int *code);

/* ------------------------------------------------------------------------
 * Activation quantizers (slm/tensor.c:683-720 and 930-950)
 *
 * Quantized activations use split planes (qs int8[n_tok][k], then per-block
 * scales, then Q8_K bsums) instead of the reference's q8k_block array; the
 * numbers are identical. Byte sizes from qh_q8k_bytes / qh_q8_0_bytes.
 * ---------------------------------------------------------------------- */
int64_t qh_q8k_bytes(int64_t k, int64_t n_tok);
int64_t qh_q8_0_bytes(int64_t k, int64_t n_tok);
/* Byte offsets of the scale and bsum planes inside a Q8_K split buffer. */
int64_t qh_q8k_d_offset(int64_t k, int64_t n_tok);
int64_t qh_q8k_bsums_offset(int64_t k, int64_t n_tok);
/* Byte offset of the fp16 scale plane inside a Q8_0 split buffer. */
int64_t qh_q8_0_d_offset(int64_t k, int64_t n_tok);

/* quantize_row_q8_K (slm/tensor.c:683) over n_tok rows; k % 256 == 0. */
int qh_quantize_q8k(const float *d_x, int64_t k, int64_t n_tok, void *d_q8k, void *stream);
/* tensor_quantize_row_q8_0 (slm/tensor.c:930) over n_tok rows; k % 32 == 0. */
int qh_quantize_q8_0(const float *d_x, int64_t k, int64_t n_tok, void *d_q8_0, void *stream);

/* ------------------------------------------------------------------------
 * Matmul entry points
 * ---------------------------------------------------------------------- */

/* Device workspace bytes a matmul of this type/shape needs (the quantized
 * activation rows the reference takes from its arena, slm/tensor.c:836). */
int64_t qh_matmul_workspace_bytes(int type, int64_t k, int64_t n_tok);

/* tensor_matmul_q4k_f32 (slm/tensor.c:827): out = W x, W Q4_K (k, out_f). */
int qh_matmul_q4k_f32(const void *d_w, int64_t out_f, int64_t k, const float *d_x,
                      int64_t n_tok, float *d_out, void *d_work, int64_t work_bytes,
                      void *stream);
/* tensor_matmul_q5k_f32 (slm/tensor.c:898). */
int qh_matmul_q5k_f32(const void *d_w, int64_t out_f, int64_t k, const float *d_x,
                      int64_t n_tok, float *d_out, void *d_work, int64_t work_bytes,
                      void *stream);
/* tensor_matmul_q6k_f32 (slm/tensor.c:1012). */
int qh_matmul_q6k_f32(const void *d_w, int64_t out_f, int64_t k, const float *d_x,
                      int64_t n_tok, float *d_out, void *d_work, int64_t work_bytes,
                      void *stream);
/* tensor_matmul_q8_0_f32 (slm/tensor.c:952); activations go through the
 * Q8_0 quantizer (roundf), not Q8_K. */
int qh_matmul_q8_0_f32(const void *d_w, int64_t out_f, int64_t k, const float *d_x,
                       int64_t n_tok, float *d_out, void *d_work, int64_t work_bytes,
                       void *stream);

/* tensor_matmul_f32 (slm/tensor.c:517), the F32 case of matmul_dispatch
 * (slm/model.c:227): out[t][j] = sum_i w[j][i] * x[t][i] with one float
 * multiply and one float add per i in index order, as the reference's loop.
 * Weights fp32 [out_f][k] (GGUF shape (k, out_f)); no workspace. */
int qh_matmul_f32(const float *d_w, int64_t out_f, int64_t k, const float *d_x, int64_t n_tok, float *d_out,
                  void *stream);

/* No counterpart in the reference (its CPU matmuls take their scratch from
 * the context arena). Same computation and results as qh_matmul_q4k_f32,
 * for callers that are not allowed to allocate device memory -- e.g. a host
 * that reserves all device memory in its own pool at start-up, or a service
 * that forbids cudaMalloc after initialization because an allocation can
 * synchronize the device. It needs no workspace: the quantized activation
 * rows go to a fixed 128 KiB device array inside this library (every GPU
 * that loads the library holds it until exit); shapes needing more than
 * 131,072 - 256 bytes of activation scratch (qh_q8k_bytes(k, n_tok)) are
 * rejected with QH_ERR_WORKSPACE. Calls allocate nothing. All calls share
 * the array, so calls whose work overlaps on the GPU race: serialize them on
 * one stream. The first call on each device (with that device current)
 * looks up the array's device address; make it before any stream capture. */
int qh_matmul_q4k_f32_noalloc(const void *d_w, int64_t out_f, int64_t k, const float *d_x,
                              int64_t n_tok, float *d_out, void *stream);

/* matmul_dispatch (slm/model.c:220): dispatch on the GGUF weight type with
 * the GGUF shape order (k = shape[0], out_f = shape[1]): F32, Q8_0, Q4_K,
 * Q5_K, Q6_K. F32 needs no workspace (qh_matmul_workspace_bytes returns 0);
 * any other type returns QH_ERR_UNSUPPORTED where the reference aborts
 * (slm/model.c:259-261). */
int qh_matmul(int type, const void *d_w, int64_t k, int64_t out_f, const float *d_x,
              int64_t n_tok, float *d_out, void *d_work, int64_t work_bytes, void *stream);

/* Same as qh_matmul with the activations already quantized by
 * qh_quantize_q8k (qh_quantize_q8_0 for Q8_0), so one quantization can feed
 * several projections of the same input (q/k/v, gate/up). */
int qh_matmul_preq(int type, const void *d_w, int64_t k, int64_t out_f, const void *d_xq,
                   int64_t n_tok, float *d_out, void *stream);

/* ------------------------------------------------------------------------
 * Grouped matvec plans: many independent (weight, quantized activation,
 * output) jobs of one weight type in ONE persistent launch. A decode step
 * issues its projections this way (e.g. q, k, v of one layer). No host
 * reference counterpart: the reference calls tensor_matmul_* once per
 * weight. Plan creation allocates a small device job table once; running a
 * plan allocates nothing and can be captured in a CUDA graph.
 * ---------------------------------------------------------------------- */
typedef struct qh_matvec_job {
    const void *d_w;   /* GGUF blocks, (k, out_f), 16-byte aligned */
    const void *d_xq;  /* split Q8_K (Q8_0) activation buffer of xq_rows rows of k */
    float *d_out;      /* fp32 [n_tok][out_f] */
    int64_t k;
    int64_t out_f;
    int64_t xq_rows;   /* rows the split buffer was quantized for (0: n_tok) */
    int64_t xq_row0;   /* first of the job's n_tok rows inside that buffer */
} qh_matvec_job;

typedef struct qh_matvec_plan_s *qh_matvec_plan;

/* n_tok in [1, 8]. */
int qh_matvec_plan_create(int type, const qh_matvec_job *h_jobs, int n_jobs, int64_t n_tok,
                          qh_matvec_plan *out_plan);
/* Fused input: instead of reading the jobs' shared Q8_K activation (d_xq of
 * the jobs), every CTA of the launch forms it itself from fp32 rows
 * [n_tok][k] -- the step that otherwise runs as its own kernel just before
 * the projections (one launch fewer, no activation round trip through
 * memory), with the same arithmetic bit for bit:
 *   QH_FUSE_RMSNORM  residual add + RMSNorm (tensor_add + tensor_rms_norm,
 *                    slm/tensor.c:285, 348-369): rows d_a (+ d_b when
 *                    given), weight d_w, eps; with d_b the sum h = a + b is
 *                    also written to d_h_out (the updated residual stream);
 *   QH_FUSE_SWIGLU   silu(d_a) * d_b (slm/qwen.c:952-955);
 *   QH_FUSE_QUANT    d_a as is;
 *   0                back to d_xq.
 * All jobs must share k (<= 4096 for RMSNorm); K-quant plans only. The
 * pointers are captured by the plan: qh_matvec_plan_run launches with them.
 * The outputs equal those of quantizing first (qh_rmsnorm_q8k,
 * qh_swiglu_q8k, qh_quantize_q8k) and running the plan on that activation. */
#define QH_FUSE_RMSNORM 1
#define QH_FUSE_SWIGLU 2
#define QH_FUSE_QUANT 3
int qh_matvec_plan_fuse_input(qh_matvec_plan plan, int mode, const float *d_a, const float *d_b, const float *d_w,
                              float eps, float *d_h_out);
/* Output tail: after the plan's matvecs, the launch's last CTA to finish
 * forms the next layer's Q8_K input (split layout, qh_q8k_bytes(k, n_tok)
 * bytes at d_xq) from fp32 rows [n_tok][k] -- typically this plan's own
 * outputs -- with the same modes and operations as qh_matvec_plan_fuse_input
 * (QH_FUSE_RMSNORM: h_out = a + b, RMSNorm with w and eps, as qh_rmsnorm_q8k;
 * QH_FUSE_SWIGLU: silu(a) * b, as qh_swiglu_q8k; QH_FUSE_QUANT: a, as
 * qh_quantize_q8k; 0 removes the tail). It replaces the separate
 * normalization / activation kernel between two projections of the
 * reference's step (slm/qwen.c:939-957, slm/model.c:949 to the next
 * layer's tensor_rms_norm), bit for bit. Allocates a 4-byte arrival counter
 * on the first call; launches of one plan must not overlap. */
int qh_matvec_plan_fuse_output(qh_matvec_plan plan, int mode, int64_t k, const float *d_a, const float *d_b,
                               const float *d_w, float eps, float *d_h_out, void *d_xq);
int qh_matvec_plan_run(qh_matvec_plan plan, void *stream);
/* Rows per tile, pipeline stages, grid size and shared memory chosen. */
int qh_matvec_plan_info(qh_matvec_plan plan, int *rows_per_tile, int *n_stages, int *grid,
                        int *smem_bytes);
int qh_matvec_plan_destroy(qh_matvec_plan plan);

/* Failure-detection test hook (no reference counterpart): the plan's next
 * runs leave out every copy of tile `tile` (-1: none), so the consumers'
 * bounded wait for that stage runs out after wait_limit polls (0: the
 * kernels' default limit, seconds) -- the path a lost copy or a stalled
 * producer takes: the CTA records the timeout in the device error word,
 * stops, waits (bounded) for its own copies in flight and returns, and
 * qh_check_device_error then reports QH_ERR_DEVICE. Nothing faults and
 * nothing is left in flight; the outputs of that launch are not defined. */
int qh_matvec_plan_test_timeout(qh_matvec_plan plan, int32_t tile, uint32_t wait_limit);

/* ------------------------------------------------------------------------
 * Tensor-core matmul for many tokens (prefill, batched decode): the same
 * results as tensor_matmul_{q4k,q5k,q6k}_f32 (slm/tensor.c:827-853, 898-919,
 * 1012-1033) with n tokens, computed by tcgen05 int8 MMAs on sm_100a. The
 * weights are read once per 64-token tile instead of once per token.
 * Q4_K, Q5_K and Q6_K; other types return QH_ERR_UNSUPPORTED.
 *
 * Formats:
 *   tiled weights  -- the GGUF blocks reordered as [row tile of 128][block]
 *                     [128 rows][block bytes padded to 16: 144, 176, 224]
 *                     (rows past out_f and padding zero):
 *                     qh_gemm_weight_bytes bytes, written by
 *                     qh_gemm_pack_weights from the GGUF (k, out_f) blocks.
 *   tiled Q8_K     -- the reference's quantize_row_q8_K per token
 *                     (slm/tensor.c:683-720); per (64-token tile, block)
 *                     18,688 bytes: the quants as the MMA operand
 *                     [16 chunks][64 tokens][16], the 64 fp32 scales, and
 *                     the sub-block sums S_j as two int8 operand rows per
 *                     token (S_j mod 128, floor(S_j / 128));
 *                     qh_q8kt_bytes bytes, written by qh_quantize_q8kt.
 * ---------------------------------------------------------------------- */
#define QH_Q8KT_TILE_TOKENS 64  /* tokens per tile of the tiled Q8_K layout */
int64_t qh_gemm_weight_bytes(int type, int64_t k, int64_t out_f);
int qh_gemm_pack_weights(int type, const void *d_w, int64_t k, int64_t out_f, void *d_wt, void *stream);
int64_t qh_q8kt_bytes(int64_t k, int64_t n_tok);
int qh_quantize_q8kt(const float *d_x, int64_t k, int64_t n_tok, void *d_q8kt, void *stream);

/* One output of a grouped GEMM: d_out[t * ld_out + j] = row j of the tiled
 * weights d_wt dotted with token t, for j < out_f, t < n_tok. */
typedef struct qh_gemm_job {
    const void *d_wt;
    int64_t out_f;
    float *d_out;
    int64_t ld_out;
} qh_gemm_job;

/* Up to 8 jobs of one type sharing the tiled activations (k, n_tok) in one
 * persistent launch; asynchronous on `stream`, allocates nothing. With a
 * scratch of at least qh_gemm_scratch_bytes (its first 4 KB, the arrival
 * counters, zero-filled before the first use; every call leaves them at
 * zero, so one scratch serves calls of any shape), launches with few output
 * tiles split each tile's super-blocks over several CTAs and add the
 * per-block terms in block order at the end (same results); d_scratch may
 * be NULL. Calls sharing a scratch must not overlap on the GPU. */
int64_t qh_gemm_scratch_bytes(const qh_gemm_job *jobs, int n_jobs, int64_t k, int64_t n_tok);
#define QH_GEMM_WEIGHTS_READY 1 /* flags: the tiled weights were complete before the previous
                                   kernel on the stream started (e.g. packed, then synchronized):
                                   the kernel streams them in while that kernel finishes */
#define QH_GEMM_EXPANDED 2      /* flags: jobs[].d_wt are expanded weights (qh_gemm_expand_weights):
                                   the kernel streams the MMA operands directly, no expansion */
int qh_gemm(int type, const qh_gemm_job *jobs, int n_jobs, int64_t k, const void *d_q8kt, int64_t n_tok,
            void *d_scratch, int64_t scratch_bytes, int32_t flags, void *stream);

/* Expanded weights: the tiled weights (qh_gemm_pack_weights) turned once
 * into the tensor-core operand image of every 128-row tile and super-block
 * -- the int8 planes whose dots with the Q8_K activations are the
 * reference's block integers (hi/lo planes of scale * weight, the min row
 * for Q4_K/Q5_K), plus the rows' fp16 d/dmin as fp32 -- so a qh_gemm with
 * QH_GEMM_EXPANDED only streams and multiplies: the form for decoding many
 * sequences, where each weight is used by one 64-token tile per step.
 * 2.09 (Q4_K/Q5_K) or 2.03 (Q6_K) bytes per weight; bit-identical results. */
int64_t qh_gemm_expanded_bytes(int type, int64_t k, int64_t out_f);
int qh_gemm_expand_weights(int type, const void *d_wt, int64_t k, int64_t out_f, void *d_we, void *stream);

/* One-call form of tensor_matmul_*_f32 for n_tok tokens: packs the weights
 * and quantizes the activations into d_work (qh_matmul_gemm_workspace_bytes)
 * and runs qh_gemm. d_out fp32 [n_tok][out_f]. */
int64_t qh_matmul_gemm_workspace_bytes(int type, int64_t k, int64_t out_f, int64_t n_tok);
int qh_matmul_gemm(int type, const void *d_w, int64_t k, int64_t out_f, const float *d_x, int64_t n_tok,
                   float *d_out, void *d_work, int64_t work_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* QH_BACKEND_H */
