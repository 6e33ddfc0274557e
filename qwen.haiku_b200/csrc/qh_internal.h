// SPDX-License-Identifier: MIT
//
// qh_internal.h -- launch-side interfaces between the C-ABI layer
// (qh_api.cu) and the kernel files. Not installed; C++ linkage.

#ifndef QH_INTERNAL_H
#define QH_INTERNAL_H

#include <cuda_runtime.h>
#include <stdint.h>

#include "qh_formats.h"

namespace qh {

// One independent matvec (or n_tok-token matmul) in a grouped launch.
// Activation pointers address the split layouts of qh_formats.h for the
// job's own K: xqs int8 [n_tok][K]; xd f32 [n_tok][K/256] (Q8_K) or fp16
// bits [n_tok][K/32] (Q8_0); xbs int16 [n_tok][K/256][16] (Q8_K only).
struct GemvJob {
    const uint8_t *w;
    const int8_t *xqs;
    const void *xd;
    const int16_t *xbs;
    float *out;
    int32_t n_rows;      // N, output features
    int32_t nb;          // blocks per row
    int32_t row_bytes;   // nb * block bytes
    int32_t k;           // K, input features
    int32_t d_stride;    // scale-plane elements per token row (f32 for Q8_K, fp16 for Q8_0)
    int32_t box_blocks;  // blocks per staged row segment (filled by the planner)
    int32_t box_pitch;   // shared-memory pitch of a staged row segment, bytes (planner)
    int32_t tile_begin;  // first global tile index of this job (filled by the planner)
    int32_t n_tiles;     // tiles of this job (filled by the planner)
};

constexpr int kGemvInlineJobs = 8;
constexpr int kGemvMaxStages = 16;

struct GemvParams {
    int32_t n_jobs;
    int32_t total_tiles;
    int32_t rows_per_tile;
    int32_t n_stages;
    int32_t stage_bytes;
    int32_t n_tok;
    int32_t x_offset;      // byte offset of the staged activation planes inside a stage
    int32_t split;         // one 8-row tile per CTA: the tile's blocks spread over the consumer warps
    int32_t terms_off;     // split: byte offset of the terms area from the stage ring base
    // Fused input (xform != 0): every CTA forms the jobs' shared Q8_K
    // activation itself from fp32 rows into a fixed shared-memory area at
    // x_fixed (the same split-plane layout as a staged one) instead of
    // copying it per stage:
    //   1 residual + RMSNorm: a = h, b = branch output (or null), w = norm
    //     weight, h_out = h + b (written by CTA 0 when b is given);
    //   2 SwiGLU: a = gate, b = up;   3 plain quantization of a.
    int32_t xform;
    int32_t x_fixed;
    int32_t xk;            // K of the fused input (every job's k)
    float eps;
    const float *xa, *xb, *xw;
    float *xh_out;
    const GemvJob *table;  // device copy of all jobs when n_jobs > kGemvInlineJobs
    // Output tail (tform != 0): after its matvecs the launch's last CTA
    // (ticket counter) forms a Q8_K row set in the split layout at txq from
    // fp32 rows of tk values, with the operations of xform's modes:
    // 1 residual + RMSNorm (ta = h, tb = branch or null, tw = weight, th_out =
    // h + b), 2 SwiGLU (ta = gate, tb = up), 3 plain quantization of ta.
    int32_t tform;
    int32_t tk;
    float teps;
    const float *ta, *tb, *tw;
    float *th_out;
    uint8_t *txq;
    unsigned *ticket;      // zero between launches
    int *err_flag;         // device error word
    // Failure-detection test hook (qh_matvec_plan_test_timeout): tile
    // test_withhold - 1 gets no copies (0: none), and bounded waits poll at
    // most wait_limit times (0: kWaitLimit).
    int32_t test_withhold;
    uint32_t wait_limit;
    GemvJob jobs[kGemvInlineJobs];
};

// Launch geometry chosen by the planner.
struct GemvGeometry {
    int grid;
    int smem_bytes;
};

// Fills tile_begin/n_tiles/box fields of `jobs`, the tiling fields of `p`
// and the launch geometry. All jobs share `type`; returns
// cudaErrorInvalidValue if a row is too long to stage. `sm_count` is the
// device's multiprocessor count.
cudaError_t gemv_plan(int type, GemvJob *jobs, int n_jobs, int n_tok, int sm_count,
                      GemvParams *p, GemvGeometry *g, int xform = 0);

// Launches the grouped GEMV kernel for `type`; p.n_tok in [1, 8].
cudaError_t gemv_launch(int type, const GemvParams &p, const GemvGeometry &g,
                        cudaStream_t stream);

// Activation quantizers: x fp32 [n_tok][k] -> split layouts.
cudaError_t quantize_q8k_launch(const float *x, int64_t k, int64_t n_tok, void *q8k,
                                cudaStream_t stream);
cudaError_t quantize_q8_0_launch(const float *x, int64_t k, int64_t n_tok, void *q8_0,
                                 cudaStream_t stream);

// Launch with programmatic stream serialization (the kernel may start
// while the previous kernel on the stream finishes; it orders itself with
// pdl_wait()). Captured into CUDA graphs as programmatic edges.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// launch_pdl with a thread-block cluster shape.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                               dim3 cluster, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster.x;
    attr[1].val.clusterDim.y = cluster.y;
    attr[1].val.clusterDim.z = cluster.z;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Device error word (lazily allocated per device) and its reset/read.
int *device_error_word();

// Quantized-input matmul through the grouped GEMV kernel: tokens in launches
// of up to 8, halved while a stage cannot hold them. Bounded-wait timeouts
// go to `err_word`. Returns a QH_ status and sets qh_last_error() on failure.
int matmul_preq_launch(int type, const void *d_w, int64_t k, int64_t out_f, const void *d_xq, int64_t n_tok,
                       float *d_out, cudaStream_t s, int sm_count, int *err_word);

// F32 weights (tensor_matmul_f32) and many-token Q8_0 (qh_small.cu).
cudaError_t matmul_f32_launch(const float *w, int64_t k, int64_t out_f, const float *x, int64_t n_tok, float *out,
                              cudaStream_t s);
cudaError_t matmul_q8_0_many_launch(const void *w, int64_t k, int64_t out_f, const void *xq, int64_t xq_rows,
                                    int64_t row0, int64_t n_tok, float *out, cudaStream_t s);

// The no-allocation entry point's own error word on device `dev`, or null
// while that entry point has not run there (qh_noalloc.cu).
int *noalloc_error_word(int dev);

// Sets the calling thread's qh_last_error() message.
void set_last_error_message(const char *msg);

}  // namespace qh

#endif  // QH_INTERNAL_H
