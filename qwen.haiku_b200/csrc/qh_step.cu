// SPDX-License-Identifier: MIT
//
// qh_step.cu -- persistent decode step for one sequence (batch 1) on sm_100a.
//
// The reference's slm_forward_step (slm/qwen.c:874-981) is a chain of ~200
// dependent operations per token: residual add + RMSNorm, the projections of
// a layer (tensor_matmul_*_f32, slm/tensor.c:827-1033), the Gated DeltaNet
// head update (slm/qwen.c:318-611), SwiGLU, the down projection, and so on.
// As separate launches each of them costs a launch's ramp and drain (3-15 us
// at batch 1) while moving only 1-5 MB. Here a run of consecutive phases is
// ONE cooperative launch of one CTA per SM:
//
//   * warp 8 (one lane) is the producer: it walks every projection phase of
//     the launch in order and streams this CTA's weight tiles (contiguous
//     row ranges, 1-D bulk copies on the TMA engine) into a byte ring of
//     shared memory. Weights do not depend on activations, so the stream
//     runs ahead across phase boundaries, limited only by the ring;
//   * warps 0-7 consume, phase after phase, with a grid-wide barrier between
//     phases (a bounded wait). A projection phase first forms its Q8_K input
//     in every CTA from the fp32 rows of the previous phase -- residual add +
//     RMSNorm, SwiGLU, or plain quantization, the operations and order of
//     resnorm_q8k_kernel / swiglu_q8k_kernel / quantize_q8k_kernel -- then
//     runs the GEMV consumers (qh_gemv_dev.cuh) on its tiles. A DeltaNet
//     phase runs one head per CTA (warps 0-3), with the head's 64 KB state
//     copied into shared memory during the phase before; the operations are
//     those of gdn_fused_kernel.
//
// Results are bit-identical to the launch-per-operation step (tested).
// Every cross-CTA read of an activation uses ld.global.cg (L2), so no SM
// reads a stale L1 line of a buffer another SM rewrote in an earlier phase.
// Every wait (ring barriers, the DeltaNet state copy, the grid barrier) is
// bounded; on timeout the CTA records kDevWaitTimeout in the device error
// word, the other CTAs see the word in their barrier wait, and all return.

#include <stdio.h>

#include <algorithm>
#include <vector>

#include "qh_backend.h"
#include "qh_common.cuh"
#include "qh_gdn.cuh"
#include "qh_gemv_dev.cuh"
#include "qh_internal.h"
#include "qh_kernels.h"
#include "qh_q8k.cuh"
#include "qh_tc.cuh"

namespace qh {

constexpr int kStepSlots = 32;                      // tiles in flight per CTA (ring slots)
constexpr int kStepThreads = 32 * (kConsumerWarps + 1);
constexpr int kStepHeader = 3072;                   // barriers + slot metadata
constexpr int kStepTerms = 4096;                    // split tiles: two buffers of per-block terms
constexpr int kStepTermsFloats = kStepTerms / 8;
constexpr int kStepTaps = 4;  // conv kernel of the DeltaNet layers (other widths run as launches)
constexpr int kStepHD = 128;
constexpr int kFormChunk = 8;  // blocks of an input row whose loads are in flight together
constexpr int kStepPairFloats = 1024;  // a paired (gate/up) phase's outputs kept per CTA
constexpr int kStepStateBytes = kStepHD * kStepHD * 4;
// DeltaNet shared-memory region: state [128 k][128 v], then the head's conv
// ring rows [3 parts][taps][128] and conv weights [3 parts][128][taps]
constexpr int kStepGdnRowBytes = 3 * kStepTaps * kStepHD * 4;
constexpr int kStepGdnBytes = kStepStateBytes + 2 * kStepGdnRowBytes;
constexpr uint64_t kStepBarrierNs = 2000000000ull;  // grid-barrier wait limit: 2 s
constexpr int kStepBarExit = 32;                    // word of the exit counter (its own 128-byte line)

enum StepKind : int32_t { kPhaseMatvec = 0, kPhaseGdn = 1, kPhaseAttn = 2 };

struct StepJob {
    const uint8_t *w;
    float *out;
    int32_t type, n_rows, nb, row_bytes, k, d_stride;
    int32_t tile_begin, n_tiles;  // tiles of this job inside its phase
};

struct StepGdn {
    const float *qkv;
    float *ring;
    const float *conv_w, *bb, *aa, *dt_bias, *ssm_a;
    float *state;
    const float *z, *norm_w;
    float *y;
    int32_t heads, kk;
    float eps;
};

// One gated-attention layer for one token (sequence 0 of the arguments of
// qh_attn_pre + qh_attn_decode): CTA j serves query head j.
struct StepAttn {
    const float *qraw, *kin, *vin, *qn_w, *kn_w, *rope;
    __half *kcache, *vcache;  // [max_pos][kvh][128]
    float *ctx;               // [nh * 128]
    int32_t nh, kvh, rope_dim, max_pos;
    float eps;
};
constexpr int kAttnChunk = 32;  // V rows per cp.async chunk
constexpr int kAttnBufs = 4;    // chunk buffers: up to 3 chunks in flight ahead
__host__ __device__ constexpr int64_t attn_scratch_bytes(int64_t max_pos) {
    // q, new K row, new V row (floats), scores, V chunks (fp16)
    return 3 * 128 * 4 + ((max_pos + 3) / 4 * 4) * 4 + kAttnBufs * kAttnChunk * 128 * 2;
}

struct StepPhase {
    int32_t kind;
    int32_t xform, xk;   // QH_STEP_X_*, input width
    float eps;
    const float *xa, *xb, *xw;
    float *xh_out;
    float *act;          // paired phase: silu(out of job 0) * out of job 1, per row
    int32_t job0, njobs, rows_per_tile, total_tiles, split;
    int32_t gdn;         // kPhaseGdn / kPhaseAttn: index into the DeltaNet / attention table
};

// What the producer tells the consumers about the tile in a ring slot.
struct SlotMeta {
    float *out;
    int32_t off;  // ring offset of the tile's first row
    int32_t row0, nrows, n_rows;
    int32_t type, nb, k, row_bytes;
};
static_assert(sizeof(SlotMeta) <= 48 && 1024 + 32 * 48 + 16 <= 3072, "slot metadata");

struct StepParams {
    const StepPhase *phases;
    const StepJob *jobs;
    const StepGdn *gdns;
    const StepAttn *attns;
    int32_t first, count;
    int32_t ring_bytes, ring_off, x_off, row_off, terms_off, state_off, w_off, w_floats;
    const int32_t *pos_ptr;
    // [0] grid-barrier arrivals (barrier n completes at n * gridDim.x),
    // [kStepBarExit] exits; zero between launches
    unsigned *bar;
    int *err_flag;
    uint64_t *stamps;  // measurement hook (qh_step_set_stamps), or null
    // failure-detection test hook (qh_step_test_timeout): tile number
    // test_tile of CTA 0 gets no copy (-1: none); mbarrier waits poll at most
    // wait_limit times (0: kWaitLimit)
    int32_t test_tile;
    uint32_t wait_limit;
};

// ---------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ldcg_f(const float *p) { return __ldcg(p); }

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until the bulk stores this thread committed have read their shared
// memory source (the region may then be overwritten).
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Tiles [t0, t1) of a phase for this CTA: a contiguous range (of whole
// pairs in a paired phase, whose tile 2u is job 0's tile u and tile 2u + 1
// job 1's).
__device__ __forceinline__ void my_tiles(const StepPhase &P, int &t0, int &t1) {
    const int units = P.act ? P.total_tiles / 2 : P.total_tiles;
    t0 = static_cast<int>(static_cast<int64_t>(units) * blockIdx.x / gridDim.x);
    t1 = static_cast<int>(static_cast<int64_t>(units) * (blockIdx.x + 1) / gridDim.x);
    if (P.act) {
        t0 *= 2;
        t1 *= 2;
    }
}

// Grid barrier over the consumer warps of every CTA: a release add on a
// counter that only grows during the launch (barrier n completes at
// n * gridDim.x) and acquire loads of it in the wait. The wait is bounded in
// time and gives up early when another CTA has recorded an error. Returns
// false (uniformly for the CTA) on either.
__device__ __forceinline__ bool step_grid_barrier(const StepParams &p, unsigned n) {
    __shared__ int s_ok;
    consumers_sync();
    if (threadIdx.x == 0) {
        // release: this CTA's writes (ordered before thread 0 by the barrier
        // above) become visible with the arrival; one trip to L2, no reply.
        // (Measured: a separate fence before or after costs ~0.4 us each;
        // copies of the counter on other L2 lines do not help.)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
        const unsigned target = n * gridDim.x;
        bool ok = false;
        const uint64_t t0 = global_ns();
        for (uint32_t it = 1;; ++it) {
            if (ld_acquire_u32(p.bar) >= target) {
                ok = true;
                break;
            }
            if ((it & 63u) == 0) {  // the error word and the time limit, now and then
                if (*reinterpret_cast<volatile int *>(p.err_flag) != 0) break;
                if (global_ns() - t0 > kStepBarrierNs) {
                    report_error(p.err_flag, kDevWaitTimeout);
                    break;
                }
            }
        }
        s_ok = ok ? 1 : 0;
    }
    consumers_sync();
    return s_ok != 0;
}

// Measurement hook (qh_step_set_stamps), per phase ph a record of
// kStampFixed + 2 * gridDim.x words: [0..3] CTA 0's %globaltimer at the phase
// start, input formed, work done, past the barrier; [4..7] points inside the
// phase's work on CTA 0; [8 + c] CTA c's work done, [8 + G + c] CTA c's input
// formed.
constexpr int kStampFixed = 8;
__device__ __forceinline__ int64_t stamp_rec(int ph) { return static_cast<int64_t>(ph) * (kStampFixed + 2 * gridDim.x); }
__device__ __forceinline__ void stamp(const StepParams &p, int ph, int what) {
    if (p.stamps && blockIdx.x == 0 && threadIdx.x == 0) p.stamps[stamp_rec(ph) + what] = global_ns();
}
// [8 + c]: CTA c's work done; [8 + G + c]: CTA c's input formed
__device__ __forceinline__ void stamp_cta(const StepParams &p, int ph, int second = 0) {
    if (p.stamps && threadIdx.x == 0)
        p.stamps[stamp_rec(ph) + kStampFixed + second * gridDim.x + blockIdx.x] = global_ns();
}

// ---------------------------------------------------------------------------
// Input formation: the Q8_K planes of one row of xk values in shared memory
// ([qs][bsums][d], the split layout a staged activation has), with the
// operations and order of resnorm_q8k_kernel (thread t sums the squares of
// elements t, t + 256, ... in double, then the warp tree and the warps in
// order), swiglu_q8k_kernel or quantize_q8k_kernel; quantized one Q8_K block
// per warp by q8k_block_warp. CTA 0 writes the residual sum when asked.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void step_form_input(const StepPhase &P, uint8_t *xs, float *rowbuf, const float *wsm,
                                                uint64_t *tstamp = nullptr) {
    __shared__ double dscr[kConsumerWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = P.xk, nb = K / QH_QK;
    int8_t *qs = reinterpret_cast<int8_t *>(xs);
    int16_t *bs = reinterpret_cast<int16_t *>(xs + K);
    float *dd = reinterpret_cast<float *>(xs + K + nb * 32);
    if (P.xform == QH_STEP_X_QUANT) {
        for (int b = warp; b < nb; b += kConsumerWarps) {
            const int e0 = b * QH_QK + 8 * lane;
            const float4 a0 = __ldcg(reinterpret_cast<const float4 *>(P.xa + e0));
            const float4 a1 = __ldcg(reinterpret_cast<const float4 *>(P.xa + e0 + 4));
            const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            q8k_block_warp(v, qs + b * QH_QK, bs + b * 16, dd + b);
        }
        return;
    }
    // First pass over all 256 threads, every load issued at once: thread t
    // takes elements t, t + 256, ... (the element order of the reference
    // norm's double sum of squares, as resnorm_q8k_kernel).
    const float *wbuf = wsm;  // RMSNorm weights, copied into shared memory a phase ahead
    float rscale = 0.0f;
    if (P.xform == QH_STEP_X_RESNORM) {
        double s = 0.0;
        for (int j0 = 0; j0 < nb; j0 += kFormChunk) {
            float xv[kFormChunk], yv[kFormChunk];
#pragma unroll
            for (int u = 0; u < kFormChunk; ++u) {
                const int i = (j0 + u) * QH_QK + tid;
                if (j0 + u < nb) {
                    xv[u] = ldcg_f(P.xa + i);
                    yv[u] = P.xb ? ldcg_f(P.xb + i) : 0.0f;
                }
            }
#pragma unroll
            for (int u = 0; u < kFormChunk; ++u) {
                const int i = (j0 + u) * QH_QK + tid;
                if (j0 + u < nb) {
                    const float x = P.xb ? __fadd_rn(xv[u], yv[u]) : xv[u];
                    rowbuf[i] = x;
                    if (P.xh_out && blockIdx.x == 0) P.xh_out[i] = x;
                    s += static_cast<double>(__fmul_rn(x, x));
                }
            }
        }
        if (tstamp && tid == 0) tstamp[4] = global_ns();
        const double ssq = consumers_sum_d(s, dscr);  // ends with a consumer barrier: rowbuf complete
        if (tstamp && tid == 0) tstamp[5] = global_ns();
        rscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ssq / static_cast<double>(K)), P.eps)));
    } else {  // SwiGLU
        for (int j0 = 0; j0 < nb; j0 += kFormChunk) {
            float gv[kFormChunk], uv[kFormChunk];
#pragma unroll
            for (int u = 0; u < kFormChunk; ++u) {
                if (j0 + u < nb) {
                    gv[u] = ldcg_f(P.xa + (j0 + u) * QH_QK + tid);
                    uv[u] = ldcg_f(P.xb + (j0 + u) * QH_QK + tid);
                }
            }
#pragma unroll
            for (int u = 0; u < kFormChunk; ++u)
                if (j0 + u < nb) rowbuf[(j0 + u) * QH_QK + tid] = __fmul_rn(silu_f(gv[u]), uv[u]);
        }
        consumers_sync();
    }
    for (int b = warp; b < nb; b += kConsumerWarps) {
        const int e0 = b * QH_QK + 8 * lane;
        float v[8];
        const float4 r0 = *reinterpret_cast<const float4 *>(rowbuf + e0);
        const float4 r1 = *reinterpret_cast<const float4 *>(rowbuf + e0 + 4);
        const float r[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
        if (P.xform == QH_STEP_X_RESNORM) {
            const float4 w0 = *reinterpret_cast<const float4 *>(wbuf + e0);
            const float4 w1 = *reinterpret_cast<const float4 *>(wbuf + e0 + 4);
            const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fmul_rn(r[e], rscale), w[e]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = r[e];
        }
        q8k_block_warp(v, qs + b * QH_QK, bs + b * 16, dd + b);
    }
}

// ---------------------------------------------------------------------------
// One Gated DeltaNet head for one token on warps 0-3 (128 threads, thread t
// owns state column t): the operations and order of gdn_fused_kernel --
// conv ring + SiLU, L2 norms (double sums: warp tree, then the 4 warps in
// order), beta / g, the recurrence over the column in shared memory with its
// two sequential double chains, the state store, the gated RMSNorm -- with
// the fp32 output row written for the next phase's quantization.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void gdn_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

__device__ __forceinline__ double gdn_sum_d(double v, double *scratch) {
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    gdn_sync();
    if (lane == 0) scratch[warp] = v;
    gdn_sync();
    double t = 0.0;
    for (int w = 0; w < kStepHD / 32; ++w) t += scratch[w];
    return t;
}

__device__ __forceinline__ double2 gdn_sum_d2(double a, double b, double *scratch) {
    for (int off = 16; off > 0; off >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, off);
        b += __shfl_xor_sync(0xffffffffu, b, off);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    gdn_sync();
    if (lane == 0) {
        scratch[warp] = a;
        scratch[4 + warp] = b;
    }
    gdn_sync();
    double ta = 0.0, tb = 0.0;
    for (int w = 0; w < kStepHD / 32; ++w) {
        ta += scratch[w];
        tb += scratch[4 + w];
    }
    return make_double2(ta, tb);
}

// beta = sigmoid(b) and g = exp(ssm_a * softplus(a + dt_bias)) of head h
// (the gdn_fused_kernel formulas), formed by warp 4 while warps 0-3 run the
// conv and the norms; named barrier 3 joins the five warps.
__device__ __forceinline__ void gdn_gates_sync() { asm volatile("bar.sync 3, 160;" ::: "memory"); }

__device__ __forceinline__ void step_gdn_gates(const StepGdn &g, int h, float *gates) {
    if ((threadIdx.x & 31) == 0) {
        gates[0] = sigmoid_f(ldcg_f(g.bb + h));
        const float a = __fadd_rn(ldcg_f(g.aa + h), __ldg(g.dt_bias + h));
        const float sp = a > 20.0f ? a : logf_ref(__fadd_rn(1.0f, expf_ref(a)));
        gates[1] = expf_ref(__fmul_rn(__ldg(g.ssm_a + h), sp));
    }
    gdn_gates_sync();
}

__device__ __forceinline__ void step_gdn_head(const StepGdn &g, int h, float *st_s, uint64_t *st_bar, uint32_t parity,
                                              const int32_t *pos_ptr, int *err, uint64_t *tstamp, const float *gates,
                                              uint32_t lim) {
    auto mark = [&](int i) {
        if (tstamp && threadIdx.x == 0) tstamp[i] = global_ns();
    };
    constexpr int HD = kStepHD;
    __shared__ double scratch[8];
    __shared__ float Ks[HD], Qs[HD];
    const int t = threadIdx.x, heads = g.heads;
    const int kdim = heads * HD, conv_dim = 3 * kdim;
    constexpr int kk = kStepTaps;
    float *st = g.state + static_cast<int64_t>(h) * HD * HD;
    const float *ring_s = st_s + HD * HD, *conv_s = ring_s + 3 * kk * HD;
    float xin[3];
#pragma unroll
    for (int part = 0; part < 3; ++part) xin[part] = ldcg_f(g.qkv + part * kdim + h * HD + t);
    const float zv = ldcg_f(g.z + h * HD + t);
    // state, conv ring rows and conv weights were copied in during the phase before
    if (!mbar_wait_n(st_bar, parity, lim)) report_error(err, kDevWaitTimeout);
    mark(5);
    float cw[3][kk], rows[3][kk];
#pragma unroll
    for (int part = 0; part < 3; ++part)
#pragma unroll
        for (int k = 0; k < kk; ++k) {
            cw[part][k] = conv_s[(part * HD + t) * kk + k];
            rows[part][k] = ring_s[(part * kk + k) * HD + t];
        }
    const int pos = max(__ldcg(pos_ptr), 0);
    const int slot = pos % kk, head_after = (pos + 1) % kk;
    float taps[3][kStepTaps - 1];
#pragma unroll
    for (int part = 0; part < 3; ++part)
#pragma unroll
        for (int k = 0; k < kStepTaps - 1; ++k) {
            const int rsel = (head_after + k) % kk;
            float v = 0.0f;
#pragma unroll
            for (int r = 0; r < kStepTaps; ++r)
                if (r == rsel) v = rows[part][r];
            taps[part][k] = v;
        }
    float mixed[3];
#pragma unroll
    for (int part = 0; part < 3; ++part) {
        const int ch = part * kdim + h * HD + t;
        g.ring[static_cast<int64_t>(slot) * conv_dim + ch] = xin[part];
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < kStepTaps; ++k)
            acc = __fadd_rn(acc, __fmul_rn(k < kk - 1 ? taps[part][k] : xin[part], cw[part][k]));
        mixed[part] = silu_f(acc);
    }
    const double2 qkss = gdn_sum_d2(static_cast<double>(__fmul_rn(mixed[0], mixed[0])),
                                    static_cast<double>(__fmul_rn(mixed[1], mixed[1])), scratch);
    const float qrs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(qkss.x)), 1e-6f));
    const float krs = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(static_cast<float>(qkss.y)), 1e-6f));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HD)));
    Qs[t] = __fmul_rn(__fmul_rn(mixed[0], qrs), scale);
    Ks[t] = __fmul_rn(mixed[1], krs);
    const float vt = mixed[2];
    gdn_gates_sync();  // with warp 4, which formed beta and g
    mark(4);
    const float gh = gates[1], bh = gates[0];
    const float o = gdn_recur_column<HD>(st_s + t, Ks, Qs, gh, bh, vt);  // qh_gdn.cuh
    mark(6);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    gdn_sync();
    if (t == 0) {
        bulk_copy_s2g(st, st_s, kStepStateBytes);
        bulk_commit_group();
    }
    const double ssq = gdn_sum_d(static_cast<double>(__fmul_rn(o, o)), scratch);
    const float mean = static_cast<float>(ssq / static_cast<double>(HD));
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, g.eps)));
    const int zi = h * HD + t;
    g.y[zi] = __fmul_rn(__fmul_rn(__fmul_rn(o, rs), __ldg(g.norm_w + t)), silu_f(zv));
    mark(7);
}

// Issues the copy of head h's state of DeltaNet layer g into st_s (thread 0
// of the CTA, which also issued the previous layer's state store).
__device__ __forceinline__ void gdn_prefetch(const StepGdn &g, int h, float *st_s, uint64_t *st_bar) {
    constexpr int HD = kStepHD, kk = kStepTaps;
    const int kdim = g.heads * HD, conv_dim = 3 * kdim;
    bulk_wait_read_all();  // the previous layer's store has read the region
    float *ring_s = st_s + HD * HD, *conv_s = ring_s + 3 * kk * HD;
    mbar_arrive_expect_tx(st_bar, kStepGdnBytes);
    bulk_copy_g2s(st_s, g.state + static_cast<int64_t>(h) * HD * HD, kStepStateBytes, st_bar);
    for (int part = 0; part < 3; ++part) {
        for (int r = 0; r < kk; ++r)
            bulk_copy_g2s(ring_s + (part * kk + r) * HD, g.ring + static_cast<int64_t>(r) * conv_dim + part * kdim + h * HD,
                          HD * 4, st_bar);
        bulk_copy_g2s(conv_s + part * HD * kk, g.conv_w + static_cast<int64_t>(part * kdim + h * HD) * kk, HD * kk * 4,
                      st_bar);
    }
}

// ---------------------------------------------------------------------------
// One query head of a gated-attention layer for one token, on the 256
// consumer threads of CTA j (query head j, KV head c = j / (nh / kvh)): the
// operations and orders of attn_pre_kernel and attn_decode_gqa_kernel.
//   * warps 0-3: RMSNorm (double sum: warp tree, then the 4 warps in order)
//     + MRoPE of the query row; warps 4-7 the same for the KV head's new K
//     row. Every CTA of a KV head forms that row itself (so no CTA waits for
//     another), and the first of them appends K and V to the caches.
//   * scores: thread t takes positions t, t + 256, ...: a sequential fp32 dot
//     over the 128 dims with the fp16 cache rows (the new row from shared
//     memory, rounded to fp16 as the cache holds it), times 1/sqrt(128);
//   * max, exp, one thread's sequential sum, scaling, then per dim (threads
//     0-127) the sequential sum over positions of p_i * V_i, the V rows
//     staged by cp.async in chunks; ctx = o * sigmoid(gate).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void attn_sync_hi() { asm volatile("bar.sync 4, 128;" ::: "memory"); }

__device__ __forceinline__ double attn_sum_hi(double v, double *scratch) {  // warps 4-7
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int w = (threadIdx.x >> 5) - 4, lane = threadIdx.x & 31;
    attn_sync_hi();
    if (lane == 0) scratch[w] = v;
    attn_sync_hi();
    double t = 0.0;
    for (int i = 0; i < 4; ++i) t += scratch[i];
    return t;
}

__device__ __forceinline__ void step_attn_head(const StepAttn &A, int j, uint8_t *scr, const int32_t *pos_ptr,
                                               uint64_t *tstamp = nullptr) {
    auto mark = [&](int i) {
        if (tstamp && threadIdx.x == 0) tstamp[i] = global_ns();
    };
    constexpr int HD = kStepHD;
    __shared__ double sq[4], sk[4];
    __shared__ float s_red[kConsumerWarps], s_inv;
    float *qs = reinterpret_cast<float *>(scr);
    float *kn = qs + HD, *vn = kn + HD;
    float *sc = vn + HD;
    __half *vbuf = reinterpret_cast<__half *>(sc + (A.max_pos + 3) / 4 * 4);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, t = tid & (HD - 1);
    const int G = A.nh / A.kvh, c = j / G;
    const int pos = min(max(__ldcg(pos_ptr), 0), A.max_pos - 1), n = pos + 1;
    const int64_t rstride = static_cast<int64_t>(A.kvh) * HD;
    const __half *kb = A.kcache + static_cast<int64_t>(c) * HD;
    const __half *vb = A.vcache + static_cast<int64_t>(c) * HD;
    // V rows of chunk q (rows below pos, from the cache) into buffer q % kAttnBufs
    const int n_old = pos, n_chunks = (n_old + kAttnChunk - 1) / kAttnChunk;
    auto issue_v = [&](int q) {
        if (q < n_chunks) {
            const int r0 = q * kAttnChunk, rows = min(kAttnChunk, n_old - r0);
            __half *dst = vbuf + (q % kAttnBufs) * kAttnChunk * HD;
            for (int piece = tid; piece < rows * (HD / 8); piece += 32 * kConsumerWarps) {
                const int r = piece / (HD / 8), q16 = piece % (HD / 8);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst + r * HD + q16 * 8)),
                             "l"(vb + (r0 + r) * rstride + q16 * 8)
                             : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int q = 0; q < kAttnBufs - 1; ++q) issue_v(q);
    // Loads that do not wait for this phase's inputs go first: the norm
    // weight and this thread's rope pair.
    const bool hi = warp >= 4;
    const float wnorm = __ldg((hi ? A.kn_w : A.qn_w) + t);
    const int half = A.rope_dim / 2;
    float rco = 1.0f, rsn = 0.0f;
    if (t < A.rope_dim) {
        const int i = t < half ? t : t - half;
        rco = __ldg(A.rope + (static_cast<int64_t>(pos) * half + i) * 2);
        rsn = __ldg(A.rope + (static_cast<int64_t>(pos) * half + i) * 2 + 1);
    }
    // ---- norms and MRoPE (attn_pre_kernel) ----
    float x, gt = 0.0f;
    if (!hi) {
        const float *src = A.qraw + static_cast<int64_t>(j) * 2 * HD;
        x = ldcg_f(src + t);
        gt = ldcg_f(src + HD + t);
    } else {
        x = ldcg_f(A.kin + static_cast<int64_t>(c) * HD + t);
    }
    const float vin = hi ? ldcg_f(A.vin + static_cast<int64_t>(c) * HD + t) : 0.0f;
    const double ssq = hi ? attn_sum_hi(static_cast<double>(__fmul_rn(x, x)), sk)
                          : gdn_sum_d(static_cast<double>(__fmul_rn(x, x)), sq);
    const float rscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ssq / static_cast<double>(HD)), A.eps)));
    const float xn = __fmul_rn(__fmul_rn(x, rscale), wnorm);
    float *xrow = hi ? kn : qs;
    xrow[t] = xn;
    consumers_sync();
    mark(4);
    float y = xn;
    if (t < A.rope_dim) {
        const int i = t < half ? t : t - half;
        const float x0 = xrow[i], x1 = xrow[i + half];
        y = t < half ? __fsub_rn(__fmul_rn(x0, rco), __fmul_rn(x1, rsn))
                     : __fadd_rn(__fmul_rn(x0, rsn), __fmul_rn(x1, rco));
    }
    consumers_sync();  // every thread has read xrow
    if (!hi) {
        qs[t] = y;
    } else {
        const __half kh = __float2half_rn(y), vh = __float2half_rn(vin);
        kn[t] = __half2float(kh);
        vn[t] = __half2float(vh);
        if (j % G == 0) {  // the first query head of the group appends the rows
            const int64_t row = (static_cast<int64_t>(pos) * A.kvh + c) * HD + t;
            A.kcache[row] = kh;
            A.vcache[row] = vh;
        }
    }
    consumers_sync();
    // ---- scores ----
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HD)));
    float lmax = -INFINITY;
    for (int i = tid; i < n; i += 32 * kConsumerWarps) {
        float dot = 0.0f;
        if (i < pos) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(kb + i * rstride);
            uint4 row[HD / 8];
#pragma unroll
            for (int q = 0; q < HD / 8; ++q) row[q] = __ldcg(kr + q);
#pragma unroll
            for (int q = 0; q < HD / 8; ++q) {
                const __half2 *hp = reinterpret_cast<const __half2 *>(&row[q]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(hp[e]);
                    dot = __fadd_rn(dot, __fmul_rn(qs[8 * q + 2 * e], f.x));
                    dot = __fadd_rn(dot, __fmul_rn(qs[8 * q + 2 * e + 1], f.y));
                }
            }
        } else {
            for (int d = 0; d < HD; ++d) dot = __fadd_rn(dot, __fmul_rn(qs[d], kn[d]));
        }
        const float sv = __fmul_rn(dot, scale);
        sc[i] = sv;
        lmax = fmaxf(lmax, sv);
    }
    for (int off = 16; off > 0; off >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, off));
    if (lane == 0) s_red[warp] = lmax;
    consumers_sync();
    mark(5);
    float m = s_red[0];
    for (int w = 1; w < kConsumerWarps; ++w) m = fmaxf(m, s_red[w]);
    for (int i = tid; i < n; i += 32 * kConsumerWarps) sc[i] = expf_ref(__fsub_rn(sc[i], m));
    consumers_sync();
    if (tid == 0) {  // the sequential sum
        float sum = 0.0f;
        int i = 0;
        for (; i + 8 <= n; i += 8) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = sc[i + e];
#pragma unroll
            for (int e = 0; e < 8; ++e) sum = __fadd_rn(sum, v[e]);
        }
        for (; i < n; ++i) sum = __fadd_rn(sum, sc[i]);
        s_inv = __fdiv_rn(1.0f, sum);
    }
    consumers_sync();
    const float inv = s_inv;
    for (int i = tid; i < n; i += 32 * kConsumerWarps) sc[i] = __fmul_rn(sc[i], inv);
    consumers_sync();
    mark(6);
    // ---- weighted V sum, per dim in position order ----
    float o = 0.0f;
    for (int q = 0; q < n_chunks; ++q) {
        issue_v(q + kAttnBufs - 1);
        asm volatile("cp.async.wait_group %0;" ::"n"(kAttnBufs - 1) : "memory");
        consumers_sync();
        if (tid < HD) {
            const __half *vc = vbuf + (q % kAttnBufs) * kAttnChunk * HD;
            const int r0 = q * kAttnChunk, rows = min(kAttnChunk, n_old - r0);
            for (int r = 0; r < rows; ++r) o = __fadd_rn(o, __fmul_rn(sc[r0 + r], __half2float(vc[r * HD + tid])));
        }
        consumers_sync();  // this buffer is refilled by the issue of chunk q + kAttnBufs
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (tid < HD) {
        o = __fadd_rn(o, __fmul_rn(sc[pos], vn[tid]));
        A.ctx[static_cast<int64_t>(j) * HD + tid] = __fmul_rn(o, sigmoid_f(gt));
    }
    mark(7);
}

// Runtime-typed 8-row group consumer (one token).
__device__ __forceinline__ void step_group(int type, const uint8_t *wbase, int trow, const GemvJob &job,
                                           const XView &x, int row0, int nvalid, int b_first, int b_step,
                                           float *terms) {
    if (type == QH_GGUF_Q4_K)
        process_group<QH_GGUF_Q4_K, 1>(wbase, 0, trow, job, x, row0, nvalid, 1, b_first, b_step, terms);
    else if (type == QH_GGUF_Q5_K)
        process_group<QH_GGUF_Q5_K, 1>(wbase, 0, trow, job, x, row0, nvalid, 1, b_first, b_step, terms);
    else
        process_group<QH_GGUF_Q6_K, 1>(wbase, 0, trow, job, x, row0, nvalid, 1, b_first, b_step, terms);
}

__device__ __forceinline__ GemvJob gemv_job_of(const StepJob &sj) {
    GemvJob j = {};
    j.out = sj.out;
    j.n_rows = sj.n_rows;
    j.nb = sj.nb;
    j.row_bytes = sj.row_bytes;
    j.k = sj.k;
    j.d_stride = sj.d_stride;
    j.box_blocks = sj.nb;
    j.box_pitch = sj.row_bytes;
    return j;
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const __grid_constant__ StepParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kStepSlots;
    uint64_t *st_bar = empty + kStepSlots;
    uint64_t *wbar = st_bar + 1;  // [2] RMSNorm weight copies
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 8 * (2 * kStepSlots + 3));
    SlotMeta *meta = reinterpret_cast<SlotMeta *>(smem + 1024);  // [kStepSlots]
    float *gates = reinterpret_cast<float *>(smem + 1024 + kStepSlots * sizeof(SlotMeta));  // DeltaNet beta, g
    uint8_t *ring = smem + p.ring_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t RB = static_cast<uint32_t>(p.ring_bytes);
    const uint32_t lim = p.wait_limit ? p.wait_limit : kWaitLimit;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStepSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(st_bar, 1);
        mbar_init(&wbar[0], 1);
        mbar_init(&wbar[1], 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ----- producer (lane 0): every projection phase's tiles of this CTA, in order -----
        if (lane != 0) return;
        auto withheld = [&](int q) { return p.test_tile >= 0 && blockIdx.x == 0 && q == p.test_tile; };
        uint32_t vstart[kStepSlots];
        uint64_t vhead = 0;
        int i = 0, oldest = 0;
        bool stop = false;
        for (int k = 0; k < p.count && !stop; ++k) {
            const StepPhase &P = p.phases[p.first + k];
            if (P.kind != kPhaseMatvec) continue;
            int t0, t1;
            my_tiles(P, t0, t1);
            int j = P.job0;
            for (int t = t0; t < t1; ++t, ++i) {
                int lt;  // tile index inside its job
                if (P.act) {
                    j = P.job0 + (t & 1);
                    lt = t >> 1;
                } else {
                    while (t >= p.jobs[j].tile_begin + p.jobs[j].n_tiles) ++j;
                    lt = t - p.jobs[j].tile_begin;
                }
                const StepJob &J = p.jobs[j];
                const int row0 = lt * P.rows_per_tile;
                const int nrows = min(P.rows_per_tile, J.n_rows - row0);
                const uint8_t *g0 = J.w + static_cast<int64_t>(row0) * J.row_bytes;
                const uint8_t *g1 = g0 + static_cast<int64_t>(nrows) * J.row_bytes;
                const uint8_t *a0 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(g0) & ~uintptr_t(15));
                const uint8_t *a1 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(g1) & ~uintptr_t(15));
                const uint32_t wbytes = static_cast<uint32_t>(a1 - a0);
                const uint32_t tail = static_cast<uint32_t>(g1 - a1);
                // room for whole 8-row groups: the consumers read all 8 rows of a
                // group (a ragged group's extra rows are garbage and never stored)
                const uint32_t rows8 = static_cast<uint32_t>((nrows + kGroupRows - 1) / kGroupRows * kGroupRows);
                const uint32_t sz =
                    (static_cast<uint32_t>(g0 - a0) + rows8 * static_cast<uint32_t>(J.row_bytes) + 32u + 127u) & ~127u;
                // place the tile: contiguous in the ring, wrapping to its start
                uint64_t vs = vhead;
                if (static_cast<uint32_t>(vs % RB) + sz > RB) vs = (vs / RB + 1) * RB;
                while (oldest < i && (i - oldest >= kStepSlots || vs + sz - vstart[oldest % kStepSlots] > RB)) {
                    if (*abort_flag ||
                        !mbar_wait_n(&empty[oldest % kStepSlots], static_cast<uint32_t>(oldest / kStepSlots) & 1u, lim)) {
                        report_error(p.err_flag, kDevWaitTimeout);
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    ++oldest;
                }
                if (stop) break;
                const int s = i % kStepSlots;
                vstart[s] = static_cast<uint32_t>(vs);
                vhead = vs + sz;
                uint8_t *dst = ring + static_cast<uint32_t>(vs % RB);
                for (uint32_t q = 0; q < tail; ++q) dst[wbytes + q] = __ldg(a1 + q);
                SlotMeta &M = meta[s];
                M.out = J.out;
                M.off = static_cast<int>(vs % RB) + static_cast<int>(g0 - a0);
                M.row0 = row0;
                M.nrows = nrows;
                M.n_rows = J.n_rows;
                M.type = J.type;
                M.nb = J.nb;
                M.k = J.k;
                M.row_bytes = J.row_bytes;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                if (withheld(i)) continue;  // test hook: this tile never arrives
                if (wbytes) {
                    mbar_arrive_expect_tx(&full[s], wbytes);
                    bulk_copy_g2s(dst, a0, wbytes, &full[s]);
                } else {
                    mbar_arrive(&full[s]);
                }
            }
        }
        // Drain: no copy of this CTA stays in flight past its exit.
        for (int q = max(0, i - kStepSlots); q < i; ++q)
            if (!withheld(q) && !mbar_wait_n(&full[q % kStepSlots], static_cast<uint32_t>(q / kStepSlots) & 1u, lim))
                report_error(p.err_flag, kDevWaitTimeout);
        return;
    }

    // ----- consumers -----
    uint8_t *xs = smem + p.x_off;
    float *rowbuf = reinterpret_cast<float *>(smem + p.row_off);
    float *terms = reinterpret_cast<float *>(smem + p.terms_off);
    float *st_s = reinterpret_cast<float *>(smem + p.state_off);
    // Launched with programmatic serialization: the producer's weight stream
    // starts while the previous kernel finishes; everything that reads or
    // writes activations, caches or states waits for it here.
    pdl_wait();
    int i = 0;              // tile sequence number, as the producer counts
    uint32_t n_gdn = 0;     // DeltaNet phases of this CTA so far (state barrier parity)
    bool ok = true;
    // A DeltaNet phase's state copy is issued at the start of the phase
    // before it (or at its own start when it opens the launch).
    auto maybe_prefetch = [&](int k) {
        if (threadIdx.x != 0 || k >= p.count) return;
        const StepPhase &N = p.phases[p.first + k];
        if (N.kind == kPhaseGdn && static_cast<int>(blockIdx.x) < p.gdns[N.gdn].heads)
            gdn_prefetch(p.gdns[N.gdn], blockIdx.x, st_s, st_bar);
    };
    // The RMSNorm weights of phase k go to buffer k & 1, copied at the start
    // of phase k - 1 by a CTA that has tiles in phase k.
    float *wpre = reinterpret_cast<float *>(smem + p.w_off);
    uint32_t wuse[2] = {0u, 0u};
    auto norm_prefetch = [&](int k) {
        if (k >= p.count) return false;
        const StepPhase &N = p.phases[p.first + k];
        if (N.kind != kPhaseMatvec || N.xform != QH_STEP_X_RESNORM) return false;
        int a, b;
        my_tiles(N, a, b);
        if (a >= b) return false;
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(&wbar[k & 1], static_cast<uint32_t>(N.xk) * 4u);
            bulk_copy_g2s(wpre + (k & 1) * p.w_floats, N.xw, static_cast<uint32_t>(N.xk) * 4u, &wbar[k & 1]);
        }
        return true;
    };
    maybe_prefetch(0);
    bool w_next = norm_prefetch(0);
    for (int k = 0; k < p.count && ok; ++k) {
        const bool w_here = w_next;
        maybe_prefetch(k + 1);
        w_next = norm_prefetch(k + 1);
        stamp(p, p.first + k, 0);
        const StepPhase &P = p.phases[p.first + k];
        if (P.kind == kPhaseAttn) {
            const StepAttn &A = p.attns[P.gdn];
            uint64_t *ts = (p.stamps && blockIdx.x == 0)
                               ? p.stamps + stamp_rec(p.first + k)
                               : nullptr;
            if (static_cast<int>(blockIdx.x) < A.nh)
                step_attn_head(A, blockIdx.x, reinterpret_cast<uint8_t *>(st_s), p.pos_ptr, ts);
        } else if (P.kind == kPhaseGdn) {
            const StepGdn &G = p.gdns[P.gdn];
            if (static_cast<int>(blockIdx.x) < G.heads) {
                uint64_t *ts = (p.stamps && blockIdx.x == 0)
                                   ? p.stamps + stamp_rec(p.first + k)
                                   : nullptr;
                if (warp < kStepHD / 32)
                    step_gdn_head(G, blockIdx.x, st_s, st_bar, n_gdn & 1u, p.pos_ptr, p.err_flag, ts, gates, lim);
                else if (warp == kStepHD / 32)
                    step_gdn_gates(G, blockIdx.x, gates);
                ++n_gdn;
            }
        } else {
            int t0, t1;
            my_tiles(P, t0, t1);
            if (w_here) {  // this phase's RMSNorm weights
                const int b = k & 1;
                if (!mbar_wait_n(&wbar[b], wuse[b] & 1u, lim)) report_error(p.err_flag, kDevWaitTimeout);
                ++wuse[b];
                stamp(p, p.first + k, 6);
            }
            uint64_t *fts = (p.stamps && blockIdx.x == 0)
                                ? p.stamps + stamp_rec(p.first + k)
                                : nullptr;
            if (t0 < t1) step_form_input(P, xs, rowbuf, wpre + (k & 1) * p.w_floats, fts);  // a CTA without tiles needs no input
            consumers_sync();
            stamp(p, p.first + k, 1);
            stamp_cta(p, p.first + k, 1);
            // paired phase: the CTA's gate / up outputs stay in shared memory
            // (rowbuf, free once the input is formed) for the SwiGLU epilogue
            const int pr0 = P.act ? (t0 >> 1) * P.rows_per_tile : 0;
            const int prows = P.act ? (t1 >> 1) * P.rows_per_tile - pr0 : 0;
            float *pair_out = rowbuf;
            XView x;
            x.qs = reinterpret_cast<const int8_t *>(xs);
            auto job_of = [&](const SlotMeta &M) {
                GemvJob jb = {};
                jb.out = M.out;
                jb.n_rows = M.n_rows;
                jb.nb = M.nb;
                jb.row_bytes = M.row_bytes;
                jb.k = M.k;
                jb.d_stride = (M.nb + 3) & ~3;
                jb.box_blocks = M.nb;
                jb.box_pitch = M.row_bytes;
                x.bs = reinterpret_cast<const int16_t *>(xs + M.k);
                x.d = xs + M.k + M.nb * 32;
                return jb;
            };
            if (P.split) {
                // one 8-row tile: its blocks spread over the 8 warps, the terms
                // meet in shared memory, warp 0 adds them in block order
                for (int t = t0; t < t1; ++t, ++i) {
                    const int s = i % kStepSlots;
                    const bool got = !*abort_flag &&
                                     mbar_wait_n(&full[s], static_cast<uint32_t>(i / kStepSlots) & 1u, lim);
                    if (bar_any(1, 32 * kConsumerWarps, !got)) {
                        if (!got) {
                            report_error(p.err_flag, kDevWaitTimeout);
                            *abort_flag = 1;
                        }
                        ok = false;
                        break;
                    }
                    const SlotMeta M = meta[s];
                    const GemvJob job = job_of(M);
                    const int nvalid = min(kGroupRows, M.nrows);
                    float *tb = terms + (i & 1) * kStepTermsFloats;
                    if (warp < M.nb)
                        step_group(M.type, ring + M.off, 0, job, x, M.row0, nvalid, warp, kConsumerWarps, tb);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[s]);
                    consumers_sync();
                    if (warp == 0 && (lane & 3) == 0 && (lane >> 2) < nvalid) {
                        const int r = lane >> 2;
                        float acc = 0.0f;
                        for (int b = 0; b < M.nb; ++b) acc = __fadd_rn(acc, tb[r * M.nb + b]);
                        M.out[M.row0 + r] = acc;
                    }
                }
            } else {
                // Group G of the CTA's tiles (tile G / gpt, its group G % gpt) goes
                // to warp G % 8; a warp waits for, and releases, only the tiles it
                // works on. A tile's empty barrier takes 8 arrivals: one per group
                // and, from the warp of group 0, the 8 - gpt groups it does not have.
                const int gpt = P.rows_per_tile / kGroupRows;  // groups per tile (<= 8)
                const int ng = (t1 - t0) * gpt;
                for (int G = warp; G < ng; G += kConsumerWarps) {
                    const int tl = G / gpt, gi = G - tl * gpt, ii = i + tl, s = ii % kStepSlots;
                    if (*abort_flag || !mbar_wait_n(&full[s], static_cast<uint32_t>(ii / kStepSlots) & 1u, lim)) {
                        report_error(p.err_flag, kDevWaitTimeout);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const SlotMeta M = meta[s];
                    if (kGroupRows * gi < M.nrows) {
                        GemvJob job = job_of(M);
                        int row0 = M.row0;
                        if (P.act) {  // rows of job 0 then job 1, relative to the CTA's first row
                            job.out = pair_out + ((t0 + tl) & 1) * prows;
                            row0 -= pr0;
                        }
                        step_group(M.type, ring + M.off, kGroupRows * gi, job, x, row0 + kGroupRows * gi,
                                   min(kGroupRows, M.nrows - kGroupRows * gi), 0, 1, nullptr);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive_n(&empty[s], gi == 0 ? kConsumerWarps + 1 - gpt : 1);
                }
                i += t1 - t0;
                // the loop's exit is per warp; the barrier below needs all of them
                ok = !bar_any(1, 32 * kConsumerWarps, !ok);
                stamp(p, p.first + k, 7);
                if (ok && P.act) {
                    // SwiGLU of the rows this CTA computed: the values
                    // swiglu_q8k_kernel forms, for the next phase to quantize;
                    // the two projections' outputs are stored as well
                    const StepJob &J0 = p.jobs[P.job0];
                    float *out1 = p.jobs[P.job0 + 1].out;
                    const int r1 = min(pr0 + prows, J0.n_rows);
                    for (int r = pr0 + static_cast<int>(threadIdx.x); r < r1; r += 32 * kConsumerWarps) {
                        const float gv = pair_out[r - pr0], uv = pair_out[prows + r - pr0];
                        P.act[r] = __fmul_rn(silu_f(gv), uv);
                        J0.out[r] = gv;
                        out1[r] = uv;
                    }
                }
            }
        }
        stamp(p, p.first + k, 2);
        stamp_cta(p, p.first + k);
        if (ok && k + 1 < p.count) ok = step_grid_barrier(p, static_cast<unsigned>(k + 1));
        stamp(p, p.first + k, 3);
        if (!ok) *abort_flag = 1;
    }
    pdl_launch_dependents();  // the next kernel may be scheduled; it waits for this one to finish
    if (threadIdx.x == 0) {
        bulk_wait_all();  // the last state store has completed
        // the last CTA to leave resets the counters for the next launch
        __threadfence();
        if (atomicAdd(p.bar + kStepBarExit, 1u) == gridDim.x - 1) {
            p.bar[0] = 0u;
            p.bar[kStepBarExit] = 0u;
            __threadfence();
        }
    }
}

}  // namespace qh

// ---------------------------------------------------------------------------
// Host side: program creation and launch.
// ---------------------------------------------------------------------------
struct qh_step_prog {
    int dev = 0, sms = 0, smem = 0;
    qh::StepParams base = {};
    qh::StepPhase *d_phases = nullptr;
    qh::StepJob *d_jobs = nullptr;
    qh::StepGdn *d_gdns = nullptr;
    qh::StepAttn *d_attns = nullptr;
    unsigned *d_bar = nullptr;
    int nphases = 0;
};

namespace {
int step_bad(const char *what) {
    qh::set_last_error_message(what);
    return QH_ERR_INVALID;
}
int step_cuda(cudaError_t e, const char *what) {
    cudaGetLastError();
    char msg[256];
    snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
    qh::set_last_error_message(msg);
    return QH_ERR_CUDA;
}
bool a16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

extern "C" {

int qh_step_create(const qh_step_phase *phases, int32_t n_phases, const int32_t *d_pos, qh_step_prog **out) {
    using namespace qh;
    if (!phases || n_phases <= 0 || !d_pos || !out) return step_bad("qh_step_create: bad arguments");
    *out = nullptr;
    int dev = 0, sms = 0, optin = 0, coop = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return step_cuda(e, "cudaGetDevice");
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev)) != cudaSuccess)
        return step_cuda(e, "cudaDeviceGetAttribute");
    if (!coop) {
        set_last_error_message("qh_step_create: the device has no cooperative launch");
        return QH_ERR_UNSUPPORTED;
    }
    int *err = device_error_word();
    if (!err) return step_bad("qh_step_create: no device error word");
    std::vector<StepPhase> hp(static_cast<size_t>(n_phases));
    std::vector<StepJob> hj;
    std::vector<StepGdn> hg;
    std::vector<StepAttn> ha;
    int64_t max_x = 0, max_row = 0, max_res_k = 0, max_norm_k = 0;
    int64_t aux_bytes = 0;  // DeltaNet state and attention scratch share one region
    for (int k = 0; k < n_phases; ++k) {
        const qh_step_phase &ph = phases[k];
        StepPhase P = {};
        P.kind = ph.kind;
        P.gdn = -1;
        if (ph.kind == QH_STEP_ATTN) {
            if (!ph.d_qraw || !ph.d_kin || !ph.d_vin || !ph.d_qnorm_w || !ph.d_knorm_w || !ph.d_rope ||
                !ph.d_kcache || !ph.d_vcache || !ph.d_ctx || ph.n_heads <= 0 || ph.n_kv_heads <= 0 ||
                ph.n_heads % ph.n_kv_heads || ph.n_heads > sms || ph.rope_dim < 0 || ph.rope_dim > kStepHD ||
                ph.rope_dim % 2 || ph.max_pos <= 0 || !a16(ph.d_kcache) || !a16(ph.d_vcache))
                return step_bad("qh_step_create: bad attention phase");
            if (ph.max_pos > QH_STEP_ATTN_MAX_POS) {
                set_last_error_message("qh_step_create: attention cache longer than QH_STEP_ATTN_MAX_POS");
                return QH_ERR_UNSUPPORTED;
            }
            if (ph.head_dim != kStepHD) {
                set_last_error_message("qh_step_create: attention head dim must be 128");
                return QH_ERR_UNSUPPORTED;
            }
            StepAttn a = {ph.d_qraw, ph.d_kin, ph.d_vin, ph.d_qnorm_w, ph.d_knorm_w, ph.d_rope,
                          reinterpret_cast<__half *>(ph.d_kcache), reinterpret_cast<__half *>(ph.d_vcache), ph.d_ctx,
                          ph.n_heads, ph.n_kv_heads, ph.rope_dim, ph.max_pos, ph.eps};
            P.kind = kPhaseAttn;
            P.gdn = static_cast<int32_t>(ha.size());
            ha.push_back(a);
            aux_bytes = std::max<int64_t>(aux_bytes, attn_scratch_bytes(ph.max_pos));
            hp[static_cast<size_t>(k)] = P;
            continue;
        }
        if (ph.kind == QH_STEP_GDN) {
            // a DeltaNet phase's state is copied in during the phase before it,
            // into one region per CTA: two in a row are refused
            if (k > 0 && (phases[k - 1].kind == QH_STEP_GDN || phases[k - 1].kind == QH_STEP_ATTN))
                return step_bad("qh_step_create: a DeltaNet phase directly after a DeltaNet or attention phase");
            if (!ph.d_qkv || !ph.d_ring || !ph.d_conv_w || !ph.d_b || !ph.d_a || !ph.d_dt_bias || !ph.d_ssm_a ||
                !ph.d_state || !ph.d_z || !ph.d_norm_w || !ph.d_y || ph.heads <= 0 || ph.heads > sms ||
                !a16(ph.d_state) || !a16(ph.d_ring) || !a16(ph.d_conv_w))
                return step_bad("qh_step_create: bad DeltaNet phase");
            if (ph.conv_kernel != kStepTaps) {
                set_last_error_message("qh_step_create: DeltaNet conv kernel must be 4");
                return QH_ERR_UNSUPPORTED;
            }
            if (ph.head_dim != kStepHD) {
                set_last_error_message("qh_step_create: DeltaNet head dim must be 128");
                return QH_ERR_UNSUPPORTED;
            }
            StepGdn g = {ph.d_qkv, ph.d_ring, ph.d_conv_w, ph.d_b, ph.d_a, ph.d_dt_bias, ph.d_ssm_a, ph.d_state,
                         ph.d_z, ph.d_norm_w, ph.d_y, ph.heads, ph.conv_kernel, ph.eps};
            P.kind = kPhaseGdn;
            P.gdn = static_cast<int32_t>(hg.size());
            hg.push_back(g);
            aux_bytes = std::max<int64_t>(aux_bytes, kStepGdnBytes);
            hp[static_cast<size_t>(k)] = P;
            continue;
        }
        if (ph.kind != QH_STEP_MATVEC) return step_bad("qh_step_create: bad phase kind");
        const int64_t K = ph.xk;
        if (ph.n_proj <= 0 || ph.n_proj > QH_STEP_MAX_PROJ || K <= 0 || K % QH_QK || !ph.d_xa ||
            ph.xform < QH_STEP_X_RESNORM || ph.xform > QH_STEP_X_QUANT || (ph.xform == QH_STEP_X_SWIGLU && !ph.d_xb) ||
            (ph.xform == QH_STEP_X_RESNORM && !ph.d_xw) || (ph.xform != QH_STEP_X_QUANT && K > kFuseMaxBlocks * QH_QK) ||
            !a16(ph.d_xa) ||
            (ph.d_xb && !a16(ph.d_xb)))
            return step_bad("qh_step_create: bad projection phase");
        P.kind = kPhaseMatvec;
        P.xform = ph.xform;
        P.xk = static_cast<int32_t>(K);
        P.eps = ph.eps;
        P.xa = ph.d_xa;
        P.xb = ph.d_xb;
        P.xw = ph.d_xw;
        P.xh_out = ph.d_xh_out;
        P.act = ph.d_act_out;
        if (ph.d_act_out &&
            (ph.n_proj != 2 || ph.proj[0].out_f != ph.proj[1].out_f || !a16(ph.d_act_out)))
            return step_bad("qh_step_create: a SwiGLU output needs two projections of one shape");
        P.job0 = static_cast<int32_t>(hj.size());
        P.njobs = ph.n_proj;
        int64_t total_rows = 0, prow = 0, max_nb = 0;
        for (int q = 0; q < ph.n_proj; ++q) {
            const qh_step_proj &pr = ph.proj[q];
            if (pr.type != QH_GGUF_Q4_K && pr.type != QH_GGUF_Q5_K && pr.type != QH_GGUF_Q6_K) {
                set_last_error_message("qh_step_create: projection weights must be Q4_K, Q5_K or Q6_K");
                return QH_ERR_UNSUPPORTED;
            }
            if (!pr.d_w || !pr.d_out || pr.k != K || pr.out_f <= 0 || pr.out_f > (1 << 24) || !a16(pr.d_w))
                return step_bad("qh_step_create: bad projection");
            StepJob J = {};
            J.w = static_cast<const uint8_t *>(pr.d_w);
            J.out = pr.d_out;
            J.type = pr.type;
            J.n_rows = static_cast<int32_t>(pr.out_f);
            J.nb = static_cast<int32_t>(K / QH_QK);
            J.row_bytes = static_cast<int32_t>(qhf_row_bytes(pr.type, K));
            J.k = static_cast<int32_t>(K);
            J.d_stride = static_cast<int32_t>(qhf_q8k_d_stride(K));
            hj.push_back(J);
            total_rows += pr.out_f;
            prow = std::max<int64_t>(prow, J.row_bytes);
            max_nb = std::max<int64_t>(max_nb, J.nb);
        }
        max_row = std::max(max_row, prow);
        // residual row + norm weights (RMSNorm) or the SwiGLU row, as fp32
        if (ph.xform == QH_STEP_X_RESNORM) {
            max_res_k = std::max<int64_t>(max_res_k, K);
            max_norm_k = std::max<int64_t>(max_norm_k, K);
            if (!a16(ph.d_xw)) return step_bad("qh_step_create: RMSNorm weights not 16-byte aligned");
        }
        if (ph.xform == QH_STEP_X_SWIGLU) max_res_k = std::max<int64_t>(max_res_k, K);
        max_x = std::max<int64_t>(max_x, K + (K / QH_QK) * 32 + qhf_q8k_d_stride(K) * 4);
        // rows per tile and split decided below, once the ring size is known
        P.total_tiles = static_cast<int32_t>(total_rows);  // rows for now
        P.split = static_cast<int32_t>(max_nb);           // max blocks for now
        P.rows_per_tile = static_cast<int32_t>(prow);     // max row bytes for now
        hp[static_cast<size_t>(k)] = P;
    }
    // shared-memory plan: header, activation planes, residual row, split
    // terms, DeltaNet state, then the ring
    const int64_t x_bytes = (max_x + 127) / 128 * 128;
    // (a paired phase keeps at most kStepPairFloats gate/up outputs per CTA
    // there too: checked below, once its rows per tile are known)
    const int64_t row_bytes = (std::max<int64_t>(max_res_k, kStepPairFloats) * 4 + 127) / 128 * 128;
    const int64_t x_off = kStepHeader, row_off = x_off + x_bytes, terms_off = row_off + row_bytes;
    const int64_t w_off = terms_off + kStepTerms, w_floats = (max_norm_k + 31) / 32 * 32;
    const int64_t state_off = w_off + 2 * w_floats * 4;
    const int64_t ring_off = (state_off + aux_bytes + 127) / 128 * 128;
    // dynamic shared memory: the opt-in maximum less the kernel's static arrays
    cudaFuncAttributes fa = {};
    if ((e = cudaFuncGetAttributes(&fa, step_kernel)) != cudaSuccess) return step_cuda(e, "cudaFuncGetAttributes");
    const int64_t dyn = (static_cast<int64_t>(optin) - static_cast<int64_t>(fa.sharedSizeBytes)) / 128 * 128;
    const int64_t ring_bytes = (dyn - ring_off) / 128 * 128;
    if (ring_bytes < 4 * 8 * max_row + 512) return step_bad("qh_step_create: rows too long for the tile ring");
    for (int k = 0; k < n_phases; ++k) {
        StepPhase &P = hp[static_cast<size_t>(k)];
        if (P.kind != kPhaseMatvec) continue;
        const int64_t total_rows = P.total_tiles, prow = P.rows_per_tile, max_nb = P.split;
        // tiles of 8 rows (one consumer warp each) unless a launch has many
        // rows per CTA; at least four tiles fit the ring
        const int64_t r_cap = std::max<int64_t>(8, ((ring_bytes / 4 - 256) / prow) / 8 * 8);
        const int64_t r_bal = (total_rows / (4 * static_cast<int64_t>(sms))) / 8 * 8;
        const int64_t R = std::min<int64_t>(std::min(r_cap, std::max<int64_t>(8, r_bal)), 8 * kGroupRows);
        int64_t tiles = 0;
        for (int q = 0; q < P.njobs; ++q) {
            StepJob &J = hj[static_cast<size_t>(P.job0 + q)];
            J.tile_begin = static_cast<int32_t>(tiles);
            J.n_tiles = static_cast<int32_t>((J.n_rows + R - 1) / R);
            tiles += J.n_tiles;
        }
        P.rows_per_tile = static_cast<int32_t>(R);
        P.total_tiles = static_cast<int32_t>(tiles);
        P.split = (!P.act && R == 8 && tiles <= sms && max_nb > 1 && 8 * max_nb <= kStepTermsFloats) ? 1 : 0;
        if (P.act && 2 * ((tiles / 2 + sms - 1) / sms) * R > kStepPairFloats)
            return step_bad("qh_step_create: a SwiGLU phase has too many rows per CTA");
    }
    qh_step_prog *prog = new qh_step_prog();
    prog->dev = dev;
    prog->sms = sms;
    prog->smem = static_cast<int>(dyn);
    prog->nphases = n_phases;
    auto cleanup = [&]() { qh_step_destroy(prog); };
    if ((e = cudaMalloc(&prog->d_phases, hp.size() * sizeof(StepPhase))) != cudaSuccess ||
        (e = cudaMalloc(&prog->d_jobs, std::max<size_t>(1, hj.size()) * sizeof(StepJob))) != cudaSuccess ||
        (e = cudaMalloc(&prog->d_gdns, std::max<size_t>(1, hg.size()) * sizeof(StepGdn))) != cudaSuccess ||
        (e = cudaMalloc(&prog->d_attns, std::max<size_t>(1, ha.size()) * sizeof(StepAttn))) != cudaSuccess ||
        (e = cudaMalloc(&prog->d_bar, (kStepBarExit + 32) * sizeof(unsigned))) != cudaSuccess) {
        cleanup();
        return step_cuda(e, "qh_step_create: cudaMalloc");
    }
    if ((e = cudaMemcpy(prog->d_phases, hp.data(), hp.size() * sizeof(StepPhase), cudaMemcpyHostToDevice)) !=
            cudaSuccess ||
        (!hj.empty() &&
         (e = cudaMemcpy(prog->d_jobs, hj.data(), hj.size() * sizeof(StepJob), cudaMemcpyHostToDevice)) !=
             cudaSuccess) ||
        (!hg.empty() &&
         (e = cudaMemcpy(prog->d_gdns, hg.data(), hg.size() * sizeof(StepGdn), cudaMemcpyHostToDevice)) !=
             cudaSuccess) ||
        (!ha.empty() &&
         (e = cudaMemcpy(prog->d_attns, ha.data(), ha.size() * sizeof(StepAttn), cudaMemcpyHostToDevice)) !=
             cudaSuccess) ||
        (e = cudaMemset(prog->d_bar, 0, (kStepBarExit + 32) * sizeof(unsigned))) != cudaSuccess) {
        cleanup();
        return step_cuda(e, "qh_step_create: upload");
    }
    if ((e = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, prog->smem)) !=
        cudaSuccess) {
        cleanup();
        return step_cuda(e, "qh_step_create: cudaFuncSetAttribute");
    }
    int per_sm = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel, kStepThreads, prog->smem)) !=
            cudaSuccess ||
        per_sm < 1) {
        cleanup();
        if (e != cudaSuccess) return step_cuda(e, "qh_step_create: occupancy");
        set_last_error_message("qh_step_create: the step kernel does not fit an SM");
        return QH_ERR_UNSUPPORTED;
    }
    StepParams &b = prog->base;
    b.phases = prog->d_phases;
    b.jobs = prog->d_jobs;
    b.gdns = prog->d_gdns;
    b.attns = prog->d_attns;
    b.ring_bytes = static_cast<int32_t>(ring_bytes);
    b.ring_off = static_cast<int32_t>(ring_off);
    b.x_off = static_cast<int32_t>(x_off);
    b.row_off = static_cast<int32_t>(row_off);
    b.terms_off = static_cast<int32_t>(terms_off);
    b.state_off = static_cast<int32_t>(state_off);
    b.w_off = static_cast<int32_t>(w_off);
    b.w_floats = static_cast<int32_t>(w_floats);
    b.pos_ptr = d_pos;
    b.bar = prog->d_bar;
    b.err_flag = err;
    b.test_tile = -1;
    b.wait_limit = 0;
    *out = prog;
    return QH_OK;
}

int qh_step_run(qh_step_prog *prog, int32_t first, int32_t count, void *stream) {
    using namespace qh;
    if (!prog || first < 0 || count <= 0 || first + count > prog->nphases)
        return step_bad("qh_step_run: bad arguments");
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != prog->dev) return step_bad("qh_step_run: program made on another device");
    StepParams p = prog->base;
    p.first = first;
    p.count = count;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(prog->sms));
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(prog->smem);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, step_kernel, p);
    if (e != cudaSuccess) return step_cuda(e, "qh_step_run");
    return QH_OK;
}

int qh_step_set_stamps(qh_step_prog *prog, uint64_t *d_stamps) {
    if (!prog) return step_bad("qh_step_set_stamps: bad arguments");
    prog->base.stamps = d_stamps;
    return QH_OK;
}

int32_t qh_step_phase_count(const qh_step_prog *prog) { return prog ? prog->nphases : -1; }

int qh_step_test_timeout(qh_step_prog *prog, int32_t tile, uint32_t wait_limit) {
    if (!prog || tile < -1) return step_bad("qh_step_test_timeout: bad arguments");
    prog->base.test_tile = tile;
    prog->base.wait_limit = wait_limit;
    return QH_OK;
}

void qh_step_destroy(qh_step_prog *prog) {
    if (!prog) return;
    if (prog->d_phases) cudaFree(prog->d_phases);
    if (prog->d_jobs) cudaFree(prog->d_jobs);
    if (prog->d_gdns) cudaFree(prog->d_gdns);
    if (prog->d_attns) cudaFree(prog->d_attns);
    if (prog->d_bar) cudaFree(prog->d_bar);
    delete prog;
}

}  // extern "C"
