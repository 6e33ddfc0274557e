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
#include "qh_gemv_dev.cuh"

namespace qh {

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
