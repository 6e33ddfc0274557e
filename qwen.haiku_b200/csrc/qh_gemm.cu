// SPDX-License-Identifier: MIT
//
// qh_gemm.cu -- K-quant x Q8_K matmul for many tokens on the 5th-generation
// tensor cores (tcgen05.mma kind::i8, accumulators in TMEM), bit-exact with
// the reference's per-row dots (simd/quants.h:267-402) and its per-block
// fp32 combination (the sequential sumf += ... of tensor_matmul_*_f32,
// slm/tensor.c:827-1033).
//
// The integer part of one super-block (256 weights) is an exact integer dot
// that the tensor core computes, once the weights are expanded in shared
// memory into int8 "planes" whose dot with the int8 activations gives the
// reference's integers:
//   Q4_K / Q5_K: a_p = scale[sb(p)] * w_p  (<= 63 * 31) split as
//                a_p = 128 * hi_p + lo_p  (hi, lo in [0, 127]); a third plane
//                holds min[sb(p)], whose dot with the activations is
//                sum_sb min[sb] * (bsums[2sb] + bsums[2sb+1]) = isum_mins.
//                isum = 128 * (hi . x) + (lo . x).
//   Q6_K:        a_p = scale[p/16] * (w_p - 32) split the same way (hi
//                signed); 128 * (hi . x) + (lo . x) = isum - 32 * isum_mins,
//                the integer the reference scales.
// Per super-block the accumulators are read back from TMEM and combined in
// fp32 exactly as the reference does, in block order.
//
// Operands (no-swizzle K-major canonical layout, see qh_tc.cuh):
//   A  128 weight rows x 256 per plane, built by the CUDA cores from the
//      raw GGUF blocks;
//   B  64 tokens x 256 int8 activations, the tiled Q8_K layout
//      (qh_formats.h) copied as one 16 KB bulk transfer per super-block.
// Weights are read in the "tiled" order [row tile][block][128 rows][block
// bytes] (qh_gemm_pack_weights), so one super-block of a row tile is one
// contiguous bulk copy.
//
// CTA: 4 expander warps (one also issues the MMAs), 4 epilogue warps and
// 1 producer warp (bulk copies into a 3-stage ring), one CTA per SM,
// persistent over (row tile, token tile) work items.

#include <cuda_runtime.h>
#include <stdio.h>

#include <algorithm>

#include "../../include/qh_backend.h"
#include "qh_common.cuh"
#include "qh_internal.h"
#include "qh_q8k.cuh"
#include "qh_tc.cuh"

namespace qh {

constexpr int kGemmRows = 128;           // MMA M: weight rows per tile
constexpr int kGemmTok = QH_Q8KT_TILE;   // MMA N: tokens per tile (64)
constexpr int kExpWarps = 8;             // expanders: 2 threads per weight row
constexpr int kEpiWarps = 8;             // epilogue: 4 lane groups x 2 token halves
// Warp roles: [expanders][epilogue][producer][MMA]; with expanded weights
// there are no expanders and the CTA is 10 warps.
__host__ __device__ constexpr int gemm_exp_warps(bool exp) { return exp ? 0 : kExpWarps; }
__host__ __device__ constexpr int gemm_threads(bool exp) { return 32 * (gemm_exp_warps(exp) + kEpiWarps + 2); }
constexpr int kGemmMaxJobs = 8;
constexpr int kGemmMaxStages = 4;
constexpr int kPlaneBytes = kGemmRows * QH_QK;  // 32 KB: one int8 operand plane
constexpr int kMinRowBytes = kGemmRows * 16;    // 2 KB: min operand (first K chunk)
constexpr int kGemmHeader = 1024;
constexpr int kGemmSmemMax = 232448;            // 227 KB per CTA
constexpr uint32_t kAccCols = 256;              // one accumulator set
constexpr int kRing = 4;                        // scale ring depth (blocks)
constexpr int kSpreadDone = 512;                // split-K: second counter of tile t at tickets[512 + t]
constexpr int kSpreadMaxNb = 16;                // spread reduction: at most 16 blocks per tile
constexpr int kSpreadPerThread = 4;             // ... and 4 elements per epilogue thread
constexpr uint64_t kSpreadWaitNs = 2000000000ull;  // wait for the tile's other chunks: 2 s

__device__ __forceinline__ uint64_t gemm_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned gemm_ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct GemmJob {
    const uint8_t *wt;  // tiled weights
    float *out;         // [n_tok][ldo]
    int32_t n_rows;
    int32_t m_tiles;
    int32_t tile_begin;  // first global row tile of this job
    int32_t ldo;
};

struct GemmParams {
    int32_t n_jobs, total_items, nb, n_tok, t_tiles, n_stages;
    int32_t kchunks, kc_blocks;  // split of the super-blocks of one output tile over CTAs
    int32_t spread;              // split-K: every chunk's CTA sums a slice of the tile (all resident)
    int32_t w_early;             // weights complete before the previous kernel: stream them before pdl_wait
    const uint8_t *xq;           // tiled Q8_K activations
    float *terms;                // split-K: per-block fp32 terms [tile][block][64 tokens][128 rows]
    unsigned *tickets;           // split-K: arrivals per output tile, then (spread) readers done at
                                 // kSpreadDone + tile (all left at zero)
    int *err_flag;
    GemmJob jobs[kGemmMaxJobs];
};

// Per type: GGUF block bytes, padded row-block bytes in the tiled weights
// (16-byte multiple), operand planes (hi, lo) and whether the min operand
// is used.
template <int TYPE>
struct KQ;
template <>
struct KQ<QH_GGUF_Q4_K> {
    static constexpr int kBytes = QH_Q4K_BYTES, kPadded = 144, kMins = 1;
};
template <>
struct KQ<QH_GGUF_Q5_K> {
    static constexpr int kBytes = QH_Q5K_BYTES, kPadded = 176, kMins = 1;
};
template <>
struct KQ<QH_GGUF_Q6_K> {
    static constexpr int kBytes = QH_Q6K_BYTES, kPadded = 224, kMins = 0;
};

__host__ __device__ constexpr int padded_block_bytes(int type) {
    return type == QH_GGUF_Q4_K ? 144 : type == QH_GGUF_Q5_K ? 176 : type == QH_GGUF_Q6_K ? 224 : 0;
}

__device__ __forceinline__ void put16(uint8_t *plane, int c, int r, uint32_t a, uint32_t b, uint32_t cc,
                                      uint32_t d) {
    *reinterpret_cast<uint4 *>(plane + c * (kGemmRows * 16) + r * 16) = make_uint4(a, b, cc, d);
}

// Q4_K/Q5_K scale and min of sub-block sb (q4k_get_scale_min,
// simd/quants.h:215-224).
__device__ __forceinline__ void scale_min(const uint8_t *s12, int sb, int &sc, int &mn) {
    if (sb < 4) {
        sc = s12[sb] & 0x3f;
        mn = s12[sb + 4] & 0x3f;
    } else {
        sc = (s12[sb + 4] & 0x0f) | ((s12[sb - 4] >> 6) << 4);
        mn = (s12[sb + 4] >> 4) | ((s12[sb] >> 6) << 4);
    }
}

// 4 weights (bytes of w) times a non-negative scale (products < 2^16),
// split into lo = a & 127 and hi = a >> 7 bytes.
// Products a < 2^11, so (a >> 7) fits the low byte of each lane and the
// byte interleave (byte_perm) needs no masking for hi.
__device__ __forceinline__ void split_pos(uint32_t w, uint32_t sc, uint32_t &hi, uint32_t &lo) {
    const uint32_t p02 = (w & 0x00ff00ffu) * sc;
    const uint32_t p13 = ((w >> 8) & 0x00ff00ffu) * sc;
    lo = __byte_perm(p02, p13, 0x6240u) & 0x7f7f7f7fu;
    hi = __byte_perm(p02 >> 7, p13 >> 7, 0x6240u);
}

// Expansion of half h (weights 128h..128h+127) of row r's super-block into
// the hi/lo planes (and, for h == 0, the row's min-operand entries).
template <int TYPE>
__device__ __forceinline__ void expand(const uint8_t *raw, int h, int r, uint8_t *planes);

template <>
__device__ __forceinline__ void expand<QH_GGUF_Q4_K>(const uint8_t *raw, int h, int r, uint8_t *planes) {
    const uint8_t *s12 = raw + 4;
    uint32_t mins[2] = {0u, 0u};
#pragma unroll
    for (int cl = 0; cl < 8; ++cl) {
        const int c = 8 * h + cl, sb = c >> 1;
        int sc, mn;
        scale_min(s12, sb, sc, mn);
        const uint4 q = *reinterpret_cast<const uint4 *>(raw + 16 + 32 * (c >> 2) + 16 * (c & 1));
        const uint32_t sh = 4u * ((c >> 1) & 1);
        uint32_t hi[4], lo[4];
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) split_pos((qw[k] >> sh) & 0x0f0f0f0fu, static_cast<uint32_t>(sc), hi[k], lo[k]);
        put16(planes, c, r, hi[0], hi[1], hi[2], hi[3]);
        put16(planes + kPlaneBytes, c, r, lo[0], lo[1], lo[2], lo[3]);
    }
    if (h == 0) {
#pragma unroll
        for (int sb = 0; sb < 8; ++sb) {
            int sc, mn;
            scale_min(s12, sb, sc, mn);
            mins[sb >> 2] |= static_cast<uint32_t>(mn) << (8 * (sb & 3));
        }
        *reinterpret_cast<uint4 *>(planes + 2 * kPlaneBytes + r * 16) = make_uint4(mins[0], mins[1], 0u, 0u);
    }
}

template <>
__device__ __forceinline__ void expand<QH_GGUF_Q5_K>(const uint8_t *raw, int h, int r, uint8_t *planes) {
    const uint8_t *s12 = raw + 4;
    uint32_t mins[2] = {0u, 0u};
#pragma unroll
    for (int cl = 0; cl < 8; ++cl) {
        const int c = 8 * h + cl, sb = c >> 1;
        int sc, mn;
        scale_min(s12, sb, sc, mn);
        const uint4 q = *reinterpret_cast<const uint4 *>(raw + 48 + 32 * (c >> 2) + 16 * (c & 1));
        const uint4 qh = *reinterpret_cast<const uint4 *>(raw + 16 + 16 * (c & 1));
        const uint32_t sh = 4u * ((c >> 1) & 1);
        uint32_t hi[4], lo[4];
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ((qw[k] >> sh) & 0x0f0f0f0fu) | (((hw[k] >> sb) & 0x01010101u) << 4);
            split_pos(w, static_cast<uint32_t>(sc), hi[k], lo[k]);
        }
        put16(planes, c, r, hi[0], hi[1], hi[2], hi[3]);
        put16(planes + kPlaneBytes, c, r, lo[0], lo[1], lo[2], lo[3]);
    }
    if (h == 0) {
#pragma unroll
        for (int sb = 0; sb < 8; ++sb) {
            int sc, mn;
            scale_min(s12, sb, sc, mn);
            mins[sb >> 2] |= static_cast<uint32_t>(mn) << (8 * (sb & 3));
        }
        *reinterpret_cast<uint4 *>(planes + 2 * kPlaneBytes + r * 16) = make_uint4(mins[0], mins[1], 0u, 0u);
    }
}

// Q6_K: a = sc * (w - 32), computed as u = a + 4096 in non-negative 16-bit
// lanes (no carries or borrows cross lanes for |sc| <= 128, w <= 63); then
// lo = u & 127 and hi = (u >> 7) - 32 = floor(a / 128). Rows are padded to
// 224 bytes in the tiled weights, so every field is 16-byte aligned.
template <>
__device__ __forceinline__ void expand<QH_GGUF_Q6_K>(const uint8_t *raw, int h, int r, uint8_t *planes) {
    const uint4 scv = *reinterpret_cast<const uint4 *>(raw + 192);
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
    for (int cl = 0; cl < 8; ++cl) {
        const int c = 8 * h + cl, rq = (c >> 1) & 3, l0 = 16 * (c & 1);
        const uint4 ql = *reinterpret_cast<const uint4 *>(raw + 64 * h + 32 * (rq & 1) + l0);
        const uint4 qh = *reinterpret_cast<const uint4 *>(raw + 128 + 32 * h + l0);
        const int sc = static_cast<int8_t>((scw[c >> 2] >> (8 * (c & 3))) & 0xffu);
        const uint32_t lsh = 4u * static_cast<uint32_t>(rq >> 1), hsh = 2u * static_cast<uint32_t>(rq);
        const uint32_t a = static_cast<uint32_t>(sc < 0 ? -sc : sc);
        const uint32_t cst = static_cast<uint32_t>(sc < 0 ? 4096 + 32 * (-sc) : 4096 - 32 * sc);
        const uint32_t c2 = cst | (cst << 16);
        const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w};
        const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ((lw[k] >> lsh) & 0x0f0f0f0fu) | (((hw[k] >> hsh) & 0x03030303u) << 4);
            const uint32_t w02 = (w & 0x00ff00ffu) * a, w13 = ((w >> 8) & 0x00ff00ffu) * a;
            const uint32_t u02 = sc < 0 ? c2 - w02 : c2 + w02;
            const uint32_t u13 = sc < 0 ? c2 - w13 : c2 + w13;
            // u < 2^14: (u >> 7) fits the low byte of each lane
            lo[k] = __byte_perm(u02, u13, 0x6240u) & 0x7f7f7f7fu;
            hi[k] = __vsub4(__byte_perm(u02 >> 7, u13 >> 7, 0x6240u), 0x20202020u);
        }
        put16(planes, c, r, hi[0], hi[1], hi[2], hi[3]);
        put16(planes + kPlaneBytes, c, r, lo[0], lo[1], lo[2], lo[3]);
    }
}

// Work item -> (job, row tile mt, token tile tt, output tile index, block
// range [b0, b1)). The k-chunks of one output tile are consecutive items.
struct Item {
    GemmJob job;
    int mt, tt, tile, b0, b1;
};
__device__ __forceinline__ Item decode_item(const GemmParams &p, int item) {
    Item it;
    const int kc = item % p.kchunks;
    it.tile = item / p.kchunks;
    const int g = it.tile / p.t_tiles;
    it.tt = it.tile - g * p.t_tiles;
    int j = 0;
    while (j + 1 < p.n_jobs && g >= p.jobs[j + 1].tile_begin) ++j;
    it.job = p.jobs[j];
    it.mt = g - it.job.tile_begin;
    it.b0 = kc * p.kc_blocks;
    it.b1 = min(p.nb, it.b0 + p.kc_blocks);
    return it;
}

// Expanded weights (qh_gemm_expand_weights): per (row tile, block) the A
// operand exactly as the expander warps build it -- hi plane, lo plane, min
// rows (Q4_K/Q5_K) -- followed by the rows' (d, dmin) as float2[128].
template <int TYPE>
struct ExpBlock {
    static constexpr int kA = 2 * kPlaneBytes + (KQ<TYPE>::kMins ? kMinRowBytes : 0);
    static constexpr int kBytes = kA + kGemmRows * 8;
};
__host__ __device__ constexpr int expanded_block_bytes(int type) {
    return type == QH_GGUF_Q6_K ? 2 * kPlaneBytes + kGemmRows * 8 : 2 * kPlaneBytes + kMinRowBytes + kGemmRows * 8;
}

// Shared-memory plan of one CTA (offsets from the dynamic smem base). EXP:
// the stages hold expanded weights and the MMAs read A from the stage (no
// A buffers, no expansion).
template <int TYPE, bool EXP = false>
struct GemmSmem {
    static constexpr int kWB = EXP ? ExpBlock<TYPE>::kBytes : kGemmRows * KQ<TYPE>::kPadded;  // weight tile block
    static constexpr int kXB = KQ<TYPE>::kMins ? QH_Q8KT_BLOCK_BYTES : QH_Q8KT_MIN_OFF;  // activation bytes copied
    static constexpr int kStage = kWB + kXB;
    static constexpr int kABuf = 2 * kPlaneBytes + (KQ<TYPE>::kMins ? kMinRowBytes : 0);
    static constexpr int kA = kGemmHeader;                                       // 2 A buffers (not EXP)
    static constexpr int kScales = kA + (EXP ? 0 : 2 * kABuf);                   // ring of token scales
    static constexpr int kRowScales = kScales + kRing * kGemmTok * 4;            // ring of row (d, dmin)
    static constexpr int kStages = kRowScales + kRing * kGemmRows * 8;           // stage ring
    static constexpr int kNStages = (kGemmSmemMax - kStages - kMinRowBytes) / kStage > kGemmMaxStages
                                        ? kGemmMaxStages
                                        : (kGemmSmemMax - kStages - kMinRowBytes) / kStage;
    // 2 KB of zeros after the stages: the second K chunk of both min
    // operands (a positive leading-dimension offset from either).
    static constexpr int kZero = kStages + kNStages * kStage;
    static constexpr int kTotal = kZero + kMinRowBytes;
    static_assert(kNStages >= 2 && kTotal <= kGemmSmemMax, "shared memory plan");
};

// Warp roles (576 threads, one CTA per SM; with expanded weights, EXP, the
// expanders are absent -- 320 threads, epilogue warps 0-7, producer 8, MMA 9 --
// and the MMAs read A straight from the stage, whose row scales the MMA warp
// moves to the ring before the stage is released):
//   warps 0-7   expanders: two threads per weight row build the A planes
//               of a super-block into one of two A buffers and copy its
//               scales to a small ring;
//   warps 8-15  epilogue: thread = (weight row, half of the token tile);
//               reads the accumulators, combines in fp32, stores;
//   warp 16     producer: one bulk copy each of the weight tile block and
//               the activation tile block per super-block;
//   warp 17     one thread issues the MMAs of each block.
// A buffers and TMEM accumulators are double-buffered, so the expansion of
// block b+1, the MMAs of block b and the epilogue of block b-1 overlap.
// mbarriers: full[s] (copies landed), empty[s] (block's MMAs done with the
// stage), mma_done[2] (MMAs of a block completed: its A buffer is free, its
// accumulators readable), acc_empty[2] (8 epilogue warps read them),
// a_ready[2] (8 expander warps wrote a block's A buffer and scales),
// scale_ready[2] (the MMA thread passes the scales on to the epilogue).
template <int TYPE, bool EXP, bool SPREAD>
__global__ void __launch_bounds__(gemm_threads(EXP), 1) gemm_kernel(const __grid_constant__ GemmParams p) {
    using L = GemmSmem<TYPE, EXP>;
    constexpr int XW = gemm_exp_warps(EXP), kProducerWarp = XW + kEpiWarps, kMmaWarp = kProducerWarp + 1;
    constexpr int kGemmThreads = gemm_threads(EXP);
    constexpr int BBP = KQ<TYPE>::kPadded, MINS = KQ<TYPE>::kMins;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kGemmMaxStages;
    uint64_t *mma_done = empty + kGemmMaxStages;
    uint64_t *acc_empty = mma_done + 2;
    uint64_t *scale_ready = acc_empty + 2;
    uint64_t *a_ready = scale_ready + 2;
    uint64_t *xfull = a_ready + 2;  // activation part of a stage landed (full[] covers the weights)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 256);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 260);
    float *tok_scale = reinterpret_cast<float *>(smem + L::kScales);     // [kRing][64]
    float2 *row_scale = reinterpret_cast<float2 *>(smem + L::kRowScales);  // [kRing][128]
    uint8_t *zero = smem + L::kZero;
    uint8_t *stages = smem + L::kStages;

    constexpr int S = L::kNStages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&xfull[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&mma_done[b], 1);
            mbar_init(&acc_empty[b], kEpiWarps);
            mbar_init(&scale_ready[b], 1);
            mbar_init(&a_ready[b], kExpWarps);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    for (int i = tid; i < kMinRowBytes / 16; i += kGemmThreads)
        reinterpret_cast<uint4 *>(zero)[i] = make_uint4(0u, 0u, 0u, 0u);
    // A CTA of this kernel never shares an SM with another one (shared
    // memory), so the TMEM it allocates is free even while the previous
    // kernel runs. Only the producer waits for earlier kernels (before the
    // first activation copy, or before any copy unless p.w_early); every other
    // global access of the kernel follows an activation copy.
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, 2 * kAccCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == kProducerWarp) {
        // ----- producer -----
        if (lane == 0) {
            int i = 0;
            bool stop = false, waited = !p.w_early;
            if (waited) pdl_wait();
            const uint8_t *xpend[kGemmMaxStages];  // activation blocks of the first ring, issued after the wait
            auto issue_x = [&](int s2, const uint8_t *src) {
                mbar_arrive_expect_tx(&xfull[s2], L::kXB);
                bulk_copy_g2s(stages + static_cast<int64_t>(s2) * L::kStage + L::kWB, src, L::kXB, &xfull[s2]);
            };
            for (int item = blockIdx.x; item < p.total_items && !stop; item += gridDim.x) {
                const Item it = decode_item(p, item);
                const uint8_t *wsrc = it.job.wt + static_cast<int64_t>(it.mt) * p.nb * L::kWB;
                const uint8_t *xsrc = p.xq + static_cast<int64_t>(it.tt) * p.nb * QH_Q8KT_BLOCK_BYTES;
                for (int b = it.b0; b < it.b1; ++b, ++i) {
                    const int s = i % S;
                    if (!waited && i == S) {
                        pdl_wait();
                        waited = true;
                        for (int j = 0; j < S; ++j) issue_x(j, xpend[j]);
                    }
                    if (*abort_flag) { stop = true; break; }
                    if (i >= S && !mbar_wait(&empty[s], (static_cast<uint32_t>(i / S) & 1u) ^ 1u)) {
                        report_error(p.err_flag, kDevWaitTimeout);
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    uint8_t *dst = stages + static_cast<int64_t>(s) * L::kStage;
                    mbar_arrive_expect_tx(&full[s], L::kWB);
                    bulk_copy_g2s(dst, wsrc + static_cast<int64_t>(b) * L::kWB, L::kWB, &full[s]);
                    const uint8_t *xb = xsrc + static_cast<int64_t>(b) * QH_Q8KT_BLOCK_BYTES;
                    if (waited) issue_x(s, xb);
                    else xpend[s] = xb;
                }
            }
            if (!waited) {  // ended inside the first ring
                pdl_wait();
                for (int j = 0; j < i; ++j) issue_x(j, xpend[j]);
            }
            // Drain: no copy of this CTA stays in flight past its exit.
            for (int j = max(0, i - S); j < i; ++j) {
                const uint32_t ph = static_cast<uint32_t>(j / S) & 1u;
                if (!mbar_wait(&full[j % S], ph) || !mbar_wait(&xfull[j % S], ph)) report_error(p.err_flag, kDevWaitTimeout);
            }
        }
    } else if (warp == kMmaWarp) {
        // ----- MMA issue: lane 0; lanes 0-15 also move the token scales -----
        constexpr uint32_t idesc64 = tc::idesc_i8(kGemmRows, kGemmTok);
        constexpr uint32_t idesc128 = tc::idesc_i8(kGemmRows, 2 * kGemmTok);
        int i = 0, ib = 0;
        bool stop = false;
        for (int item = blockIdx.x; item < p.total_items && !stop; item += gridDim.x) {
            const Item it = decode_item(p, item);
            for (int b = it.b0; b < it.b1; ++b, ++i, ++ib) {
                const int s = i % S, buf = ib & 1, ring = ib % kRing;
                const uint32_t ph = static_cast<uint32_t>(ib >> 1) & 1u;
                // expanders done with this block's A buffer and row scales; the
                // activations landed; the epilogue done with the accumulators
                // two blocks back
                bool ok = true;
                if (lane == 0)
                    ok = !*abort_flag &&
                         (EXP ? mbar_wait(&full[s], static_cast<uint32_t>(i / S) & 1u) : mbar_wait(&a_ready[buf], ph)) &&
                         mbar_wait(&xfull[s], static_cast<uint32_t>(i / S) & 1u) &&
                         (ib < 2 || mbar_wait(&acc_empty[buf], ph ^ 1u));
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) {
                    if (lane == 0) {
                        report_error(p.err_flag, kDevWaitTimeout);
                        *abort_flag = 1;
                    }
                    stop = true;
                    break;
                }
                const uint8_t *wst = stages + static_cast<int64_t>(s) * L::kStage;
                const uint8_t *xst = wst + L::kWB;
                if (lane < kGemmTok / 4)
                    reinterpret_cast<uint4 *>(tok_scale + ring * kGemmTok)[lane] =
                        reinterpret_cast<const uint4 *>(xst + QH_Q8KT_D_OFF)[lane];
                if (EXP) {
                    // the rows' (d, dmin) leave the stage before it is released
                    const uint4 *src = reinterpret_cast<const uint4 *>(wst + L::kABuf);
                    uint4 *dst = reinterpret_cast<uint4 *>(row_scale + ring * kGemmRows);
                    dst[lane] = src[lane];
                    dst[lane + 32] = src[lane + 32];
                }
                __syncwarp();
                if (lane == 0) {
                    tc::fence_after_sync();
                    const uint32_t a0 = EXP ? smem_addr(wst) : smem_addr(smem + L::kA + buf * L::kABuf);
                    const uint32_t b0 = smem_addr(xst);
                    const uint32_t dcol = tmem + buf * kAccCols;
                    const uint64_t ad0 = tc::smem_desc(a0, kGemmRows * 16, 128);
                    const uint64_t bd0 = tc::smem_desc(b0, kGemmTok * 16, 128);
#pragma unroll
                    for (int pl = 0; pl < 2; ++pl)
#pragma unroll
                        for (int ks = 0; ks < QH_QK / 32; ++ks)
                            tc::mma_i8(dcol + pl * kGemmTok,
                                       ad0 + static_cast<uint64_t>((pl * kPlaneBytes + ks * 2 * kGemmRows * 16) >> 4),
                                       bd0 + static_cast<uint64_t>((ks * 2 * kGemmTok * 16) >> 4), idesc64, ks > 0);
                    if (MINS) {
                        // [S mod 128 | floor(S/128)] (128 columns) = min row x min operand;
                        // the second K chunk of both operands is the zero area.
                        const uint32_t am = a0 + 2 * kPlaneBytes, bm = b0 + QH_Q8KT_MIN_OFF, z = smem_addr(zero);
                        tc::mma_i8(dcol + 2 * kGemmTok, tc::smem_desc(am, z - am, 128), tc::smem_desc(bm, z - bm, 128),
                                   idesc128, false);
                    }
                    tc::commit(&mma_done[buf]);
                    tc::commit(&empty[s]);
                    // release the block's scales (row scales from the expanders,
                    // token scales from this warp) to the epilogue
                    mbar_arrive(&scale_ready[buf]);
                }
            }
        }
    } else if (warp < XW) {
        // ----- expanders (idle with expanded weights) -----
        if constexpr (!EXP) {
            const int r = tid >> 1, h = tid & 1;
            int i = 0, ib = 0;
            bool stop = false;
            for (int item = blockIdx.x; item < p.total_items && !stop; item += gridDim.x) {
                const Item it = decode_item(p, item);
                for (int b = it.b0; b < it.b1; ++b, ++i, ++ib) {
                    const int s = i % S, buf = ib & 1, ring = ib % kRing;
                    // stage landed; the MMAs two blocks back are done with this A buffer
                    const bool ok = __all_sync(0xffffffffu,
                                               !*abort_flag && mbar_wait(&full[s], static_cast<uint32_t>(i / S) & 1u) &&
                                                   (ib < 2 || mbar_wait(&mma_done[buf], static_cast<uint32_t>((ib - 2) >> 1) & 1u)));
                    if (!ok) {
                        stop = true;
                        break;
                    }
                    const uint8_t *wst = stages + static_cast<int64_t>(s) * L::kStage;
                    const uint8_t *raw = wst + r * BBP;
                    expand<TYPE>(raw, h, r, smem + L::kA + buf * L::kABuf);
                    if (h == 0) {
                        const uint32_t dd = *reinterpret_cast<const uint32_t *>(raw + (TYPE == QH_GGUF_Q6_K ? 208 : 0));
                        row_scale[ring * kGemmRows + r] =
                            make_float2(h2f_bits(dd), TYPE == QH_GGUF_Q6_K ? 0.0f : h2f_bits(dd >> 16));
                    }
                    tc::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_ready[buf]);
                }
            }
            if (stop && lane == 0) {
                report_error(p.err_flag, kDevWaitTimeout);
                *abort_flag = 1;
            }
        }
    } else {
        // ----- epilogue -----
        const int ew = warp - XW;
        const int er = 32 * (ew & 3) + lane;  // weight row = TMEM lane
        const int th = ew >> 2;               // token half of the tile
        const uint32_t lane_base = static_cast<uint32_t>(32 * (ew & 3)) << 16;
        volatile int &last_flag = *reinterpret_cast<volatile int *>(smem + 264);
        const bool split = p.kchunks > 1;
        int ib = 0;
        bool stop = false;
        for (int item = blockIdx.x; item < p.total_items && !stop; item += gridDim.x) {
            const Item it = decode_item(p, item);
            float acc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
            const int t0 = it.tt * kGemmTok + 32 * th;
            // split-K: this tile's per-block terms, [block][64 tokens][128 rows]
            float *tterms = split ? p.terms + static_cast<int64_t>(it.tile) * p.nb * (kGemmTok * kGemmRows) : nullptr;
            for (int b = it.b0; b < it.b1; ++b, ++ib) {
                const int buf = ib & 1, ring = ib % kRing;
                const uint32_t ph = static_cast<uint32_t>(ib >> 1) & 1u;
                const bool ok = __all_sync(0xffffffffu, mbar_wait(&scale_ready[buf], ph) && mbar_wait(&mma_done[buf], ph));
                if (!ok || *abort_flag) {
                    stop = true;
                    break;
                }
                tc::fence_after_sync();
                const float2 rs = row_scale[ring * kGemmRows + er];
                const float *ts = tok_scale + ring * kGemmTok + 32 * th;
                const uint32_t tcol = tmem + lane_base + buf * kAccCols + 32 * th;
                // With expanded weights (320 threads, registers to spare) both
                // halves' accumulator loads are issued before one wait; the
                // 576-thread form loads and waits per half.
                constexpr bool kBoth = EXP && !MINS;
                constexpr int kHalves = kBoth ? 2 : 1;
                uint32_t vhi[kHalves][16], vlo[kHalves][16], vsl[kHalves][16], vsh[kHalves][16];
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int hv = kBoth ? c : 0;
                    if (!kBoth || c == 0) {
#pragma unroll
                        for (int c2 = 0; c2 < (kBoth ? 2 : 1); ++c2) {
                            const int cc = kBoth ? c2 : c, hh = kBoth ? c2 : 0;
                            tc::ld_32x32b_x16(tcol + 16 * cc, vhi[hh]);
                            tc::ld_32x32b_x16(tcol + kGemmTok + 16 * cc, vlo[hh]);
                            if (MINS) {
                                tc::ld_32x32b_x16(tcol + 2 * kGemmTok + 16 * cc, vsl[hh]);
                                tc::ld_32x32b_x16(tcol + 3 * kGemmTok + 16 * cc, vsh[hh]);
                            }
                        }
                        tc::wait_ld();
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float yd = ts[16 * c + j];
                        const int isum = static_cast<int>(vhi[hv][j]) * 128 + static_cast<int>(vlo[hv][j]);
                        float term;
                        if (!MINS) {
                            term = __fmul_rn(__fmul_rn(rs.x, yd), __int2float_rn(isum));
                        } else {
                            const int imin = static_cast<int>(vsl[hv][j]) + 128 * static_cast<int>(vsh[hv][j]);
                            const float d = __fmul_rn(yd, rs.x), dm = __fmul_rn(yd, rs.y);
                            term = __fsub_rn(__fmul_rn(d, __int2float_rn(isum)), __fmul_rn(dm, __int2float_rn(imin)));
                        }
                        if (split)
                            tterms[(static_cast<int64_t>(b) * kGemmTok + 32 * th + 16 * c + j) * kGemmRows + er] = term;
                        else
                            acc[16 * c + j] = __fadd_rn(acc[16 * c + j], term);
                    }
                }
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
            }
            if (split) {
                // The CTA that brings the tile's last chunk adds every block's
                // term in block order (the reference's sequential sum). The
                // barrier also makes a stop of any epilogue warp uniform.
                __threadfence();
                if (bar_any(2, 32 * kEpiWarps, stop)) {
                    stop = true;
                    break;
                }
                if constexpr (SPREAD) {
                    // Every chunk's CTA of the tile is resident (one item per
                    // CTA): each waits for all the chunks' terms, then sums a
                    // slice of the tile's elements, all blocks' terms loaded
                    // before the in-order adds.
                    if (warp == XW && lane == 0) {
                        atomicAdd(&p.tickets[it.tile], 1u);
                        const unsigned target = static_cast<unsigned>(p.kchunks);
                        const uint64_t t_start = gemm_ns();
                        int ok = 0;
                        for (uint32_t n = 1;; ++n) {
                            if (gemm_ld_acquire(&p.tickets[it.tile]) >= target) { ok = 1; break; }
                            if ((n & 63u) == 0) {
                                if (*reinterpret_cast<volatile int *>(p.err_flag) != 0) break;
                                if (gemm_ns() - t_start > kSpreadWaitNs) {
                                    report_error(p.err_flag, kDevWaitTimeout);
                                    break;
                                }
                            }
                        }
                        last_flag = ok;
                    }
                    asm volatile("bar.sync 2, %0;" ::"n"(32 * kEpiWarps) : "memory");
                    if (!last_flag) {
                        stop = true;
                        break;
                    }
                    __threadfence();  // acquire the other chunks' terms
                    constexpr int E = kGemmTok * kGemmRows;
                    const int c = it.b0 / p.kc_blocks;
                    const int lo = c * E / p.kchunks, hi = (c + 1) * E / p.kchunks;
                    const int et = ew * 32 + lane;
                    // two elements per round trip to L2 (bounded registers)
#pragma unroll 1
                    for (int e0 = 0; e0 < kSpreadPerThread; e0 += 2) {
                        float v[2][kSpreadMaxNb];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int idx = lo + et + 32 * kEpiWarps * (e0 + e);
#pragma unroll
                            for (int b = 0; b < kSpreadMaxNb; ++b)
                                if (idx < hi && b < p.nb) v[e][b] = __ldcg(tterms + static_cast<int64_t>(b) * E + idx);
                        }
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int idx = lo + et + 32 * kEpiWarps * (e0 + e);
                            if (idx < hi) {
                                float sum = 0.0f;
#pragma unroll
                                for (int b = 0; b < kSpreadMaxNb; ++b)
                                    if (b < p.nb) sum = __fadd_rn(sum, v[e][b]);
                                const int tok = it.tt * kGemmTok + idx / kGemmRows;
                                const int n = it.mt * kGemmRows + idx % kGemmRows;
                                if (n < it.job.n_rows && tok < p.n_tok)
                                    it.job.out[static_cast<int64_t>(tok) * it.job.ldo + n] = sum;
                            }
                        }
                    }
                    // every read of the tile's terms is done: the last reader
                    // returns both counters to zero
                    asm volatile("bar.sync 2, %0;" ::"n"(32 * kEpiWarps) : "memory");
                    if (warp == XW && lane == 0) {
                        const unsigned prev = atomicAdd(&p.tickets[kSpreadDone + it.tile], 1u);
                        if (prev == static_cast<unsigned>(p.kchunks - 1)) {
                            p.tickets[it.tile] = 0u;
                            p.tickets[kSpreadDone + it.tile] = 0u;
                        }
                    }
                    continue;
                }
                if (warp == XW && lane == 0) {
                    const unsigned prev = atomicAdd(&p.tickets[it.tile], 1u);
                    last_flag = prev == static_cast<unsigned>(p.kchunks - 1);
                    if (last_flag) p.tickets[it.tile] = 0u;
                }
                asm volatile("bar.sync 2, %0;" ::"n"(32 * kEpiWarps) : "memory");
                if (!last_flag) continue;
                __threadfence();  // acquire the other chunks' terms
                // with expanded weights (registers to spare) two blocks'
                // terms are in flight per round trip to L2; the adds stay in
                // block order
                auto term = [&](int b, int j) {
                    return __ldcg(tterms + (static_cast<int64_t>(b) * kGemmTok + 32 * th + j) * kGemmRows + er);
                };
                int b = 0;
                if constexpr (EXP) {
                    for (; b + 2 <= p.nb; b += 2) {
                        float v0[32], v1[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            v0[j] = term(b, j);
                            v1[j] = term(b + 1, j);
                        }
#pragma unroll
                        for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(__fadd_rn(acc[j], v0[j]), v1[j]);
                    }
                }
                for (; b < p.nb; ++b) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(acc[j], term(b, j));
                }
            } else if (stop) {
                break;
            }
            const int n = it.mt * kGemmRows + er;
            if (n < it.job.n_rows) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (t0 + j < p.n_tok) it.job.out[static_cast<int64_t>(t0 + j) * it.job.ldo + n] = acc[j];
            }
        }
        if (stop && lane == 0) {
            report_error(p.err_flag, kDevWaitTimeout);
            *abort_flag = 1;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 2 * kAccCols);
    }
}

// Weight repacking: GGUF rows -> [row tile][block][128 rows][padded block
// bytes], padding and rows past n_rows zero. CTA (row tile, block), one
// thread per row; 2-byte copies (GGUF rows are 2-byte aligned).
__global__ void pack_tiles_kernel(const uint8_t *__restrict__ w, int64_t n_rows, int nb, int bb, int bbp,
                                  uint8_t *__restrict__ wt) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t mt = blockIdx.x;
    const int b = blockIdx.y, r = threadIdx.x;
    const int64_t row = mt * kGemmRows + r;
    uint16_t *dst = reinterpret_cast<uint16_t *>(wt + ((mt * nb + b) * kGemmRows + r) * bbp);
    int i = 0;
    if (row < n_rows) {
        const uint16_t *src = reinterpret_cast<const uint16_t *>(w + row * nb * bb + static_cast<int64_t>(b) * bb);
        for (; i < bb / 2; ++i) dst[i] = src[i];
    }
    for (; i < bbp / 2; ++i) dst[i] = 0;
}

// Expansion of tiled weights into the A-operand image of every (row tile,
// block) (ExpBlock): CTA (row tile, block), two threads per row running the
// expander warps' code into global memory, plus the rows' (d, dmin).
template <int TYPE>
__global__ void __launch_bounds__(256) expand_tiles_kernel(const uint8_t *__restrict__ wt, int nb,
                                                           uint8_t *__restrict__ we) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int BBP = KQ<TYPE>::kPadded;
    const int64_t tb = static_cast<int64_t>(blockIdx.x) * nb + blockIdx.y;
    const int r = threadIdx.x >> 1, h = threadIdx.x & 1;
    const uint8_t *raw = wt + (tb * kGemmRows + r) * BBP;
    uint8_t *dst = we + tb * ExpBlock<TYPE>::kBytes;
    expand<TYPE>(raw, h, r, dst);
    if (h == 0) {
        const uint32_t dd = *reinterpret_cast<const uint32_t *>(raw + (TYPE == QH_GGUF_Q6_K ? 208 : 0));
        reinterpret_cast<float2 *>(dst + ExpBlock<TYPE>::kA)[r] =
            make_float2(h2f_bits(dd), TYPE == QH_GGUF_Q6_K ? 0.0f : h2f_bits(dd >> 16));
    }
}

// Q8_K quantization into the tiled layout: CTA (block, token).
__global__ void __launch_bounds__(256) quantize_q8kt_kernel(const float *__restrict__ x, int k, int n_tok,
                                                            uint8_t *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ Q8KScratch sc;
    const int b = blockIdx.x, t = blockIdx.y;
    const float v = x[static_cast<int64_t>(t) * k + b * QH_QK + threadIdx.x];
    q8k_block256(v, sc, q8k_row(out, k, n_tok, t, QH_Q8KT_TILE), b);
}

template <int TYPE, bool EXP>
static cudaError_t gemm_launch_t(const GemmParams &p0, int sm_count, cudaStream_t stream) {
    using L = GemmSmem<TYPE, EXP>;
    GemmParams p = p0;
    p.n_stages = L::kNStages;
    const int smem = L::kTotal;
    // the spread split-K reduction is its own instantiation, so the kernels
    // of the other launches stay compact (registers, instruction cache)
    static bool attr_done[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool spread = EXP && p.spread;
    auto kern = spread ? gemm_kernel<TYPE, EXP, EXP> : gemm_kernel<TYPE, EXP, false>;
    if (dev >= 0 && dev < 64 && !attr_done[dev][spread]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
        if (e != cudaSuccess) return e;
        attr_done[dev][spread] = true;
    }
    const int grid = std::min(p.total_items, sm_count);
    return launch_pdl(kern, dim3(grid), dim3(gemm_threads(EXP)), smem, stream, p);
}

}  // namespace qh

// ---------------------------------------------------------------------------
// C-ABI
// ---------------------------------------------------------------------------
namespace {
int gfail(int code, const char *msg) {
    qh::set_last_error_message(msg);
    return code;
}
int gcuda(cudaError_t e, const char *what) {
    char msg[256];
    snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
    qh::set_last_error_message(msg);
    return QH_ERR_CUDA;
}
bool gemm_type_ok(int type) { return type == QH_TYPE_Q4_K || type == QH_TYPE_Q5_K || type == QH_TYPE_Q6_K; }
bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

extern "C" {

int64_t qh_gemm_weight_bytes(int type, int64_t k, int64_t out_f) {
    if (!gemm_type_ok(type) || k <= 0 || k % 256 || out_f <= 0) return -1;
    return ((out_f + qh::kGemmRows - 1) / qh::kGemmRows) * qh::kGemmRows * (k / 256) * qh::padded_block_bytes(type);
}

int qh_gemm_pack_weights(int type, const void *d_w, int64_t k, int64_t out_f, void *d_wt, void *stream) {
    if (!gemm_type_ok(type)) return gfail(QH_ERR_UNSUPPORTED, "gemm_pack_weights: type must be Q4_K, Q5_K or Q6_K");
    if (!d_w || !d_wt || k <= 0 || k % 256 || out_f <= 0 || k / 256 > 65535 || out_f > 0x7fffffffll)
        return gfail(QH_ERR_INVALID, "gemm_pack_weights: bad arguments");
    if ((reinterpret_cast<uintptr_t>(d_w) & 1u) || !al16(d_wt))
        return gfail(QH_ERR_ALIGN, "gemm_pack_weights: misaligned pointer");
    const int64_t mt = (out_f + qh::kGemmRows - 1) / qh::kGemmRows;
    cudaError_t e = qh::launch_pdl(qh::pack_tiles_kernel, dim3(static_cast<unsigned>(mt), static_cast<unsigned>(k / 256)),
                                   dim3(qh::kGemmRows), 0, static_cast<cudaStream_t>(stream),
                                   static_cast<const uint8_t *>(d_w), out_f, static_cast<int>(k / 256),
                                   static_cast<int>(qhf_block_bytes(type)), qh::padded_block_bytes(type),
                                   static_cast<uint8_t *>(d_wt));
    if (e != cudaSuccess) return gcuda(e, "gemm_pack_weights launch");
    return QH_OK;
}

int64_t qh_gemm_expanded_bytes(int type, int64_t k, int64_t out_f) {
    if (!gemm_type_ok(type) || k <= 0 || k % 256 || out_f <= 0) return -1;
    return ((out_f + qh::kGemmRows - 1) / qh::kGemmRows) * (k / 256) * qh::expanded_block_bytes(type);
}

int qh_gemm_expand_weights(int type, const void *d_wt, int64_t k, int64_t out_f, void *d_we, void *stream) {
    if (!gemm_type_ok(type)) return gfail(QH_ERR_UNSUPPORTED, "gemm_expand_weights: type must be Q4_K, Q5_K or Q6_K");
    if (!d_wt || !d_we || k <= 0 || k % 256 || out_f <= 0 || k / 256 > 65535 || out_f > 0x7fffffffll)
        return gfail(QH_ERR_INVALID, "gemm_expand_weights: bad arguments");
    if (!al16(d_wt) || !al16(d_we)) return gfail(QH_ERR_ALIGN, "gemm_expand_weights: misaligned pointer");
    const dim3 grid(static_cast<unsigned>((out_f + qh::kGemmRows - 1) / qh::kGemmRows), static_cast<unsigned>(k / 256));
    const uint8_t *wt = static_cast<const uint8_t *>(d_wt);
    uint8_t *we = static_cast<uint8_t *>(d_we);
    const int nb = static_cast<int>(k / 256);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    switch (type) {
        case QH_TYPE_Q4_K: e = qh::launch_pdl(qh::expand_tiles_kernel<QH_GGUF_Q4_K>, grid, dim3(256), 0, s, wt, nb, we); break;
        case QH_TYPE_Q5_K: e = qh::launch_pdl(qh::expand_tiles_kernel<QH_GGUF_Q5_K>, grid, dim3(256), 0, s, wt, nb, we); break;
        default: e = qh::launch_pdl(qh::expand_tiles_kernel<QH_GGUF_Q6_K>, grid, dim3(256), 0, s, wt, nb, we); break;
    }
    if (e != cudaSuccess) return gcuda(e, "gemm_expand_weights launch");
    return QH_OK;
}

int64_t qh_q8kt_bytes(int64_t k, int64_t n_tok) {
    if (k <= 0 || k % 256 || n_tok <= 0) return -1;
    return qhf_q8kt_total_bytes(k, n_tok);
}

int qh_quantize_q8kt(const float *d_x, int64_t k, int64_t n_tok, void *d_q8kt, void *stream) {
    if (!d_x || !d_q8kt || k <= 0 || k % 256 || k / 256 > 65535 || n_tok <= 0 || n_tok > 65535)
        return gfail(QH_ERR_INVALID, "quantize_q8kt: bad arguments");
    if (!al16(d_q8kt)) return gfail(QH_ERR_ALIGN, "quantize_q8kt: output not 16-byte aligned");
    cudaError_t e = qh::launch_pdl(qh::quantize_q8kt_kernel, dim3(static_cast<unsigned>(k / 256), static_cast<unsigned>(n_tok)),
                                   dim3(256), 0, static_cast<cudaStream_t>(stream), d_x, static_cast<int>(k),
                                   static_cast<int>(n_tok), static_cast<uint8_t *>(d_q8kt));
    if (e != cudaSuccess) return gcuda(e, "quantize_q8kt launch");
    return QH_OK;
}

static int64_t gemm_tiles(const qh_gemm_job *jobs, int n_jobs, int64_t n_tok) {
    int64_t t = 0;
    for (int j = 0; j < n_jobs; ++j) t += (jobs[j].out_f + qh::kGemmRows - 1) / qh::kGemmRows;
    return t * qhf_q8kt_tiles(n_tok);
}

// Scratch: a fixed area of arrival counters (one per output tile, so calls
// of different shapes sharing one scratch never see another call's terms in
// their counters), then the per-block terms.
constexpr int64_t kMaxSplitTiles = 1024;
constexpr int64_t kTicketBytes = kMaxSplitTiles * 4;

int64_t qh_gemm_scratch_bytes(const qh_gemm_job *jobs, int n_jobs, int64_t k, int64_t n_tok) {
    if (!jobs || n_jobs <= 0 || n_jobs > qh::kGemmMaxJobs || k <= 0 || k % 256 || n_tok <= 0) return -1;
    for (int j = 0; j < n_jobs; ++j)
        if (jobs[j].out_f <= 0) return -1;
    const int64_t tiles = std::min(gemm_tiles(jobs, n_jobs, n_tok), kMaxSplitTiles);
    return kTicketBytes + tiles * (k / 256) * qh::kGemmTok * qh::kGemmRows * 4;
}

int qh_gemm(int type, const qh_gemm_job *jobs, int n_jobs, int64_t k, const void *d_q8kt, int64_t n_tok,
            void *d_scratch, int64_t scratch_bytes, int32_t flags, void *stream) {
    if (!gemm_type_ok(type)) return gfail(QH_ERR_UNSUPPORTED, "gemm: type must be Q4_K, Q5_K or Q6_K");
    if (!jobs || n_jobs <= 0 || n_jobs > qh::kGemmMaxJobs || !d_q8kt || k <= 0 || k % 256 || n_tok <= 0 ||
        n_tok > 65535)
        return gfail(QH_ERR_INVALID, "gemm: bad arguments");
    if (!al16(d_q8kt) || (d_scratch && !al16(d_scratch))) return gfail(QH_ERR_ALIGN, "gemm: buffer not 16-byte aligned");
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return gcuda(e, "gemm: device query");
    qh::GemmParams p = {};
    p.n_jobs = n_jobs;
    p.nb = static_cast<int32_t>(k / 256);
    p.n_tok = static_cast<int32_t>(n_tok);
    p.t_tiles = static_cast<int32_t>(qhf_q8kt_tiles(n_tok));
    p.xq = static_cast<const uint8_t *>(d_q8kt);
    p.w_early = (flags & QH_GEMM_WEIGHTS_READY) ? 1 : 0;
    p.err_flag = qh::device_error_word();
    if (!p.err_flag) return gfail(QH_ERR_CUDA, "gemm: no device error word");
    int64_t tiles = 0;
    for (int j = 0; j < n_jobs; ++j) {
        const qh_gemm_job &jb = jobs[j];
        if (!jb.d_wt || !jb.d_out || jb.out_f <= 0 || jb.out_f > 0x7fffffffll || jb.ld_out < jb.out_f ||
            jb.ld_out > 0x7fffffffll)
            return gfail(QH_ERR_INVALID, "gemm: bad job");
        if (!al16(jb.d_wt)) return gfail(QH_ERR_ALIGN, "gemm: weights not 16-byte aligned");
        qh::GemmJob g;
        g.wt = static_cast<const uint8_t *>(jb.d_wt);
        g.out = jb.d_out;
        g.n_rows = static_cast<int32_t>(jb.out_f);
        g.m_tiles = static_cast<int32_t>((jb.out_f + qh::kGemmRows - 1) / qh::kGemmRows);
        g.tile_begin = static_cast<int32_t>(tiles);
        g.ldo = static_cast<int32_t>(jb.ld_out);
        tiles += g.m_tiles;
        p.jobs[j] = g;
    }
    const int64_t out_tiles = tiles * p.t_tiles;
    // Split the super-blocks of each output tile over several CTAs when the
    // tiles alone would leave most SMs idle (needs the scratch).
    p.kchunks = 1;
    p.kc_blocks = p.nb;
    p.spread = 0;
    const int64_t need = qh_gemm_scratch_bytes(jobs, n_jobs, k, n_tok);
    // Expanded weights stream at the memory rate, so a split (whose last CTA
    // re-reads every block's terms) pays only for very few tiles.
    const int64_t split_below = (flags & QH_GEMM_EXPANDED) ? sms / 4 : sms / 2;
    if (d_scratch && scratch_bytes >= need && out_tiles < split_below && out_tiles <= kMaxSplitTiles && p.nb > 1) {
        const int64_t want = std::min<int64_t>(p.nb, (sms + out_tiles - 1) / out_tiles);
        p.kc_blocks = static_cast<int32_t>((p.nb + want - 1) / want);
        p.kchunks = static_cast<int32_t>((p.nb + p.kc_blocks - 1) / p.kc_blocks);
        p.tickets = static_cast<unsigned *>(d_scratch);
        p.terms = reinterpret_cast<float *>(static_cast<uint8_t *>(d_scratch) + kTicketBytes);
        // Spread reduction when every item has its own resident CTA (the
        // chunks of a tile wait for one another) and a slice fits the
        // per-thread registers.
        const int64_t items = out_tiles * p.kchunks;
        const int64_t slice = (static_cast<int64_t>(qh::kGemmTok) * qh::kGemmRows + p.kchunks - 1) / p.kchunks;
        p.spread = (flags & QH_GEMM_EXPANDED) && items <= sms && out_tiles <= qh::kSpreadDone &&
                   p.nb <= qh::kSpreadMaxNb &&
                   slice <= static_cast<int64_t>(qh::kSpreadPerThread) * 32 * qh::kEpiWarps;
    }
    if (out_tiles * p.kchunks > 0x7fffffffll) return gfail(QH_ERR_INVALID, "gemm: too many tiles");
    p.total_items = static_cast<int32_t>(out_tiles * p.kchunks);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool xp = (flags & QH_GEMM_EXPANDED) != 0;
    switch (type) {
        case QH_TYPE_Q4_K: e = xp ? qh::gemm_launch_t<QH_GGUF_Q4_K, true>(p, sms, s)
                                  : qh::gemm_launch_t<QH_GGUF_Q4_K, false>(p, sms, s); break;
        case QH_TYPE_Q5_K: e = xp ? qh::gemm_launch_t<QH_GGUF_Q5_K, true>(p, sms, s)
                                  : qh::gemm_launch_t<QH_GGUF_Q5_K, false>(p, sms, s); break;
        default: e = xp ? qh::gemm_launch_t<QH_GGUF_Q6_K, true>(p, sms, s)
                        : qh::gemm_launch_t<QH_GGUF_Q6_K, false>(p, sms, s); break;
    }
    if (e != cudaSuccess) return gcuda(e, "gemm launch");
    return QH_OK;
}

int64_t qh_matmul_gemm_workspace_bytes(int type, int64_t k, int64_t out_f, int64_t n_tok) {
    const int64_t w = qh_gemm_weight_bytes(type, k, out_f), x = qh_q8kt_bytes(k, n_tok);
    if (w < 0 || x < 0) return -1;
    const qh_gemm_job job = {nullptr, out_f, nullptr, out_f};
    return qhf_align16(w) + qhf_align16(x) + qh_gemm_scratch_bytes(&job, 1, k, n_tok);
}

int qh_matmul_gemm(int type, const void *d_w, int64_t k, int64_t out_f, const float *d_x, int64_t n_tok,
                   float *d_out, void *d_work, int64_t work_bytes, void *stream) {
    const int64_t need = qh_matmul_gemm_workspace_bytes(type, k, out_f, n_tok);
    if (need < 0) return gemm_type_ok(type) ? gfail(QH_ERR_INVALID, "matmul_gemm: bad shape")
                                            : gfail(QH_ERR_UNSUPPORTED, "matmul_gemm: type must be Q4_K, Q5_K or Q6_K");
    if (!d_work || work_bytes < need) return gfail(QH_ERR_WORKSPACE, "matmul_gemm: workspace too small");
    if (!al16(d_work)) return gfail(QH_ERR_ALIGN, "matmul_gemm: workspace not 16-byte aligned");
    uint8_t *wt = static_cast<uint8_t *>(d_work);
    uint8_t *xq = wt + qhf_align16(qh_gemm_weight_bytes(type, k, out_f));
    uint8_t *scratch = xq + qhf_align16(qh_q8kt_bytes(k, n_tok));
    qh_gemm_job job = {wt, out_f, d_out, out_f};
    const int64_t sb = qh_gemm_scratch_bytes(&job, 1, k, n_tok);
    // the split-K arrival counters start at zero (the kernel leaves them so)
    cudaError_t e = cudaMemsetAsync(scratch, 0, static_cast<size_t>(kTicketBytes), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return gcuda(e, "matmul_gemm: clear counters");
    int rc = qh_gemm_pack_weights(type, d_w, k, out_f, wt, stream);
    if (rc) return rc;
    rc = qh_quantize_q8kt(d_x, k, n_tok, xq, stream);
    if (rc) return rc;
    return qh_gemm(type, &job, 1, k, xq, n_tok, scratch, sb, 0, stream);
}

}  // extern "C"
