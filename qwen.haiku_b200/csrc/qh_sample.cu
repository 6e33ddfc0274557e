// SPDX-License-Identifier: MIT
//
// qh_sample.cu -- the reference's sampler chain (sample_with,
// slm/sampler.c:134-180) on sm_100a: one CTA of 1024 threads per row.
//
//   1. repetition penalty (slm/sampler.c:49-63): every thread takes the
//      first occurrence of a token in the window, counts its occurrences
//      and applies the divide-or-multiply that many times in order, which
//      is what the reference's per-occurrence loop does to that logit;
//   2. temperature <= 0: block argmax, first index of the strict maximum
//      (sample_argmax, slm/model.c:401-412);
//   3. top-k collect (slm/sampler.c:70-93): the reference scans the vocabulary
//      once, keeping k slots and replacing the slot that holds the current
//      minimum (the first such slot) whenever a logit beats it. The slot
//      order matters downstream (the softmax sum runs over it, and the
//      stable sort keeps it among equal probabilities), so the scan is
//      replayed exactly: the block filters 8192 logits at a time against
//      the current minimum (which only grows, so every logit that enters
//      the slots passes the filter), compacts the survivors in vocabulary
//      order, and warp 0 replays them 32 at a time: a ballot finds the next
//      one that beats the minimum, the owning lane rewrites its slot, and a
//      warp min-reduction (redux.sync on an order-preserving key, lowest
//      lane among equals) finds the new first minimum;
//   4. softmax over the slots in slot order (slm/sampler.c:97-112): the
//      exponentials in parallel, the sum sequential in one thread;
//   5. stable descending sort by rank counting (slm/sampler.c:117-130);
//   6. top-p, min-p, renormalising sum and roulette pick: sequential float
//      sums in one thread over at most 256 values, with one generator draw
//      (rng_uniform, slm/model.c:444-447).
//
// The model's sampled decode step uses the same kernel with a feed stage:
// the pick is recorded by position, appended to the row's history and fed
// as the next input token, and the last row to finish advances the
// position (ticket counter, left at zero).

#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>

#include "../../include/qh_backend.h"
#include "../../include/qh_kernels.h"
#include "../../include/qh_sampler.h"
#include "qh_common.cuh"
#include "qh_internal.h"

namespace qh {
namespace {

constexpr int kThreads = 1024;
constexpr int kPerThread = 8;
constexpr int kChunk = kThreads * kPerThread;  // logits filtered per round
constexpr int kTopK = QH_SAMPLE_TOPK_MAX;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

// rng_next + rng_uniform (slm/model.c:420-447)
__device__ __forceinline__ float rng_uniform(uint64_t &s0, uint64_t &s1) {
    const uint64_t a = s0;
    const uint64_t res = rotl64(a * 5u, 7) * 9u;
    s1 ^= a;
    s0 = rotl64(a, 24) ^ s1 ^ (s1 << 16);
    s1 = rotl64(s1, 37);
    return __fdiv_rn(static_cast<float>(static_cast<uint32_t>(res >> 40)), 16777216.0f);
}

// Order-preserving unsigned key of a float (-0 and +0 map to the same key,
// as they compare equal).
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Feed stage of the model's sampled decode step (nullptr in qh_sample).
struct Feed {
    int32_t *hist_w;      // history rows, written (the pick is appended)
    int32_t *hist_n_w;    // history lengths, incremented
    int32_t *next;        // [B] picks
    int32_t *tokens;      // [B] next step's input tokens
    int32_t *picks;       // [B][stride] picks by position
    int32_t *ctl;         // [0] position (advanced by the last row)
    unsigned *ticket;     // rows finished (kept at zero between launches)
    int32_t stride;
    int32_t B;
};

struct Shared {
    float val[kTopK];
    int32_t idx[kTopK];
    float sval[kTopK];
    int32_t sidx[kTopK];
    int32_t wsum[kThreads / 32];
    float wbest[kThreads / 32];
    int32_t wbi[kThreads / 32];
    float mval;
    float sum;
    int32_t ncand;
    int32_t result;
};

__global__ void __launch_bounds__(kThreads)
    sample_kernel(float *__restrict__ logits, int64_t vocab, const qh_sample_ctl *__restrict__ dctl, qh_sample_ctl hctl,
                  const int32_t *__restrict__ hist, int32_t hist_stride, const int32_t *__restrict__ hist_n,
                  uint64_t *__restrict__ rng, int32_t *__restrict__ out, Feed feed) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ Shared sh;
    extern __shared__ __align__(16) uint8_t dyn[];
    float *cand_v = reinterpret_cast<float *>(dyn);
    int32_t *cand_i = reinterpret_cast<int32_t *>(dyn + kChunk * 4);

    const int row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const qh_sample_ctl c = dctl ? *dctl : hctl;
    const qh_sampler &sp = c.sp;
    float *lr = logits + static_cast<int64_t>(row) * vocab;
    const int32_t *h = hist + static_cast<int64_t>(row) * hist_stride;
    const int32_t hn = hist_n[row];

    // slm_generate_raw masks eos/eot while fewer than min_new tokens were
    // generated (slm/slm.c:303-322): saved, set to -inf, restored after.
    int pos = 0;
    bool mask = false;
    float saved_eos = 0.0f, saved_eot = 0.0f;
    if (feed.ctl) {
        pos = feed.ctl[0];
        mask = (pos - c.gen0) < c.min_new;
        if (mask) {
            __syncthreads();
            if (tid == 0) {
                if (c.eos_id >= 0 && c.eos_id < vocab) { saved_eos = lr[c.eos_id]; lr[c.eos_id] = -INFINITY; }
                if (c.eot_id >= 0 && c.eot_id < vocab) { saved_eot = lr[c.eot_id]; lr[c.eot_id] = -INFINITY; }
            }
            __syncthreads();
        }
    }

    // 1. repetition penalty: the window is staged in shared memory (the
    // candidate buffer is free here) unless it is longer than the buffer
    if (sp.repetition_penalty != 1.0f && hn != 0) {
        const int32_t start = (sp.repetition_window > 0 && sp.repetition_window < hn) ? hn - sp.repetition_window : 0;
        const int32_t W = hn - start;
        const int32_t *win = h + start;
        if (W <= kChunk) {
            for (int32_t i = tid; i < W; i += kThreads) cand_i[i] = h[start + i];
            __syncthreads();
            win = cand_i;
        }
        for (int32_t i = tid; i < W; i += kThreads) {
            const int32_t t = win[i];
            if (t < 0 || static_cast<int64_t>(t) >= vocab) continue;
            bool first = true;
            for (int32_t j = 0; j < i; ++j)
                if (win[j] == t) { first = false; break; }
            if (!first) continue;
            int32_t n = 1;
            for (int32_t j = i + 1; j < W; ++j) n += (win[j] == t);
            float lv = lr[t];
            for (int32_t r = 0; r < n; ++r)
                lv = (lv > 0.0f) ? __fdiv_rn(lv, sp.repetition_penalty) : __fmul_rn(lv, sp.repetition_penalty);
            lr[t] = lv;
        }
        __syncthreads();
    }

    if (!(sp.temperature > 0.0f)) {
        // 2. greedy: first index of the strict maximum, element 0 the start
        float best = -INFINITY;
        int bi = 0x7fffffff;
        for (int64_t i = tid; i < vocab; i += kThreads) {
            const float v = lr[i];
            if (v > best) { best = v; bi = static_cast<int>(i); }
        }
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(kFull, best, off);
            const int oi = __shfl_xor_sync(kFull, bi, off);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
        if (lane == 0) { sh.wbest[warp] = best; sh.wbi[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < kThreads / 32; ++w)
                if (sh.wbest[w] > best || (sh.wbest[w] == best && sh.wbi[w] < bi)) { best = sh.wbest[w]; bi = sh.wbi[w]; }
            const float f0 = lr[0];
            sh.result = (f0 != f0 || bi == 0x7fffffff || !(best > f0)) ? 0 : bi;
        }
        __syncthreads();
    } else {
        // 3. top-k collect in the reference's slot order
        int k = sp.top_k > 0 ? sp.top_k : kTopK;
        if (k > kTopK) k = kTopK;
        const int filled = static_cast<int64_t>(k) < vocab ? k : static_cast<int>(vocab);
        if (tid < filled) { sh.val[tid] = lr[tid]; sh.idx[tid] = tid; }
        __syncthreads();
        if (vocab > k) {
            // warp 0 keeps the slots in registers -- lane l holds slots
            // 8l .. 8l+7 (values rv, token ids ri) -- and the current first
            // minimum (mval, mslot); lmin/lslot are the lane's own first
            // minimum
            float rv[8], mval = 0.0f, lmin = INFINITY;
            int32_t ri[8];
            int mslot = 0, lslot = 0x7fffffff;
            auto lane_min = [&]() {
                lmin = INFINITY;
                lslot = 0x7fffffff;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (lane * 8 + j < k && (lslot == 0x7fffffff || rv[j] < lmin)) { lmin = rv[j]; lslot = lane * 8 + j; }
            };
            auto warp_min = [&]() {
                const uint32_t key = lslot == 0x7fffffff ? 0xffffffffu : order_key(lmin);
                const uint32_t mk = __reduce_min_sync(kFull, key);
                const int wl = __ffs(__ballot_sync(kFull, key == mk)) - 1;
                mval = __shfl_sync(kFull, lmin, wl);
                mslot = __shfl_sync(kFull, lslot, wl);
            };
            if (warp == 0) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int slot = lane * 8 + j;
                    rv[j] = slot < k ? sh.val[slot] : INFINITY;
                    ri[j] = slot < k ? sh.idx[slot] : 0;
                }
                lane_min();
                warp_min();
                if (lane == 0) sh.mval = mval;
            }
            __syncthreads();
            // Rounds: the first covers kThreads logits (one per thread), the
            // others kChunk; each thread's logits of the next round are loaded
            // while warp 0 replays this one.
            int64_t base = k;
            int per = 1;
            float v[kPerThread];
            auto load_round = [&](int64_t b0, int pt) {
#pragma unroll
                for (int r = 0; r < kPerThread; ++r) {
                    const int64_t i = b0 + static_cast<int64_t>(tid) * pt + r;
                    v[r] = (r < pt && i < vocab) ? lr[i] : -INFINITY;
                }
            };
            load_round(base, per);
            while (base < vocab) {
                const float thr = sh.mval;
                const int64_t i0 = base + static_cast<int64_t>(tid) * per;
                unsigned pass = 0;
#pragma unroll
                for (int r = 0; r < kPerThread; ++r)
                    if (r < per && i0 + r < vocab && v[r] > thr) pass |= 1u << r;
                const int cnt = __popc(pass);
                int incl = cnt;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const int y = __shfl_up_sync(kFull, incl, off);
                    if (lane >= off) incl += y;
                }
                if (lane == 31) sh.wsum[warp] = incl;
                __syncthreads();
                if (warp == 0) {
                    const int w = sh.wsum[lane];
                    int wi = w;
#pragma unroll
                    for (int off = 1; off < 32; off <<= 1) {
                        const int y = __shfl_up_sync(kFull, wi, off);
                        if (lane >= off) wi += y;
                    }
                    sh.wsum[lane] = wi - w;
                    if (lane == 31) sh.ncand = wi;
                }
                __syncthreads();
                int o = sh.wsum[warp] + incl - cnt;
#pragma unroll
                for (int r = 0; r < kPerThread; ++r)
                    if (pass & (1u << r)) { cand_v[o] = v[r]; cand_i[o] = static_cast<int32_t>(i0 + r); ++o; }
                __syncthreads();
                const int64_t next = base + static_cast<int64_t>(kThreads) * per;
                per = kPerThread;
                if (next < vocab) load_round(next, per);
                if (warp == 0) {
                    const int ncand = sh.ncand;
                    for (int g = 0; g < ncand; g += 32) {
                        const bool valid = g + lane < ncand;
                        const float cv = valid ? cand_v[g + lane] : -INFINITY;
                        const int32_t ci = valid ? cand_i[g + lane] : 0;
                        unsigned live = __ballot_sync(kFull, valid);
                        while (true) {
                            const unsigned enter = __ballot_sync(kFull, valid && cv > mval) & live;
                            if (enter == 0u) break;
                            const int src = __ffs(enter) - 1;
                            const float nv = __shfl_sync(kFull, cv, src);
                            const int32_t ni = __shfl_sync(kFull, ci, src);
                            if (lane == (mslot >> 3)) {
                                const int jj = mslot & 7;
#pragma unroll
                                for (int j = 0; j < 8; ++j)
                                    if (j == jj) { rv[j] = nv; ri[j] = ni; }
                                lane_min();
                            }
                            warp_min();
                            live &= src == 31 ? 0u : (kFull << (src + 1));
                        }
                    }
                    if (lane == 0) sh.mval = mval;
                }
                __syncthreads();
                base = next;
            }
            if (warp == 0) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int slot = lane * 8 + j;
                    if (slot < k) { sh.val[slot] = rv[j]; sh.idx[slot] = ri[j]; }
                }
            }
            __syncthreads();
        }
        // 4. softmax with temperature over the slots, in slot order
        if (tid < 32) {
            float m = -INFINITY;
            for (int j = tid; j < filled; j += 32) m = fmaxf(m, sh.val[j]);
            for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, off));
            if (tid == 0) sh.sum = m;
        }
        __syncthreads();
        const float m = sh.sum;
        if (tid < filled) sh.val[tid] = expf_ref(__fdiv_rn(__fsub_rn(sh.val[tid], m), sp.temperature));
        __syncthreads();
        if (tid == 0) {
            float s = 0.0f;
            for (int j = 0; j < filled; ++j) s = __fadd_rn(s, sh.val[j]);
            sh.sum = s;
        }
        __syncthreads();
        const float sum = sh.sum;
        if (sum > 0.0f && tid < filled) sh.val[tid] = __fdiv_rn(sh.val[tid], sum);
        __syncthreads();
        // 5. stable descending sort: rank = larger values + equal ones before
        if (tid < filled) {
            const float v = sh.val[tid];
            int rank = 0;
            for (int i = 0; i < filled; ++i) {
                const float u = sh.val[i];
                rank += (u > v) || (u == v && i < tid);
            }
            if (rank < filled) { sh.sval[rank] = v; sh.sidx[rank] = sh.idx[tid]; }
        }
        __syncthreads();
        // 6. top-p, min-p, roulette
        if (tid == 0) {
            int cutoff = filled;
            if (sp.top_p > 0.0f && sp.top_p < 1.0f) {
                float acc = 0.0f;
                for (int j = 0; j < filled; ++j) {
                    acc = __fadd_rn(acc, sh.sval[j]);
                    if (acc >= sp.top_p) { cutoff = j + 1; break; }
                }
            }
            if (sp.min_p > 0.0f) {
                const float thresh = __fmul_rn(sp.min_p, sh.sval[0]);
                int j2 = 1;
                while (j2 < cutoff && sh.sval[j2] >= thresh) ++j2;
                cutoff = j2;
            }
            float s = 0.0f;
            for (int j = 0; j < cutoff; ++j) s = __fadd_rn(s, sh.sval[j]);
            uint64_t s0 = rng[2 * row], s1 = rng[2 * row + 1];
            const float u = __fmul_rn(rng_uniform(s0, s1), s);
            rng[2 * row] = s0;
            rng[2 * row + 1] = s1;
            float cacc = 0.0f;
            int picked = 0;
            for (int j = 0; j < cutoff; ++j) {
                cacc = __fadd_rn(cacc, sh.sval[j]);
                if (u <= cacc) { picked = j; break; }
            }
            sh.result = sh.sidx[picked];
        }
        __syncthreads();
    }
    if (tid != 0) return;
    const int32_t pick = sh.result;
    if (mask) {
        if (c.eos_id >= 0 && c.eos_id < vocab) lr[c.eos_id] = saved_eos;
        if (c.eot_id >= 0 && c.eot_id < vocab) lr[c.eot_id] = saved_eot;
    }
    if (out) out[row] = pick;
    if (!feed.ctl) return;
    feed.next[row] = pick;
    if (pos >= 0 && pos < feed.stride) feed.picks[static_cast<int64_t>(row) * feed.stride + pos] = pick;
    feed.tokens[row] = pick;
    if (hn < hist_stride) {
        feed.hist_w[static_cast<int64_t>(row) * hist_stride + hn] = pick;
        feed.hist_n_w[row] = hn + 1;
    }
    __threadfence();
    if (atomicAdd(feed.ticket, 1u) == static_cast<unsigned>(feed.B - 1)) {
        feed.ctl[0] = pos + 1;
        *feed.ticket = 0u;
    }
}

bool g_attr_done[64] = {false};

cudaError_t launch_sample(float *logits, int B, int64_t vocab, const qh_sample_ctl *dctl, const qh_sample_ctl &hctl,
                          const int32_t *hist, int32_t hist_stride, const int32_t *hist_n, uint64_t *rng,
                          int32_t *out, const Feed &feed, cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int smem = kChunk * 8;
    if (dev >= 0 && dev < 64 && !g_attr_done[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        g_attr_done[dev] = true;
    }
    return launch_pdl(sample_kernel, dim3(static_cast<unsigned>(B)), dim3(kThreads), smem, s, logits, vocab, dctl,
                      hctl, hist, hist_stride, hist_n, rng, out, feed);
}

int fail_invalid(const char *what) {
    set_last_error_message(what);
    return QH_ERR_INVALID;
}

int status_of(cudaError_t e, const char *what) {
    const cudaError_t last = cudaGetLastError();
    if (e == cudaSuccess) e = last;
    if (e == cudaSuccess) return QH_OK;
    char msg[256];
    snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
    set_last_error_message(msg);
    return QH_ERR_CUDA;
}

}  // namespace
}  // namespace qh

extern "C" {

void qh_sampler_defaults(qh_sampler *s) {
    if (!s) return;
    s->temperature = 0.7f;
    s->top_k = 40;
    s->top_p = 0.9f;
    s->min_p = 0.05f;
    s->repetition_penalty = 1.25f;
    s->repetition_window = 64;
}

void qh_rng_seed(uint64_t seed, uint64_t state[2]) {
    if (!state) return;
    // SplitMix64, two outputs (slm/model.c:431-442)
    uint64_t z = seed + 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    state[0] = z ^ (z >> 31);
    z = state[0] + 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    state[1] = z ^ (z >> 31);
    if (state[0] == 0 && state[1] == 0) state[0] = 1;
}

int qh_sample(const qh_sampler *sp, float *d_logits, int32_t B, int64_t vocab, const int32_t *d_hist,
              int32_t hist_stride, const int32_t *d_hist_n, uint64_t *d_rng, int32_t *d_out, void *stream) {
    if (!sp || !d_logits || !d_hist || !d_hist_n || !d_rng || !d_out || B <= 0 || B > 0x7fffffff ||
        vocab <= 0 || vocab > 0x7ffffffe || hist_stride < 0)
        return qh::fail_invalid("qh_sample: bad arguments");
    qh_sample_ctl c = {};
    c.sp = *sp;
    c.eos_id = c.eot_id = -1;
    const qh::Feed feed = {};
    return qh::status_of(qh::launch_sample(d_logits, B, vocab, nullptr, c, d_hist, hist_stride, d_hist_n, d_rng, d_out,
                                           feed, static_cast<cudaStream_t>(stream)),
                         "qh_sample");
}

int qh_sample_feed(float *d_logits, int32_t B, int64_t vocab, const qh_sample_ctl *d_sctl, int32_t *d_hist,
                   int32_t hist_stride, int32_t *d_hist_n, uint64_t *d_rng, int32_t *d_next, int32_t stride,
                   int32_t *d_ctl, int32_t *d_tokens, int32_t *d_picks, unsigned *d_ticket, void *stream) {
    if (!d_logits || !d_sctl || !d_hist || !d_hist_n || !d_rng || !d_next || !d_ctl || !d_tokens || !d_picks ||
        !d_ticket || B <= 0 || B > 0x7fffffff || vocab <= 0 || vocab > 0x7ffffffe || hist_stride <= 0 || stride <= 0)
        return qh::fail_invalid("qh_sample_feed: bad arguments");
    qh_sample_ctl unused = {};
    qh::Feed feed;
    feed.hist_w = d_hist;
    feed.hist_n_w = d_hist_n;
    feed.next = d_next;
    feed.tokens = d_tokens;
    feed.picks = d_picks;
    feed.ctl = d_ctl;
    feed.ticket = d_ticket;
    feed.stride = stride;
    feed.B = B;
    return qh::status_of(qh::launch_sample(d_logits, B, vocab, d_sctl, unused, d_hist, hist_stride, d_hist_n, d_rng,
                                           nullptr, feed, static_cast<cudaStream_t>(stream)),
                         "qh_sample_feed");
}

}  // extern "C"
