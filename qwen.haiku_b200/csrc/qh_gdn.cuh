// SPDX-License-Identifier: MIT
//
// qh_gdn.cuh -- the Gated DeltaNet recurrence of one state column, shared by
// the DeltaNet kernels (qh_model.cu, qh_step.cu). slm/qwen.c:499-557 per
// column v of a head's state S [k][v], with the decay g, the normalized K and
// Q rows and beta:
//   kv    = sum_k double(fl(fl(S[k][v] * g) * K[k]))          (k in order)
//   delta = fl(fl(V[v] - float(kv)) * beta)
//   S[k][v] = fl(fl(S[k][v] * g) + fl(K[k] * delta))
//   out   = float(sum_k double(fl(S[k][v] * Q[k])))          (k in order)
// The two sums are sequential chains of double adds (8 cycles each on
// sm_100a); the helper keeps the additions and their order and only moves
// the shared-memory loads ahead of them.

#ifndef QH_GDN_CUH
#define QH_GDN_CUH

namespace qh {

constexpr int kGdnBatch = 16;

// Column in shared memory: sc = &S[0][v], row stride HD floats; K, Q in
// shared memory (broadcast reads). Updates the column in place; returns out.
// Software-pipelined: the raw operands of the next 16 k are loaded before
// the current 16 are added (bounded registers, ~100 per thread), so the
// loads overlap the chain: 23 % faster than loads inside the add loop on
// sm_100a (5.9 K against 7.6 K cycles for the two chains, measured).
template <int HD>
__device__ __forceinline__ float gdn_recur_column(float *__restrict__ sc, const float *__restrict__ K,
                                                  const float *__restrict__ Q, float g, float beta, float v) {
    constexpr int B = kGdnBatch;
    static_assert(HD % B == 0, "column length");
    float s[B], k[B], q[B], s_next[B], k_next[B], q_next[B];
#pragma unroll
    for (int j = 0; j < B; ++j) {
        s[j] = sc[j * HD];
        k[j] = K[j];
    }
    double acc = 0.0;
#pragma unroll 1
    for (int k0 = 0; k0 < HD; k0 += B) {
        if (k0 + B < HD) {
#pragma unroll
            for (int j = 0; j < B; ++j) {
                s_next[j] = sc[(k0 + B + j) * HD];
                k_next[j] = K[k0 + B + j];
            }
        }
#pragma unroll
        for (int j = 0; j < B; ++j) acc += static_cast<double>(__fmul_rn(__fmul_rn(s[j], g), k[j]));
#pragma unroll
        for (int j = 0; j < B; ++j) {
            s[j] = s_next[j];
            k[j] = k_next[j];
        }
    }
    const float delta = __fmul_rn(__fsub_rn(v, static_cast<float>(acc)), beta);
#pragma unroll
    for (int j = 0; j < B; ++j) {
        s[j] = sc[j * HD];
        k[j] = K[j];
        q[j] = Q[j];
    }
    double acc2 = 0.0;
#pragma unroll 1
    for (int k0 = 0; k0 < HD; k0 += B) {
        if (k0 + B < HD) {
#pragma unroll
            for (int j = 0; j < B; ++j) {
                s_next[j] = sc[(k0 + B + j) * HD];
                k_next[j] = K[k0 + B + j];
                q_next[j] = Q[k0 + B + j];
            }
        }
#pragma unroll
        for (int j = 0; j < B; ++j) {
            const float sn = __fadd_rn(__fmul_rn(s[j], g), __fmul_rn(k[j], delta));
            sc[(k0 + j) * HD] = sn;
            acc2 += static_cast<double>(__fmul_rn(sn, q[j]));
        }
#pragma unroll
        for (int j = 0; j < B; ++j) {
            s[j] = s_next[j];
            k[j] = k_next[j];
            q[j] = q_next[j];
        }
    }
    return static_cast<float>(acc2);
}

}  // namespace qh

#endif  // QH_GDN_CUH
