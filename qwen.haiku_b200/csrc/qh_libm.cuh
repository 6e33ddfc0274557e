// SPDX-License-Identifier: MIT
//
// qh_libm.cuh -- the reference's expf and logf on the device, bit for bit.
//
// The reference calls the host C library's expf/logf (SiLU and sigmoid,
// the DeltaNet gate and softplus, softmax, the sampler; on Linux that is
// glibc). Those functions are not correctly rounded: glibc's expf differs
// from the correctly rounded value on ~7.6e-5 of inputs, and the model's
// Q8_K re-quantization of every layer input turns such one-ulp differences
// into different greedy tokens after tens of steps. So the device evaluates
// them the way glibc (2.28 and later, x86-64 FMA variant) does -- the
// table-driven method of ARM's optimized-routines (published under the MIT /
// Apache-2.0 licences):
//
//   expf: k = round(x 32/ln2), r = x 32/ln2 - k (one fma each), result
//         2^(k/32) p(r) with 2^(k/32) built from a 32-entry table of
//         2^(i/32) (exponent added to the bits) and p a cubic, in double
//         precision, rounded once to float.
//   logf: x = 2^k z, z in [0x3f330000, 0x3f330000 + 2^23) as bit patterns,
//         split into 16 subintervals; r = z invc_i - 1 (fma), result
//         logc_i + k ln2 + r + r^2 q(r) with q a quadratic, in double
//         precision, rounded once to float.
//
// The constants (qh_libm_consts.h) are not transcribed from any source: the
// 2^(i/32) table is computed from its definition, and the polynomials and the
// log table were measured against the host library by oracle/libm/fit.py,
// which moves textbook starting values until the result equals the host's
// on every float input. For logf a handful of inputs remain whose unrounded
// value lies within ~1e-6 ulp of a rounding boundary and which no nearby
// parameter set rounds as the host does; they are listed with the host's
// results and looked up first. tests/test_libm_gpu.py compares these device
// functions with the host library over all 2^32 inputs.
//
// Every double operation is an explicit round-to-nearest intrinsic, so the
// compiler cannot contract or reorder them.

#ifndef QH_LIBM_CUH
#define QH_LIBM_CUH

#include <cuda_runtime.h>
#include <stdint.h>

#include "qh_libm_consts.h"

namespace qh {

__device__ __forceinline__ float expf_ref(float x) {
    using namespace libm;
    const uint32_t ix = __float_as_uint(x);
    if (ix == 0xff800000u) return 0.0f;                                // -inf
    if ((ix & 0x7f800000u) == 0x7f800000u) return __fadd_rn(x, x);    // +inf, nan
    if (x > 89.0f) return __uint_as_float(0x7f800000u);                // overflow
    if (x < -104.0f) return 0.0f;                                      // underflow
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32, shift = 0x1.8p+52;
    const double xd = static_cast<double>(x);
    double kd = __fma_rn(inv_ln2_n, xd, shift);
    const uint64_t ki = static_cast<uint64_t>(__double_as_longlong(kd));
    kd = __dsub_rn(kd, shift);
    const double r = __fma_rn(inv_ln2_n, xd, -kd);
    const double s = __longlong_as_double(static_cast<long long>(__ldg(&kExp2Tab[ki & 31]) + (ki << 47)));
    const double z = __fma_rn(kExpC0, r, kExpC1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(kExpC2, r, 1.0);
    y = __fma_rn(z, r2, y);
    return __double2float_rn(__dmul_rn(y, s));
}

__device__ __forceinline__ float logf_ref(float x) {
    using namespace libm;
    uint32_t ix = __float_as_uint(x);
    if (ix == 0x3f800000u) return 0.0f;
    if (ix - 0x00800000u >= 0x7f800000u - 0x00800000u) {
        if (ix * 2u == 0) return __uint_as_float(0xff800000u);          // +-0 -> -inf
        if (ix == 0x7f800000u) return x;                                // +inf
        if ((ix & 0x80000000u) || ix * 2u >= 0xff000000u) return __uint_as_float(0xffc00000u);  // < 0, nan
        ix = __float_as_uint(__fmul_rn(x, 0x1p23f)) - (23u << 23);      // subnormal
    }
    if (kLogExcN > 0) {  // the measured inputs the evaluation below rounds the other way
        // one pass over the short list, every load independent (one memory
        // latency, where a binary search waits for log2(n) of them)
        const uint32_t xb = __float_as_uint(x);
        int hit = -1;
#pragma unroll
        for (int e = 0; e < kLogExcN; ++e)
            if (__ldg(&kLogExcIn[e]) == xb) hit = e;
        if (hit >= 0) return __uint_as_float(__ldg(&kLogExcOut[hit]));
    }
    const uint32_t tmp = ix - 0x3f330000u;
    const int i = static_cast<int>((tmp >> 19) & 15u);
    const int k = static_cast<int32_t>(tmp) >> 23;
    const double z = static_cast<double>(__uint_as_float(ix - (tmp & 0xff800000u)));
    const double r = __fma_rn(z, __ldg(&kLogInvC[i]), -1.0);
    const double y0 = __fma_rn(static_cast<double>(k), kLn2, __ldg(&kLogLogC[i]));
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(kLogA1, r, kLogA2);
    y = __fma_rn(kLogA0, r2, y);
    y = __fma_rn(y, r2, __dadd_rn(y0, r));
    return __double2float_rn(y);
}

// Brings the tables of expf_ref / logf_ref into this SM's L1 (a hint: no
// result, no fault). Called by lanes 0-9 of one warp before a kernel's
// programmatic-launch wait (the tables are constants), so its first expf or
// logf after the wait does not wait for a memory round trip per table step.
__device__ __forceinline__ void libm_prefetch_l1(int lane) {
    using namespace libm;
    const void *p = nullptr;
    switch (lane) {
        case 0: p = &kExp2Tab[0]; break;
        case 1: p = &kExp2Tab[31]; break;
        case 2: p = &kLogInvC[0]; break;
        case 3: p = &kLogInvC[15]; break;
        case 4: p = &kLogLogC[0]; break;
        case 5: p = &kLogLogC[15]; break;
        case 6: p = &kLogExcIn[0]; break;
        case 7: p = &kLogExcIn[kLogExcN > 0 ? kLogExcN - 1 : 0]; break;
        case 8: p = &kLogExcOut[0]; break;
        case 9: p = &kLogExcOut[kLogExcN > 0 ? kLogExcN - 1 : 0]; break;
        default: break;
    }
    if (p) asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

}  // namespace qh

#endif  // QH_LIBM_CUH
