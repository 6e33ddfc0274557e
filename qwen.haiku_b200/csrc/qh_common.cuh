// SPDX-License-Identifier: MIT
//
// qh_common.cuh -- sm_100a device helpers shared by the kernels: shared
// memory addressing, mbarrier and bulk-copy (TMA engine, 1-D) wrappers in
// inline PTX, bounded waits, exact-rounding fp helpers and the device error
// flag every spin-wait reports to.

#ifndef QH_COMMON_CUH
#define QH_COMMON_CUH

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qh_formats.h"
#include "qh_libm.cuh"

namespace qh {

// Device-side error codes written to the error word (first error wins).
enum DeviceError : int {
    kDevOk = 0,
    kDevWaitTimeout = 1,   // an mbarrier wait ran out of iterations
};

// Iteration limit of a bounded mbarrier wait. try_wait suspends the thread
// for a hardware-chosen interval per call, so this is seconds of waiting:
// far beyond any legitimate stall, short enough to return control.
constexpr uint32_t kWaitLimit = 1u << 22;

// Programmatic dependent launch. Every kernel of this library starts with
// pdl_launch_dependents() (the next kernel on the stream may be scheduled
// as soon as all CTAs of this one run) and calls pdl_wait() before it reads
// or writes memory that an earlier kernel touches: pdl_wait returns once the
// preceding grid has completed and its writes are visible. Both are no-ops
// in a launch without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// `count` arrivals at once.
__device__ __forceinline__ void mbar_arrive_n(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// The same with at most `limit` polls.
__device__ __forceinline__ bool mbar_wait_n(uint64_t *bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// 1-D bulk copy global -> shared through the TMA engine, completing `bytes`
// of transaction count on `bar`. src and dst 16-byte aligned, bytes a
// non-zero multiple of 16. The global source is this GPU's own memory.
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes,
                                              uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 1-D bulk copy shared -> global (bulk-group completion). Writers of the
// shared source must have executed fence.proxy.async.shared::cta and
// synchronized with the issuing thread first.
__device__ __forceinline__ void bulk_copy_s2g(void *dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_addr(src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void report_error(int *flag, int code) {
    if (flag != nullptr) atomicCAS(flag, 0, code);
}

// --- loads ----------------------------------------------------------------

__device__ __forceinline__ uint4 lds128(const uint8_t *p) {
    return *reinterpret_cast<const uint4 *>(p);
}
__device__ __forceinline__ uint32_t lds32(const uint8_t *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}
// 16 bytes from a 2-byte-aligned shared address: five aligned words, then a
// funnel shift by 0 or 16 bits.
__device__ __forceinline__ uint4 lds128_a2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(a & 2) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
    uint4 r;
    r.x = __funnelshift_r(w0, w1, sh);
    r.y = __funnelshift_r(w1, w2, sh);
    r.z = __funnelshift_r(w2, w3, sh);
    r.w = __funnelshift_r(w3, w4, sh);
    return r;
}
// 4 bytes from a 2-byte-aligned shared address.
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    return __funnelshift_r(w[0], w[1], static_cast<uint32_t>(a & 2) * 8u);
}

__device__ __forceinline__ int4 ldg128(const void *p) {
    return __ldg(reinterpret_cast<const int4 *>(p));
}

// expf / logf: the host C library's values, bit for bit (qh_libm.cuh); and
// the SiLU / sigmoid the reference builds from expf.
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf_ref(-x))); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_ref(-x))); }

__device__ __forceinline__ float h2f_bits(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

}  // namespace qh

#endif  // QH_COMMON_CUH
