// SPDX-License-Identifier: MIT
//
// qh_tc.cuh -- 5th-generation tensor core (tcgen05) and tensor memory (TMEM)
// wrappers in inline PTX for sm_100a, as used by the GEMM kernel:
//   * TMEM allocation (one warp allocates, the same warp frees),
//   * shared-memory matrix descriptors for the no-swizzle K-major canonical
//     layout,
//   * the instruction descriptor of kind::i8 (s8 x s8 -> s32),
//   * tcgen05.mma issue, commit to an mbarrier, and tcgen05.ld of 32 lanes x
//     32 columns of 32-bit accumulators.
//
// Canonical K-major, no-swizzle operand layout (per 16-byte "chunk" of K):
//   byte (row r, k-byte c) of an R-row operand lives at
//       (c / 16) * (R * 16) + r * 16 + (c % 16)
//   i.e. chunks of R rows x 16 bytes; 8-row core matrices are 128 contiguous
//   bytes (stride-dimension byte offset SBO = 128), and the two K-adjacent
//   core matrices one MMA reads (K = 32 int8) are R * 16 bytes apart
//   (leading-dimension byte offset LBO = R * 16).

#ifndef QH_TC_CUH
#define QH_TC_CUH

#include <stdint.h>

#include "qh_common.cuh"

namespace qh {
namespace tc {

// ---- TMEM ----------------------------------------------------------------
// Allocates `cols` columns (power of two >= 32) and writes the TMEM base
// address to *dst (shared memory). Whole warp, converged.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// ---- ordering --------------------------------------------------------------
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes (operands built by threads) become
// visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- descriptors -----------------------------------------------------------
// Shared-memory matrix descriptor, no swizzle (layout type 0), version 1,
// base offset 0, relative LBO mode.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version of sm_100
    return d;
}

// Instruction descriptor of kind::i8: D s32, A and B signed 8-bit, both
// K-major, no negation, no saturation, dense. M in {64, 128, 256}, N a
// multiple of 16 in [16, 256] (for M = 128).
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4)                                 // D format: s32
           | (1u << 7)                               // A: s8
           | (1u << 10)                              // B: s8
           | (static_cast<uint32_t>(N >> 3) << 17)   // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);  // M / 16
}

// ---- MMA -------------------------------------------------------------------
// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}

// Arrives once on `bar` when every MMA issued so far by this thread has
// completed (and its shared-memory reads are done).
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// ---- TMEM -> registers -----------------------------------------------------
// Warp w (w % 4 = subpartition) reads lanes 32(w%4)..+31: thread i gets row
// 32(w%4)+i, columns taddr.col .. +31. Call wait_ld() before using v.
__device__ __forceinline__ void ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace tc

// Named barrier over `count` threads (a multiple of 32) that also ORs a
// predicate across them: every participant gets the same answer, so a
// failed bounded wait in any thread can be acted on uniformly.
__device__ __forceinline__ bool bar_any(uint32_t id, uint32_t count, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.cta.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(v ? 1u : 0u), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

}  // namespace qh

#endif  // QH_TC_CUH
