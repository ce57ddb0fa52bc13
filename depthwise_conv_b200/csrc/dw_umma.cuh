// dw_umma.cuh -- sm_100a tensor-core (tcgen05) helpers for the pointwise
// block's GEMM: tensor-memory allocation, shared-memory matrix descriptors,
// the single-thread MMA issue, its completion signal and the tensor-memory
// loads of the epilogue.  All forms are cta_group::1 (one SM per tile) and
// no load anywhere uses cluster multicast.
#pragma once

#include <stdint.h>

#include "dw_device.cuh"

namespace dwb {

// ---- tensor memory (TMEM) ------------------------------------------------------
// A warp allocates `ncols` columns (a power of two, >= 32) of the SM's 512 x
// 128-lane tensor memory and writes the base address to shared memory; the same
// warp frees them at the end.  The relinquish lets other CTAs on the SM
// allocate while this one runs.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Ordering of tcgen05 operations across a thread synchronisation (barrier or
// mbarrier): "before" on the signalling side, "after" on the waiting side.
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- shared-memory matrix descriptors ------------------------------------------
// An operand tile of R rows x 64 fp16 (128 bytes) per row, K-major, written by
// TMA with the 128-byte swizzle: rows grouped in 8-row (1024-byte) swizzle
// atoms.  Descriptor fields (64 bits): start address >> 4 in bits 0-13, leading
// byte offset >> 4 in bits 16-29 (unused by swizzled K-major layouts; 1),
// stride byte offset >> 4 in bits 32-45 (1024 bytes between 8-row groups),
// descriptor version 1 in bits 46-47, base offset 0 in bits 49-51 (the tile
// starts on a 1024-byte boundary), layout type 2 (128-byte swizzle) in bits
// 61-63.  The 16-element K slice k of the tile starts 32 k bytes into each
// row, which is the start address plus 32 k (the swizzle is applied to the
// absolute address bits, so the atom's alignment carries it).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_byte_addr) {
  return static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor of kind::f16 with fp16 A and B (both K-major) and an
// fp32 accumulator: D format (bits 4-5) = 1 (f32), A and B formats (bits 7-9,
// 10-12) = 0 (f16), A/B major (bits 15, 16) = 0 (K), N >> 3 in bits 17-22,
// M >> 4 in bits 24-28.
template <int M, int N>
__host__ __device__ constexpr uint32_t f16_f32acc_idesc() {
  static_assert(M == 128, "one-SM tiles of 128 rows");
  static_assert(N % 16 == 0 && N >= 16 && N <= 256, "N: a multiple of 16 in [16, 256] for M = 128");
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T for one 128 x N x 16 block, issued by one
// thread; `accumulate` = 0 overwrites D (the first K slice of a tile).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on an mbarrier of this CTA when every tcgen05 operation the
// calling thread issued so far has completed (the MMAs have read their shared
// memory operands and written D).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// Warp-collective load of 16 consecutive fp32 columns of the warp's 32 TMEM
// lanes (lane i of the warp receives lane base+i); wait before use.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 2-D tiled TMA load (no multicast), completion on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
      : "memory");
}

}  // namespace dwb
