// tc.cuh -- tcgen05 (5th-generation tensor core) building blocks for sm_100a:
// shared-memory matrix descriptors, the block-scaled instruction descriptor,
// TMEM allocation, scale-factor copies, MMA issue, commit and TMEM loads.
//
// Layout conventions used by every caller:
//  - A and B operands are K-major with 128-byte swizzle: a tile of R rows is
//    R x 128 B (128 E4M3 values of K per row), row r at r*128 B, its 16-byte
//    chunk j stored at chunk j ^ (r & 7); 8-row groups are 1024 B apart and the
//    tile base is 1024-byte aligned (TMA SWIZZLE_128B writes exactly this).
//  - UE8M0 scale factors, one per 32 values of K, for 128 rows x 4 K-blocks
//    (one 128-wide K tile) are a 512-byte block: row m0 + 32*m1, K-block k at
//    byte m0*16 + m1*4 + k.  tcgen05.cp .32x128b.warpx4 copies it to 4 TMEM
//    columns (replicated over the four 32-lane sub-partitions); the MMA for
//    K-block k selects byte k.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace wh {
namespace tc {

// K-major, SWIZZLE_128B operand: start address, LBO 16 B (unused), SBO 1024 B,
// descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t smem_addr) {
  uint64_t d = (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}
// No-swizzle K-major source of a 32 x 16 B scale-factor block (8-row core
// matrices of 128 B, 128 B apart).
__device__ __forceinline__ uint64_t desc_sf_block(uint32_t smem_addr) {
  uint64_t d = (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(128u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}
// kind::mxf8f6f4 block-scaled instruction descriptor: A and B E4M3, K-major,
// UE8M0 scales, M = 128, N = n (multiple of 8 up to 256), scale bytes sfa/sfb.
__host__ __device__ __forceinline__ uint32_t idesc_mxf8(int n, uint32_t sfa, uint32_t sfb) {
  return (sfb & 3u) << 4 | (uint32_t(n) >> 3) << 17 | 1u << 23 | (128u >> 4) << 24 |
         (sfa & 3u) << 29;
}

// TMEM allocation by one whole warp; the base address lands in *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes -> visible to the tensor core
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void cp_sf_block(uint32_t taddr, uint64_t src_desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc)
               : "memory");
}
// D[tmem_d] (+)= A * B with block scales; accumulate = 0 overwrites D.
__device__ __forceinline__ void mma_mxf8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p; }"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}
// Arrive on an mbarrier when every earlier tcgen05 operation of this thread
// has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 16 columns of 32-bit values: thread t of the warp gets lane
// (taddr.lane + t), columns taddr.col .. +15.
__device__ __forceinline__ void ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace wh
