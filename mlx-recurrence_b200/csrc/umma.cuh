// 5th-generation tensor core (tcgen05) building blocks for sm_100a:
// shared-memory matrix descriptors, instruction descriptors, TMEM
// allocation, MMA issue/commit and TMEM -> register loads.
//
// Encodings follow the PTX ISA's tcgen05 "shared memory descriptor" and
// "instruction descriptor" formats (the same bit layout CUTLASS's
// cute::UMMA::SmemDescriptor / InstrDescriptor use):
//   smem descriptor (64 bit): [0,14) start address >> 4, [16,30) leading
//     byte offset >> 4, [32,46) stride byte offset >> 4, [46,48) version = 1,
//     [49,52) base offset, [52] LBO mode, [61,64) layout (2 = 128B swizzle).
//   instruction descriptor (32 bit, kind::f16): [4,6) D format (1 = f32),
//     [7,10) A format, [10,13) B format (0 = f16, 1 = bf16), [15] A major,
//     [16] B major (0 = K-major, 1 = MN-major), [17,23) N >> 3, [24,29) M >> 4.
//
// Operand tiles used here are all 128-byte-swizzled with 64 bf16 (128 B)
// per row, 1024-byte aligned:
//   K-major  [rows = M or N][64 K]: row r at r*128 B; SBO = 1024 B between
//            8-row groups; K steps of 16 advance the start address by 32 B.
//   MN-major [rows = K][64 MN]:     row k at k*128 B; SBO = 1024 B between
//            8-row groups of K; LBO = distance between 64-wide MN blocks;
//            K steps of 16 advance the start address by 2048 B.
// In both, the 16-byte chunk c of row r sits at chunk position c ^ (r & 7),
// which is what TMA writes with CU_TENSOR_MAP_SWIZZLE_128B.
#pragma once

#include <stdint.h>

namespace mr {
namespace umma {

constexpr uint32_t kLayoutSW128 = 2;

__device__ __forceinline__ uint64_t sdesc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)kLayoutSW128 << 61;
  return d;
}

// K-major 128B-swizzled tile: SBO 1024, LBO 16 (unused inside one swizzle atom).
__device__ __forceinline__ uint64_t sdesc_k(uint32_t smem_addr) { return sdesc(smem_addr, 16, 1024); }

// MN-major 128B-swizzled tile; lbo = byte distance between 64-wide MN blocks.
__device__ __forceinline__ uint64_t sdesc_mn(uint32_t smem_addr, uint32_t lbo) { return sdesc(smem_addr, lbo, 1024); }

// fmt: 0 = f16, 1 = bf16; major: 0 = K, 1 = MN.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int fmt, int a_major, int b_major) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)a_major << 15) |
         ((uint32_t)b_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- TMEM allocation (one full warp executes these) -------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- MMA (one thread issues) ------------------------------------------------
// D[tmem] (+)= A[smem] * B[smem]^T (per the descriptors' majorness).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}

// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- TMEM -> registers: lane = thread's row, 16 consecutive f32 columns -----
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column) relative to an allocation base.
__device__ __forceinline__ uint32_t taddr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// Byte offset of element (row, col) in a 128B-swizzled tile of 64-element
// (128-byte) rows of 2-byte elements.
__device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t col) {
  const uint32_t chunk = (col >> 3) ^ (row & 7);
  return row * 128u + chunk * 16u + (col & 7) * 2u;
}

// Byte offset of float (row, col) in a 128B-swizzled tile of 32-float
// (128-byte) rows: TMA's CU_TENSOR_MAP_SWIZZLE_128B layout for 4-byte data.
__device__ __forceinline__ uint32_t sw128_off_f32(uint32_t row, uint32_t col) {
  const uint32_t chunk = (col >> 2) ^ (row & 7);
  return row * 128u + chunk * 16u + (col & 3) * 4u;
}

}  // namespace umma
}  // namespace mr
