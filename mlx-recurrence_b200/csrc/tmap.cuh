// TMA tensor maps (host) and tiled bulk-tensor copies (device).
//
// A tensor map describes a 2-D row-major view [rows, cols] of a global array
// and the box (tile) one copy moves into shared memory. The driver's encoder
// is fetched once through cudaGetDriverEntryPoint, so the library needs no
// link-time dependency on libcuda. Every CTA loads its own tiles from this
// GPU's memory; no copy is shared across the CTAs of a cluster.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mr {

// Encode a 2-D tiled map: inner (contiguous) extent `cols`, outer `rows`,
// row pitch `row_bytes`, box [box_rows, box_cols], no swizzle unless given.
// Out-of-bounds box elements read as zero. Returns MR_OK or an MR_E_* code.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

// 3-D tiled map over [d2, d1, d0] (d0 contiguous) with byte pitches s1, s2
// for dims 1 and 2 and box [b2, b1, b0].
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0,
                 uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

template <typename T> struct TmapType;
template <> struct TmapType<float> { static constexpr CUtensorMapDataType v = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; };
template <> struct TmapType<__nv_bfloat16> { static constexpr CUtensorMapDataType v = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; };
template <> struct TmapType<__half> { static constexpr CUtensorMapDataType v = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; };

// Tiled 2-D load of the box at (col x, row y) into shared memory, completing
// on `bar`. x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
      "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
      "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
      : "memory");
}

// Tiled 3-D store of a shared-memory box to global memory (bulk group).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int x, int y, int z, const void* src) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(z), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(src)))
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// wait until at most N of this thread's committed bulk groups are still reading shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
// Wait until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace mr
