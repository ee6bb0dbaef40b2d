// Diagnostic: one 128x128x128 bf16 tcgen05 tile for every shared-memory
// operand form the chunked SSD/GLA kernels use, checked by a GPU test
// against a float64 matmul:
//   D1 = A * Bk^T   A K-major (TMA, 128B swizzle), Bk K-major (TMA)
//   D2 = A * Bmn    A K-major written by threads, Bmn MN-major (TMA)
//   D3 = Amn^T * Bmn  A MN-major (TMA, two 64-wide MN blocks), Bmn MN-major
// A, Bk, Amn are [128, 128] bf16 row-major, Bmn is [128, 64]; D1 is
// [128, 128] f32, D2 and D3 are [128, 64] f32.
#include "common.cuh"
#include "tma.cuh"
#include "tmap.cuh"
#include "umma.cuh"

namespace mr {

constexpr int kTile = 16384;  // one [128 rows x 64 bf16] swizzled tile

__global__ void __launch_bounds__(256, 1)
umma_selftest_kernel(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tBk,
                     const __grid_constant__ CUtensorMap tBmn, const __grid_constant__ CUtensorMap tAmn,
                     const __nv_bfloat16* __restrict__ A, float* __restrict__ D1, float* __restrict__ D2,
                     float* __restrict__ D3) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;                  // 2 tiles: K 0-63, 64-127
  unsigned char* sB = sA + 2 * kTile;        // 2 tiles
  unsigned char* sBmn = sB + 2 * kTile;      // 1 tile [K=128][N=64]
  unsigned char* sAmn = sBmn + kTile;        // 2 tiles [K=128][M 0-63], [K][M 64-127]
  unsigned char* sAt = sAmn + 2 * kTile;     // 2 tiles, thread-written K-major A
  uint64_t* bars = reinterpret_cast<uint64_t*>(sAt + 2 * kTile);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);

  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    umma::tmem_alloc(tmem_slot, 256);
    umma::tmem_relinquish();
  }
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tbase = *tmem_slot;

  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], 7 * kTile);
    tma_load_2d(sA, &tA, 0, 0, &bars[0]);
    tma_load_2d(sA + kTile, &tA, 64, 0, &bars[0]);
    tma_load_2d(sB, &tBk, 0, 0, &bars[0]);
    tma_load_2d(sB + kTile, &tBk, 64, 0, &bars[0]);
    tma_load_2d(sBmn, &tBmn, 0, 0, &bars[0]);
    tma_load_2d(sAmn, &tAmn, 0, 0, &bars[0]);
    tma_load_2d(sAmn + kTile, &tAmn, 64, 0, &bars[0]);
  }
  // thread-written K-major copy of A: thread -> (row, half)
  {
    const int row = tid >> 1, half = tid & 1;
    unsigned char* dst = sAt + half * kTile;
#pragma unroll
    for (int c = 0; c < 64; c += 8) {
      const int4 v = *reinterpret_cast<const int4*>(A + row * 128 + half * 64 + c);
      *reinterpret_cast<int4*>(dst + umma::sw128_off(row, c)) = v;
    }
    fence_proxy_async_smem();
  }
  __syncthreads();
  mbar_wait(&bars[0], 0);

  if (tid == 0) {
    umma::fence_after_sync();
    const uint32_t aK = smem_u32(sA), bK = smem_u32(sB), bMN = smem_u32(sBmn), aMN = smem_u32(sAmn),
                   aT = smem_u32(sAt);
    const uint32_t id1 = umma::idesc_f16(128, 128, 1, 0, 0);
    const uint32_t id2 = umma::idesc_f16(128, 64, 1, 0, 1);
    const uint32_t id3 = umma::idesc_f16(128, 64, 1, 1, 1);
    for (int k = 0; k < 8; ++k) {
      const uint32_t ko = (k >> 2) * kTile + (k & 3) * 32;  // K-major: tile switch + 32 B per K16
      umma::mma_f16(tbase + 0, umma::sdesc_k(aK + ko), umma::sdesc_k(bK + ko), id1, k > 0);
      umma::mma_f16(tbase + 128, umma::sdesc_k(aT + ko), umma::sdesc_mn(bMN + k * 2048, kTile), id2, k > 0);
      umma::mma_f16(tbase + 192, umma::sdesc_mn(aMN + k * 2048, kTile), umma::sdesc_mn(bMN + k * 2048, kTile),
                    id3, k > 0);
    }
    umma::commit(&bars[1]);
  }
  mbar_wait(&bars[1], 0);
  umma::fence_after_sync();

  if (warp < 4) {
    const int row = tid;  // TMEM lane = row
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float v[16];
    for (int c = 0; c < 128; c += 16) {
      umma::tmem_ld16(tbase + lane_base + c, v);
      umma::tmem_wait_ld();
      for (int i = 0; i < 16; ++i) D1[row * 128 + c + i] = v[i];
    }
    for (int c = 0; c < 64; c += 16) {
      umma::tmem_ld16(tbase + lane_base + 128 + c, v);
      umma::tmem_wait_ld();
      for (int i = 0; i < 16; ++i) D2[row * 64 + c + i] = v[i];
      umma::tmem_ld16(tbase + lane_base + 192 + c, v);
      umma::tmem_wait_ld();
      for (int i = 0; i < 16; ++i) D3[row * 64 + c + i] = v[i];
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tbase, 256);
}

int umma_selftest_launch(const void* A, const void* Bk, const void* Bmn, const void* Amn, float* D1,
                         float* D2, float* D3, cudaStream_t st) {
  CUtensorMap tA, tBk, tBmn, tAmn;
  const auto BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  if (int rc = make_tmap_2d(&tA, A, BF, 2, 128, 128, 256, 64, 128, SW)) return rc;
  if (int rc = make_tmap_2d(&tBk, Bk, BF, 2, 128, 128, 256, 64, 128, SW)) return rc;
  if (int rc = make_tmap_2d(&tBmn, Bmn, BF, 2, 64, 128, 128, 64, 128, SW)) return rc;
  if (int rc = make_tmap_2d(&tAmn, Amn, BF, 2, 128, 128, 256, 64, 128, SW)) return rc;
  // the whole opt-in shared memory, so every descriptor-derived address of
  // the tile stays inside this CTA's allocation
  const size_t sm = 227 * 1024;
  cudaError_t e = cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return set_error(MR_E_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  umma_selftest_kernel<<<1, 256, sm, st>>>(tA, tBk, tBmn, tAmn, (const __nv_bfloat16*)A, D1, D2, D3);
  return check_launch("umma_selftest_kernel");
}

// Bounded-wait diagnostic: every CTA waits on a barrier that never completes,
// once with `limit_ns`, once with the standard limit, and records both
// durations. Nothing is in flight, so giving up leaves no copy behind.
__global__ void __launch_bounds__(32, 1) wait_timeout_selftest_kernel(uint64_t limit_ns, uint64_t* elapsed_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    uint64_t t0 = globaltimer_ns();
    mbar_wait_ns(&bar, 0, limit_ns);
    uint64_t t1 = globaltimer_ns();
    mbar_wait(&bar, 0);
    uint64_t t2 = globaltimer_ns();
    elapsed_ns[2 * blockIdx.x] = t1 - t0;
    elapsed_ns[2 * blockIdx.x + 1] = t2 - t1;
  }
}

int wait_selftest_launch(int ctas, uint64_t limit_ns, uint64_t* elapsed_ns, cudaStream_t st) {
  wait_timeout_selftest_kernel<<<(unsigned)ctas, 32, 0, st>>>(limit_ns, elapsed_ns);
  return check_launch("wait_timeout_selftest_kernel");
}

int selftest_device_error(bool clear) { return read_device_error(clear); }

}  // namespace mr
