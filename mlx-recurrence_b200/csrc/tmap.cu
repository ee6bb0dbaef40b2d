// Host-side TMA tensor-map encoding (see tmap.cuh).
#include <mutex>

#include "common.cuh"
#include "tmap.cuh"

namespace mr {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// The encoder checks the address against the calling thread's current context.
// A thread that has made no CUDA runtime call yet (an autograd worker thread
// that only reused cached allocations, say) has none: bind its current device's
// primary context (the runtime does so on cudaSetDevice) and encode again.
static bool bind_current_device() {
  int d = 0;
  return cudaGetDevice(&d) == cudaSuccess && cudaSetDevice(d) == cudaSuccess;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = encoder();
  if (enc == nullptr) return set_error(MR_E_DEVICE, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (row_bytes & 15u) || ((box_cols * elem_bytes) & 15u))
    return set_error(MR_E_ALIGN, "tensor map: base, row pitch and box row must be 16-byte multiples");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  auto encode = [&] {
    return enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT && bind_current_device()) r = encode();
  if (r != CUDA_SUCCESS)
    return set_error(MR_E_LAUNCH, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, box %u x %u",
                     (int)r, (unsigned long long)cols, (unsigned long long)rows, box_cols, box_rows);
  return MR_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0,
                 uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = encoder();
  if (enc == nullptr) return set_error(MR_E_DEVICE, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (s1 & 15u) || (s2 & 15u) || ((b0 * elem_bytes) & 15u))
    return set_error(MR_E_ALIGN, "tensor map: base, pitches and box row must be 16-byte multiples");
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  auto encode = [&] {
    return enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT && bind_current_device()) r = encode();
  if (r != CUDA_SUCCESS)
    return set_error(MR_E_LAUNCH, "cuTensorMapEncodeTiled (3d) failed (%d)", (int)r);
  return MR_OK;
}

}  // namespace mr
