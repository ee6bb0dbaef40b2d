// Shared device helpers for the scan kernels: element conversion, vector
// loads/stores of V consecutive elements, and the launch-error plumbing.
#pragma once

#include <type_traits>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mlrec.h"

namespace mr {

// ---- scalar conversion ------------------------------------------------------
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// ---- GLA gate range of the tensor-core path ----------------------------------
// Gates the chunked GLA kernels compute to within tolerance (their algebra works
// in log g and divides by g for the gate gradient). A unit (batch row, head) with
// any other gate is marked by the chunk kernel with a NaN in its first output
// element (y[b, 0, h, 0] forward, grad_gates[b, 0, h] backward) and recomputed
// by the per-step kernels, which recompute every marked unit (a NaN there for any
// other reason is recomputed to the same value).
__device__ __forceinline__ bool gla_gate_in_range(float g) { return g >= 1e-3f && g <= 1.f; }
constexpr unsigned kMarkNaN = 0x7fc00000u;

// ---- V consecutive elements as one vector access ----------------------------
// Raw storage of V elements of T (V*sizeof(T) bytes: 2..16), loaded/stored as
// a single aligned vector instruction.
template <typename T, int V> struct alignas(sizeof(T) * V) Vec {
  T v[V];
};

template <typename T, int V>
__device__ __forceinline__ Vec<T, V> ld_vec(const T* p) {
  return *reinterpret_cast<const Vec<T, V>*>(p);
}

// Streaming (read-once) load: bypasses L1 allocation.
template <typename T, int V>
__device__ __forceinline__ Vec<T, V> ld_stream(const T* p) {
  Vec<T, V> r;
  constexpr int B = sizeof(T) * V;
  if constexpr (B == 16) {
    int4 t = __ldcs(reinterpret_cast<const int4*>(p));
    r = *reinterpret_cast<Vec<T, V>*>(&t);
  } else if constexpr (B == 8) {
    int2 t = __ldcs(reinterpret_cast<const int2*>(p));
    r = *reinterpret_cast<Vec<T, V>*>(&t);
  } else if constexpr (B == 4) {
    int t = __ldcs(reinterpret_cast<const int*>(p));
    r = *reinterpret_cast<Vec<T, V>*>(&t);
  } else {
    r = *reinterpret_cast<const Vec<T, V>*>(p);
  }
  return r;
}

template <typename T, int V>
__device__ __forceinline__ void st_vec(T* p, const float (&f)[V]) {
  Vec<T, V> r;
  if constexpr (V % 2 == 0 && std::is_same_v<T, __nv_bfloat16>) {
    // pairs by the packed conversion (one instruction per pair, off the XU pipe)
#pragma unroll
    for (int i = 0; i < V; i += 2) *reinterpret_cast<__nv_bfloat162*>(&r.v[i]) = __floats2bfloat162_rn(f[i], f[i + 1]);
  } else if constexpr (V % 2 == 0 && std::is_same_v<T, __half>) {
#pragma unroll
    for (int i = 0; i < V; i += 2) *reinterpret_cast<__half2*>(&r.v[i]) = __floats2half2_rn(f[i], f[i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r.v[i] = from_f<T>(f[i]);
  }
  *reinterpret_cast<Vec<T, V>*>(p) = r;
}

// Streaming (write-once) store of V floats.
template <int V>
__device__ __forceinline__ void st_stream_f32(float* p, const float (&f)[V]) {
  if constexpr (V == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(f[0], f[1], f[2], f[3]));
  } else if constexpr (V == 2) {
    __stcs(reinterpret_cast<float2*>(p), make_float2(f[0], f[1]));
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) __stcs(p + i, f[i]);
  }
}

}  // namespace mr

// ---- host-side error plumbing (defined in mlrec_abi.cu) ---------------------
namespace mr {
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
}  // namespace mr
