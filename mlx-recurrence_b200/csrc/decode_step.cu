// One-token decode steps: the recurrence advanced by a single time step on a
// float32 state cache held in the final state's layout ([B,H,Dh,N] SSD,
// [B,H,Dk,Dv] GLA, [B,D] RG-LRU, [B,2Dp] rotLRU), updated in place, with that
// step's output. The reference has no decode entry point (a decode step there
// is a scan of length 1, each a separate Metal dispatch); the update is one
// step of its pure loops (ssd.py:382-394, gla.py:336-346, rglru.py:274-282,
// rotlru.py:338-351).
//
// The steps are HBM-bound: the state is read and written once (the inputs of
// one token are small), so each kernel streams the state with coalesced
// accesses, one CTA per (batch row, head) for SSD and GLA and a grid-stride
// loop over channels for the diagonal scans.
#include "common.cuh"

namespace mr {

constexpr int kStepThreads = 256;
constexpr int kStepWarps = kStepThreads / 32;

__device__ __forceinline__ float step_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// SSD: lanes own state columns n = lane + 32k (k < NK), warps own rows d.
//   h[d,n] <- exp(delta A[h,n]) h[d,n] + delta B[n] u[d];  y[d] = sum_n h[d,n] C[n]
template <typename T, int NK>
__global__ void __launch_bounds__(kStepThreads)
ssd_step_kernel(const T* __restrict__ u, const T* __restrict__ delta, const T* __restrict__ Bm,
                const T* __restrict__ Cm, const float* __restrict__ A, int64_t ash, int64_t asn, int H,
                int Dh, int N, float* __restrict__ state, float* __restrict__ y) {
  const int64_t bh = blockIdx.x;
  const int h = (int)(bh % H);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float dt = to_f(delta[bh]);
  float dec[NK], dB[NK], cv[NK];
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    const int n = lane + 32 * k;
    const bool ok = n < N;
    dec[k] = ok ? expf(dt * A[h * ash + n * asn]) : 0.f;
    dB[k] = ok ? dt * to_f(Bm[bh * N + n]) : 0.f;
    cv[k] = ok ? to_f(Cm[bh * N + n]) : 0.f;
  }
  for (int d = warp; d < Dh; d += kStepWarps) {
    const float ud = to_f(u[bh * Dh + d]);
    float* row = state + (bh * Dh + d) * (int64_t)N;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < NK; ++k) {
      const int n = lane + 32 * k;
      if (n < N) {
        const float hv = dec[k] * row[n] + dB[k] * ud;
        row[n] = hv;
        acc += hv * cv[k];
      }
    }
    acc = step_warp_sum(acc);
    if (lane == 0) y[bh * Dh + d] = acc;
  }
}

// GLA: lanes own columns j = lane + 32c (the v dimension), warps own rows i.
//   S[i,j] <- g S[i,j] + k_i v_j;  y_j = sum_i q_i S[i,j]
template <typename T, int NC>
__global__ void __launch_bounds__(kStepThreads)
gla_step_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                const T* __restrict__ gates, int Dh, float* __restrict__ state, float* __restrict__ y) {
  __shared__ float red[kStepWarps][32 * NC];
  const int64_t bh = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float g = to_f(gates[bh]);
  float vj[NC], acc[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int j = lane + 32 * c;
    vj[c] = j < Dh ? to_f(v[bh * Dh + j]) : 0.f;
    acc[c] = 0.f;
  }
  for (int i = warp; i < Dh; i += kStepWarps) {
    const float ki = to_f(k[bh * Dh + i]), qi = to_f(q[bh * Dh + i]);
    float* row = state + (bh * Dh + i) * (int64_t)Dh;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int j = lane + 32 * c;
      if (j < Dh) {
        const float s = g * row[j] + ki * vj[c];
        row[j] = s;
        acc[c] += qi * s;
      }
    }
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) red[warp][lane + 32 * c] = acc[c];
  __syncthreads();
  for (int j = threadIdx.x; j < Dh; j += kStepThreads) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kStepWarps; ++w) s += red[w][j];
    y[bh * Dh + j] = s;
  }
}

// RG-LRU: h <- a h + x, y = h (per channel)
template <typename T>
__global__ void __launch_bounds__(kStepThreads)
rglru_step_kernel(const T* __restrict__ a, const T* __restrict__ x, int64_t n, float* __restrict__ state,
                  float* __restrict__ y) {
  for (int64_t i = (int64_t)blockIdx.x * kStepThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kStepThreads) {
    const float hv = to_f(a[i]) * state[i] + to_f(x[i]);
    state[i] = hv;
    y[i] = hv;
  }
}

// rotLRU: per pair p, (u, w) <- a R(theta) (u, w) + (x_2p, x_2p+1), y = the new pair
template <typename T>
__global__ void __launch_bounds__(kStepThreads)
rotlru_step_kernel(const T* __restrict__ a, const T* __restrict__ cs, const T* __restrict__ sn,
                   const T* __restrict__ x, int64_t npairs, float* __restrict__ state, float* __restrict__ y) {
  for (int64_t p = (int64_t)blockIdx.x * kStepThreads + threadIdx.x; p < npairs;
       p += (int64_t)gridDim.x * kStepThreads) {
    const float av = to_f(a[p]), c = to_f(cs[p]), s = to_f(sn[p]);
    const float2 h = reinterpret_cast<const float2*>(state)[p];
    const float un = av * (c * h.x - s * h.y) + to_f(x[2 * p]);
    const float wn = av * (s * h.x + c * h.y) + to_f(x[2 * p + 1]);
    reinterpret_cast<float2*>(state)[p] = make_float2(un, wn);
    reinterpret_cast<float2*>(y)[p] = make_float2(un, wn);
  }
}

static unsigned stream_grid(int64_t n) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + kStepThreads - 1) / kStepThreads;
  const int64_t cap = (int64_t)sms * 8;  // resident CTAs of 256 threads, grid-stride beyond
  return (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
}

template <typename T>
int ssd_step_launch(const void* u, const void* delta, const void* Bm, const void* Cm, const float* A, int64_t ash,
                    int64_t asn, int64_t batch, int64_t H, int64_t Dh, int64_t N, float* state, float* y,
                    cudaStream_t st) {
  const dim3 grid((unsigned)(batch * H));
  const T *u_ = (const T*)u, *d_ = (const T*)delta, *B_ = (const T*)Bm, *C_ = (const T*)Cm;
  if (N <= 32)
    ssd_step_kernel<T, 1><<<grid, kStepThreads, 0, st>>>(u_, d_, B_, C_, A, ash, asn, (int)H, (int)Dh, (int)N, state, y);
  else if (N <= 64)
    ssd_step_kernel<T, 2><<<grid, kStepThreads, 0, st>>>(u_, d_, B_, C_, A, ash, asn, (int)H, (int)Dh, (int)N, state, y);
  else
    ssd_step_kernel<T, 4><<<grid, kStepThreads, 0, st>>>(u_, d_, B_, C_, A, ash, asn, (int)H, (int)Dh, (int)N, state, y);
  return check_launch("ssd_step_kernel");
}

template <typename T>
int gla_step_launch(const void* q, const void* k, const void* v, const void* gates, int64_t batch, int64_t H,
                    int64_t Dh, float* state, float* y, cudaStream_t st) {
  const dim3 grid((unsigned)(batch * H));
  const T *q_ = (const T*)q, *k_ = (const T*)k, *v_ = (const T*)v, *g_ = (const T*)gates;
  if (Dh <= 32)
    gla_step_kernel<T, 1><<<grid, kStepThreads, 0, st>>>(q_, k_, v_, g_, (int)Dh, state, y);
  else if (Dh <= 64)
    gla_step_kernel<T, 2><<<grid, kStepThreads, 0, st>>>(q_, k_, v_, g_, (int)Dh, state, y);
  else
    gla_step_kernel<T, 4><<<grid, kStepThreads, 0, st>>>(q_, k_, v_, g_, (int)Dh, state, y);
  return check_launch("gla_step_kernel");
}

template <typename T>
int rglru_step_launch(const void* a, const void* x, int64_t batch, int64_t D, float* state, float* y,
                      cudaStream_t st) {
  const int64_t n = batch * D;
  rglru_step_kernel<T><<<stream_grid(n), kStepThreads, 0, st>>>((const T*)a, (const T*)x, n, state, y);
  return check_launch("rglru_step_kernel");
}

template <typename T>
int rotlru_step_launch(const void* a, const void* cs, const void* sn, const void* x, int64_t batch, int64_t Dp,
                       float* state, float* y, cudaStream_t st) {
  const int64_t np = batch * Dp;
  rotlru_step_kernel<T><<<stream_grid(np), kStepThreads, 0, st>>>((const T*)a, (const T*)cs, (const T*)sn,
                                                                  (const T*)x, np, state, y);
  return check_launch("rotlru_step_kernel");
}

#define MR_INST(T)                                                                                         \
  template int ssd_step_launch<T>(const void*, const void*, const void*, const void*, const float*, int64_t, \
                                  int64_t, int64_t, int64_t, int64_t, int64_t, float*, float*, cudaStream_t); \
  template int gla_step_launch<T>(const void*, const void*, const void*, const void*, int64_t, int64_t,     \
                                  int64_t, float*, float*, cudaStream_t);                                  \
  template int rglru_step_launch<T>(const void*, const void*, int64_t, int64_t, float*, float*,           \
                                    cudaStream_t);                                                         \
  template int rotlru_step_launch<T>(const void*, const void*, const void*, const void*, int64_t, int64_t, \
                                     float*, float*, cudaStream_t);
MR_INST(float)
MR_INST(__nv_bfloat16)
MR_INST(__half)
#undef MR_INST

}  // namespace mr
