// Gated DeltaNet scan, per-step form with segment checkpoints and a
// recompute backward. The reference carries this recurrence as a design only
// (docs/DESIGN_gated_deltanet.md), which plans this per-step kernel pair first
// (its section 7, phase 2) and the chunked WY form after it. Per (batch row b,
// head h) the state is S [Dh(i, key axis), Dh(j, value axis)]:
//
//   p_t = S_{t-1}^T k_t,  w_t = beta_t (v_t - alpha_t p_t)
//   S_t = alpha_t S_{t-1} + k_t w_t^T          (= alpha (I - beta k k^T) S + beta k v^T, R1'')
//   o_t = S_t^T q_t = alpha_t S_{t-1}^T q_t + (k_t . q_t) w_t                       (R2')
//
// Inputs q, k, v [B,L,H,Dh] (q, k L2-normalised by the caller), alpha, beta
// [B,L,H] already activated (the design's "caller pre-activates" contract,
// section 7), all in one dtype; o [B,L,H,Dh] float32; checkpoints
// [B, L/seg, H, Dh, Dh] float32 (i-major, j fastest; the last one is the final
// state); the optional initial state h0 and its gradient in the same [B,H,Dh,Dh]
// layout.
//
// Layout on the GPU: one CTA per unit (b, h) of 4*Dh threads. Thread (j, g)
// owns column j of S, rows g*Dh/4 .. (g+1)*Dh/4 - 1, in registers; the four
// row groups of a column sit in lanes 8 apart of one warp, so the reductions
// over i that the recurrence needs each step (p, S^T q, the adjoint's d) are
// a register dot product plus two shuffles. The backward's reductions over j
// (grad_q = S_t go, grad_k = G w + S_{t-1} gp) go through shared memory once
// per step.
//
// Backward: per segment (newest first), phase A replays the forward from the
// segment's checkpoint, storing w_t and p_t per step and a sub-checkpoint of
// S every kGdnK steps in a per-CTA scratch (short-lived, L2-resident); phase B
// walks the sub-blocks newest first, replays the kGdnK states S_{t-1} of the
// sub-block from its sub-checkpoint into thread-private shared-memory slots
// (with the stored w, two operations per element and step), and runs the
// adjoint step (docs/DESIGN_gated_deltanet.md:334-401):
//   G += q go^T;  d = G^T k;  gp = -alpha beta d
//   grad_q = S_t go,  grad_k = G w + S_{t-1} gp,  grad_v = beta d
//   grad_alpha = <G, S_{t-1}> - beta d.p,  grad_beta = d.(v - alpha p)
//   G <- alpha G + k gp^T
// The replays use the forward's operations in the forward's order, so they
// reproduce its states bit for bit.
#include "common.cuh"

namespace mr {

constexpr int kGdnK = 4;           // steps per replayed sub-block of the backward
constexpr int kGdnMaxCtas = 4096;  // backward CTAs (each walks units), bounds the scratch

// R consecutive elements of T at p (16-byte aligned) as floats
template <typename T, int R>
__device__ __forceinline__ void gdn_load_rows(const T* p, float (&f)[R]) {
  constexpr int VN = 16 / (int)sizeof(T);
  static_assert(R % VN == 0, "rows per thread must fill 16-byte vectors");
#pragma unroll
  for (int c = 0; c < R / VN; ++c) {
    const Vec<T, VN> x = ld_vec<T, VN>(p + c * VN);
#pragma unroll
    for (int e = 0; e < VN; ++e) f[c * VN + e] = to_f(x.v[e]);
  }
}

// sum over the four row groups of a column (lanes 8 and 16 apart); every lane
// of the group gets the same bits
__device__ __forceinline__ float gdn_group_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 8);
  x += __shfl_xor_sync(0xffffffffu, x, 16);
  return x;
}

__device__ __forceinline__ float gdn_warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// one step of the state update, shared by the forward and both replays
template <int R>
__device__ __forceinline__ void gdn_update(float (&S)[R], const float (&kr)[R], float a, float w) {
#pragma unroll
  for (int r = 0; r < R; ++r) S[r] = fmaf(a, S[r], __fmul_rn(kr[r], w));
}

template <int R>
__device__ __forceinline__ float gdn_dot(const float (&x)[R], const float (&y)[R]) {
  float acc = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) acc = fmaf(x[r], y[r], acc);
  return acc;
}

template <typename T, int DH, bool kH0>
__global__ void __launch_bounds__(DH * 4)
gdn_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               const T* __restrict__ alpha, const T* __restrict__ beta, int L, int H, int seg,
               float* __restrict__ y, float* __restrict__ ckpt, const float* __restrict__ h0) {
  constexpr int R = DH / 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 3, j = warp * 8 + (lane & 7), i0 = g * R;
  const int64_t b = blockIdx.x / H;
  const int h = blockIdx.x % H;
  const int nseg = L / seg;
  const int64_t sbase = ((b * H + h) * DH + i0) * (int64_t)DH + j;  // element (i0, j) of [B,H,DH,DH]
  float S[R];
#pragma unroll
  for (int r = 0; r < R; ++r) S[r] = kH0 ? h0[sbase + r * DH] : 0.f;

  for (int t = 0; t < L; ++t) {
    const int64_t row = (b * L + t) * H + h;
    float kr[R], qr[R];
    gdn_load_rows<T, R>(k + row * DH + i0, kr);
    gdn_load_rows<T, R>(q + row * DH + i0, qr);
    const float vj = to_f(v[row * DH + j]);
    const float a = to_f(alpha[row]), bt = to_f(beta[row]);
    const float p = gdn_group_sum(gdn_dot(kr, S));
    const float sq = gdn_group_sum(gdn_dot(qr, S));
    const float kq = gdn_group_sum(gdn_dot(kr, qr));
    const float w = bt * fmaf(-a, p, vj);
    if (g == 0) y[row * DH + j] = fmaf(a, sq, kq * w);
    gdn_update(S, kr, a, w);
    if ((t + 1) % seg == 0) {
      float* c = ckpt + ((b * nseg + (t + 1) / seg - 1) * H + h) * (int64_t)DH * DH + (int64_t)i0 * DH + j;
#pragma unroll
      for (int r = 0; r < R; ++r) c[r * DH] = S[r];
    }
  }
}

template <int DH>
struct GdnBwdSmem {
  static constexpr int NT = DH * 4;
  static constexpr size_t slots = (size_t)kGdnK * DH * DH;  // [K][R][NT], thread-private
  static constexpr size_t red = (size_t)2 * DH * (DH + 4);  // [2][DH(j)][DH + 4 (i)]
  static constexpr size_t bytes = (slots + red + 2 * (NT / 32)) * sizeof(float);
};

// per-CTA scratch: sub-checkpoints [ceil(seg/K)][R][NT], then w and p [seg][DH]
__host__ __device__ __forceinline__ int64_t gdn_scratch_floats(int64_t Dh, int64_t seg) {
  return (seg + kGdnK - 1) / kGdnK * Dh * Dh + 2 * seg * Dh;
}

template <typename T, int DH, bool kH0>
__global__ void __launch_bounds__(DH * 4, DH == 64 ? 2 : 4)
gdn_bwd_kernel(const float* __restrict__ gy, const float* __restrict__ gfinal, const float* __restrict__ ckpt,
               const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               const T* __restrict__ alpha, const T* __restrict__ beta, int L, int H, int seg, int units,
               T* __restrict__ gq, T* __restrict__ gk, T* __restrict__ gv, T* __restrict__ galpha,
               T* __restrict__ gbeta, float* __restrict__ ws, const float* __restrict__ h0,
               float* __restrict__ gh0) {
  constexpr int R = DH / 4, NT = DH * 4, NW = NT / 32, K = kGdnK, RS = DH + 4;
  extern __shared__ float4 gdn_smem[];
  float* slots = reinterpret_cast<float*>(gdn_smem);
  float* red = slots + K * DH * DH;
  float* rsc = red + 2 * DH * RS;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 3, j = warp * 8 + (lane & 7), i0 = g * R;
  const int nseg = L / seg, nsb = (seg + K - 1) / K;
  float* sub = ws + (int64_t)blockIdx.x * gdn_scratch_floats(DH, seg);
  float* vw = sub + (int64_t)nsb * DH * DH;  // [seg][DH]
  float* vp = vw + (int64_t)seg * DH;        // [seg][DH]
  // role in the reduction over j: vector (0 grad_q, 1 grad_k), quad of rows, column phase
  const int rv = tid / (NT / 2), rq = (tid % (NT / 2)) / 8, rj = tid & 7;

  for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
    const int64_t b = unit / H;
    const int h = unit % H;
    const int64_t sbase = ((b * H + h) * DH + i0) * (int64_t)DH + j;
    float G[R];
#pragma unroll
    for (int r = 0; r < R; ++r) G[r] = gfinal != nullptr ? gfinal[sbase + r * DH] : 0.f;

    for (int s = nseg - 1; s >= 0; --s) {
      const int64_t t0 = (int64_t)s * seg;
      // ---- phase A: replay the segment, keep w, p and every K-th state
      {
        float S[R];
        const float* src = s > 0 ? ckpt + ((b * nseg + s - 1) * H + h) * (int64_t)DH * DH + (int64_t)i0 * DH + j
                           : kH0 ? h0 + sbase : nullptr;
#pragma unroll
        for (int r = 0; r < R; ++r) S[r] = src != nullptr ? src[r * DH] : 0.f;
        for (int tl = 0; tl < seg; ++tl) {
          if (tl % K == 0) {
            float* d = sub + (int64_t)(tl / K) * DH * DH + tid;
#pragma unroll
            for (int r = 0; r < R; ++r) d[r * NT] = S[r];
          }
          const int64_t row = (b * L + t0 + tl) * H + h;
          float kr[R];
          gdn_load_rows<T, R>(k + row * DH + i0, kr);
          const float vj = to_f(v[row * DH + j]);
          const float a = to_f(alpha[row]), bt = to_f(beta[row]);
          const float p = gdn_group_sum(gdn_dot(kr, S));
          const float w = bt * fmaf(-a, p, vj);
          if (g == 0) {
            vw[tl * DH + j] = w;
            vp[tl * DH + j] = p;
          }
          gdn_update(S, kr, a, w);
        }
      }
      __syncthreads();  // w, p of the segment visible to the column's four row groups

      // ---- phase B: sub-blocks newest first
      for (int sb = nsb - 1; sb >= 0; --sb) {
        const int tb = sb * K, nk = min(K, seg - tb);
        {
          float cur[R];
          const float* src = sub + (int64_t)sb * DH * DH + tid;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            cur[r] = src[r * NT];
            slots[r * NT + tid] = cur[r];
          }
#pragma unroll
          for (int m = 1; m < K; ++m) {
            if (m < nk) {
              const int tl = tb + m - 1;
              const int64_t row = (b * L + t0 + tl) * H + h;
              float kr[R];
              gdn_load_rows<T, R>(k + row * DH + i0, kr);
              gdn_update(cur, kr, to_f(alpha[row]), vw[tl * DH + j]);
#pragma unroll
              for (int r = 0; r < R; ++r) slots[(m * R + r) * NT + tid] = cur[r];
            }
          }
        }
#pragma unroll
        for (int m = K - 1; m >= 0; --m) {
          if (m < nk) {
            const int tl = tb + m;
            const int64_t row = (b * L + t0 + tl) * H + h;
            float kr[R], Sp[R];
            gdn_load_rows<T, R>(k + row * DH + i0, kr);
            const float go = gy[row * DH + j];
            {
              float qr[R];
              gdn_load_rows<T, R>(q + row * DH + i0, qr);
#pragma unroll
              for (int r = 0; r < R; ++r) G[r] = fmaf(qr[r], go, G[r]);  // output seed (B0)
            }
#pragma unroll
            for (int r = 0; r < R; ++r) Sp[r] = slots[(m * R + r) * NT + tid];
            const float vj = to_f(v[row * DH + j]);
            const float a = to_f(alpha[row]), bt = to_f(beta[row]);
            const float w = vw[tl * DH + j], p = vp[tl * DH + j];
            const float d = gdn_group_sum(gdn_dot(kr, G));
            const float gp = -a * bt * d;
            float gaP = gdn_dot(G, Sp), gbP = 0.f;
            if (g == 0) {
              gaP = fmaf(-bt * d, p, gaP);
              gbP = d * fmaf(-a, p, vj);
              gv[row * DH + j] = from_f<T>(bt * d);
            }
            // this column's terms of grad_q (S_t go) and grad_k (G w + S_{t-1} gp)
            float* rw = red + (int64_t)j * RS + i0;
#pragma unroll
            for (int c = 0; c < R / 4; ++c) {
              float4 r1, r2;
              float* p1 = &r1.x;
              float* p2 = &r2.x;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int r = 4 * c + e;
                p1[e] = fmaf(a, Sp[r], kr[r] * w) * go;
                p2[e] = fmaf(G[r], w, Sp[r] * gp);
              }
              *reinterpret_cast<float4*>(rw + 4 * c) = r1;
              *reinterpret_cast<float4*>(rw + DH * RS + 4 * c) = r2;
            }
#pragma unroll
            for (int r = 0; r < R; ++r) G[r] = fmaf(a, G[r], kr[r] * gp);  // adjoint to t-1 (Bp')
            gaP = gdn_warp_sum(gaP);
            gbP = gdn_warp_sum(gbP);
            if (lane == 0) {
              rsc[warp] = gaP;
              rsc[NW + warp] = gbP;
            }
            __syncthreads();
            {
              float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
              const float* rr = red + (int64_t)rv * DH * RS + 4 * rq;
#pragma unroll
              for (int jj = rj; jj < DH; jj += 8) {
                const float4 x = *reinterpret_cast<const float4*>(rr + jj * RS);
                acc.x += x.x, acc.y += x.y, acc.z += x.z, acc.w += x.w;
              }
#pragma unroll
              for (int o = 1; o < 8; o <<= 1) {
                acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
                acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
                acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
                acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
              }
              if (rj == 0) {
                const float out[4] = {acc.x, acc.y, acc.z, acc.w};
                st_vec<T, 4>((rv == 0 ? gq : gk) + row * DH + 4 * rq, out);
              }
              if (tid == 0) {
                float sa = 0.f, sbeta = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < NW; ++w2) {
                  sa += rsc[w2];
                  sbeta += rsc[NW + w2];
                }
                galpha[row] = from_f<T>(sa);
                gbeta[row] = from_f<T>(sbeta);
              }
            }
            __syncthreads();
          }
        }
      }
    }
    // the adjoint carried past step 0 is the gradient of the initial state
    if (kH0 && gh0 != nullptr)
#pragma unroll
      for (int r = 0; r < R; ++r) gh0[sbase + r * DH] = G[r];
  }
}

// ============================================================================
// host launchers
// ============================================================================

template <typename Kern>
static int gdn_set_smem(Kern kernel, size_t bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return set_error(MR_E_LAUNCH, "gated_deltanet: cannot reserve %zu bytes of shared memory", bytes);
  return MR_OK;
}

template <typename T, int DH>
static int gdn_fwd_dh(const T* q, const T* k, const T* v, const T* al, const T* be, int64_t batch, int64_t L,
                      int64_t H, int64_t seg, float* y, float* ckpt, const float* h0, cudaStream_t st) {
  const dim3 grid((unsigned)(batch * H));
  auto kern = h0 != nullptr ? gdn_fwd_kernel<T, DH, true> : gdn_fwd_kernel<T, DH, false>;
  kern<<<grid, DH * 4, 0, st>>>(q, k, v, al, be, (int)L, (int)H, (int)seg, y, ckpt, h0);
  return check_launch("gdn_fwd_kernel");
}

template <typename T>
int gdn_fwd_launch(const void* q, const void* k, const void* v, const void* alpha, const void* beta, int64_t batch,
                   int64_t L, int64_t H, int64_t Dh, int64_t seg, float* y, float* ckpt, const float* h0,
                   cudaStream_t st) {
  const T *q_ = (const T*)q, *k_ = (const T*)k, *v_ = (const T*)v, *a_ = (const T*)alpha, *b_ = (const T*)beta;
  if (Dh == 32) return gdn_fwd_dh<T, 32>(q_, k_, v_, a_, b_, batch, L, H, seg, y, ckpt, h0, st);
  return gdn_fwd_dh<T, 64>(q_, k_, v_, a_, b_, batch, L, H, seg, y, ckpt, h0, st);
}

static int64_t gdn_bwd_grid(int64_t batch, int64_t H) {
  const int64_t units = batch * H;
  return units < kGdnMaxCtas ? units : kGdnMaxCtas;
}

size_t gdn_bwd_ws_bytes(int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg) {
  (void)L;
  return (size_t)gdn_bwd_grid(batch, H) * gdn_scratch_floats(Dh, seg) * sizeof(float);
}

template <typename T, int DH>
static int gdn_bwd_dh(const float* gy, const float* gf, const float* ckpt, const T* q, const T* k, const T* v,
                      const T* al, const T* be, int64_t batch, int64_t L, int64_t H, int64_t seg, T* gq, T* gk,
                      T* gv, T* ga, T* gb, float* ws, const float* h0, float* gh0, cudaStream_t st) {
  constexpr size_t sm = GdnBwdSmem<DH>::bytes;
  auto kern = h0 != nullptr ? gdn_bwd_kernel<T, DH, true> : gdn_bwd_kernel<T, DH, false>;
  if (int rc = gdn_set_smem(kern, sm)) return rc;
  const dim3 grid((unsigned)gdn_bwd_grid(batch, H));
  kern<<<grid, DH * 4, sm, st>>>(gy, gf, ckpt, q, k, v, al, be, (int)L, (int)H, (int)seg, (int)(batch * H), gq, gk,
                                 gv, ga, gb, ws, h0, gh0);
  return check_launch("gdn_bwd_kernel");
}

template <typename T>
int gdn_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* q, const void* k, const void* v,
                   const void* alpha, const void* beta, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg,
                   void* gq, void* gk, void* gv, void* galpha, void* gbeta, void* ws, const float* h0, float* gh0,
                   cudaStream_t st) {
  const T *q_ = (const T*)q, *k_ = (const T*)k, *v_ = (const T*)v, *a_ = (const T*)alpha, *b_ = (const T*)beta;
  T *gq_ = (T*)gq, *gk_ = (T*)gk, *gv_ = (T*)gv, *ga_ = (T*)galpha, *gb_ = (T*)gbeta;
  if (Dh == 32)
    return gdn_bwd_dh<T, 32>(gy, gf, ckpt, q_, k_, v_, a_, b_, batch, L, H, seg, gq_, gk_, gv_, ga_, gb_,
                             (float*)ws, h0, gh0, st);
  return gdn_bwd_dh<T, 64>(gy, gf, ckpt, q_, k_, v_, a_, b_, batch, L, H, seg, gq_, gk_, gv_, ga_, gb_, (float*)ws,
                           h0, gh0, st);
}

#define MR_INST(T)                                                                                              \
  template int gdn_fwd_launch<T>(const void*, const void*, const void*, const void*, const void*, int64_t,     \
                                 int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t); \
  template int gdn_bwd_launch<T>(const float*, const float*, const float*, const void*, const void*,           \
                                 const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t,    \
                                 int64_t, void*, void*, void*, void*, void*, void*, const float*, float*,      \
                                 cudaStream_t);
MR_INST(float)
MR_INST(__nv_bfloat16)
MR_INST(__half)
#undef MR_INST

}  // namespace mr
