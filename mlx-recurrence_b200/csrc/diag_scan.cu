// Diagonal scans: RG-LRU (real, h <- a*h + x) and rotational LRU (complex
// pair, h <- a*R(theta)*h + x), forward with segment checkpoints and
// checkpoint-recompute backward.
//
// Reference kernels: mlx_recurrence/rglru.py:64-203, rotlru.py:80-266.
// The reference walks all L steps with one thread per channel (rglru.py:81-101);
// at B*D = 20,480 channels that leaves a B200 far from HBM saturation.
//
// Layout of the work. A CTA (8 warps) owns a tile of W adjacent channels
// (pairs for rotLRU) of one batch row and walks L in blocks of TB steps.
// Each block's input rows are streamed global -> shared memory by the TMA
// unit (one cp.async.bulk per row and input, completing on a per-stage
// mbarrier) through an S-stage ring, so S-1 blocks are in flight while one
// is computed and the registers stay free. Inside a block warp w owns TW =
// TB/8 consecutive steps and lane l owns W/32 adjacent channels.
//
// The scan inside a block is the three-phase chunk scan over the affine step
// maps h -> a*h + x:
//   1. each thread folds its TW steps into one map (A, H),
//   2. the 8 per-warp maps go through shared memory and each thread folds
//      the maps of the warps before it into its carry-in,
//   3. each thread re-runs its steps from the carry-in with the reference's
//      exact per-step update (rglru.py:92, rotlru.py:110-111), writing y and
//      the segment checkpoints.
// The backward walks blocks newest -> oldest. Blocks are aligned to segments
// so each block starts from a checkpoint; it regenerates h_{t-1} with the
// same three phases forward, then runs the adjoint c_{t-1} = a_t (gy_t + c_t)
// (rotLRU: conj(z_t) (gy_t + c_t)) with the three phases in reverse.
// Segments longer than one block first regenerate the state at each of
// their block starts (plain loads) into the workspace.
#include "common.cuh"
#include "tma.cuh"
#include "tmap.cuh"

namespace mr {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct cf {
  float r, i;
};
__device__ __forceinline__ cf cmul(cf p, cf q) { return {p.r * q.r - p.i * q.i, p.r * q.i + p.i * q.r}; }
__device__ __forceinline__ cf cfma(cf p, cf q, cf s) {  // p*q + s
  return {p.r * q.r - p.i * q.i + s.r, p.r * q.i + p.i * q.r + s.i};
}

// Block q of the backward's block sequence (segment aligned). Small segments:
// blocks of tbe = (TB/seg)*seg steps. Long segments: nsub blocks per
// segment, the last one possibly short.
struct BlockMap {
  int L, seg, TB, tbe, nsub, nq;
  __device__ __host__ BlockMap(int L_, int seg_, int TB_) : L(L_), seg(seg_), TB(TB_) {
    if (seg <= TB) {
      tbe = (TB / seg) * seg;
      nsub = 1;
      nq = (L + tbe - 1) / tbe;
    } else {
      tbe = TB;
      nsub = (seg + TB - 1) / TB;
      nq = (L / seg) * nsub;
    }
  }
  __device__ void range(int q, int& t0, int& nt, int& j) const {
    if (nsub == 1) {
      t0 = q * tbe;
      nt = min(tbe, L - t0);
      j = 0;
    } else {
      const int s = q / nsub;
      j = q % nsub;
      t0 = s * seg + j * TB;
      nt = min(TB, (s + 1) * seg - t0);
    }
  }
};

// ============================================================================
// RG-LRU forward
// ============================================================================

// Input gating folded into the RG-LRU kernels (kG): the stored inputs are x,
// r, i (three tiles) and a per-channel Lambda, and the scan's gate and input
// are formed on load, a_t = sigmoid(Lambda)^(c r_t), b_t = sqrt(1 - a_t^2) i_t x_t
// (the prologue the reference leaves to MLX host code, rglru.py:8-27; with r
// the activated recurrence gate this is Griffin's exp(-c softplus(-Lambda) r_t)).
struct RgGate {
  const float* lam;  // [D] Lambda
  float c;           // the gate exponent scale
};

// log sigmoid(x), stable for either sign
__device__ __forceinline__ float log_sigmoid(float x) { return x >= 0.f ? -log1pf(expf(-x)) : x - log1pf(expf(x)); }

// a = exp(z) (z = c r log sigmoid(Lambda) <= 0) and s = sqrt(1 - a^2) from one
// e = expm1(z): a = 1 + e, 1 - a^2 = -e (2 + e), no cancellation as a -> 1
__device__ __forceinline__ void rg_gate(float z, float& a, float& s) {
  const float e = expm1f(z);
  a = 1.f + e;
  s = sqrtf(fmaxf(-e * (2.f + e), 0.f));
}

template <typename T, int W, int TB, int S, int NIN>
struct RgFwdSmem {
  static constexpr size_t bytes = (size_t)NIN * S * TB * W * sizeof(T) + 2 * 2 * kWarps * W * 4 + S * 8;
};

template <typename T, int W, int TB, int S, bool kH0, bool kG>
__global__ void __launch_bounds__(kThreads, 3)
rglru_fwd_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_x,
                 const __grid_constant__ CUtensorMap tm_i, RgGate gate, int L, int64_t D, int seg,
                 float* __restrict__ y, float* __restrict__ ckpt, const float* __restrict__ h0) {
  // kG: tm_a, tm_x, tm_i map x, r, i; else a and x (tm_i unused)
  constexpr int V = W / 32, TW = TB / kWarps, NIN = kG ? 3 : 2;
  extern __shared__ __align__(128) unsigned char smem[];
  T* sa = reinterpret_cast<T*>(smem);
  T* sx = sa + S * TB * W;
  T* si = sx + S * TB * W;  // kG only
  float* sA = reinterpret_cast<float*>(sa + NIN * S * TB * W);
  float* sH = sA + 2 * kWarps * W;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sH + 2 * kWarps * W);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * W;
  const int Wv = (int)min((int64_t)W, D - c0);
  const int cl = lane * V;
  const bool act = cl < Wv;
  const int nseg = L / seg;
  const int nblk = (L + TB - 1) / TB;
  const int64_t gbase = b * (int64_t)L * D + c0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int blk) {  // one thread: a [TB x W] box per input
    const int s = blk % S, row = (int)(b * L) + blk * TB;
    mbar_arrive_expect_tx(&bar[s], (uint32_t)NIN * TB * W * sizeof(T));
    tma_load_2d(sa + s * TB * W, &tm_a, (int)c0, row, &bar[s]);
    tma_load_2d(sx + s * TB * W, &tm_x, (int)c0, row, &bar[s]);
    if constexpr (kG) tma_load_2d(si + s * TB * W, &tm_i, (int)c0, row, &bar[s]);
  };
  if (threadIdx.x == 0)
    for (int k = 0; k < S - 1 && k < nblk; ++k) issue(k);

  float carry[V];  // the state before the block: h0 [B, D] or zero
#pragma unroll
  for (int v = 0; v < V; ++v) carry[v] = (kH0 && act) ? h0[b * D + c0 + cl + v] : 0.f;
  float cl2[V];  // kG: c log sigmoid(Lambda) of the lane's channels
#pragma unroll
  for (int v = 0; v < V; ++v) cl2[v] = (kG && act) ? gate.c * log_sigmoid(gate.lam[c0 + cl + v]) : 0.f;

  for (int blk = 0; blk < nblk; ++blk) {
    const int s = blk % S;
    mbar_wait(&bar[s], (blk / S) & 1);
    const int buf = blk & 1;
    const int r0 = warp * TW;
    const int t0 = blk * TB + r0;
    const T* ra = sa + (s * TB + r0) * W + cl;
    const T* rx = sx + (s * TB + r0) * W + cl;

    float fa[TW][V], fx[TW][V];
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const bool ok = t0 + i < L;
      const Vec<T, V> va = ld_vec<T, V>(ra + i * W);
      const Vec<T, V> vx = ld_vec<T, V>(rx + i * W);
      if constexpr (kG) {  // (va, vx, vi) = (x, r, i)
        const Vec<T, V> vi = ld_vec<T, V>(si + (s * TB + r0) * W + cl + i * W);
#pragma unroll
        for (int v = 0; v < V; ++v) {
          float av, sv;
          rg_gate(cl2[v] * to_f(vx.v[v]), av, sv);
          fa[i][v] = ok ? av : 1.f;
          fx[i][v] = ok ? sv * to_f(vi.v[v]) * to_f(va.v[v]) : 0.f;
        }
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v) {
          fa[i][v] = ok ? to_f(va.v[v]) : 1.f;
          fx[i][v] = ok ? to_f(vx.v[v]) : 0.f;
        }
      }
    }
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float A = 1.f, H = 0.f;
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        H = fa[i][v] * H + fx[i][v];
        A = fa[i][v] * A;
      }
      sA[(buf * kWarps + warp) * W + cl + v] = A;
      sH[(buf * kWarps + warp) * W + cl + v] = H;
    }
    __syncthreads();
    // every thread is past block blk-1: its stage can be refilled
    if (threadIdx.x == 0 && blk + S - 1 < nblk) {
      fence_proxy_async_smem();
      issue(blk + S - 1);
    }

    float cin[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float cur = carry[v];
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (w == warp) cin[v] = cur;
        cur = sA[(buf * kWarps + w) * W + cl + v] * cur + sH[(buf * kWarps + w) * W + cl + v];
      }
      carry[v] = cur;
    }

    if (act) {
      float* yr = y + gbase + (int64_t)t0 * D + cl;
      int rem = (t0 + 1) % seg;  // (t + 1) mod seg, advanced per step
      int sidx = (t0 + 1) / seg;
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        const int t = t0 + i;
        if (t < L) {
          float hv[V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            cin[v] = fa[i][v] * cin[v] + fx[i][v];  // rglru.py:92
            hv[v] = cin[v];
          }
          st_stream_f32<V>(yr, hv);
          if (rem == 0) st_stream_f32<V>(ckpt + (b * nseg + sidx - 1) * D + c0 + cl, hv);
        }
        yr += D;
        if (++rem == seg) {
          rem = 0;
          ++sidx;
        }
      }
    }
  }
}

// ============================================================================
// RG-LRU backward
// ============================================================================

template <typename T, int W, int TB, int S, int NIN>
struct RgBwdSmem {
  static constexpr size_t bytes =
      (size_t)S * TB * W * (NIN * sizeof(T) + 4) + 4 * 2 * kWarps * W * 4 + S * 8;
};

// kG: the inputs (a, x, ig) are (x, r, i) and the gradients (ga, gx, gi) are those
// of (x, r, i); glam_part [B, D] receives each batch row's d loss / d Lambda.
template <typename T, int W, int TB, int S, bool kH0, bool kG>
__global__ void __launch_bounds__(kThreads, kG ? 2 : 3)  // gated: 2 CTAs per SM by shared memory anyway
rglru_bwd_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_x,
                 const __grid_constant__ CUtensorMap tm_g, const __grid_constant__ CUtensorMap tm_i,
                 RgGate gate, const float* __restrict__ gfinal, const float* __restrict__ ckpt,
                 const T* __restrict__ a, const T* __restrict__ x, const T* __restrict__ ig, int L, int64_t D,
                 int seg, T* __restrict__ ga, T* __restrict__ gx, T* __restrict__ gi,
                 float* __restrict__ glam_part, float* __restrict__ ws, const float* __restrict__ h0,
                 float* __restrict__ gh0) {
  constexpr int V = W / 32, TW = TB / kWarps, NIN = kG ? 3 : 2;
  extern __shared__ __align__(128) unsigned char smem[];
  T* sa = reinterpret_cast<T*>(smem);
  T* sx = sa + S * TB * W;
  T* si = sx + S * TB * W;  // kG only
  float* sg = reinterpret_cast<float*>(sa + NIN * S * TB * W);
  float* sA = sg + S * TB * W;
  float* sH = sA + 2 * kWarps * W;
  float* sR = sH + 2 * kWarps * W;
  float* sG = sR + 2 * kWarps * W;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sG + 2 * kWarps * W);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * W;
  const int Wv = (int)min((int64_t)W, D - c0);
  const int cl = lane * V;
  const bool act = cl < Wv;
  const int nseg = L / seg;
  const BlockMap bm(L, seg, TB);
  const int64_t gbase = b * (int64_t)L * D + c0;
  float* wsb = ws + ((b * gridDim.x + blockIdx.x) * (int64_t)bm.nsub) * W + cl;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // pipeline position p streams block q = nq-1-p
  auto issue = [&](int p) {  // one thread: [TB x W] boxes of a, x, grad_y
    const int s = p % S;
    int t0, nt, j;
    bm.range(bm.nq - 1 - p, t0, nt, j);
    const int row = (int)(b * L) + t0;
    mbar_arrive_expect_tx(&bar[s], (uint32_t)TB * W * (NIN * (uint32_t)sizeof(T) + 4u));
    tma_load_2d(sa + s * TB * W, &tm_a, (int)c0, row, &bar[s]);
    tma_load_2d(sx + s * TB * W, &tm_x, (int)c0, row, &bar[s]);
    if constexpr (kG) tma_load_2d(si + s * TB * W, &tm_i, (int)c0, row, &bar[s]);
    tma_load_2d(sg + s * TB * W, &tm_g, (int)c0, row, &bar[s]);
  };
  if (threadIdx.x == 0)
    for (int k = 0; k < S - 1 && k < bm.nq; ++k) issue(k);

  float cr[V];
#pragma unroll
  for (int v = 0; v < V; ++v) cr[v] = (gfinal != nullptr && act) ? gfinal[b * D + c0 + cl + v] : 0.f;
  // kG: c log sigmoid(Lambda), c (1 - sigmoid(Lambda)) and the d loss / d Lambda sum of the lane
  float cl2[V], klam[V], glam[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const float lm = (kG && act) ? gate.lam[c0 + cl + v] : 0.f;
    cl2[v] = kG ? gate.c * log_sigmoid(lm) : 0.f;
    klam[v] = kG ? gate.c / (1.f + expf(lm)) : 0.f;  // c (1 - sigmoid(Lambda)) = c sigmoid(-Lambda)
    glam[v] = 0.f;
  }
  // kG: the scan's gate and input from (x, r, i) at global offset o of the lane's channel v
  auto gated_ab = [&](int64_t o, int v, float& av, float& bv) {
    float sv;
    rg_gate(cl2[v] * to_f(x[o]), av, sv);
    bv = sv * to_f(ig[o]) * to_f(a[o]);
  };
  int it = 0;  // exchange-buffer parity

  for (int p = 0; p < bm.nq; ++p) {
    const int q = bm.nq - 1 - p;
    int tb0, ntb, j;
    bm.range(q, tb0, ntb, j);

    // long segments: regenerate the state at every block start of the segment
    if (bm.nsub > 1 && j == bm.nsub - 1) {
      const int sidx = tb0 / seg;
      const int s0 = sidx * seg;
      float cur[V];
#pragma unroll
      for (int v = 0; v < V; ++v)
        cur[v] = !act ? 0.f : sidx > 0 ? ckpt[(b * nseg + sidx - 1) * D + c0 + cl + v]
                 : kH0 ? h0[b * D + c0 + cl + v] : 0.f;
      for (int jj = 0; jj + 1 < bm.nsub; ++jj, ++it) {
        const int buf = it & 1;
        const int t0 = s0 + jj * TB + warp * TW;
        const int tend = min(s0 + (jj + 1) * TB, s0 + seg);
#pragma unroll
        for (int v = 0; v < V; ++v) {
          float A = 1.f, H = 0.f;
#pragma unroll
          for (int i = 0; i < TW; ++i) {
            if (act && t0 + i < tend) {
              const int64_t o = gbase + (int64_t)(t0 + i) * D + cl + v;
              float av, bv;
              if constexpr (kG) {
                gated_ab(o, v, av, bv);
              } else {
                av = to_f(a[o]);
                bv = to_f(x[o]);
              }
              H = av * H + bv;
              A = av * A;
            }
          }
          sA[(buf * kWarps + warp) * W + cl + v] = A;
          sH[(buf * kWarps + warp) * W + cl + v] = H;
        }
        __syncthreads();
#pragma unroll
        for (int v = 0; v < V; ++v) {
#pragma unroll
          for (int w = 0; w < kWarps; ++w)
            cur[v] = sA[(buf * kWarps + w) * W + cl + v] * cur[v] + sH[(buf * kWarps + w) * W + cl + v];
          if (warp == 0 && act) wsb[(int64_t)(jj + 1) * W + v] = cur[v];
        }
      }
      __syncthreads();
    }

    const int s = p % S;
    mbar_wait(&bar[s], (p / S) & 1);
    const int buf = it & 1;
    ++it;
    const int r0 = warp * TW;
    const int t0 = tb0 + r0;
    const int tend = tb0 + ntb;
    const T* ra = sa + (s * TB + r0) * W + cl;
    const T* rx = sx + (s * TB + r0) * W + cl;
    const float* rg = sg + (s * TB + r0) * W + cl;

    const T* ri = si + (s * TB + r0) * W + cl;  // kG: i
    float fa[TW][V], fx[TW][V], fg[TW][V];
    float fsg[kG ? TW : 1][V];  // kG: sqrt(1 - a^2) of each step
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const bool ok = t0 + i < tend;
      const Vec<T, V> va = ld_vec<T, V>(ra + i * W);
      const Vec<T, V> vx = ld_vec<T, V>(rx + i * W);
      const Vec<float, V> vg = ld_vec<float, V>(rg + i * W);
      if constexpr (kG) {  // (va, vx, vi) = (x, r, i)
        const Vec<T, V> vi = ld_vec<T, V>(ri + i * W);
#pragma unroll
        for (int v = 0; v < V; ++v) {
          float av, sv;
          rg_gate(cl2[v] * to_f(vx.v[v]), av, sv);
          fa[i][v] = ok ? av : 1.f;
          fx[i][v] = ok ? sv * to_f(vi.v[v]) * to_f(va.v[v]) : 0.f;
          fg[i][v] = ok ? vg.v[v] : 0.f;
          fsg[i][v] = sv;
        }
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v) {
          fa[i][v] = ok ? to_f(va.v[v]) : 1.f;
          fx[i][v] = ok ? to_f(vx.v[v]) : 0.f;
          fg[i][v] = ok ? vg.v[v] : 0.f;
        }
      }
    }
    float hs[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (j > 0)
        hs[v] = act ? wsb[(int64_t)j * W + v] : 0.f;
      else
        hs[v] = !act ? 0.f : tb0 > 0 ? ckpt[(b * nseg + tb0 / seg - 1) * D + c0 + cl + v]
                : kH0 ? h0[b * D + c0 + cl + v] : 0.f;
    }

#pragma unroll
    for (int v = 0; v < V; ++v) {
      float A = 1.f, H = 0.f, R = 1.f, G = 0.f;
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        H = fa[i][v] * H + fx[i][v];
        A = fa[i][v] * A;
      }
#pragma unroll
      for (int i = TW - 1; i >= 0; --i) {  // c_out = a * (gy + c_in)
        G = fa[i][v] * (fg[i][v] + G);
        R = fa[i][v] * R;
      }
      sA[(buf * kWarps + warp) * W + cl + v] = A;
      sH[(buf * kWarps + warp) * W + cl + v] = H;
      sR[(buf * kWarps + warp) * W + cl + v] = R;
      sG[(buf * kWarps + warp) * W + cl + v] = G;
    }
    __syncthreads();
    if (threadIdx.x == 0 && p + S - 1 < bm.nq) {
      fence_proxy_async_smem();
      issue(p + S - 1);
    }

    float hp[TW][V], crin[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float cur = hs[v];
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (w == warp) break;
        cur = sA[(buf * kWarps + w) * W + cl + v] * cur + sH[(buf * kWarps + w) * W + cl + v];
      }
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        hp[i][v] = cur;
        cur = fa[i][v] * cur + fx[i][v];
      }
      float rc = cr[v];
#pragma unroll
      for (int w = kWarps - 1; w >= 0; --w) {
        if (w == warp) crin[v] = rc;
        rc = sR[(buf * kWarps + w) * W + cl + v] * rc + sG[(buf * kWarps + w) * W + cl + v];
      }
      cr[v] = rc;
    }

    // adjoint per step, newest -> oldest (rglru.py:173-178)
#pragma unroll
    for (int i = TW - 1; i >= 0; --i) {
      const int t = t0 + i;
      float o_x[V], o_a[V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const float adj = fg[i][v] + crin[v];
        o_x[v] = adj;
        o_a[v] = adj * hp[i][v];
        crin[v] = adj * fa[i][v];
      }
      if constexpr (kG) {
        // chain through b = sqrt(1 - a^2) i x and a = exp(c log sigmoid(Lambda) r):
        // grads of x, r, i and the Lambda sum (out of range steps have adj = 0)
        const Vec<T, V> vxx = ld_vec<T, V>(ra + i * W), vr = ld_vec<T, V>(rx + i * W), vi = ld_vec<T, V>(ri + i * W);
        float o_gx[V], o_gr[V], o_gi[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const float xx = to_f(vxx.v[v]), rr = to_f(vr.v[v]), ii = to_f(vi.v[v]);
          const float av = fa[i][v], sg_ = fsg[i][v];
          o_gx[v] = o_x[v] * sg_ * ii;
          o_gi[v] = o_x[v] * sg_ * xx;
          const float gat = o_a[v] - (sg_ > 0.f ? o_x[v] * ii * xx * av / sg_ : 0.f);
          o_gr[v] = gat * cl2[v] * av;
          if (t < tend) glam[v] += gat * rr * av * klam[v];
        }
        if (act && t < tend) {
          const int64_t o = gbase + (int64_t)t * D + cl;
          st_vec<T, V>(ga + o, o_gx);
          st_vec<T, V>(gx + o, o_gr);
          st_vec<T, V>(gi + o, o_gi);
        }
      } else if (act && t < tend) {
        const int64_t o = gbase + (int64_t)t * D + cl;
        st_vec<T, V>(gx + o, o_x);
        st_vec<T, V>(ga + o, o_a);
      }
    }
  }
  if constexpr (kG) {  // the CTA's d loss / d Lambda: a sum over its warps' steps
    __syncthreads();
#pragma unroll
    for (int v = 0; v < V; ++v) sA[warp * W + cl + v] = glam[v];
    __syncthreads();
    if (warp == 0 && act)
#pragma unroll
      for (int v = 0; v < V; ++v) {
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) acc += sA[w * W + cl + v];
        glam_part[b * D + c0 + cl + v] = acc;
      }
  }
  // the reverse carry past step 0 is the gradient of the initial state
  if (kH0 && gh0 != nullptr && act)
#pragma unroll
    for (int v = 0; v < V; ++v) gh0[b * D + c0 + cl + v] = cr[v];
}

// ============================================================================
// rotLRU forward (pairs interleaved in x / y; rotlru.py:80-146)
// ============================================================================

// cos and sin of an angle for the rotLRU angle input. Cody-Waite reduction
// (Cody & Waite, "Software Manual for the Elementary Functions", 1980): k =
// rint(t 2/pi), r = t - k pi/2 with pi/2 split in two floats (hi = pi/2
// rounded to float, lo = the float nearest pi/2 - hi) and fused multiply-adds,
// so r is exact to a few float ulps for |t| < 2^17 pi/2; then the Taylor series
// of sin r to r^9 and cos r to r^10 on |r| <= pi/4 (truncation below 2e-9), and
// the quadrant k mod 4 picks and signs the pair. About 20 instructions with no
// taken branch, small enough to unroll across a tile (the library's sincosf
// carries a long path for huge arguments that bloats an unrolled loop);
// arguments beyond the reduction's range, and non-finite ones, go to sincosf
// out of line.
__device__ __noinline__ float2 rot_sincos_wide(float t) {
  float sv, cv;
  sincosf(t, &sv, &cv);
  return make_float2(sv, cv);
}

__device__ __forceinline__ void rot_sincos(float t, float& sv, float& cv) {
  constexpr float kTwoOverPi = (float)(2.0 / 3.14159265358979323846);
  constexpr float kHalfPiHi = (float)(3.14159265358979323846 / 2.0);
  constexpr float kHalfPiLo = (float)(3.14159265358979323846 / 2.0 - (double)kHalfPiHi);
  if (!(fabsf(t) < 205887.4f)) {  // 2^17 pi/2; NaN takes this branch too
    const float2 w = rot_sincos_wide(t);
    sv = w.x, cv = w.y;
    return;
  }
  const float k = rintf(t * kTwoOverPi);
  float r = fmaf(-k, kHalfPiHi, t);
  r = fmaf(-k, kHalfPiLo, r);
  const float r2 = r * r;
  float ps = (float)(1.0 / 362880.0);
  ps = fmaf(ps, r2, (float)(-1.0 / 5040.0));
  ps = fmaf(ps, r2, (float)(1.0 / 120.0));
  ps = fmaf(ps, r2, (float)(-1.0 / 6.0));
  const float sr = fmaf(ps * r2, r, r);
  float pc = (float)(-1.0 / 3628800.0);
  pc = fmaf(pc, r2, (float)(1.0 / 40320.0));
  pc = fmaf(pc, r2, (float)(-1.0 / 720.0));
  pc = fmaf(pc, r2, (float)(1.0 / 24.0));
  pc = fmaf(pc, r2, -0.5f);
  const float cr = fmaf(pc, r2, 1.f);
  const int q = __float2int_rn(k);
  const float a = (q & 1) ? cr : sr, b = (q & 1) ? sr : cr;
  sv = (q & 2) ? -a : a;
  cv = ((q + 1) & 2) ? -b : b;
}

// kTh: the rotation comes as its angle theta (one tile, in the cs slot) and the
// kernels form cos and sin on load; the reference takes cos and sin from host
// code (rotlru.py:18-22). NT: input tiles per stage (5 units of T: a, cs, sn, x;
// 4 with the angle).
template <typename T, int W, int TB, int S, int NT = 5>
struct RotFwdSmem {
  static constexpr size_t bytes = (size_t)S * TB * W * NT * sizeof(T) + 2 * 2 * kWarps * W * 8 + S * 8;
};

template <typename T, int W, int TB, int S, bool kH0, bool kTh>
__global__ void __launch_bounds__(kThreads, 2)
rotlru_fwd_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_c,
                  const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_x,
                  int L, int64_t Dp, int seg, float* __restrict__ y, float* __restrict__ ckpt,
                  const float* __restrict__ h0) {
  constexpr int V = W / 32, TW = TB / kWarps;
  extern __shared__ __align__(128) unsigned char smem[];
  T* sa = reinterpret_cast<T*>(smem);
  T* sc = sa + S * TB * W;                     // cs, or theta (kTh)
  T* ss = sc + (kTh ? 0 : S * TB * W);         // sn (kTh: unused)
  T* sx = ss + S * TB * W;  // [S][TB][2W]
  cf* sZ = reinterpret_cast<cf*>(sx + S * TB * 2 * W);
  cf* sH = sZ + 2 * kWarps * W;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sH + 2 * kWarps * W);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t p0 = (int64_t)blockIdx.x * W;
  const int Wv = (int)min((int64_t)W, Dp - p0);
  const int pl = lane * V;
  const bool act = pl < Wv;
  const int64_t D = 2 * Dp;
  const int nseg = L / seg;
  const int nblk = (L + TB - 1) / TB;
  const int64_t xbase = b * (int64_t)L * D + 2 * p0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int blk) {  // one thread: [TB x W] boxes of a, cs, sn; [TB x 2W] of x
    const int s = blk % S, row = (int)(b * L) + blk * TB;
    mbar_arrive_expect_tx(&bar[s], (uint32_t)TB * W * (kTh ? 4u : 5u) * sizeof(T));
    tma_load_2d(sa + s * TB * W, &tm_a, (int)p0, row, &bar[s]);
    tma_load_2d(sc + s * TB * W, &tm_c, (int)p0, row, &bar[s]);
    if constexpr (!kTh) tma_load_2d(ss + s * TB * W, &tm_s, (int)p0, row, &bar[s]);
    tma_load_2d(sx + s * TB * 2 * W, &tm_x, (int)(2 * p0), row, &bar[s]);
  };
  if (threadIdx.x == 0)
    for (int k = 0; k < S - 1 && k < nblk; ++k) issue(k);

  cf carry[V];  // the state before the block: h0 [B, 2Dp] (pairs) or zero
#pragma unroll
  for (int v = 0; v < V; ++v)
    carry[v] = (kH0 && act) ? cf{h0[b * D + 2 * (p0 + pl + v)], h0[b * D + 2 * (p0 + pl + v) + 1]}
                            : cf{0.f, 0.f};

  for (int blk = 0; blk < nblk; ++blk) {
    const int s = blk % S;
    mbar_wait(&bar[s], (blk / S) & 1);
    const int buf = blk & 1;
    const int r0 = warp * TW;
    const int t0 = blk * TB + r0;

    float fa[TW][V], fc[TW][V], fs[TW][V];
    cf fx[TW][V];
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const bool ok = t0 + i < L;
      const int row = s * TB + r0 + i;
      const Vec<T, V> va = ld_vec<T, V>(sa + row * W + pl);
      const Vec<T, V> vc = ld_vec<T, V>(sc + row * W + pl);
      const Vec<T, V> vs = ld_vec<T, V>(ss + row * W + pl);
      const Vec<T, 2 * V> vx = ld_vec<T, 2 * V>(sx + row * 2 * W + 2 * pl);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        float cv, sv;
        if constexpr (kTh)
          rot_sincos(to_f(vc.v[v]), sv, cv);
        else
          cv = to_f(vc.v[v]), sv = to_f(vs.v[v]);
        fa[i][v] = ok ? to_f(va.v[v]) : 1.f;
        fc[i][v] = ok ? cv : 1.f;
        fs[i][v] = ok ? sv : 0.f;
        fx[i][v] = ok ? cf{to_f(vx.v[2 * v]), to_f(vx.v[2 * v + 1])} : cf{0.f, 0.f};
      }
    }
#pragma unroll
    for (int v = 0; v < V; ++v) {
      cf Z = {1.f, 0.f}, H = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        const cf z = {fa[i][v] * fc[i][v], fa[i][v] * fs[i][v]};
        H = cfma(z, H, fx[i][v]);
        Z = cmul(z, Z);
      }
      sZ[(buf * kWarps + warp) * W + pl + v] = Z;
      sH[(buf * kWarps + warp) * W + pl + v] = H;
    }
    __syncthreads();
    if (threadIdx.x == 0 && blk + S - 1 < nblk) {
      fence_proxy_async_smem();
      issue(blk + S - 1);
    }

    cf cin[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      cf cur = carry[v];
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (w == warp) cin[v] = cur;
        cur = cfma(sZ[(buf * kWarps + w) * W + pl + v], cur, sH[(buf * kWarps + w) * W + pl + v]);
      }
      carry[v] = cur;
    }

    if (act) {
      int rem = (t0 + 1) % seg;  // (t + 1) mod seg, advanced per step
      int sidx = (t0 + 1) / seg;
#pragma unroll
      for (int i = 0; i < TW; ++i, ++rem) {
        if (rem == seg) {
          rem = 0;
          ++sidx;
        }
        const int t = t0 + i;
        if (t < L) {
          float hv[2 * V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const float av = fa[i][v], c = fc[i][v], sv = fs[i][v];
            const float u = cin[v].r, w = cin[v].i;
            const float un = av * (c * u - sv * w) + fx[i][v].r;  // rotlru.py:110
            const float wn = av * (sv * u + c * w) + fx[i][v].i;  // rotlru.py:111
            cin[v] = {un, wn};
            hv[2 * v] = un;
            hv[2 * v + 1] = wn;
          }
          st_stream_f32<2 * V>(y + xbase + (int64_t)t * D + 2 * pl, hv);
          if (rem == 0) st_stream_f32<2 * V>(ckpt + (b * nseg + sidx - 1) * D + 2 * (p0 + pl), hv);
        }
      }
    }
  }
}

// ============================================================================
// rotLRU backward (rotlru.py:153-266)
// ============================================================================

template <typename T, int W, int TB, int S, int NT = 5>
struct RotBwdSmem {
  static constexpr size_t bytes =
      (size_t)S * TB * W * (NT * sizeof(T) + 8) + 4 * 2 * kWarps * W * 8 + S * 8;
};

// kTh: cs holds theta and gcs receives d loss / d theta (sn, gsn unused)
template <typename T, int W, int TB, int S, bool kH0, bool kTh>
__global__ void __launch_bounds__(kThreads, 2)
rotlru_bwd_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_c,
                  const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_x,
                  const __grid_constant__ CUtensorMap tm_g, const float* __restrict__ gfinal,
                  const float* __restrict__ ckpt, const T* __restrict__ a, const T* __restrict__ cs,
                  const T* __restrict__ sn, const T* __restrict__ x, int L, int64_t Dp, int seg,
                  T* __restrict__ ga, T* __restrict__ gcs, T* __restrict__ gsn, T* __restrict__ gx,
                  float* __restrict__ ws, const float* __restrict__ h0, float* __restrict__ gh0) {
  constexpr int V = W / 32, TW = TB / kWarps;
  extern __shared__ __align__(128) unsigned char smem[];
  T* sa = reinterpret_cast<T*>(smem);
  T* sc = sa + S * TB * W;                                  // cs, or theta (kTh)
  T* ss = sc + (kTh ? 0 : S * TB * W);                      // sn (kTh: unused)
  T* sx = ss + S * TB * W;                                  // [S][TB][2W]
  float* sg = reinterpret_cast<float*>(sx + S * TB * 2 * W);  // [S][TB][2W]
  cf* sZ = reinterpret_cast<cf*>(sg + S * TB * 2 * W);
  cf* sH = sZ + 2 * kWarps * W;
  cf* sR = sH + 2 * kWarps * W;
  cf* sG = sR + 2 * kWarps * W;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sG + 2 * kWarps * W);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t p0 = (int64_t)blockIdx.x * W;
  const int Wv = (int)min((int64_t)W, Dp - p0);
  const int pl = lane * V;
  const bool act = pl < Wv;
  const int64_t D = 2 * Dp;
  const int nseg = L / seg;
  const BlockMap bm(L, seg, TB);
  const int64_t pbase = b * (int64_t)L * Dp + p0;
  const int64_t xbase = b * (int64_t)L * D + 2 * p0;
  float* wsb = ws + ((b * gridDim.x + blockIdx.x) * (int64_t)bm.nsub) * (2 * W) + 2 * pl;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int p) {  // one thread: boxes of a, cs, sn, x and grad_y
    const int s = p % S;
    int t0, nt, j;
    bm.range(bm.nq - 1 - p, t0, nt, j);
    const int row = (int)(b * L) + t0;
    mbar_arrive_expect_tx(&bar[s], (uint32_t)TB * W * ((kTh ? 4u : 5u) * sizeof(T) + 8u));
    tma_load_2d(sa + s * TB * W, &tm_a, (int)p0, row, &bar[s]);
    tma_load_2d(sc + s * TB * W, &tm_c, (int)p0, row, &bar[s]);
    if constexpr (!kTh) tma_load_2d(ss + s * TB * W, &tm_s, (int)p0, row, &bar[s]);
    tma_load_2d(sx + s * TB * 2 * W, &tm_x, (int)(2 * p0), row, &bar[s]);
    tma_load_2d(sg + s * TB * 2 * W, &tm_g, (int)(2 * p0), row, &bar[s]);
  };
  if (threadIdx.x == 0)
    for (int k = 0; k < S - 1 && k < bm.nq; ++k) issue(k);

  cf cr[V];
#pragma unroll
  for (int v = 0; v < V; ++v)
    cr[v] = (gfinal != nullptr && act)
                ? cf{gfinal[b * D + 2 * (p0 + pl + v)], gfinal[b * D + 2 * (p0 + pl + v) + 1]}
                : cf{0.f, 0.f};
  int it = 0;

  for (int p = 0; p < bm.nq; ++p) {
    const int q = bm.nq - 1 - p;
    int tb0, ntb, j;
    bm.range(q, tb0, ntb, j);

    if (bm.nsub > 1 && j == bm.nsub - 1) {
      const int sidx = tb0 / seg;
      const int s0 = sidx * seg;
      cf cur[V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const float* ck = sidx > 0 ? ckpt + (b * nseg + sidx - 1) * D + 2 * (p0 + pl + v)
                          : kH0 ? h0 + b * D + 2 * (p0 + pl + v) : nullptr;
        cur[v] = (act && ck != nullptr) ? cf{ck[0], ck[1]} : cf{0.f, 0.f};
      }
      for (int jj = 0; jj + 1 < bm.nsub; ++jj, ++it) {
        const int buf = it & 1;
        const int t0 = s0 + jj * TB + warp * TW;
        const int tend = min(s0 + (jj + 1) * TB, s0 + seg);
#pragma unroll
        for (int v = 0; v < V; ++v) {
          cf Z = {1.f, 0.f}, H = {0.f, 0.f};
#pragma unroll
          for (int i = 0; i < TW; ++i) {
            if (act && t0 + i < tend) {
              const int64_t o = pbase + (int64_t)(t0 + i) * Dp + pl + v;
              const int64_t ox = xbase + (int64_t)(t0 + i) * D + 2 * (pl + v);
              const float av = to_f(a[o]);
              float cv, sv;
              if constexpr (kTh)
                rot_sincos(to_f(cs[o]), sv, cv);
              else
                cv = to_f(cs[o]), sv = to_f(sn[o]);
              const cf z = {av * cv, av * sv};
              H = cfma(z, H, {to_f(x[ox]), to_f(x[ox + 1])});
              Z = cmul(z, Z);
            }
          }
          sZ[(buf * kWarps + warp) * W + pl + v] = Z;
          sH[(buf * kWarps + warp) * W + pl + v] = H;
        }
        __syncthreads();
#pragma unroll
        for (int v = 0; v < V; ++v) {
#pragma unroll
          for (int w = 0; w < kWarps; ++w)
            cur[v] = cfma(sZ[(buf * kWarps + w) * W + pl + v], cur[v], sH[(buf * kWarps + w) * W + pl + v]);
          if (warp == 0 && act) {
            wsb[(int64_t)(jj + 1) * 2 * W + 2 * v] = cur[v].r;
            wsb[(int64_t)(jj + 1) * 2 * W + 2 * v + 1] = cur[v].i;
          }
        }
      }
      __syncthreads();
    }

    const int s = p % S;
    mbar_wait(&bar[s], (p / S) & 1);
    const int buf = it & 1;
    ++it;
    const int r0 = warp * TW;
    const int t0 = tb0 + r0;
    const int tend = tb0 + ntb;

    float fa[TW][V], fc[TW][V], fs[TW][V];
    cf fx[TW][V], fg[TW][V];
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const bool ok = t0 + i < tend;
      const int row = s * TB + r0 + i;
      const Vec<T, V> va = ld_vec<T, V>(sa + row * W + pl);
      const Vec<T, V> vc = ld_vec<T, V>(sc + row * W + pl);
      const Vec<T, V> vs = ld_vec<T, V>(ss + row * W + pl);
      const Vec<T, 2 * V> vx = ld_vec<T, 2 * V>(sx + row * 2 * W + 2 * pl);
      const Vec<float, 2 * V> vg = ld_vec<float, 2 * V>(sg + row * 2 * W + 2 * pl);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        float cv, sv;
        if constexpr (kTh)
          rot_sincos(to_f(vc.v[v]), sv, cv);
        else
          cv = to_f(vc.v[v]), sv = to_f(vs.v[v]);
        fa[i][v] = ok ? to_f(va.v[v]) : 1.f;
        fc[i][v] = ok ? cv : 1.f;
        fs[i][v] = ok ? sv : 0.f;
        fx[i][v] = ok ? cf{to_f(vx.v[2 * v]), to_f(vx.v[2 * v + 1])} : cf{0.f, 0.f};
        fg[i][v] = ok ? cf{vg.v[2 * v], vg.v[2 * v + 1]} : cf{0.f, 0.f};
      }
    }
    cf hs[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (j > 0) {
        hs[v] = act ? cf{wsb[(int64_t)j * 2 * W + 2 * v], wsb[(int64_t)j * 2 * W + 2 * v + 1]} : cf{0.f, 0.f};
      } else {
        const float* ck = tb0 > 0 ? ckpt + (b * nseg + tb0 / seg - 1) * D + 2 * (p0 + pl + v)
                          : kH0 ? h0 + b * D + 2 * (p0 + pl + v) : nullptr;
        hs[v] = (act && ck != nullptr) ? cf{ck[0], ck[1]} : cf{0.f, 0.f};
      }
    }

#pragma unroll
    for (int v = 0; v < V; ++v) {
      cf Z = {1.f, 0.f}, H = {0.f, 0.f}, R = {1.f, 0.f}, G = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        const cf z = {fa[i][v] * fc[i][v], fa[i][v] * fs[i][v]};
        H = cfma(z, H, fx[i][v]);
        Z = cmul(z, Z);
      }
#pragma unroll
      for (int i = TW - 1; i >= 0; --i) {  // c_out = conj(z) * (gy + c_in)
        const cf zc = {fa[i][v] * fc[i][v], -fa[i][v] * fs[i][v]};
        G = cmul(zc, {fg[i][v].r + G.r, fg[i][v].i + G.i});
        R = cmul(zc, R);
      }
      sZ[(buf * kWarps + warp) * W + pl + v] = Z;
      sH[(buf * kWarps + warp) * W + pl + v] = H;
      sR[(buf * kWarps + warp) * W + pl + v] = R;
      sG[(buf * kWarps + warp) * W + pl + v] = G;
    }
    __syncthreads();
    if (threadIdx.x == 0 && p + S - 1 < bm.nq) {
      fence_proxy_async_smem();
      issue(p + S - 1);
    }

    cf hp[TW][V], crin[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      cf cur = hs[v];
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (w == warp) break;
        cur = cfma(sZ[(buf * kWarps + w) * W + pl + v], cur, sH[(buf * kWarps + w) * W + pl + v]);
      }
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        hp[i][v] = cur;
        const float u = cur.r, w = cur.i, c = fc[i][v], sv = fs[i][v], av = fa[i][v];
        cur = {av * (c * u - sv * w) + fx[i][v].r, av * (sv * u + c * w) + fx[i][v].i};
      }
      cf rc = cr[v];
#pragma unroll
      for (int w = kWarps - 1; w >= 0; --w) {
        if (w == warp) crin[v] = rc;
        rc = cfma(sR[(buf * kWarps + w) * W + pl + v], rc, sG[(buf * kWarps + w) * W + pl + v]);
      }
      cr[v] = rc;
    }

    // adjoint per step (rotlru.py:206-235)
#pragma unroll
    for (int i = TW - 1; i >= 0; --i) {
      const int t = t0 + i;
      float o_a[V], o_c[V], o_s[V], o_x[2 * V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const float aU = fg[i][v].r + crin[v].r;
        const float aW = fg[i][v].i + crin[v].i;
        const float up = hp[i][v].r, wp = hp[i][v].i;
        const float c = fc[i][v], sv = fs[i][v], av = fa[i][v];
        o_x[2 * v] = aU;
        o_x[2 * v + 1] = aW;
        const float ru = c * up - sv * wp;
        const float rw = sv * up + c * wp;
        o_a[v] = aU * ru + aW * rw;
        o_c[v] = av * (aU * up + aW * wp);
        o_s[v] = av * (aW * up - aU * wp);
        if constexpr (kTh) o_c[v] = c * o_s[v] - sv * o_c[v];  // d/dtheta = cos d/dsn - sin d/dcs
        crin[v] = {av * (c * aU + sv * aW), av * (-sv * aU + c * aW)};
      }
      if (act && t < tend) {
        const int64_t o = pbase + (int64_t)t * Dp + pl;
        st_vec<T, V>(ga + o, o_a);
        st_vec<T, V>(gcs + o, o_c);
        if constexpr (!kTh) st_vec<T, V>(gsn + o, o_s);
        st_vec<T, 2 * V>(gx + xbase + (int64_t)t * D + 2 * pl, o_x);
      }
    }
  }
  // the reverse carry past step 0 is the gradient of the initial state
  if (kH0 && gh0 != nullptr && act)
#pragma unroll
    for (int v = 0; v < V; ++v) {
      gh0[b * D + 2 * (p0 + pl + v)] = cr[v].r;
      gh0[b * D + 2 * (p0 + pl + v) + 1] = cr[v].i;
    }
}

// ============================================================================
// host launchers
// ============================================================================

// Tile shapes (channels per CTA W, steps per block TB, pipeline stages S),
// from a sweep on B200 at c2/c3 (bf16): one channel per lane with long blocks
// for RG-LRU (more CTAs, shorter per-thread chains in phase 1), 64-pair tiles
// for the rotLRU forward, 32-pair tiles of 64 steps for its backward. The
// rotLRU forward with the angle input takes three stages (112 KB of shared
// memory, two CTAs per SM): its cos/sin work wants the second CTA's warps to
// overlap it (0.71 -> 0.55 ms at c3, against 0.63 with 32-pair tiles).
template <typename T> struct DiagCfg {
  static constexpr int RgFW = 32, RgFTB = 128, RgFS = sizeof(T) == 4 ? 2 : 4;
  static constexpr int RgBW = 32, RgBTB = 128, RgBS = 2;
  static constexpr int RotFW = 64, RotFTB = 64, RotFS = sizeof(T) == 4 ? 2 : 4;
  static constexpr int RotAFW = 64, RotAFTB = 64, RotAFS = sizeof(T) == 4 ? 2 : 3;  // angle input
  static constexpr int RotBW = 32, RotBTB = 64, RotBS = 2;
};

template <typename K>
static int set_smem(K kernel, size_t bytes) {
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return set_error(MR_E_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return MR_OK;
}

int diag_device_error(bool clear) { return read_device_error(clear); }

size_t rglru_bwd_ws_bytes(int64_t batch, int64_t L, int64_t D, int64_t seg) {
  using C = DiagCfg<__nv_bfloat16>;
  static_assert(DiagCfg<float>::RgBTB == C::RgBTB && DiagCfg<float>::RgBW == C::RgBW, "");
  const BlockMap bm((int)L, (int)seg, C::RgBTB);
  if (bm.nsub <= 1) return 0;
  return (size_t)batch * ((D + C::RgBW - 1) / C::RgBW) * bm.nsub * C::RgBW * sizeof(float);
}

size_t rotlru_bwd_ws_bytes(int64_t batch, int64_t L, int64_t Dp, int64_t seg) {
  using C = DiagCfg<__nv_bfloat16>;
  const BlockMap bm((int)L, (int)seg, C::RotBTB);
  if (bm.nsub <= 1) return 0;
  return (size_t)batch * ((Dp + C::RotBW - 1) / C::RotBW) * bm.nsub * 2 * C::RotBW * sizeof(float);
}

template <typename T>
static int tmap_rows(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int W, int TB) {
  return make_tmap_2d(m, base, TmapType<T>::v, sizeof(T), (uint64_t)cols, (uint64_t)rows,
                      (uint64_t)cols * sizeof(T), (uint32_t)W, (uint32_t)TB);
}

// kG: (a, x, ig) are (x, r, i) with the gate in `gate`; else ig is unused
template <typename T, bool kG>
static int rglru_fwd_any(const void* a, const void* x, const void* ig, RgGate gate, int64_t batch, int64_t L,
                         int64_t D, int64_t seg, float* y, float* ckpt, const float* h0, cudaStream_t st) {
  using C = DiagCfg<T>;
  // three input tiles per stage when gated: one stage fewer keeps three CTAs per SM (bf16)
  constexpr int W = C::RgFW, TB = C::RgFTB, S = kG && C::RgFS > 3 ? 3 : C::RgFS;
  constexpr size_t sm = RgFwdSmem<T, W, TB, S, kG ? 3 : 2>::bytes;
  CUtensorMap ma, mx, mi;
  if (int rc = tmap_rows<T>(&ma, a, batch * L, D, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&mx, x, batch * L, D, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&mi, kG ? ig : a, batch * L, D, W, TB)) return rc;
  // an initial state selects its own instantiation (the common case's code stays as it was)
  auto k = h0 != nullptr ? rglru_fwd_kernel<T, W, TB, S, true, kG> : rglru_fwd_kernel<T, W, TB, S, false, kG>;
  if (int rc = set_smem(k, sm)) return rc;
  dim3 grid((unsigned)((D + W - 1) / W), (unsigned)batch);
  k<<<grid, kThreads, sm, st>>>(ma, mx, mi, gate, (int)L, D, (int)seg, y, ckpt, h0);
  return check_launch("rglru_fwd_kernel");
}

template <typename T>
int rglru_fwd_launch(const void* a, const void* x, int64_t batch, int64_t L, int64_t D, int64_t seg,
                     float* y, float* ckpt, const float* h0, cudaStream_t st) {
  return rglru_fwd_any<T, false>(a, x, nullptr, RgGate{nullptr, 0.f}, batch, L, D, seg, y, ckpt, h0, st);
}

template <typename T>
int rglru_gated_fwd_launch(const void* x, const void* r, const void* i, const float* lam, float c, int64_t batch,
                           int64_t L, int64_t D, int64_t seg, float* y, float* ckpt, const float* h0,
                           cudaStream_t st) {
  return rglru_fwd_any<T, true>(x, r, i, RgGate{lam, c}, batch, L, D, seg, y, ckpt, h0, st);
}

// d loss / d Lambda [D] = sum over batch rows of the per-row partials [B, D]
__global__ void lambda_sum_kernel(const float* __restrict__ part, int64_t batch, int64_t D,
                                  float* __restrict__ glam) {
  const int64_t d = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float acc = 0.f;
  for (int64_t b = 0; b < batch; ++b) acc += part[b * D + d];
  glam[d] = acc;
}

template <typename T, bool kG>
static int rglru_bwd_any(const float* gy, const float* gf, const float* ckpt, const void* a, const void* x,
                         const void* ig, RgGate gate, int64_t batch, int64_t L, int64_t D, int64_t seg, void* ga,
                         void* gx, void* gi, float* glam_part, float* ws, const float* h0, float* gh0,
                         cudaStream_t st) {
  using C = DiagCfg<T>;
  constexpr int W = C::RgBW, TB = C::RgBTB, S = C::RgBS;
  constexpr size_t sm = RgBwdSmem<T, W, TB, S, kG ? 3 : 2>::bytes;
  CUtensorMap ma, mx, mg, mi;
  if (int rc = tmap_rows<T>(&ma, a, batch * L, D, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&mx, x, batch * L, D, W, TB)) return rc;
  if (int rc = tmap_rows<float>(&mg, gy, batch * L, D, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&mi, kG ? ig : a, batch * L, D, W, TB)) return rc;
  auto k = h0 != nullptr ? rglru_bwd_kernel<T, W, TB, S, true, kG> : rglru_bwd_kernel<T, W, TB, S, false, kG>;
  if (int rc = set_smem(k, sm)) return rc;
  dim3 grid((unsigned)((D + W - 1) / W), (unsigned)batch);
  k<<<grid, kThreads, sm, st>>>(ma, mx, mg, mi, gate, gf, ckpt, (const T*)a, (const T*)x, (const T*)ig, (int)L, D,
                                (int)seg, (T*)ga, (T*)gx, (T*)gi, glam_part, ws, h0, gh0);
  return check_launch("rglru_bwd_kernel");
}

template <typename T>
int rglru_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* a, const void* x,
                     int64_t batch, int64_t L, int64_t D, int64_t seg, void* ga, void* gx, float* ws,
                     const float* h0, float* gh0, cudaStream_t st) {
  return rglru_bwd_any<T, false>(gy, gf, ckpt, a, x, nullptr, RgGate{nullptr, 0.f}, batch, L, D, seg, ga, gx,
                                 nullptr, nullptr, ws, h0, gh0, st);
}

// workspace: the plain backward's (long segments), then the [B, D] Lambda partials
size_t rglru_gated_bwd_ws_bytes(int64_t batch, int64_t L, int64_t D, int64_t seg) {
  return (rglru_bwd_ws_bytes(batch, L, D, seg) + 255) / 256 * 256 + (size_t)batch * D * sizeof(float);
}

template <typename T>
int rglru_gated_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* x, const void* r,
                           const void* i, const float* lam, float c, int64_t batch, int64_t L, int64_t D,
                           int64_t seg, void* gx, void* gr, void* gi, float* glam, void* ws, const float* h0,
                           float* gh0, cudaStream_t st) {
  float* part = (float*)((char*)ws + (rglru_bwd_ws_bytes(batch, L, D, seg) + 255) / 256 * 256);
  if (int rc = rglru_bwd_any<T, true>(gy, gf, ckpt, x, r, i, RgGate{lam, c}, batch, L, D, seg, gx, gr, gi, part,
                                      (float*)ws, h0, gh0, st))
    return rc;
  lambda_sum_kernel<<<(unsigned)((D + 255) / 256), 256, 0, st>>>(part, batch, D, glam);
  return check_launch("lambda_sum_kernel");
}

// sn == nullptr: cs holds the angle theta (the kernels form cos and sin)
template <typename T, bool kTh>
int rotlru_fwd_any(const void* a, const void* cs, const void* sn, const void* x, int64_t batch, int64_t L,
                   int64_t Dp, int64_t seg, float* y, float* ckpt, const float* h0, cudaStream_t st) {
  using C = DiagCfg<T>;
  constexpr int W = kTh ? C::RotAFW : C::RotFW, TB = kTh ? C::RotAFTB : C::RotFTB, S = kTh ? C::RotAFS : C::RotFS;
  constexpr size_t sm = RotFwdSmem<T, W, TB, S, kTh ? 4 : 5>::bytes;
  CUtensorMap ma, mc, ms, mx;
  if (int rc = tmap_rows<T>(&ma, a, batch * L, Dp, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&mc, cs, batch * L, Dp, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&ms, kTh ? cs : sn, batch * L, Dp, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&mx, x, batch * L, 2 * Dp, 2 * W, TB)) return rc;
  auto k = h0 != nullptr ? rotlru_fwd_kernel<T, W, TB, S, true, kTh> : rotlru_fwd_kernel<T, W, TB, S, false, kTh>;
  if (int rc = set_smem(k, sm)) return rc;
  dim3 grid((unsigned)((Dp + W - 1) / W), (unsigned)batch);
  k<<<grid, kThreads, sm, st>>>(ma, mc, ms, mx, (int)L, Dp, (int)seg, y, ckpt, h0);
  return check_launch("rotlru_fwd_kernel");
}

template <typename T>
int rotlru_fwd_launch(const void* a, const void* cs, const void* sn, const void* x, int64_t batch,
                      int64_t L, int64_t Dp, int64_t seg, float* y, float* ckpt, const float* h0,
                      cudaStream_t st) {
  return rotlru_fwd_any<T, false>(a, cs, sn, x, batch, L, Dp, seg, y, ckpt, h0, st);
}

template <typename T>
int rotlru_angle_fwd_launch(const void* a, const void* theta, const void* x, int64_t batch, int64_t L, int64_t Dp,
                            int64_t seg, float* y, float* ckpt, const float* h0, cudaStream_t st) {
  return rotlru_fwd_any<T, true>(a, theta, nullptr, x, batch, L, Dp, seg, y, ckpt, h0, st);
}

// sn == nullptr: cs holds theta and gcs receives its gradient (gsn unused)
template <typename T, bool kTh>
int rotlru_bwd_any(const float* gy, const float* gf, const float* ckpt, const void* a, const void* cs,
                   const void* sn, const void* x, int64_t batch, int64_t L, int64_t Dp, int64_t seg, void* ga,
                   void* gcs, void* gsn, void* gx, float* ws, const float* h0, float* gh0, cudaStream_t st) {
  using C = DiagCfg<T>;
  constexpr int W = C::RotBW, TB = C::RotBTB, S = C::RotBS;  // the angle input shares the workspace layout
  constexpr size_t sm = RotBwdSmem<T, W, TB, S, kTh ? 4 : 5>::bytes;
  CUtensorMap ma, mc, ms, mx, mg;
  if (int rc = tmap_rows<T>(&ma, a, batch * L, Dp, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&mc, cs, batch * L, Dp, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&ms, kTh ? cs : sn, batch * L, Dp, W, TB)) return rc;
  if (int rc = tmap_rows<T>(&mx, x, batch * L, 2 * Dp, 2 * W, TB)) return rc;
  if (int rc = tmap_rows<float>(&mg, gy, batch * L, 2 * Dp, 2 * W, TB)) return rc;
  auto k = h0 != nullptr ? rotlru_bwd_kernel<T, W, TB, S, true, kTh> : rotlru_bwd_kernel<T, W, TB, S, false, kTh>;
  if (int rc = set_smem(k, sm)) return rc;
  dim3 grid((unsigned)((Dp + W - 1) / W), (unsigned)batch);
  k<<<grid, kThreads, sm, st>>>(ma, mc, ms, mx, mg, gf, ckpt, (const T*)a, (const T*)cs, (const T*)sn,
                                (const T*)x, (int)L, Dp, (int)seg, (T*)ga, (T*)gcs, (T*)gsn, (T*)gx, ws, h0,
                                gh0);
  return check_launch("rotlru_bwd_kernel");
}

template <typename T>
int rotlru_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* a,
                      const void* cs, const void* sn, const void* x, int64_t batch, int64_t L,
                      int64_t Dp, int64_t seg, void* ga, void* gcs, void* gsn, void* gx, float* ws,
                      const float* h0, float* gh0, cudaStream_t st) {
  return rotlru_bwd_any<T, false>(gy, gf, ckpt, a, cs, sn, x, batch, L, Dp, seg, ga, gcs, gsn, gx, ws, h0, gh0, st);
}

template <typename T>
int rotlru_angle_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* a, const void* theta,
                            const void* x, int64_t batch, int64_t L, int64_t Dp, int64_t seg, void* ga,
                            void* gtheta, void* gx, float* ws, const float* h0, float* gh0, cudaStream_t st) {
  return rotlru_bwd_any<T, true>(gy, gf, ckpt, a, theta, nullptr, x, batch, L, Dp, seg, ga, gtheta, nullptr, gx,
                                 ws, h0, gh0, st);
}

#define MR_INST(T)                                                                                  \
  template int rglru_fwd_launch<T>(const void*, const void*, int64_t, int64_t, int64_t, int64_t,    \
                                   float*, float*, const float*, cudaStream_t);                    \
  template int rglru_bwd_launch<T>(const float*, const float*, const float*, const void*,          \
                                   const void*, int64_t, int64_t, int64_t, int64_t, void*, void*,  \
                                   float*, const float*, float*, cudaStream_t);                    \
  template int rotlru_fwd_launch<T>(const void*, const void*, const void*, const void*, int64_t,   \
                                    int64_t, int64_t, int64_t, float*, float*, const float*,       \
                                    cudaStream_t);                                                 \
  template int rglru_gated_fwd_launch<T>(const void*, const void*, const void*, const float*, float, \
                                         int64_t, int64_t, int64_t, int64_t, float*, float*,       \
                                         const float*, cudaStream_t);                              \
  template int rglru_gated_bwd_launch<T>(const float*, const float*, const float*, const void*,     \
                                         const void*, const void*, const float*, float, int64_t,   \
                                         int64_t, int64_t, int64_t, void*, void*, void*, float*,   \
                                         void*, const float*, float*, cudaStream_t);               \
  template int rotlru_bwd_launch<T>(const float*, const float*, const float*, const void*,         \
                                    const void*, const void*, const void*, int64_t, int64_t,       \
                                    int64_t, int64_t, void*, void*, void*, void*, float*,          \
                                    const float*, float*, cudaStream_t);                           \
  template int rotlru_angle_fwd_launch<T>(const void*, const void*, const void*, int64_t, int64_t, \
                                          int64_t, int64_t, float*, float*, const float*,          \
                                          cudaStream_t);                                           \
  template int rotlru_angle_bwd_launch<T>(const float*, const float*, const float*, const void*,   \
                                          const void*, const void*, int64_t, int64_t, int64_t,     \
                                          int64_t, void*, void*, void*, float*, const float*,      \
                                          float*, cudaStream_t);
MR_INST(float)
MR_INST(__nv_bfloat16)
MR_INST(__half)
#undef MR_INST

}  // namespace mr
