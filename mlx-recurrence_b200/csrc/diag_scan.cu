// Diagonal scans: RG-LRU (real, h <- a*h + x) and rotational LRU (complex
// pair, h <- a*R(theta)*h + x), forward with segment checkpoints and
// checkpoint-recompute backward.
//
// Reference kernels: mlx_recurrence/rglru.py:64-203, rotlru.py:80-266.
// The reference walks all L steps with one thread per channel (rglru.py:81-101);
// at B*D = 20,480 channels that leaves a B200 far from HBM saturation. Here a
// CTA owns a tile of W = 32*V adjacent channels of one batch row and walks L
// in blocks of 8*TW steps; inside a block each of the 8 warps owns TW
// consecutive steps, so every warp-wide load is one contiguous row segment
// (coalesced, V elements per lane) and 8 steps' worth of loads are in flight
// per thread, with the next block prefetched into registers.
//
// Within a block the scan is the classic three-phase chunk scan over the
// affine step maps h -> a*h + x:
//   1. each thread folds its TW steps into one map (A, H),
//   2. the 8 per-warp maps are exchanged through shared memory and each thread
//      folds the maps of the warps before it into its carry-in,
//   3. each thread re-runs its TW steps from the carry-in with the reference's
//      exact per-step update (rglru.py:92), writing y and the checkpoints.
// The backward applies the same three phases twice per block: forward to
// regenerate h_{t-1} from the block's starting checkpoint, then in reverse
// to run the adjoint c_{t-1} = a_t * (gy_t + c_t) (rglru.py:36-39).
#include "common.cuh"

namespace mr {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// ============================================================================
// RG-LRU
// ============================================================================

template <typename T, int V, int TW>
__global__ void __launch_bounds__(kThreads)
rglru_fwd_kernel(const T* __restrict__ a, const T* __restrict__ x, int L, int64_t D, int seg,
                 float* __restrict__ y, float* __restrict__ ckpt) {
  constexpr int W = 32 * V;
  constexpr int TB = kWarps * TW;
  __shared__ float sA[2][kWarps][W];
  __shared__ float sH[2][kWarps][W];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t c = (int64_t)blockIdx.x * W + lane * V;
  const bool act = c < D;
  const int64_t base = b * (int64_t)L * D + c;
  const int nseg = L / seg;
  const int nblk = (L + TB - 1) / TB;

  Vec<T, V> ca[TW], cx[TW];
  auto load = [&](int blk, Vec<T, V>(&ra)[TW], Vec<T, V>(&rx)[TW]) {
    const int t0 = blk * TB + warp * TW;
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      if (act && t0 + i < L) {
        ra[i] = ld_stream<T, V>(a + base + (int64_t)(t0 + i) * D);
        rx[i] = ld_stream<T, V>(x + base + (int64_t)(t0 + i) * D);
      }
    }
  };
  load(0, ca, cx);

  float carry[V];
#pragma unroll
  for (int v = 0; v < V; ++v) carry[v] = 0.f;

  for (int blk = 0; blk < nblk; ++blk) {
    Vec<T, V> na[TW], nx[TW];
    if (blk + 1 < nblk) load(blk + 1, na, nx);
    const int buf = blk & 1;
    const int t0 = blk * TB + warp * TW;

    // phase 1: fold this thread's TW steps
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float A = 1.f, H = 0.f;
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        if (t0 + i < L) {
          const float av = to_f(ca[i].v[v]);
          H = av * H + to_f(cx[i].v[v]);
          A = av * A;
        }
      }
      sA[buf][warp][lane * V + v] = A;
      sH[buf][warp][lane * V + v] = H;
    }
    __syncthreads();

    // phase 2: carry-in for this warp, carry-out of the block
    float cin[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float cur = carry[v];
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (w == warp) cin[v] = cur;
        cur = sA[buf][w][lane * V + v] * cur + sH[buf][w][lane * V + v];
      }
      carry[v] = cur;
    }

    // phase 3: exact per-step recurrence from the carry-in (rglru.py:92-99)
    if (act) {
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        const int t = t0 + i;
        if (t < L) {
          float hv[V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            cin[v] = to_f(ca[i].v[v]) * cin[v] + to_f(cx[i].v[v]);
            hv[v] = cin[v];
          }
          st_stream_f32<V>(y + base + (int64_t)t * D, hv);
          if ((t + 1) % seg == 0) {
            const int64_t s = (t + 1) / seg - 1;
            st_stream_f32<V>(ckpt + (b * nseg + s) * D + c, hv);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      ca[i] = na[i];
      cx[i] = nx[i];
    }
  }
}

template <typename T, int V, int TW>
__global__ void __launch_bounds__(kThreads)
rglru_bwd_kernel(const float* __restrict__ gy, const float* __restrict__ gfinal,
                 const float* __restrict__ ckpt, const T* __restrict__ a, const T* __restrict__ x,
                 int L, int64_t D, int seg, int grp, T* __restrict__ ga, T* __restrict__ gx,
                 float* __restrict__ ws) {
  constexpr int W = 32 * V;
  constexpr int TB = kWarps * TW;
  __shared__ float sA[2][kWarps][W];
  __shared__ float sH[2][kWarps][W];
  __shared__ float sR[2][kWarps][W];
  __shared__ float sG[2][kWarps][W];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t c = (int64_t)blockIdx.x * W + lane * V;
  const bool act = c < D;
  const int64_t base = b * (int64_t)L * D + c;
  const int nseg = L / seg;
  const int glen = grp * seg;                  // steps per segment group
  const int ngrp = (nseg + grp - 1) / grp;
  const int nsub_max = (glen + TB - 1) / TB;   // > 1 only when seg > TB
  float* wsb = ws + ((b * gridDim.x + blockIdx.x) * (int64_t)nsub_max) * W + lane * V;
  int it = 0;                                  // shared-buffer parity counter

  // incoming adjoint carry c_L = dL/dh_final (rglru.py drops it; see mlrec.h)
  float cr[V];
#pragma unroll
  for (int v = 0; v < V; ++v) cr[v] = (gfinal != nullptr && act) ? gfinal[b * D + c + v] : 0.f;

  for (int g = ngrp - 1; g >= 0; --g) {
    const int g0 = g * glen;
    const int gl = min(glen, L - g0);
    const int nsub = (gl + TB - 1) / TB;
    float hstart[V];
#pragma unroll
    for (int v = 0; v < V; ++v)
      hstart[v] = (g0 > 0 && act) ? ckpt[(b * nseg + g0 / seg - 1) * D + c + v] : 0.f;

    // pass 1 (segments longer than one block): states at sub-block starts
    if (nsub > 1) {
      float cur[V];
#pragma unroll
      for (int v = 0; v < V; ++v) cur[v] = hstart[v];
      for (int j = 0; j + 1 < nsub; ++j, ++it) {
        const int buf = it & 1;
        const int t0 = g0 + j * TB + warp * TW;
        const int tend = g0 + gl;
#pragma unroll
        for (int v = 0; v < V; ++v) {
          float A = 1.f, H = 0.f;
#pragma unroll
          for (int i = 0; i < TW; ++i) {
            if (act && t0 + i < tend) {
              const float av = to_f(a[base + (int64_t)(t0 + i) * D + v]);
              H = av * H + to_f(x[base + (int64_t)(t0 + i) * D + v]);
              A = av * A;
            }
          }
          sA[buf][warp][lane * V + v] = A;
          sH[buf][warp][lane * V + v] = H;
        }
        __syncthreads();
#pragma unroll
        for (int v = 0; v < V; ++v) {
#pragma unroll
          for (int w = 0; w < kWarps; ++w) cur[v] = sA[buf][w][lane * V + v] * cur[v] + sH[buf][w][lane * V + v];
          if (warp == 0 && act) wsb[(int64_t)(j + 1) * W + v] = cur[v];
        }
      }
      __syncthreads();
    }

    // pass 2: sub-blocks newest -> oldest
    for (int j = nsub - 1; j >= 0; --j, ++it) {
      const int buf = it & 1;
      const int s0 = g0 + j * TB;
      const int sl = min(TB, g0 + gl - s0);
      const int t0 = s0 + warp * TW;
      const int tend = s0 + sl;

      float fa[TW][V], fxv[TW][V], fg[TW][V];
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        const bool ok = act && (t0 + i < tend);
        if (ok) {
          const int64_t off = base + (int64_t)(t0 + i) * D;
          Vec<T, V> ra = ld_stream<T, V>(a + off);
          Vec<T, V> rx = ld_stream<T, V>(x + off);
          Vec<float, V> rg = ld_stream<float, V>(gy + off);
#pragma unroll
          for (int v = 0; v < V; ++v) {
            fa[i][v] = to_f(ra.v[v]);
            fxv[i][v] = to_f(rx.v[v]);
            fg[i][v] = rg.v[v];
          }
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            fa[i][v] = 1.f;
            fxv[i][v] = 0.f;
            fg[i][v] = 0.f;
          }
        }
      }
      float hs[V];
#pragma unroll
      for (int v = 0; v < V; ++v) hs[v] = (j == 0) ? hstart[v] : (act ? wsb[(int64_t)j * W + v] : 0.f);

      // forward phase 1
#pragma unroll
      for (int v = 0; v < V; ++v) {
        float A = 1.f, H = 0.f;
#pragma unroll
        for (int i = 0; i < TW; ++i) {
          H = fa[i][v] * H + fxv[i][v];
          A = fa[i][v] * A;
        }
        sA[buf][warp][lane * V + v] = A;
        sH[buf][warp][lane * V + v] = H;
      }
      // reverse phase 1: c_out = a*(gy + c_in), folded newest -> oldest
#pragma unroll
      for (int v = 0; v < V; ++v) {
        float A = 1.f, G = 0.f;
#pragma unroll
        for (int i = TW - 1; i >= 0; --i) {
          G = fa[i][v] * (fg[i][v] + G);
          A = fa[i][v] * A;
        }
        sR[buf][warp][lane * V + v] = A;
        sG[buf][warp][lane * V + v] = G;
      }
      __syncthreads();

      float hp[TW][V];   // h_{t-1} for each owned step
      float crin[V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        float cur = hs[v];
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          if (w == warp) break;
          cur = sA[buf][w][lane * V + v] * cur + sH[buf][w][lane * V + v];
        }
#pragma unroll
        for (int i = 0; i < TW; ++i) {
          hp[i][v] = cur;
          cur = fa[i][v] * cur + fxv[i][v];
        }
        float rc = cr[v];
#pragma unroll
        for (int w = kWarps - 1; w >= 0; --w) {
          if (w == warp) crin[v] = rc;
          rc = sR[buf][w][lane * V + v] * rc + sG[buf][w][lane * V + v];
        }
        cr[v] = rc;
      }

      // reverse phase 3: adjoint per step (rglru.py:173-178)
#pragma unroll
      for (int i = TW - 1; i >= 0; --i) {
        const int t = t0 + i;
        float gxa[V], gaa[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const float adj = fg[i][v] + crin[v];
          gxa[v] = adj;
          gaa[v] = adj * hp[i][v];
          crin[v] = adj * fa[i][v];
        }
        if (act && t < tend) {
          const int64_t off = base + (int64_t)t * D;
          st_vec<T, V>(gx + off, gxa);
          st_vec<T, V>(ga + off, gaa);
        }
      }
    }
  }
}

// ============================================================================
// Rotational LRU (complex pair per channel; rotlru.py:80-266)
// ============================================================================

struct cf {
  float r, i;
};
__device__ __forceinline__ cf cmul(cf p, cf q) { return {p.r * q.r - p.i * q.i, p.r * q.i + p.i * q.r}; }
__device__ __forceinline__ cf cfma(cf p, cf q, cf s) {  // p*q + s
  return {p.r * q.r - p.i * q.i + s.r, p.r * q.i + p.i * q.r + s.i};
}

template <typename T, int V, int TW>
__global__ void __launch_bounds__(kThreads)
rotlru_fwd_kernel(const T* __restrict__ a, const T* __restrict__ cs, const T* __restrict__ sn,
                  const T* __restrict__ x, int L, int64_t Dp, int seg, float* __restrict__ y,
                  float* __restrict__ ckpt) {
  constexpr int W = 32 * V;
  constexpr int TB = kWarps * TW;
  __shared__ cf sZ[2][kWarps][W];
  __shared__ cf sH[2][kWarps][W];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t p = (int64_t)blockIdx.x * W + lane * V;  // first pair
  const bool act = p < Dp;
  const int64_t D = 2 * Dp;
  const int64_t pbase = b * (int64_t)L * Dp + p;
  const int64_t xbase = b * (int64_t)L * D + 2 * p;
  const int nseg = L / seg;
  const int nblk = (L + TB - 1) / TB;

  Vec<T, V> ca[TW], cc[TW], cs_[TW];
  Vec<T, 2 * V> cx[TW];
  auto load = [&](int blk, Vec<T, V>(&ra)[TW], Vec<T, V>(&rc)[TW], Vec<T, V>(&rs)[TW],
                  Vec<T, 2 * V>(&rx)[TW]) {
    const int t0 = blk * TB + warp * TW;
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      if (act && t0 + i < L) {
        const int64_t o = pbase + (int64_t)(t0 + i) * Dp;
        ra[i] = ld_stream<T, V>(a + o);
        rc[i] = ld_stream<T, V>(cs + o);
        rs[i] = ld_stream<T, V>(sn + o);
        rx[i] = ld_stream<T, 2 * V>(x + xbase + (int64_t)(t0 + i) * D);
      }
    }
  };
  load(0, ca, cc, cs_, cx);

  cf carry[V];
#pragma unroll
  for (int v = 0; v < V; ++v) carry[v] = {0.f, 0.f};

  for (int blk = 0; blk < nblk; ++blk) {
    Vec<T, V> na[TW], nc[TW], ns[TW];
    Vec<T, 2 * V> nx[TW];
    if (blk + 1 < nblk) load(blk + 1, na, nc, ns, nx);
    const int buf = blk & 1;
    const int t0 = blk * TB + warp * TW;

#pragma unroll
    for (int v = 0; v < V; ++v) {
      cf Z = {1.f, 0.f}, H = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        if (t0 + i < L) {
          const float av = to_f(ca[i].v[v]);
          const cf z = {av * to_f(cc[i].v[v]), av * to_f(cs_[i].v[v])};
          H = cfma(z, H, {to_f(cx[i].v[2 * v]), to_f(cx[i].v[2 * v + 1])});
          Z = cmul(z, Z);
        }
      }
      sZ[buf][warp][lane * V + v] = Z;
      sH[buf][warp][lane * V + v] = H;
    }
    __syncthreads();

    cf cin[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      cf cur = carry[v];
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (w == warp) cin[v] = cur;
        cur = cfma(sZ[buf][w][lane * V + v], cur, sH[buf][w][lane * V + v]);
      }
      carry[v] = cur;
    }

    if (act) {
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        const int t = t0 + i;
        if (t < L) {
          float hv[2 * V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const float av = to_f(ca[i].v[v]), c = to_f(cc[i].v[v]), s = to_f(cs_[i].v[v]);
            const float u = cin[v].r, w = cin[v].i;
            // rotlru.py:110-111, same operation order
            const float un = av * (c * u - s * w) + to_f(cx[i].v[2 * v]);
            const float wn = av * (s * u + c * w) + to_f(cx[i].v[2 * v + 1]);
            cin[v] = {un, wn};
            hv[2 * v] = un;
            hv[2 * v + 1] = wn;
          }
          st_stream_f32<2 * V>(y + xbase + (int64_t)t * D, hv);
          if ((t + 1) % seg == 0) {
            const int64_t s = (t + 1) / seg - 1;
            st_stream_f32<2 * V>(ckpt + (b * nseg + s) * D + 2 * p, hv);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      ca[i] = na[i];
      cc[i] = nc[i];
      cs_[i] = ns[i];
      cx[i] = nx[i];
    }
  }
}

template <typename T, int V, int TW>
__global__ void __launch_bounds__(kThreads)
rotlru_bwd_kernel(const float* __restrict__ gy, const float* __restrict__ gfinal,
                  const float* __restrict__ ckpt, const T* __restrict__ a, const T* __restrict__ cs,
                  const T* __restrict__ sn, const T* __restrict__ x, int L, int64_t Dp, int seg,
                  int grp, T* __restrict__ ga, T* __restrict__ gcs, T* __restrict__ gsn,
                  T* __restrict__ gx, float* __restrict__ ws) {
  constexpr int W = 32 * V;
  constexpr int TB = kWarps * TW;
  __shared__ cf sZ[2][kWarps][W];
  __shared__ cf sH[2][kWarps][W];
  __shared__ cf sR[2][kWarps][W];
  __shared__ cf sG[2][kWarps][W];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t p = (int64_t)blockIdx.x * W + lane * V;
  const bool act = p < Dp;
  const int64_t D = 2 * Dp;
  const int64_t pbase = b * (int64_t)L * Dp + p;
  const int64_t xbase = b * (int64_t)L * D + 2 * p;
  const int nseg = L / seg;
  const int glen = grp * seg;
  const int ngrp = (nseg + grp - 1) / grp;
  const int nsub_max = (glen + TB - 1) / TB;
  float* wsb = ws + ((b * gridDim.x + blockIdx.x) * (int64_t)nsub_max) * (2 * W) + 2 * lane * V;
  int it = 0;

  cf cr[V];
#pragma unroll
  for (int v = 0; v < V; ++v)
    cr[v] = (gfinal != nullptr && act) ? cf{gfinal[b * D + 2 * (p + v)], gfinal[b * D + 2 * (p + v) + 1]}
                                       : cf{0.f, 0.f};

  for (int g = ngrp - 1; g >= 0; --g) {
    const int g0 = g * glen;
    const int gl = min(glen, L - g0);
    const int nsub = (gl + TB - 1) / TB;
    cf hstart[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (g0 > 0 && act) {
        const float* ck = ckpt + (b * nseg + g0 / seg - 1) * D + 2 * (p + v);
        hstart[v] = {ck[0], ck[1]};
      } else {
        hstart[v] = {0.f, 0.f};
      }
    }

    if (nsub > 1) {
      cf cur[V];
#pragma unroll
      for (int v = 0; v < V; ++v) cur[v] = hstart[v];
      for (int j = 0; j + 1 < nsub; ++j, ++it) {
        const int buf = it & 1;
        const int t0 = g0 + j * TB + warp * TW;
        const int tend = g0 + gl;
#pragma unroll
        for (int v = 0; v < V; ++v) {
          cf Z = {1.f, 0.f}, H = {0.f, 0.f};
#pragma unroll
          for (int i = 0; i < TW; ++i) {
            if (act && t0 + i < tend) {
              const int64_t o = pbase + (int64_t)(t0 + i) * Dp + v;
              const float av = to_f(a[o]);
              const cf z = {av * to_f(cs[o]), av * to_f(sn[o])};
              const int64_t ox = xbase + (int64_t)(t0 + i) * D + 2 * v;
              H = cfma(z, H, {to_f(x[ox]), to_f(x[ox + 1])});
              Z = cmul(z, Z);
            }
          }
          sZ[buf][warp][lane * V + v] = Z;
          sH[buf][warp][lane * V + v] = H;
        }
        __syncthreads();
#pragma unroll
        for (int v = 0; v < V; ++v) {
#pragma unroll
          for (int w = 0; w < kWarps; ++w) cur[v] = cfma(sZ[buf][w][lane * V + v], cur[v], sH[buf][w][lane * V + v]);
          if (warp == 0 && act) {
            wsb[(int64_t)(j + 1) * 2 * W + 2 * v] = cur[v].r;
            wsb[(int64_t)(j + 1) * 2 * W + 2 * v + 1] = cur[v].i;
          }
        }
      }
      __syncthreads();
    }

    for (int j = nsub - 1; j >= 0; --j, ++it) {
      const int buf = it & 1;
      const int s0 = g0 + j * TB;
      const int sl = min(TB, g0 + gl - s0);
      const int t0 = s0 + warp * TW;
      const int tend = s0 + sl;

      float fa[TW][V], fc[TW][V], fs[TW][V];
      cf fx[TW][V], fg[TW][V];
#pragma unroll
      for (int i = 0; i < TW; ++i) {
        const bool ok = act && (t0 + i < tend);
        if (ok) {
          const int64_t o = pbase + (int64_t)(t0 + i) * Dp;
          const int64_t ox = xbase + (int64_t)(t0 + i) * D;
          Vec<T, V> ra = ld_stream<T, V>(a + o);
          Vec<T, V> rc = ld_stream<T, V>(cs + o);
          Vec<T, V> rs = ld_stream<T, V>(sn + o);
          Vec<T, 2 * V> rx = ld_stream<T, 2 * V>(x + ox);
          Vec<float, 2 * V> rg = ld_stream<float, 2 * V>(gy + ox);
#pragma unroll
          for (int v = 0; v < V; ++v) {
            fa[i][v] = to_f(ra.v[v]);
            fc[i][v] = to_f(rc.v[v]);
            fs[i][v] = to_f(rs.v[v]);
            fx[i][v] = {to_f(rx.v[2 * v]), to_f(rx.v[2 * v + 1])};
            fg[i][v] = {rg.v[2 * v], rg.v[2 * v + 1]};
          }
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            fa[i][v] = 1.f;
            fc[i][v] = 1.f;
            fs[i][v] = 0.f;
            fx[i][v] = {0.f, 0.f};
            fg[i][v] = {0.f, 0.f};
          }
        }
      }
      cf hs[V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        if (j == 0) {
          hs[v] = hstart[v];
        } else if (act) {
          hs[v] = {wsb[(int64_t)j * 2 * W + 2 * v], wsb[(int64_t)j * 2 * W + 2 * v + 1]};
        } else {
          hs[v] = {0.f, 0.f};
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
        sZ[buf][warp][lane * V + v] = Z;
        sH[buf][warp][lane * V + v] = H;
        // reverse map: c_out = conj(z) * (gy + c_in)
        cf R = {1.f, 0.f}, G = {0.f, 0.f};
#pragma unroll
        for (int i = TW - 1; i >= 0; --i) {
          const cf zc = {fa[i][v] * fc[i][v], -fa[i][v] * fs[i][v]};
          G = cmul(zc, {fg[i][v].r + G.r, fg[i][v].i + G.i});
          R = cmul(zc, R);
        }
        sR[buf][warp][lane * V + v] = R;
        sG[buf][warp][lane * V + v] = G;
      }
      __syncthreads();

      cf hp[TW][V];
      cf crin[V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        cf cur = hs[v];
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          if (w == warp) break;
          cur = cfma(sZ[buf][w][lane * V + v], cur, sH[buf][w][lane * V + v]);
        }
#pragma unroll
        for (int i = 0; i < TW; ++i) {
          hp[i][v] = cur;
          const float u = cur.r, w = cur.i;
          const float c = fc[i][v], s = fs[i][v], av = fa[i][v];
          cur = {av * (c * u - s * w) + fx[i][v].r, av * (s * u + c * w) + fx[i][v].i};
        }
        cf rc = cr[v];
#pragma unroll
        for (int w = kWarps - 1; w >= 0; --w) {
          if (w == warp) crin[v] = rc;
          rc = cfma(sR[buf][w][lane * V + v], rc, sG[buf][w][lane * V + v]);
        }
        cr[v] = rc;
      }

      // adjoint per step (rotlru.py:499-516)
#pragma unroll
      for (int i = TW - 1; i >= 0; --i) {
        const int t = t0 + i;
        float o_a[V], o_c[V], o_s[V], o_x[2 * V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const float aU = fg[i][v].r + crin[v].r;
          const float aW = fg[i][v].i + crin[v].i;
          const float up = hp[i][v].r, wp = hp[i][v].i;
          const float c = fc[i][v], s = fs[i][v], av = fa[i][v];
          o_x[2 * v] = aU;
          o_x[2 * v + 1] = aW;
          const float ru = c * up - s * wp;
          const float rw = s * up + c * wp;
          o_a[v] = aU * ru + aW * rw;
          o_c[v] = av * (aU * up + aW * wp);
          o_s[v] = av * (aW * up - aU * wp);
          crin[v] = {av * (c * aU + s * aW), av * (-s * aU + c * aW)};
        }
        if (act && t < tend) {
          const int64_t o = pbase + (int64_t)t * Dp;
          st_vec<T, V>(ga + o, o_a);
          st_vec<T, V>(gcs + o, o_c);
          st_vec<T, V>(gsn + o, o_s);
          st_vec<T, 2 * V>(gx + xbase + (int64_t)t * D, o_x);
        }
      }
    }
  }
}

// ============================================================================
// host launchers
// ============================================================================

// Forward tiles: V channels per lane (W = 32*V per CTA), TW steps per warp.
constexpr int kRgFwdV = 2, kRgFwdTW = 16;
constexpr int kRgBwdV = 2, kRgBwdTW = 8;
constexpr int kRotFwdV = 2, kRotFwdTW = 8;
constexpr int kRotBwdV = 1, kRotBwdTW = 8;

static int seg_group(int seg, int TB) { return seg >= TB ? 1 : TB / seg; }

size_t rglru_bwd_ws_bytes(int64_t batch, int64_t L, int64_t D, int64_t seg) {
  constexpr int W = 32 * kRgBwdV, TB = kWarps * kRgBwdTW;
  const int grp = seg_group((int)seg, TB);
  const int64_t nsub = (grp * seg + TB - 1) / TB;
  if (nsub <= 1) return 0;
  return (size_t)batch * ((D + W - 1) / W) * nsub * W * sizeof(float);
}

size_t rotlru_bwd_ws_bytes(int64_t batch, int64_t L, int64_t Dp, int64_t seg) {
  constexpr int W = 32 * kRotBwdV, TB = kWarps * kRotBwdTW;
  const int grp = seg_group((int)seg, TB);
  const int64_t nsub = (grp * seg + TB - 1) / TB;
  if (nsub <= 1) return 0;
  return (size_t)batch * ((Dp + W - 1) / W) * nsub * 2 * W * sizeof(float);
}

template <typename T>
int rglru_fwd_launch(const void* a, const void* x, int64_t batch, int64_t L, int64_t D, int64_t seg,
                     float* y, float* ckpt, cudaStream_t st) {
  constexpr int W = 32 * kRgFwdV;
  dim3 grid((unsigned)((D + W - 1) / W), (unsigned)batch);
  rglru_fwd_kernel<T, kRgFwdV, kRgFwdTW><<<grid, kThreads, 0, st>>>(
      (const T*)a, (const T*)x, (int)L, D, (int)seg, y, ckpt);
  return check_launch("rglru_fwd_kernel");
}

template <typename T>
int rglru_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* a, const void* x,
                     int64_t batch, int64_t L, int64_t D, int64_t seg, void* ga, void* gx, float* ws,
                     cudaStream_t st) {
  constexpr int W = 32 * kRgBwdV, TB = kWarps * kRgBwdTW;
  dim3 grid((unsigned)((D + W - 1) / W), (unsigned)batch);
  rglru_bwd_kernel<T, kRgBwdV, kRgBwdTW><<<grid, kThreads, 0, st>>>(
      gy, gf, ckpt, (const T*)a, (const T*)x, (int)L, D, (int)seg, seg_group((int)seg, TB), (T*)ga,
      (T*)gx, ws);
  return check_launch("rglru_bwd_kernel");
}

template <typename T>
int rotlru_fwd_launch(const void* a, const void* cs, const void* sn, const void* x, int64_t batch,
                      int64_t L, int64_t Dp, int64_t seg, float* y, float* ckpt, cudaStream_t st) {
  constexpr int W = 32 * kRotFwdV;
  dim3 grid((unsigned)((Dp + W - 1) / W), (unsigned)batch);
  rotlru_fwd_kernel<T, kRotFwdV, kRotFwdTW><<<grid, kThreads, 0, st>>>(
      (const T*)a, (const T*)cs, (const T*)sn, (const T*)x, (int)L, Dp, (int)seg, y, ckpt);
  return check_launch("rotlru_fwd_kernel");
}

template <typename T>
int rotlru_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* a,
                      const void* cs, const void* sn, const void* x, int64_t batch, int64_t L,
                      int64_t Dp, int64_t seg, void* ga, void* gcs, void* gsn, void* gx, float* ws,
                      cudaStream_t st) {
  constexpr int W = 32 * kRotBwdV, TB = kWarps * kRotBwdTW;
  dim3 grid((unsigned)((Dp + W - 1) / W), (unsigned)batch);
  rotlru_bwd_kernel<T, kRotBwdV, kRotBwdTW><<<grid, kThreads, 0, st>>>(
      gy, gf, ckpt, (const T*)a, (const T*)cs, (const T*)sn, (const T*)x, (int)L, Dp, (int)seg,
      seg_group((int)seg, TB), (T*)ga, (T*)gcs, (T*)gsn, (T*)gx, ws);
  return check_launch("rotlru_bwd_kernel");
}

#define MR_INST(T)                                                                                  \
  template int rglru_fwd_launch<T>(const void*, const void*, int64_t, int64_t, int64_t, int64_t,    \
                                   float*, float*, cudaStream_t);                                  \
  template int rglru_bwd_launch<T>(const float*, const float*, const float*, const void*,          \
                                   const void*, int64_t, int64_t, int64_t, int64_t, void*, void*,  \
                                   float*, cudaStream_t);                                          \
  template int rotlru_fwd_launch<T>(const void*, const void*, const void*, const void*, int64_t,   \
                                    int64_t, int64_t, int64_t, float*, float*, cudaStream_t);      \
  template int rotlru_bwd_launch<T>(const float*, const float*, const float*, const void*,         \
                                    const void*, const void*, const void*, int64_t, int64_t,       \
                                    int64_t, int64_t, void*, void*, void*, void*, float*,          \
                                    cudaStream_t);
MR_INST(float)
MR_INST(__nv_bfloat16)
MR_INST(__half)
#undef MR_INST

}  // namespace mr
