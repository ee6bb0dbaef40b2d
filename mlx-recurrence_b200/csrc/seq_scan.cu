// SSD and GLA on CUDA cores, step by step in fp32: the exact-arithmetic
// path. It serves fp32 inputs (parity 1e-5), SSD with a decay rate that
// varies along N, and every shape the tensor-core path does not take.
//
// Reference kernels: mlx_recurrence/ssd.py:54-307, gla.py:49-270.
// One CTA (8 warps) owns one (batch, head). The state matrix is spread over
// the CTA: lane l holds state columns l, l+32, ... (the N axis for SSD, the
// i axis for GLA) and warp w holds rows w, w+8, ... (Dh for SSD, j for GLA),
// so the per-step contraction over the lane axis is a warp shuffle reduction
// and each thread carries R*NK state values in registers. The backward
// recomputes each segment from its checkpoint into a per-thread slice of
// the workspace (coalesced: element e of thread tid sits at e*256 + tid), then
// runs the reference's reverse sweep (ssd.py:204-260, gla.py:185-235).
// Sums over the warp axis (SSD grad_B/grad_C, GLA grad_q/grad_k) go through
// shared memory TS steps at a time; grad_A partials per batch row are
// reduced by a second small kernel.
#include "common.cuh"

namespace mr {

constexpr int kSeqThreads = 256;
constexpr int kTS = 4;  // steps per cross-warp partial flush
constexpr int kStage = 16;  // steps of inputs staged in shared memory at a time (at most)
// steps per staged block for rows of at most wmax floats: at most 16 prefetched values
// per thread (they stay in registers while the block before is computed)
constexpr int stage_steps(int wmax) {
  return 16 * kSeqThreads / wmax < kStage ? (16 * kSeqThreads / wmax < 1 ? 1 : 16 * kSeqThreads / wmax) : kStage;
}

// The first unit at or after `unit` in a CTA's walk (unit, + stride, ...) whose flag
// element (`flag(b * L * H + h)`, b = unit / H, h = unit % H) is NaN, or `units` when
// none is left. kSeqThreads candidates are read at once, one load per thread: a walk
// that tested one unit per iteration put a global load's latency on the path of every
// unit it skipped. Called by every thread of the CTA.
template <typename F>
__device__ int next_marked_unit(int unit, int units, int stride, int64_t L, int H, F flag) {
  __shared__ int first;
  for (; unit < units; unit += kSeqThreads * stride) {
    const int cand = unit + (int)threadIdx.x * stride;
    const bool m = cand < units && isnan(flag(((int64_t)(cand / H) * L) * H + cand % H));
    if (threadIdx.x == 0) first = units;
    __syncthreads();
    if (m) atomicMin(&first, cand);
    __syncthreads();
    const int f = first;
    __syncthreads();  // every thread has read it before the next group resets it
    if (f < units) return f;
  }
  return units;
}

// Per-step inputs staged a block of steps at a time: every thread loads its share of
// the next block (consecutive elements of a step's rows, coalesced) into registers
// while the block before is computed from shared memory, then writes them into the
// other buffer. A step's global-load latency (about a microsecond) was otherwise on
// the path of every step. A staged step is the kernel's input rows of that step side
// by side, as floats.
template <int EPT>
struct StepStage {
  float r[EPT];
};
// the SSD backward's staged row (at most): [B (N) | C (N) | u (Dh) | grad_y (Dh) | delta]
template <int R, int NK>
constexpr int ssd_bwd_wmax() { return 2 * 32 * NK + 2 * 8 * R + 1; }
// bytes of its two staging buffers (dynamic shared memory)
template <int R, int NK>
constexpr size_t ssd_bwd_stage_bytes() {
  return (size_t)2 * stage_steps(ssd_bwd_wmax<R, NK>()) * ssd_bwd_wmax<R, NK>() * sizeof(float);
}
// the GLA backward's: [k (Dh) | q (Dh) | v (Dh) | grad_y (Dh) | gate]
template <int R>
constexpr int gla_bwd_wmax() { return 4 * 8 * R + 1; }
template <int R>
constexpr size_t gla_bwd_stage_bytes() { return (size_t)2 * stage_steps(gla_bwd_wmax<R>()) * gla_bwd_wmax<R>() * sizeof(float); }

// The warp totals of R per-lane values at once (R rows of a step's outputs): a
// transposing butterfly, where each exchange hands over half of the values still
// held, so the R sums take log2(32) levels of dependent shuffles instead of R times
// as many. Returns the total of row (lane >> (5 - log2 RP)) (RP: R rounded up to a
// power of two, rows R.. are zero); every lane of a row's group holds it.
constexpr int pow2_ceil(int r) { return r <= 1 ? 1 : r <= 2 ? 2 : r <= 4 ? 4 : r <= 8 ? 8 : r <= 16 ? 16 : 32; }
// lanes sharing a row's total in warp_sum_rows<R>; the first of each group stores it
template <int R>
__device__ __forceinline__ bool row_leader(int lane) { return (lane & (32 / pow2_ceil(R) - 1)) == 0; }
template <int R>
__device__ __forceinline__ float warp_sum_rows(const float (&x)[R], int lane, int& row) {
  constexpr int RP = pow2_ceil(R);
  constexpr int LG = RP == 1 ? 0 : RP == 2 ? 1 : RP == 4 ? 2 : RP == 8 ? 3 : RP == 16 ? 4 : 5;
  float v[RP];
#pragma unroll
  for (int i = 0; i < RP; ++i) v[i] = i < R ? x[i] : 0.f;
  int o = 16;
#pragma unroll
  for (int live = RP; live > 1; live >>= 1, o >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < live / 2; ++i) {
      const float send = hi ? v[i] : v[i + live / 2];
      const float keep = hi ? v[i + live / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
#pragma unroll
  for (; o > 0; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
  row = lane >> (5 - LG);
  return v[0];
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ============================================================================
// SSD
// ============================================================================

// The state rows d of a unit evolve independently in the forward (each row's update and
// output read only that row), so a unit's Dh rows may be split over rsplit CTAs of 8R
// rows each (rows d0 .. d0 + 8R - 1, d0 = (blockIdx.x % rsplit) * 8R): with few units,
// more SMs walk the steps (c0: 36 units). rsplit = 1 in the only_marked mode (its flag
// sits in row 0 of the unit's output).
template <typename T, int R, int NK>
__global__ void __launch_bounds__(kSeqThreads)
ssd_seq_fwd_kernel(const T* __restrict__ u, const T* __restrict__ delta, const T* __restrict__ Bm,
                   const T* __restrict__ Cm, const float* __restrict__ A, int64_t ash, int64_t asn,
                   int L, int H, int Dh, int N, int seg, float* __restrict__ y,
                   float* __restrict__ ckpt, const float* __restrict__ h0, int only_marked, int rsplit) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int unit = blockIdx.x / rsplit;
  const int d0 = (blockIdx.x % rsplit) * 8 * R;  // this CTA's first row
  const int64_t b = unit / H;
  const int h = unit % H;
  const int nseg = L / seg;
  // after the dense-A tensor-core path: only the units it marked (NaN in y[b, 0, h, 0])
  if (only_marked && !isnan(y[(b * L * H + h) * Dh])) return;

  float An[NK];
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    const int n = lane + 32 * k;
    An[k] = n < N ? A[h * ash + n * asn] : 0.f;
  }
  // initial state h0 [B,H,Dh,N] (the final-state layout) or zero
  float st[R][NK];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int k = 0; k < NK; ++k) {
      const int n = lane + 32 * k;
      st[r][k] = (h0 != nullptr && n < N) ? h0[((b * H + h) * Dh + d0 + warp + 8 * r) * (int64_t)N + n] : 0.f;
    }

  // staged step rows [B (N) | C (N) | u (this CTA's 8R rows) | delta (1)], TS steps per buffer
  constexpr int WMAX = 2 * 32 * NK + 8 * R + 1;
  constexpr int TS = stage_steps(WMAX);
  constexpr int EPT = (TS * WMAX + kSeqThreads - 1) / kSeqThreads;
  __shared__ float sIn[2][TS * WMAX];
  const int W = 2 * N + 8 * R + 1;
  StepStage<EPT> pre;
  auto load_block = [&](int t0) {
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = threadIdx.x + kSeqThreads * i;
      float v = 0.f;
      if (e < TS * W) {
        const int tt = e / W, col = e - tt * W, t = t0 + tt;
        if (t < L) {
          const int64_t row = (b * L + t) * H + h;
          v = col < N               ? to_f(Bm[row * N + col])
              : col < 2 * N          ? to_f(Cm[row * N + col - N])
              : col < 2 * N + 8 * R ? to_f(u[row * Dh + d0 + col - 2 * N])
                                     : to_f(delta[row]);
        }
      }
      pre.r[i] = v;
    }
  };
  auto store_block = [&](int buf) {
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = threadIdx.x + kSeqThreads * i;
      if (e < TS * W) sIn[buf][e] = pre.r[i];
    }
  };
  const int nblk = (L + TS - 1) / TS;
  load_block(0);
  store_block(0);
  __syncthreads();

  for (int blk = 0; blk < nblk; ++blk) {
  if (blk + 1 < nblk) load_block((blk + 1) * TS);
  const int nt = min(TS, L - blk * TS);
  int tend = seg - 1 - (blk * TS) % seg;  // the block's next step that ends a segment
  auto step = [&](int tt) {
    const int t = blk * TS + tt;
    const int64_t row = (b * L + t) * H + h;
    const float* sr = sIn[blk & 1] + tt * W;
    const float dt = sr[2 * N + 8 * R];
    float dB[NK], cv[NK], dec[NK];
#pragma unroll
    for (int k = 0; k < NK; ++k) {
      const int n = lane + 32 * k;
      const bool ok = n < N;
      dB[k] = ok ? dt * sr[n] : 0.f;
      cv[k] = ok ? sr[N + n] : 0.f;
      dec[k] = ok ? expf(dt * An[k]) : 0.f;
    }
    float accs[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int d = warp + 8 * r;
      const float ud = sr[2 * N + d];
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < NK; ++k) {
        st[r][k] = dec[k] * st[r][k] + dB[k] * ud;  // ssd.py:97-98
        acc += st[r][k] * cv[k];                    // ssd.py:99
      }
      accs[r] = acc;
    }
    {
      int ri;
      const float tot = warp_sum_rows<R>(accs, lane, ri);
      if (row_leader<R>(lane) && ri < R) y[row * Dh + d0 + warp + 8 * ri] = tot;
    }
    if (tt == tend) {
      tend += seg;
      const int64_t s = (t + 1) / seg - 1;
      float* ck = ckpt + ((b * nseg + s) * H + h) * (int64_t)N * Dh + d0;
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const int n = lane + 32 * k;
          if (n < N) ck[(int64_t)n * Dh + warp + 8 * r] = st[r][k];
        }
    }
  };
  // Only the state update carries from step to step; with few state values a thread, a
  // whole block of steps is unrolled so that the independent work of later steps (the
  // decay factors, the loads, the output reduction) overlaps the earlier ones.
  if constexpr (R * NK <= 4) {
    if (nt == TS) {
#pragma unroll
      for (int tt = 0; tt < TS; ++tt) step(tt);
    } else {
      for (int tt = 0; tt < nt; ++tt) step(tt);
    }
  } else {
    for (int tt = 0; tt < nt; ++tt) step(tt);
  }
  if (blk + 1 < nblk) store_block((blk + 1) & 1);
  __syncthreads();  // the next block reads the buffer written above; this one is refilled after it
  }
}

template <typename T, int R, int NK>
__global__ void __launch_bounds__(kSeqThreads, 1)  // registers over occupancy: the per-step chain is latency-bound
ssd_seq_bwd_kernel(const float* __restrict__ gy, const float* __restrict__ gfinal,
                   const float* __restrict__ ckpt, const T* __restrict__ u,
                   const T* __restrict__ delta, const T* __restrict__ Bm, const T* __restrict__ Cm,
                   const float* __restrict__ A, int64_t ash, int64_t asn, int L, int H, int Dh,
                   int N, int seg, T* __restrict__ gu, T* __restrict__ gdelta, T* __restrict__ gB,
                   T* __restrict__ gC, float* __restrict__ gA_part, float* __restrict__ scratch,
                   const float* __restrict__ h0, float* __restrict__ gh0, int units, int only_marked,
                   int rsplit, float* __restrict__ part) {
  constexpr int NP = 32 * NK;
  __shared__ float pB[kTS][8][NP];
  __shared__ float pC[kTS][8][NP];
  __shared__ float pdt[kTS][8];
  // staged step rows (dynamic shared memory, two buffers of TS steps): the recompute
  // reads [B (N) | u (Dh) | delta], the adjoint sweep [B (N) | C (N) | u (Dh) | grad_y (Dh) | delta]
  constexpr int WMAX = ssd_bwd_wmax<R, NK>();
  constexpr int TS = stage_steps(WMAX);
  constexpr int EPT = (TS * WMAX + kSeqThreads - 1) / kSeqThreads;
  extern __shared__ float sIn[];  // [2][TS * WMAX]
  StepStage<EPT> pre;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nseg = L / seg;
  constexpr int E = R * NK;  // state values per thread
  // one scratch slot per CTA; a CTA walks units blockIdx.x, + gridDim.x, ... (one each
  // unless only_marked: then a few CTAs recompute the units the dense-A tensor-core
  // path marked, NaN in grad_delta[b, 0, h])
  float* scr = scratch + (int64_t)blockIdx.x * (seg + 1) * E * kSeqThreads + tid;
  // With rsplit > 1 (never with only_marked) a unit's rows are split over rsplit CTAs of 8R
  // rows each, d0 the CTA's first: their sums over the rows (grad_B, grad_C, grad_delta)
  // go to float32 partials part[rs] ([gB | gC] of B*L*H*N each, then gdelta of B*L*H),
  // summed over rs by a second kernel; grad_A's partial is per (batch row, rs, head).
  const int rs = blockIdx.x % rsplit, d0 = rs * 8 * R;
  const int64_t BLH = (int64_t)(units / H) * L * H;
  float* pgB = rsplit > 1 ? part + (int64_t)rs * BLH * N : nullptr;
  float* pgC = rsplit > 1 ? part + (int64_t)(rsplit + rs) * BLH * N : nullptr;
  float* pgd = rsplit > 1 ? part + (int64_t)2 * rsplit * BLH * N + (int64_t)rs * BLH : nullptr;
  for (int unit = blockIdx.x / rsplit; unit < units; unit += gridDim.x / rsplit) {
  if (only_marked) {
    unit = next_marked_unit(unit, units, gridDim.x, L, H, [&](int64_t i) { return to_f(gdelta[i]); });
    if (unit >= units) break;
  }
  const int64_t b = unit / H;
  const int h = unit % H;

  float An[NK];
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    const int n = lane + 32 * k;
    An[k] = n < N ? A[h * ash + n * asn] : 0.f;
  }
  // steps tl0 .. tl0 + n - 1 of segment s into the registers, in the recompute's (adj = false)
  // or the adjoint sweep's row layout
  // staged rows: [B | u (this CTA's 8R rows) | delta], [B | C | u | grad_y (8R rows) | delta]
  const int Wa = N + 8 * R + 1, Wb = 2 * N + 16 * R + 1;
  auto load_steps = [&](int s, int tl0, int n, bool adjl) {
    const int W = adjl ? Wb : Wa;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = threadIdx.x + kSeqThreads * i;
      float v = 0.f;
      if (e < n * W) {
        const int tt = e / W, col = e - tt * W;
        const int64_t rowt = (b * L + (int64_t)s * seg + tl0 + tt);
        const int64_t row = rowt * H + h;
        if (!adjl) {
          v = col < N ? to_f(Bm[row * N + col]) : col < N + 8 * R ? to_f(u[row * Dh + d0 + col - N]) : to_f(delta[row]);
        } else {
          v = col < N            ? to_f(Bm[row * N + col])
              : col < 2 * N      ? to_f(Cm[row * N + col - N])
              : col < 2 * N + 8 * R ? to_f(u[row * Dh + d0 + col - 2 * N])
              : col < 2 * N + 16 * R ? gy[row * Dh + d0 + col - 2 * N - 8 * R]
                                     : to_f(delta[row]);
        }
      }
      pre.r[i] = v;
    }
  };
  auto store_steps = [&](int buf, int n, bool adjl) {
    const int W = adjl ? Wb : Wa;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = threadIdx.x + kSeqThreads * i;
      if (e < n * W) sIn[buf * TS * WMAX + e] = pre.r[i];
    }
  };
  const int nb = (seg + TS - 1) / TS;  // staged blocks per segment
  auto blk_n = [&](int j) { return min(TS, seg - j * TS); };

  float adj[R][NK], gAacc[NK];
#pragma unroll
  for (int k = 0; k < NK; ++k) gAacc[k] = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int k = 0; k < NK; ++k) {
      const int n = lane + 32 * k;
      const int d = d0 + warp + 8 * r;
      adj[r][k] = (gfinal != nullptr && n < N) ? gfinal[((b * H + h) * Dh + d) * (int64_t)N + n] : 0.f;
    }

  for (int s = nseg - 1; s >= 0; --s) {
    // ---- recompute this segment's states into the thread's scratch slice
    {
      float st[R][NK];
      const float* ck = ckpt + ((b * nseg + (s - 1)) * H + h) * (int64_t)N * Dh;
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const int n = lane + 32 * k;
          const int d = d0 + warp + 8 * r;
          st[r][k] = n >= N                ? 0.f
                     : s > 0               ? ck[(int64_t)n * Dh + d]
                     : h0 != nullptr       ? h0[((b * H + h) * Dh + d) * (int64_t)N + n]
                                           : 0.f;
          scr[(int64_t)(r * NK + k) * kSeqThreads] = st[r][k];
        }
      load_steps(s, 0, blk_n(0), false);
      store_steps(0, blk_n(0), false);
      __syncthreads();
      for (int j = 0; j < nb; ++j) {
        if (j + 1 < nb) load_steps(s, (j + 1) * TS, blk_n(j + 1), false);
        const float* sb = sIn + (j & 1) * TS * WMAX;
        for (int tt = 0; tt < blk_n(j); ++tt) {
          const int tl = j * TS + tt;
          const float* sr = sb + tt * Wa;
          const float dt = sr[N + 8 * R];
          float dB[NK], dec[NK];
#pragma unroll
          for (int k = 0; k < NK; ++k) {
            const int n = lane + 32 * k;
            dB[k] = n < N ? dt * sr[n] : 0.f;
            dec[k] = n < N ? expf(dt * An[k]) : 0.f;
          }
          float* sp = scr + (int64_t)(tl + 1) * E * kSeqThreads;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const float ud = sr[N + warp + 8 * r];
#pragma unroll
            for (int k = 0; k < NK; ++k) {
              st[r][k] = dec[k] * st[r][k] + dB[k] * ud;
              sp[(int64_t)(r * NK + k) * kSeqThreads] = st[r][k];
            }
          }
        }
        if (j + 1 < nb) store_steps((j + 1) & 1, blk_n(j + 1), false);
        __syncthreads();
      }
    }

    // ---- adjoint sweep, newest -> oldest (ssd.py:204-260), its inputs staged block by block
    load_steps(s, (nb - 1) * TS, blk_n(nb - 1), true);
    store_steps(0, blk_n(nb - 1), true);
    __syncthreads();
    // The recomputed states of steps tl + 1 and tl in registers, the one of step tl - 1
    // loaded a step ahead (where a thread holds at most 16 state values): the scratch is
    // read from L2 and its latency was on every step's path.
    constexpr bool kRing = E <= 16;
    constexpr int EP = kRing ? E : 1;
    float hcr[EP], hpr[EP];
    if constexpr (kRing) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        hcr[e] = scr[((int64_t)seg * E + e) * kSeqThreads];
        hpr[e] = scr[((int64_t)(seg - 1) * E + e) * kSeqThreads];
      }
    }
    for (int j = nb - 1, q = 0; j >= 0; --j, ++q) {
    if (j > 0) load_steps(s, (j - 1) * TS, blk_n(j - 1), true);
    const float* sbuf = sIn + (q & 1) * TS * WMAX;
    for (int tl = j * TS + blk_n(j) - 1; tl >= j * TS; --tl) {
      float hnr[EP];
      if constexpr (kRing)
        if (tl > 0) {
#pragma unroll
          for (int e = 0; e < E; ++e) hnr[e] = scr[((int64_t)(tl - 1) * E + e) * kSeqThreads];
        }
      const int slot = (seg - 1 - tl) % kTS;
      const int64_t t = (int64_t)s * seg + tl;
      const int64_t row = (b * L + t) * H + h;
      const float* sr = sbuf + (tl - j * TS) * Wb;
      const float dt = sr[2 * N + 16 * R];
      float bv[NK], cv[NK], dec[NK];
#pragma unroll
      for (int k = 0; k < NK; ++k) {
        const int n = lane + 32 * k;
        const bool ok = n < N;
        bv[k] = ok ? sr[n] : 0.f;
        cv[k] = ok ? sr[N + n] : 0.f;
        dec[k] = ok ? expf(dt * An[k]) : 0.f;
      }
      const float* sc = scr + (int64_t)(tl + 1) * E * kSeqThreads;
      const float* sprev = scr + (int64_t)tl * E * kSeqThreads;
      float gdt = 0.f, pb[NK], pc[NK], gus[R];
#pragma unroll
      for (int k = 0; k < NK; ++k) pb[k] = pc[k] = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int d = warp + 8 * r;
        const float ud = sr[2 * N + d];
        const float g = sr[2 * N + 8 * R + d];
        float gu_r = 0.f;
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const float hc = kRing ? hcr[kRing ? r * NK + k : 0] : sc[(int64_t)(r * NK + k) * kSeqThreads];
          const float hp = kRing ? hpr[kRing ? r * NK + k : 0] : sprev[(int64_t)(r * NK + k) * kSeqThreads];
          float ad = adj[r][k] + g * cv[k];
          gu_r += ad * dt * bv[k];
          gdt += ad * (An[k] * dec[k] * hp + bv[k] * ud);
          gAacc[k] += ad * dt * dec[k] * hp;
          pb[k] += ad * dt * ud;
          pc[k] += hc * g;
          adj[r][k] = ad * dec[k];
        }
        gus[r] = gu_r;
      }
      {
        int ri;
        const float tot = warp_sum_rows<R>(gus, lane, ri);
        if (row_leader<R>(lane) && ri < R) gu[row * Dh + d0 + warp + 8 * ri] = from_f<T>(tot);
      }
      gdt = warp_sum(gdt);
      if (lane == 0) pdt[slot][warp] = gdt;
#pragma unroll
      for (int k = 0; k < NK; ++k) {
        pB[slot][warp][lane + 32 * k] = pb[k];
        pC[slot][warp][lane + 32 * k] = pc[k];
      }
      if (slot == kTS - 1 || tl == 0) {
        __syncthreads();
        const int nsl = slot + 1;
        for (int idx = tid; idx < nsl * N; idx += kSeqThreads) {
          const int sl = idx / N, n = idx % N;
          float sb = 0.f, scc = 0.f;
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            sb += pB[sl][w][n];
            scc += pC[sl][w][n];
          }
          const int64_t tt = t + (slot - sl);  // slot sl was step t + (slot - sl)
          const int64_t rr = (b * L + tt) * H + h;
          if (rsplit > 1) {
            pgB[rr * N + n] = sb;
            pgC[rr * N + n] = scc;
          } else {
            gB[rr * N + n] = from_f<T>(sb);
            gC[rr * N + n] = from_f<T>(scc);
          }
        }
        if (tid < nsl) {
          float sd = 0.f;
#pragma unroll
          for (int w = 0; w < 8; ++w) sd += pdt[tid][w];
          const int64_t tt = t + (slot - tid);
          if (rsplit > 1)
            pgd[(b * L + tt) * H + h] = sd;
          else
            gdelta[(b * L + tt) * H + h] = from_f<T>(sd);
        }
        __syncthreads();
      }
      if constexpr (kRing) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          hcr[e] = hpr[e];
          hpr[e] = hnr[e];
        }
      }
    }
    if (j > 0) store_steps((q + 1) & 1, blk_n(j - 1), true);
    __syncthreads();
    }
  }

  // gradient of the initial state: the adjoint carried past step 0
  if (gh0 != nullptr)
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int k = 0; k < NK; ++k) {
        const int n = lane + 32 * k;
        if (n < N) gh0[((b * H + h) * Dh + d0 + warp + 8 * r) * (int64_t)N + n] = adj[r][k];
      }
  // grad_A partial for this (b, h): sum over rows (in-thread) and warps
  __syncthreads();
#pragma unroll
  for (int k = 0; k < NK; ++k) pB[0][warp][lane + 32 * k] = gAacc[k];
  __syncthreads();
  for (int n = tid; n < N; n += kSeqThreads) {
    float sa = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) sa += pB[0][w][n];
    gA_part[((b * rsplit + rs) * H + h) * (int64_t)N + n] = sa;
  }
  __syncthreads();  // pB is reused by the next unit
  }
}

// grad_A[h,n] = sum_b part[b,h,n]   (ssd.py:305)
__global__ void sum_over_batch_kernel(const float* __restrict__ part, int64_t batch, int64_t HN,
                                      float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= HN) return;
  float s = 0.f;
  for (int64_t b = 0; b < batch; ++b) s += part[b * HN + i];
  out[i] = s;
}

// ============================================================================
// GLA
// ============================================================================

// After the tensor-core GLA path ("only_marked"), these kernels recompute the
// units it marked (a gate outside gla_gate_in_range; common.cuh).

template <typename T, int R, int IK>
__global__ void __launch_bounds__(kSeqThreads)
gla_seq_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                   const T* __restrict__ gates, int L, int H, int Dh, int seg,
                   float* __restrict__ y, float* __restrict__ ckpt, int only_marked,
                   const float* __restrict__ h0) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.x / H;
  const int h = blockIdx.x % H;
  const int nseg = L / seg;
  if (only_marked && !isnan(y[(b * L * H + h) * Dh])) return;
  // initial state h0 [B,H,Dh(i),Dh(j)] (the final-state layout) or zero
  float S[IK][R];
#pragma unroll
  for (int i = 0; i < IK; ++i)
#pragma unroll
    for (int r = 0; r < R; ++r)
      S[i][r] = h0 != nullptr ? h0[((b * H + h) * Dh + lane + 32 * i) * (int64_t)Dh + warp + 8 * r] : 0.f;

  // staged step rows [k (Dh) | q (Dh) | v (Dh) | gate], TS steps per buffer
  constexpr int WMAX = 3 * 8 * R + 1;
  constexpr int TS = stage_steps(WMAX);
  constexpr int EPT = (TS * WMAX + kSeqThreads - 1) / kSeqThreads;
  __shared__ float sIn[2][TS * WMAX];
  const int W = 3 * Dh + 1;
  StepStage<EPT> pre;
  auto load_block = [&](int t0) {
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = threadIdx.x + kSeqThreads * i;
      float x = 0.f;
      if (e < TS * W) {
        const int tt = e / W, col = e - tt * W, t = t0 + tt;
        if (t < L) {
          const int64_t row = (b * L + t) * H + h;
          x = col < Dh       ? to_f(k[row * Dh + col])
              : col < 2 * Dh ? to_f(q[row * Dh + col - Dh])
              : col < 3 * Dh ? to_f(v[row * Dh + col - 2 * Dh])
                             : to_f(gates[row]);
        }
      }
      pre.r[i] = x;
    }
  };
  auto store_block = [&](int buf) {
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = threadIdx.x + kSeqThreads * i;
      if (e < TS * W) sIn[buf][e] = pre.r[i];
    }
  };
  const int nblk = (L + TS - 1) / TS;
  load_block(0);
  store_block(0);
  __syncthreads();

  for (int blk = 0; blk < nblk; ++blk) {
  if (blk + 1 < nblk) load_block((blk + 1) * TS);
  const int nt = min(TS, L - blk * TS);
  for (int tt = 0; tt < nt; ++tt) {
    const int t = blk * TS + tt;
    const int64_t row = (b * L + t) * H + h;
    const float* sr = sIn[blk & 1] + tt * W;
    const float g = sr[3 * Dh];
    float ki[IK], qi[IK];
#pragma unroll
    for (int i = 0; i < IK; ++i) {
      ki[i] = sr[lane + 32 * i];
      qi[i] = sr[Dh + lane + 32 * i];
    }
    float os[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int j = warp + 8 * r;
      const float vj = sr[2 * Dh + j];
      float o = 0.f;
#pragma unroll
      for (int i = 0; i < IK; ++i) {
        S[i][r] = g * S[i][r] + ki[i] * vj;  // gla.py:87
        o += qi[i] * S[i][r];                // gla.py:88
      }
      os[r] = o;
    }
    {
      int ri;
      const float tot = warp_sum_rows<R>(os, lane, ri);
      if (row_leader<R>(lane) && ri < R) y[row * Dh + warp + 8 * ri] = tot;
    }
    if ((t + 1) % seg == 0) {
      const int64_t s = (t + 1) / seg - 1;
      float* ck = ckpt + ((b * nseg + s) * H + h) * (int64_t)Dh * Dh;
#pragma unroll
      for (int i = 0; i < IK; ++i)
#pragma unroll
        for (int r = 0; r < R; ++r) ck[(int64_t)(lane + 32 * i) * Dh + warp + 8 * r] = S[i][r];
    }
  }
  if (blk + 1 < nblk) store_block((blk + 1) & 1);
  __syncthreads();  // the next block reads the buffer written above; this one is refilled after it
  }
}

template <typename T, int R, int IK>
__global__ void __launch_bounds__(kSeqThreads, 1)  // as the SSD backward
gla_seq_bwd_kernel(const float* __restrict__ gy, const float* __restrict__ gfinal,
                   const float* __restrict__ ckpt, const T* __restrict__ q,
                   const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ gates,
                   int L, int H, int Dh, int seg, T* __restrict__ gq, T* __restrict__ gk,
                   T* __restrict__ gv, T* __restrict__ gg, float* __restrict__ scratch, int units,
                   int only_marked, const float* __restrict__ h0, float* __restrict__ gh0) {
  constexpr int NP = 32 * IK;
  __shared__ float pQ[kTS][8][NP];
  __shared__ float pK[kTS][8][NP];
  __shared__ float pg[kTS][8];
  // staged step rows (dynamic shared memory, two buffers of TS steps): the recompute reads
  // [k (Dh) | v (Dh) | gate], the adjoint sweep [k (Dh) | q (Dh) | v (Dh) | grad_y (Dh) | gate]
  constexpr int WMAX = gla_bwd_wmax<R>();
  constexpr int TS = stage_steps(WMAX);
  constexpr int EPT = (TS * WMAX + kSeqThreads - 1) / kSeqThreads;
  extern __shared__ float sIn[];  // [2][TS * WMAX]
  StepStage<EPT> pre;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nseg = L / seg;
  constexpr int E = R * IK;
  // one scratch slot per CTA; a CTA walks units blockIdx.x, + gridDim.x, ...
  float* scr = scratch + (int64_t)blockIdx.x * (seg + 1) * E * kSeqThreads + tid;
  for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
    if (only_marked) {
      unit = next_marked_unit(unit, units, gridDim.x, L, H, [&](int64_t i) { return to_f(gg[i]); });
      if (unit >= units) break;
    }
    const int64_t b = unit / H;
    const int h = unit % H;

    // steps tl0 .. tl0 + n - 1 of segment s into the registers, in the recompute's (adjl =
    // false) or the adjoint sweep's row layout
    const int Wa = 2 * Dh + 1, Wb = 4 * Dh + 1;
    auto load_steps = [&](int s, int tl0, int n, bool adjl) {
      const int W = adjl ? Wb : Wa;
#pragma unroll
      for (int i = 0; i < EPT; ++i) {
        const int e = threadIdx.x + kSeqThreads * i;
        float x = 0.f;
        if (e < n * W) {
          const int tt = e / W, col = e - tt * W;
          const int64_t row = (b * L + (int64_t)s * seg + tl0 + tt) * H + h;
          if (!adjl) {
            x = col < Dh ? to_f(k[row * Dh + col]) : col < 2 * Dh ? to_f(v[row * Dh + col - Dh]) : to_f(gates[row]);
          } else {
            x = col < Dh           ? to_f(k[row * Dh + col])
                : col < 2 * Dh     ? to_f(q[row * Dh + col - Dh])
                : col < 3 * Dh     ? to_f(v[row * Dh + col - 2 * Dh])
                : col < 4 * Dh     ? gy[row * Dh + col - 3 * Dh]
                                   : to_f(gates[row]);
          }
        }
        pre.r[i] = x;
      }
    };
    auto store_steps = [&](int buf, int n, bool adjl) {
      const int W = adjl ? Wb : Wa;
#pragma unroll
      for (int i = 0; i < EPT; ++i) {
        const int e = threadIdx.x + kSeqThreads * i;
        if (e < n * W) sIn[buf * TS * WMAX + e] = pre.r[i];
      }
    };
    const int nb = (seg + TS - 1) / TS;  // staged blocks per segment
    auto blk_n = [&](int j) { return min(TS, seg - j * TS); };

    float adj[IK][R];
#pragma unroll
    for (int i = 0; i < IK; ++i)
#pragma unroll
      for (int r = 0; r < R; ++r)
        adj[i][r] = gfinal != nullptr
                        ? gfinal[((b * H + h) * Dh + lane + 32 * i) * (int64_t)Dh + warp + 8 * r]
                        : 0.f;

    for (int s = nseg - 1; s >= 0; --s) {
      {
        float S[IK][R];
        const float* ck = ckpt + ((b * nseg + (s - 1)) * H + h) * (int64_t)Dh * Dh;
#pragma unroll
        for (int i = 0; i < IK; ++i)
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int64_t e = (int64_t)(lane + 32 * i) * Dh + warp + 8 * r;
            S[i][r] = s > 0 ? ck[e] : h0 != nullptr ? h0[(b * H + h) * (int64_t)Dh * Dh + e] : 0.f;
            scr[(int64_t)(i * R + r) * kSeqThreads] = S[i][r];
          }
        load_steps(s, 0, blk_n(0), false);
        store_steps(0, blk_n(0), false);
        __syncthreads();
        for (int jb = 0; jb < nb; ++jb) {
          if (jb + 1 < nb) load_steps(s, (jb + 1) * TS, blk_n(jb + 1), false);
          const float* sb = sIn + (jb & 1) * TS * WMAX;
          for (int tt = 0; tt < blk_n(jb); ++tt) {
            const int tl = jb * TS + tt;
            const float* sr = sb + tt * Wa;
            const float g = sr[2 * Dh];
            float ki[IK];
#pragma unroll
            for (int i = 0; i < IK; ++i) ki[i] = sr[lane + 32 * i];
            float* sp = scr + (int64_t)(tl + 1) * E * kSeqThreads;
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const float vj = sr[Dh + warp + 8 * r];
#pragma unroll
              for (int i = 0; i < IK; ++i) {
                S[i][r] = g * S[i][r] + ki[i] * vj;
                sp[(int64_t)(i * R + r) * kSeqThreads] = S[i][r];
              }
            }
          }
          if (jb + 1 < nb) store_steps((jb + 1) & 1, blk_n(jb + 1), false);
          __syncthreads();
        }
      }

      load_steps(s, (nb - 1) * TS, blk_n(nb - 1), true);
      store_steps(0, blk_n(nb - 1), true);
      __syncthreads();
      // the recomputed states of steps tl + 1 and tl in registers, step tl - 1's loaded a
      // step ahead (at most 16 state values a thread), as in the SSD backward
      constexpr bool kRing = E <= 16;
      constexpr int EP = kRing ? E : 1;
      float hcr[EP], hpr[EP];
      if constexpr (kRing) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          hcr[e] = scr[((int64_t)seg * E + e) * kSeqThreads];
          hpr[e] = scr[((int64_t)(seg - 1) * E + e) * kSeqThreads];
        }
      }
      for (int jb = nb - 1, qb = 0; jb >= 0; --jb, ++qb) {
      if (jb > 0) load_steps(s, (jb - 1) * TS, blk_n(jb - 1), true);
      const float* sbuf = sIn + (qb & 1) * TS * WMAX;
      for (int tl = jb * TS + blk_n(jb) - 1; tl >= jb * TS; --tl) {
        float hnr[EP];
        if constexpr (kRing)
          if (tl > 0) {
#pragma unroll
            for (int e = 0; e < E; ++e) hnr[e] = scr[((int64_t)(tl - 1) * E + e) * kSeqThreads];
          }
        const int slot = (seg - 1 - tl) % kTS;
        const int64_t t = (int64_t)s * seg + tl;
        const int64_t row = (b * L + t) * H + h;
        const float* sr = sbuf + (tl - jb * TS) * Wb;
        const float g = sr[4 * Dh];
        float ki[IK], qi[IK];
#pragma unroll
        for (int i = 0; i < IK; ++i) {
          ki[i] = sr[lane + 32 * i];
          qi[i] = sr[Dh + lane + 32 * i];
        }
        const float* sc = scr + (int64_t)(tl + 1) * E * kSeqThreads;
        const float* sprev = scr + (int64_t)tl * E * kSeqThreads;
        float ggs = 0.f, pq[IK], pk[IK], gvs[R];
#pragma unroll
        for (int i = 0; i < IK; ++i) pq[i] = pk[i] = 0.f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int j = warp + 8 * r;
          const float vj = sr[2 * Dh + j];
          const float go = sr[3 * Dh + j];
          float gv_r = 0.f;
#pragma unroll
          for (int i = 0; i < IK; ++i) {
            const float hc = kRing ? hcr[kRing ? i * R + r : 0] : sc[(int64_t)(i * R + r) * kSeqThreads];
            const float hp = kRing ? hpr[kRing ? i * R + r : 0] : sprev[(int64_t)(i * R + r) * kSeqThreads];
            const float ad = adj[i][r] + qi[i] * go;  // gla.py:213
            gv_r += ad * ki[i];
            ggs += ad * hp;
            pq[i] += go * hc;
            pk[i] += ad * vj;
            adj[i][r] = ad * g;
          }
          gvs[r] = gv_r;
        }
        {
          int ri;
          const float tot = warp_sum_rows<R>(gvs, lane, ri);
          if (row_leader<R>(lane) && ri < R) gv[row * Dh + warp + 8 * ri] = from_f<T>(tot);
        }
        ggs = warp_sum(ggs);
        if (lane == 0) pg[slot][warp] = ggs;
#pragma unroll
        for (int i = 0; i < IK; ++i) {
          pQ[slot][warp][lane + 32 * i] = pq[i];
          pK[slot][warp][lane + 32 * i] = pk[i];
        }
        if (slot == kTS - 1 || tl == 0) {
          __syncthreads();
          const int nsl = slot + 1;
          for (int idx = tid; idx < nsl * Dh; idx += kSeqThreads) {
            const int sl = idx / Dh, i = idx % Dh;
            float sq = 0.f, sk = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
              sq += pQ[sl][w][i];
              sk += pK[sl][w][i];
            }
            const int64_t rr = (b * L + t + (slot - sl)) * H + h;
            gq[rr * Dh + i] = from_f<T>(sq);
            gk[rr * Dh + i] = from_f<T>(sk);
          }
          if (tid < nsl) {
            float sd = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) sd += pg[tid][w];
            gg[(b * L + t + (slot - tid)) * H + h] = from_f<T>(sd);
          }
          __syncthreads();
        }
        if constexpr (kRing) {
#pragma unroll
          for (int e = 0; e < E; ++e) {
            hcr[e] = hpr[e];
            hpr[e] = hnr[e];
          }
        }
      }
      if (jb > 0) store_steps((qb + 1) & 1, blk_n(jb - 1), true);
      __syncthreads();
      }
    }
    // gradient of the initial state: the adjoint carried past step 0
    if (gh0 != nullptr)
#pragma unroll
      for (int i = 0; i < IK; ++i)
#pragma unroll
        for (int r = 0; r < R; ++r)
          gh0[((b * H + h) * Dh + lane + 32 * i) * (int64_t)Dh + warp + 8 * r] = adj[i][r];
    __syncthreads();  // the slot's scratch is reused by the next unit
  }
}

// ============================================================================
// host launchers
// ============================================================================

static int ceil32(int n) { return (n + 31) / 32; }
// lanes hold 1, 2 or 4 state columns (N <= 32, 64, 128)
static int nk_of(int64_t N) { const int c = ceil32((int)N); return c <= 1 ? 1 : c <= 2 ? 2 : 4; }

static int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// CTAs per unit of the per-step SSD backward: its rows split in halves while the grid
// stays within one CTA per SM (the kernel's registers allow one; Dh / 8 a power of two)
static int ssd_bwd_rsplit(int64_t batch, int64_t H, int64_t Dh) {
  const int rf = (int)Dh / 8;
  int rs = 1;
  if ((rf & (rf - 1)) == 0) {
    const int64_t cap = sm_count();
    while (rs * 2 <= rf && batch * H * rs * 2 <= cap) rs *= 2;
  }
  return rs;
}

// workspace of the per-step SSD backward: the scratch of every CTA, grad_A partials
// [B, rsplit, H, N], and with rsplit > 1 the float32 partials of grad_B, grad_C
// ([rsplit][B, L, H, N] each) and grad_delta ([rsplit][B, L, H])
static size_t align256(size_t x) { return (x + 255) / 256 * 256; }
size_t ssd_seq_bwd_ws_bytes(int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t N, int64_t seg) {
  const int64_t R = Dh / 8, NK = nk_of(N);
  const int rs = ssd_bwd_rsplit(batch, H, Dh);
  const size_t scr = (size_t)batch * H * (seg + 1) * R * NK * kSeqThreads * sizeof(float);
  const size_t gap = (size_t)batch * rs * H * N * sizeof(float);
  const size_t part = rs > 1 ? (size_t)rs * batch * L * H * (2 * N + 1) * sizeof(float) : 0;
  return align256(scr) + align256(gap) + part;
}

size_t gla_seq_bwd_ws_bytes(int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg) {
  const int64_t R = Dh / 8, IK = Dh / 32;
  return (size_t)batch * H * (seg + 1) * R * IK * kSeqThreads * sizeof(float);
}
// scratch slots of the GLA fallback after the tensor-core backward (units with
// out-of-range gates, walked by this many CTAs)
constexpr int64_t kGlaFallbackSlots = 16;
// the scratch of kGlaFallbackSlots units walked in turn
size_t gla_fallback_ws_bytes(int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg) {
  const int64_t slots = batch * H < kGlaFallbackSlots ? batch * H : kGlaFallbackSlots;
  return gla_seq_bwd_ws_bytes(slots, L, 1, Dh, seg);
}

// the dense-A tensor-core backward: its per-unit grad A partials [B, H, N], then the
// scratch of kSsdFallbackSlots units recomputed in turn by the per-step kernel
constexpr int64_t kSsdFallbackSlots = 16;
size_t ssd_fallback_ws_bytes(int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t N, int64_t seg) {
  const int64_t units = batch * H;
  const int64_t slots = units < kSsdFallbackSlots ? units : kSsdFallbackSlots;
  const size_t part = ((units * N * sizeof(float) + 255) / 256) * 256;
  return part + (size_t)slots * (seg + 1) * (Dh / 8) * nk_of(N) * kSeqThreads * sizeof(float);
}

bool ssd_seq_supported(int64_t Dh, int64_t N) {
  return (Dh == 32 || Dh == 64 || Dh == 96 || Dh == 128) && N >= 1 && N <= 128;
}
bool gla_seq_supported(int64_t Dh) { return Dh == 32 || Dh == 64 || Dh == 96 || Dh == 128; }

#define MR_SSD_DISPATCH(Dh, N, MACRO)                \
  do {                                               \
    const int nk2_ = nk_of(N);                       \
    switch ((int)(Dh) / 8) {                         \
      case 4: MACRO(4, nk2_); break;                 \
      case 8: MACRO(8, nk2_); break;                 \
      case 12: MACRO(12, nk2_); break;               \
      default: MACRO(16, nk2_); break;               \
    }                                                \
  } while (0)

template <typename T, int R>
static void ssd_fwd_nk(int nk, dim3 g, cudaStream_t st, const T* u, const T* dl, const T* Bm,
                       const T* Cm, const float* A, int64_t ash, int64_t asn, int L, int H, int Dh,
                       int N, int seg, float* y, float* ck, const float* h0, int om, int rs) {
  if (nk == 1)
    ssd_seq_fwd_kernel<T, R, 1><<<g, kSeqThreads, 0, st>>>(u, dl, Bm, Cm, A, ash, asn, L, H, Dh, N, seg, y, ck, h0, om, rs);
  else if (nk == 2)
    ssd_seq_fwd_kernel<T, R, 2><<<g, kSeqThreads, 0, st>>>(u, dl, Bm, Cm, A, ash, asn, L, H, Dh, N, seg, y, ck, h0, om, rs);
  else
    ssd_seq_fwd_kernel<T, R, 4><<<g, kSeqThreads, 0, st>>>(u, dl, Bm, Cm, A, ash, asn, L, H, Dh, N, seg, y, ck, h0, om, rs);
}

// only_marked: recompute just the units the dense-A tensor-core path marked
template <typename T>
int ssd_seq_fwd_launch(const void* u, const void* delta, const void* Bm, const void* Cm,
                       const float* A, int64_t ash, int64_t asn, int64_t batch, int64_t L, int64_t H,
                       int64_t Dh, int64_t N, int64_t seg, float* y, float* ckpt, const float* h0,
                       cudaStream_t st, int only_marked) {
  // CTAs per unit: its rows split in halves while the grid stays within two CTAs per SM
  // (Dh / 8 a power of two; one CTA per unit in the only_marked mode)
  const int64_t units = batch * H;
  const int rf = (int)Dh / 8;
  int rs = 1;
  if (!only_marked && (rf & (rf - 1)) == 0) {
    const int64_t cap = 2 * (int64_t)sm_count();
    while (rs * 2 <= rf && units * rs * 2 <= cap) rs *= 2;
  }
  dim3 g((unsigned)(units * rs));
  const int nk = nk_of(N);
#define MR_CALL(R_)                                                                                 \
  ssd_fwd_nk<T, R_>(nk, g, st, (const T*)u, (const T*)delta, (const T*)Bm, (const T*)Cm, A, ash, asn, \
                    (int)L, (int)H, (int)Dh, (int)N, (int)seg, y, ckpt, h0, only_marked, rs)
  switch (rf / rs) {
    case 1: MR_CALL(1); break;
    case 2: MR_CALL(2); break;
    case 4: MR_CALL(4); break;
    case 8: MR_CALL(8); break;
    case 12: MR_CALL(12); break;
    default: MR_CALL(16); break;
  }
#undef MR_CALL
  return check_launch("ssd_seq_fwd_kernel");
}

template <typename T, int R>
static void ssd_bwd_nk(int nk, dim3 g, cudaStream_t st, const float* gy, const float* gf,
                       const float* ck, const T* u, const T* dl, const T* Bm, const T* Cm,
                       const float* A, int64_t ash, int64_t asn, int L, int H, int Dh, int N, int seg,
                       T* gu, T* gd, T* gB, T* gC, float* gAp, float* scr, const float* h0, float* gh0,
                       int units, int om, int rs = 1, float* part = nullptr) {
  auto go = [&](auto kern, size_t sm) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    kern<<<g, kSeqThreads, sm, st>>>(gy, gf, ck, u, dl, Bm, Cm, A, ash, asn, L, H, Dh, N, seg, gu, gd, gB, gC, gAp,
                                     scr, h0, gh0, units, om, rs, part);
  };
  if (nk == 1)
    go(ssd_seq_bwd_kernel<T, R, 1>, ssd_bwd_stage_bytes<R, 1>());
  else if (nk == 2)
    go(ssd_seq_bwd_kernel<T, R, 2>, ssd_bwd_stage_bytes<R, 2>());
  else
    go(ssd_seq_bwd_kernel<T, R, 4>, ssd_bwd_stage_bytes<R, 4>());
}

// out[i] = sum over r < rsplit of part[r * n + i], in the output dtype
template <typename T>
__global__ void sum_parts_kernel(const float* __restrict__ part, int rsplit, int64_t n, T* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < rsplit; ++r) s += part[r * n + i];
    out[i] = from_f<T>(s);
  }
}

template <typename T>
int ssd_seq_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* u,
                       const void* delta, const void* Bm, const void* Cm, const float* A,
                       int64_t ash, int64_t asn, int64_t batch, int64_t L, int64_t H, int64_t Dh,
                       int64_t N, int64_t seg, void* gu, void* gd, void* gB, void* gC, float* gA,
                       void* ws, const float* h0, float* gh0, cudaStream_t st) {
  const int64_t R = Dh / 8, NK = nk_of(N), units = batch * H;
  const int rs = ssd_bwd_rsplit(batch, H, Dh);
  const size_t scr_bytes = (size_t)units * (seg + 1) * R * NK * kSeqThreads * sizeof(float);
  float* scr = (float*)ws;
  float* gAp = (float*)((char*)ws + align256(scr_bytes));
  float* part = rs > 1 ? (float*)((char*)gAp + align256((size_t)batch * rs * H * N * sizeof(float))) : nullptr;
  dim3 g((unsigned)(units * rs));
#define MR_CALL(R_)                                                                                 \
  ssd_bwd_nk<T, R_>((int)NK, g, st, gy, gf, ckpt, (const T*)u, (const T*)delta, (const T*)Bm, (const T*)Cm, A, \
                    ash, asn, (int)L, (int)H, (int)Dh, (int)N, (int)seg, (T*)gu, (T*)gd, (T*)gB, (T*)gC, gAp, \
                    scr, h0, gh0, (int)units, 0, rs, part)
  switch ((int)R / rs) {
    case 1: MR_CALL(1); break;
    case 2: MR_CALL(2); break;
    case 4: MR_CALL(4); break;
    case 8: MR_CALL(8); break;
    case 12: MR_CALL(12); break;
    default: MR_CALL(16); break;
  }
#undef MR_CALL
  int rc = check_launch("ssd_seq_bwd_kernel");
  if (rc) return rc;
  if (rs > 1) {
    const int64_t nBC = units * L * N, nd = units * L;
    const unsigned gs = (unsigned)(2 * sm_count());
    sum_parts_kernel<T><<<gs, 256, 0, st>>>(part, rs, nBC, (T*)gB);
    sum_parts_kernel<T><<<gs, 256, 0, st>>>(part + (int64_t)rs * nBC, rs, nBC, (T*)gC);
    sum_parts_kernel<T><<<gs, 256, 0, st>>>(part + (int64_t)2 * rs * nBC, rs, nd, (T*)gd);
    rc = check_launch("sum_parts_kernel");
    if (rc) return rc;
  }
  const int64_t HN = H * N;
  sum_over_batch_kernel<<<(unsigned)((HN + 255) / 256), 256, 0, st>>>(gAp, batch * rs, HN, gA);
  return check_launch("sum_over_batch_kernel");
}

// After the dense-A tensor-core backward: ws = ssd_fallback_ws_bytes, its first part the
// per-unit grad A partials [B, H, N] that path wrote. A few CTAs recompute the units it
// marked (rewriting their partials), then the partials are summed over the batch.
template <typename T>
int ssd_seq_bwd_marked_launch(const float* gy, const float* gf, const float* ckpt, const void* u,
                              const void* delta, const void* Bm, const void* Cm, const float* A,
                              int64_t ash, int64_t asn, int64_t batch, int64_t L, int64_t H, int64_t Dh,
                              int64_t N, int64_t seg, void* gu, void* gd, void* gB, void* gC, float* gA,
                              void* ws, const float* h0, float* gh0, cudaStream_t st) {
  const int64_t units = batch * H;
  float* gAp = (float*)ws;
  float* scr = (float*)((char*)ws + ((units * N * sizeof(float) + 255) / 256) * 256);
  dim3 g((unsigned)(units < kSsdFallbackSlots ? units : kSsdFallbackSlots));
#define MR_CALL(R_, NK_)                                                                        \
  ssd_bwd_nk<T, R_>(NK_, g, st, gy, gf, ckpt, (const T*)u, (const T*)delta, (const T*)Bm,         \
                    (const T*)Cm, A, ash, asn, (int)L, (int)H, (int)Dh, (int)N, (int)seg, (T*)gu,  \
                    (T*)gd, (T*)gB, (T*)gC, gAp, scr, h0, gh0, (int)units, 1)
  MR_SSD_DISPATCH(Dh, N, MR_CALL);
#undef MR_CALL
  int rc = check_launch("ssd_seq_bwd_kernel");
  if (rc) return rc;
  const int64_t HN = H * N;
  sum_over_batch_kernel<<<(unsigned)((HN + 255) / 256), 256, 0, st>>>(gAp, batch, HN, gA);
  return check_launch("sum_over_batch_kernel");
}

// only_bad: recompute just the units the tensor-core path marked (a gate
// outside gla_gate_in_range), after that path has written every unit.
template <typename T>
int gla_seq_fwd_launch(const void* q, const void* k, const void* v, const void* g, int64_t batch,
                       int64_t L, int64_t H, int64_t Dh, int64_t seg, float* y, float* ckpt,
                       const float* h0, cudaStream_t st, int only_bad) {
  dim3 grid((unsigned)(batch * H));
  const T *q_ = (const T*)q, *k_ = (const T*)k, *v_ = (const T*)v, *g_ = (const T*)g;
  const int L_ = (int)L, H_ = (int)H, s_ = (int)seg;
  switch ((int)Dh) {
    case 32: gla_seq_fwd_kernel<T, 4, 1><<<grid, kSeqThreads, 0, st>>>(q_, k_, v_, g_, L_, H_, 32, s_, y, ckpt, only_bad, h0); break;
    case 64: gla_seq_fwd_kernel<T, 8, 2><<<grid, kSeqThreads, 0, st>>>(q_, k_, v_, g_, L_, H_, 64, s_, y, ckpt, only_bad, h0); break;
    case 96: gla_seq_fwd_kernel<T, 12, 3><<<grid, kSeqThreads, 0, st>>>(q_, k_, v_, g_, L_, H_, 96, s_, y, ckpt, only_bad, h0); break;
    default: gla_seq_fwd_kernel<T, 16, 4><<<grid, kSeqThreads, 0, st>>>(q_, k_, v_, g_, L_, H_, 128, s_, y, ckpt, only_bad, h0); break;
  }
  return check_launch("gla_seq_fwd_kernel");
}

// ws: gla_seq_bwd_ws_bytes (every unit) or, with only_bad, gla_fallback_ws_bytes
template <typename T>
int gla_seq_bwd_launch(const float* gy, const float* gf, const float* ckpt, const void* q,
                       const void* k, const void* v, const void* g, int64_t batch, int64_t L,
                       int64_t H, int64_t Dh, int64_t seg, void* gq, void* gk, void* gv, void* gg,
                       void* ws, const float* h0, float* gh0, cudaStream_t st, int only_bad) {
  const int64_t units = batch * H;
  const T *q_ = (const T*)q, *k_ = (const T*)k, *v_ = (const T*)v, *g_ = (const T*)g;
  T *gq_ = (T*)gq, *gk_ = (T*)gk, *gv_ = (T*)gv, *gg_ = (T*)gg;
  float* scr = (float*)ws;
  const int L_ = (int)L, H_ = (int)H, s_ = (int)seg, u_ = (int)units;
  // only_bad: a few CTAs walk the units and recompute the marked ones
  const int flags = only_bad ? 1 : 0;
  dim3 grid((unsigned)(only_bad ? (units < kGlaFallbackSlots ? units : kGlaFallbackSlots) : units));
  auto go = [&](auto kern, int dh, size_t sm) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    kern<<<grid, kSeqThreads, sm, st>>>(gy, gf, ckpt, q_, k_, v_, g_, L_, H_, dh, s_, gq_, gk_, gv_, gg_, scr, u_, flags,
                                        h0, gh0);
  };
  switch ((int)Dh) {
    case 32: go(gla_seq_bwd_kernel<T, 4, 1>, 32, gla_bwd_stage_bytes<4>()); break;
    case 64: go(gla_seq_bwd_kernel<T, 8, 2>, 64, gla_bwd_stage_bytes<8>()); break;
    case 96: go(gla_seq_bwd_kernel<T, 12, 3>, 96, gla_bwd_stage_bytes<12>()); break;
    default: go(gla_seq_bwd_kernel<T, 16, 4>, 128, gla_bwd_stage_bytes<16>()); break;
  }
  return check_launch("gla_seq_bwd_kernel");
}

#define MR_INST(T)                                                                                  \
  template int ssd_seq_fwd_launch<T>(const void*, const void*, const void*, const void*,           \
                                     const float*, int64_t, int64_t, int64_t, int64_t, int64_t,   \
                                     int64_t, int64_t, int64_t, float*, float*, const float*,     \
                                     cudaStream_t, int);                                           \
  template int ssd_seq_bwd_marked_launch<T>(const float*, const float*, const float*, const void*, \
                                            const void*, const void*, const void*, const float*,  \
                                            int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, \
                                            int64_t, int64_t, void*, void*, void*, void*, float*, \
                                            void*, const float*, float*, cudaStream_t);            \
  template int ssd_seq_bwd_launch<T>(const float*, const float*, const float*, const void*,        \
                                     const void*, const void*, const void*, const float*, int64_t, \
                                     int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, \
                                     void*, void*, void*, void*, float*, void*, const float*,      \
                                     float*, cudaStream_t);                                        \
  template int gla_seq_fwd_launch<T>(const void*, const void*, const void*, const void*, int64_t,  \
                                     int64_t, int64_t, int64_t, int64_t, float*, float*,           \
                                     const float*, cudaStream_t, int);                             \
  template int gla_seq_bwd_launch<T>(const float*, const float*, const float*, const void*,        \
                                     const void*, const void*, const void*, int64_t, int64_t,      \
                                     int64_t, int64_t, int64_t, void*, void*, void*, void*, void*, \
                                     const float*, float*, cudaStream_t, int);
MR_INST(float)
MR_INST(__nv_bfloat16)
MR_INST(__half)
#undef MR_INST

}  // namespace mr
