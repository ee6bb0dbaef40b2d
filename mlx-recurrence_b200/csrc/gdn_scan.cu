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
// (grad_q = S_t go, grad_k = G w + S_{t-1} gp) sum each warp's 8 columns through
// a per-warp transpose buffer every step and the warps' partial sums once per
// four-step sub-block.
//
// The forward also keeps w_t per step ([B,L,H,Dh] float32, the size of the
// output), so the backward's replays need no dot products: per segment
// (newest first), phase A replays the states from the segment's checkpoint with
// the stored w (S <- alpha S + k w^T, two operations per element and step) and
// keeps a sub-checkpoint of S every kGdnK steps in a per-CTA scratch
// (short-lived, L2-resident); phase B walks the sub-blocks newest first,
// replays the kGdnK states S_{t-1} of the sub-block from its sub-checkpoint into
// thread-private shared-memory slots, and runs the adjoint step
// (docs/DESIGN_gated_deltanet.md:334-401):
//   G += q go^T;  d = G^T k;  gp = -alpha beta d
//   grad_q = S_t go,  grad_k = G w + S_{t-1} gp,  grad_v = beta d
//   grad_alpha = <G, S_{t-1}> - beta d.p,  grad_beta = d.(v - alpha p)
//   G <- alpha G + k gp^T
// The replays use the forward's operations in the forward's order, so they
// reproduce its states bit for bit.
#include "common.cuh"

namespace mr {

constexpr int kGdnK = 4;           // steps per replayed sub-block of the backward
constexpr int kGdnMaxCtas = 4096;  // backward CTAs at most (each walks units)
// The backward's scratch (ceil(seg/4) states of Dh x Dh floats per CTA) is kept
// under this many bytes by walking more units per CTA: long segments (small
// checkpoint memory) do not turn into a large workspace.
constexpr int64_t kGdnScratchBudget = (int64_t)1 << 30;

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

// sum over the P row groups of a column (lanes 32/P apart); every lane of the
// group gets the same bits
template <int P>
__device__ __forceinline__ float gdn_group_sum_p(float x) {
#pragma unroll
  for (int o = 32 / P; o < 32; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float gdn_warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Pairs of float32 lanes in one instruction (sm_100's packed f32x2 arithmetic,
// each lane rounded as its scalar operation): the per-step loops here are bound by
// float32 issue, so the element-wise updates and the dot products go two at a time.
__device__ __forceinline__ float2 gdn_pair(const float* x) { return make_float2(x[0], x[1]); }
__device__ __forceinline__ float2 gdn_bcast(float x) { return make_float2(x, x); }

// one step of the state update, shared by the forward and both replays:
// S = fma(a, S, k * w) per element (the same rounding as the scalar form)
template <int R>
__device__ __forceinline__ void gdn_update(float (&S)[R], const float (&kr)[R], float a, float w) {
  const float2 a2 = gdn_bcast(a), w2 = gdn_bcast(w);
#pragma unroll
  for (int r = 0; r < R; r += 2) {
    const float2 x = __ffma2_rn(a2, gdn_pair(S + r), __fmul2_rn(gdn_pair(kr + r), w2));
    S[r] = x.x, S[r + 1] = x.y;
  }
}

// 16-byte asynchronous global -> shared copies (each thread waits for its own
// groups; the block barrier after the wait publishes them)
__device__ __forceinline__ void gdn_cp16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void gdn_cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void gdn_cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// rows of TS steps of NV (<= 3) [B,L,H,DH] tensors of one (b, h) into shared
// [NV][TS][DH] (steps past L are not copied)
template <typename T, int DH, int TS, int NV, int NT>
__device__ __forceinline__ void gdn_stage_rows(T* dst, const T* s0, const T* s1, const T* s2, int64_t b, int h,
                                               int L, int H, int t0) {
  constexpr int CH = DH * (int)sizeof(T) / 16;  // 16-byte chunks per row
  constexpr int VN = 16 / (int)sizeof(T);
  for (int c = threadIdx.x; c < NV * TS * CH; c += NT) {
    const int which = c / (TS * CH), rem = c % (TS * CH), tt = rem / CH, ch = rem % CH;
    const int t = t0 + tt;
    const T* src = which == 0 ? s0 : which == 1 ? s1 : s2;
    if (t < L) gdn_cp16(dst + (which * TS + tt) * DH + ch * VN, src + ((b * L + t) * H + h) * DH + ch * VN);
  }
}

// 4 consecutive elements of T (shared memory) as floats
template <typename T>
__device__ __forceinline__ float4 gdn_ld4(const T* p) {
  const Vec<T, 4> x = ld_vec<T, 4>(p);
  return make_float4(to_f(x.v[0]), to_f(x.v[1]), to_f(x.v[2]), to_f(x.v[3]));
}

// R consecutive floats (shared memory, 16-byte aligned)
template <int R>
__device__ __forceinline__ void gdn_ld_f32(const float* p, float (&f)[R]) {
#pragma unroll
  for (int c = 0; c < R / 4; ++c) {
    const float4 x = *reinterpret_cast<const float4*>(p + 4 * c);
    f[4 * c] = x.x, f[4 * c + 1] = x.y, f[4 * c + 2] = x.z, f[4 * c + 3] = x.w;
  }
}

// Sum over a warp's 8 columns (lanes jl = lane & 7) of each lane's R values
// (rows g R .. g R + R - 1, g = lane >> 3) through the warp's transpose buffer
// wb (8 rows of 4R + 4 floats); out[DH] (shared) receives the warp's sums.
template <int R>
__device__ __forceinline__ void gdn_warp_colsum(float* wb, const float (&x)[R], float* out) {
  constexpr int RS = 4 * R + 4, E = R / 8;  // buffer row stride; rows summed per lane
  static_assert(E == 1 || E == 2, "R must be 8 or 16");
  const int lane = threadIdx.x & 31, g = lane >> 3, jl = lane & 7;
  float* dst = wb + jl * RS + g * R;
#pragma unroll
  for (int c = 0; c < R / 4; ++c)
    *reinterpret_cast<float4*>(dst + 4 * c) = make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
  __syncwarp();
  const float* src = wb + g * R + E * jl;
  if constexpr (E == 2) {
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const float2 v = *reinterpret_cast<const float2*>(src + jj * RS);
      acc.x += v.x, acc.y += v.y;
    }
    __syncwarp();  // the buffer is written again next
    *reinterpret_cast<float2*>(out + g * R + E * jl) = acc;
  } else {
    float acc = 0.f;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) acc += src[jj * RS];
    __syncwarp();
    out[g * R + jl] = acc;
  }
}

// sum_r x[r] y[r]: the even and the odd terms in the two lanes of a pair
template <int R>
__device__ __forceinline__ float gdn_dot(const float (&x)[R], const float (&y)[R]) {
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int r = 0; r < R; r += 2) acc = __ffma2_rn(gdn_pair(x + r), gdn_pair(y + r), acc);
  return acc.x + acc.y;
}
// x = fma(a, x, y * c) per element
template <int R>
__device__ __forceinline__ void gdn_axpy_scaled(float (&x)[R], float a, const float (&y)[R], float c) {
  const float2 a2 = gdn_bcast(a), c2 = gdn_bcast(c);
#pragma unroll
  for (int r = 0; r < R; r += 2) {
    const float2 v = __ffma2_rn(a2, gdn_pair(x + r), __fmul2_rn(gdn_pair(y + r), c2));
    x[r] = v.x, x[r + 1] = v.y;
  }
}

constexpr int kGdnTS = 16;  // steps per staged block of the forward and the backward's replay

// The forward splits each column over P row groups (P threads, Dh/P rows each).
// Four: eight at Dh = 64 was slower on B200 (c6 forward 4.8 ms against 3.15; the
// same registers per thread, so no more warps per SM, and a third shuffle level).
template <int DH> struct GdnFwdP { static constexpr int v = 4; };

template <typename T, int DH, bool kH0>
__global__ void __launch_bounds__(DH * GdnFwdP<DH>::v)
gdn_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               const T* __restrict__ alpha, const T* __restrict__ beta, int L, int H, int seg,
               float* __restrict__ y, float* __restrict__ ckpt, float* __restrict__ wp,
               const float* __restrict__ h0, const int* __restrict__ only) {
  if (only != nullptr && only[blockIdx.x] == 0) return;  // recompute flagged units only
  constexpr int P = GdnFwdP<DH>::v, R = DH / P, NT = DH * P, TS = kGdnTS, CW = 32 / P;
  static_assert(TS * (DH / 4) <= NT && (TS * (DH / 4)) % 32 == 0, "the conversion pass: 4 elements a thread");
  // staged inputs: k, q, v rows as copied [2 buffers][3][TS][DH] of T, as floats
  // [3][TS][DH], k.q per step [TS], alpha and beta [2][2][TS]
  __shared__ __align__(16) T srow[2][3 * TS * DH];
  __shared__ __align__(16) float sf[3 * TS * DH];
  __shared__ float skq[TS];
  __shared__ float sab[2][2][TS];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane / CW, j = warp * CW + (lane % CW), i0 = g * R;
  const int64_t b = blockIdx.x / H;
  const int h = blockIdx.x % H;
  const int nseg = L / seg, nblk = (L + TS - 1) / TS;
  const int64_t sbase = ((b * H + h) * DH + i0) * (int64_t)DH + j;  // element (i0, j) of [B,H,DH,DH]
  float S[R];
#pragma unroll
  for (int r = 0; r < R; ++r) S[r] = kH0 ? h0[sbase + r * DH] : 0.f;

  // alpha, beta of a block: thread tid < 2*TS holds one value until it is stored
  auto load_ab = [&](int blk) {
    const int t = blk * TS + (tid % TS);
    return (tid < 2 * TS && t < L) ? to_f((tid < TS ? alpha : beta)[(b * L + t) * H + h]) : 0.f;
  };
  gdn_stage_rows<T, DH, TS, 3, NT>(srow[0], k, q, v, b, h, L, H, 0);
  gdn_cp_commit();
  float ab = load_ab(0);
  if (tid < 2 * TS) sab[0][tid / TS][tid % TS] = ab;

  for (int blk = 0; blk < nblk; ++blk) {
    const int buf = blk & 1;
    if (blk + 1 < nblk) {
      gdn_stage_rows<T, DH, TS, 3, NT>(srow[buf ^ 1], k, q, v, b, h, L, H, (blk + 1) * TS);
      ab = load_ab(blk + 1);
    }
    gdn_cp_commit();
    gdn_cp_wait<1>();
    __syncthreads();
    if (tid < TS * (DH / 4)) {  // one pass per block: rows to floats (4 elements of k, q, v
                                // per thread) and k.q per step
      const int tt = tid / (DH / 4), c4 = (tid % (DH / 4)) * 4;
      const T* src = srow[buf] + tt * DH + c4;
      const float4 kk = gdn_ld4(src), qq = gdn_ld4(src + TS * DH), vv = gdn_ld4(src + 2 * TS * DH);
      float* dst = sf + tt * DH + c4;
      *reinterpret_cast<float4*>(dst) = kk;
      *reinterpret_cast<float4*>(dst + TS * DH) = qq;
      *reinterpret_cast<float4*>(dst + 2 * TS * DH) = vv;
      float part = fmaf(kk.x, qq.x, fmaf(kk.y, qq.y, fmaf(kk.z, qq.z, kk.w * qq.w)));
#pragma unroll
      for (int o = 1; o < DH / 4; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (c4 == 0) skq[tt] = part;
    }
    __syncthreads();
    const float* fk = sf;
    const float* fq = sf + TS * DH;
    const float* fv = sf + 2 * TS * DH;
    const int nt = min(TS, L - blk * TS);
    for (int tt = 0; tt < nt; ++tt) {
      const int t = blk * TS + tt;
      float kr[R], qr[R];
      gdn_ld_f32<R>(fk + tt * DH + i0, kr);
      gdn_ld_f32<R>(fq + tt * DH + i0, qr);
      const float vj = fv[tt * DH + j];
      const float a = sab[buf][0][tt], bt = sab[buf][1][tt];
      const float p = gdn_group_sum_p<P>(gdn_dot(kr, S));
      const float sqv = gdn_group_sum_p<P>(gdn_dot(qr, S));
      const float kq = skq[tt];
      const float w = bt * fmaf(-a, p, vj);
      if (g == 0) {
        const int64_t row = (b * L + t) * H + h;
        y[row * DH + j] = fmaf(a, sqv, kq * w);
        if (wp != nullptr) wp[row * DH + j] = w;
      }
      gdn_update(S, kr, a, w);
      if ((t + 1) % seg == 0) {
        float* c = ckpt + ((b * nseg + (t + 1) / seg - 1) * H + h) * (int64_t)DH * DH + (int64_t)i0 * DH + j;
#pragma unroll
        for (int r = 0; r < R; ++r) c[r * DH] = S[r];
      }
    }
    if (blk + 1 < nblk && tid < 2 * TS) sab[buf ^ 1][tid / TS][tid % TS] = ab;
    __syncthreads();  // the next block's copies go into this buffer
  }
}

// Shared memory of the backward (bytes): thread-private state slots
// [K][R/4][NT] float4, one transpose buffer per warp [8][DH + 4], the per-warp
// column sums of the sub-block [K][NW][2][DH] and its scalars [K][NW][2], and the
// staged inputs, phase A's ([2][alpha][TS], [2][w][TS][DH] float, [2 buffers][k][TS][DH] of T)
// and phase B's ([2][go, w, p][K][DH] float, [2][alpha, beta][K], the
// current sub-block's q, k, v as floats [3][K][DH] and w.go [K], [2][q, k, v][K][DH]
// of T) sharing one region.
template <typename T, int DH>
struct GdnBwdSmem {
  static constexpr int NT = DH * 4, K = kGdnK, TS = kGdnTS;
  static constexpr size_t slots = (size_t)K * DH * DH * 4;  // [K][R/4][NT] float4, thread-private
  static constexpr size_t red = (size_t)(NT / 32) * 8 * (DH + 4) * 4;  // per-warp transpose buffers
  static constexpr size_t part = (size_t)K * (NT / 32) * 2 * DH * 4;   // [K][NW][2][DH] partial sums
  static constexpr size_t rsc = ((size_t)K * (NT / 32) * 2 * 4 + 15) / 16 * 16;  // [K][NW][2] scalars
  static constexpr size_t a_ab = (size_t)2 * TS * 4, a_w = (size_t)2 * TS * DH * 4;
  static constexpr size_t a_rows = (size_t)2 * TS * DH * sizeof(T);
  static constexpr size_t b_f32 = (size_t)2 * 2 * K * DH * 4, b_ab = (size_t)2 * 2 * K * 4;
  static constexpr size_t b_cvt = (size_t)3 * K * DH * 4, b_wgo = 16;
  static constexpr size_t b_rows = (size_t)2 * 3 * K * DH * sizeof(T);
  static constexpr size_t stage_a = a_ab + a_w + a_rows, stage_b = b_f32 + b_ab + b_cvt + b_wgo + b_rows;
  static constexpr size_t stage = stage_a > stage_b ? stage_a : stage_b;
  static constexpr size_t bytes = slots + red + part + rsc + stage;
};

// per-CTA scratch: sub-checkpoints [ceil(seg/K)][R/4][NT] of float4
__host__ __device__ __forceinline__ int64_t gdn_scratch_floats(int64_t Dh, int64_t seg) {
  return (seg + kGdnK - 1) / kGdnK * Dh * Dh;
}

template <typename T, int DH, bool kH0>
__global__ void __launch_bounds__(DH * 4, DH == 64 ? 2 : 4)
gdn_bwd_kernel(const float* __restrict__ gy, const float* __restrict__ gfinal, const float* __restrict__ ckpt,
               const float* __restrict__ wp, const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               const T* __restrict__ alpha, const T* __restrict__ beta, int L, int H, int seg, int units,
               T* __restrict__ gq, T* __restrict__ gk, T* __restrict__ gv, T* __restrict__ galpha,
               T* __restrict__ gbeta, float* __restrict__ ws, const float* __restrict__ h0,
               float* __restrict__ gh0) {
  using SM = GdnBwdSmem<T, DH>;
  constexpr int R = DH / 4, NT = DH * 4, NW = NT / 32, K = kGdnK, TS = kGdnTS, RS = DH + 4;
  constexpr int CHF = DH * 4 / 16;  // 16-byte chunks of a float row
  extern __shared__ float4 gdn_smem[];
  unsigned char* base = reinterpret_cast<unsigned char*>(gdn_smem);
  float4* slots4 = reinterpret_cast<float4*>(base);  // [K][R/4][NT]
  float* ppart = reinterpret_cast<float*>(base + SM::slots + SM::red);
  float* psc = reinterpret_cast<float*>(base + SM::slots + SM::red + SM::part);
  unsigned char* stg = base + SM::slots + SM::red + SM::part + SM::rsc;
  // phase A staging
  float* a_ab = reinterpret_cast<float*>(stg);                 // [2][TS]: alpha
  float* a_w = reinterpret_cast<float*>(stg + SM::a_ab);       // [2][TS][DH]: w
  T* a_rows = reinterpret_cast<T*>(stg + SM::a_ab + SM::a_w);  // [2][TS][DH]: k
  // phase B staging
  float* b_f32 = reinterpret_cast<float*>(stg);                // [2][2][K][DH]: go, w
  float* b_ab = reinterpret_cast<float*>(stg + SM::b_f32);     // [2][2][K]
  float* b_cvt = reinterpret_cast<float*>(stg + SM::b_f32 + SM::b_ab);  // [3][K][DH]: q, k, v
  float* b_wgo = b_cvt + 3 * K * DH;                                   // [K]
  T* b_rows = reinterpret_cast<T*>(stg + SM::b_f32 + SM::b_ab + SM::b_cvt + SM::b_wgo);  // [2][3][K][DH]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 3, j = warp * 8 + (lane & 7), i0 = g * R;
  const int nseg = L / seg, nsb = (seg + K - 1) / K, nblk = (seg + TS - 1) / TS;
  float* wbuf = reinterpret_cast<float*>(base + SM::slots) + warp * 8 * RS;  // this warp's transpose buffer
  float* sub = ws + (int64_t)blockIdx.x * gdn_scratch_floats(DH, seg);

  for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
    const int64_t b = unit / H;
    const int h = unit % H;
    const int64_t sbase = ((b * H + h) * DH + i0) * (int64_t)DH + j;
    float G[R];
#pragma unroll
    for (int r = 0; r < R; ++r) G[r] = gfinal != nullptr ? gfinal[sbase + r * DH] : 0.f;

    for (int s = nseg - 1; s >= 0; --s) {
      const int t0 = s * seg;
      // alpha / beta of NS steps from step tl0 of the segment (thread tid < 2*NS holds one)
      auto load_ab = [&](int tl0, int NS) {
        const int tl = tl0 + tid % NS;
        return (tid < 2 * NS && tl < seg) ? to_f((tid < NS ? alpha : beta)[(b * L + t0 + tl) * H + h]) : 0.f;
      };
      // ---- phase A: replay the segment's states with the stored w, keep every K-th
      {
        float S[R];
        const float* src = s > 0 ? ckpt + ((b * nseg + s - 1) * H + h) * (int64_t)DH * DH + (int64_t)i0 * DH + j
                           : kH0 ? h0 + sbase : nullptr;
#pragma unroll
        for (int r = 0; r < R; ++r) S[r] = src != nullptr ? src[r * DH] : 0.f;
        // k rows (T) and w rows (float) of TS steps from step tl0 of the segment into buffer bb
        auto stage_a = [&](int tl0, int bb) {
          gdn_stage_rows<T, DH, TS, 1, NT>(a_rows + bb * TS * DH, k, k, k, b, h, L, H, t0 + tl0);
          for (int c = tid; c < TS * CHF; c += NT) {
            const int tt = c / CHF, ch = c % CHF, tl = tl0 + tt;
            if (tl < seg) gdn_cp16(a_w + (bb * TS + tt) * DH + ch * 4, wp + ((b * L + t0 + tl) * H + h) * DH + ch * 4);
          }
        };
        stage_a(0, 0);
        gdn_cp_commit();
        float ab = load_ab(0, TS);
        if (tid < TS) a_ab[tid] = ab;
        for (int blk = 0; blk < nblk; ++blk) {
          const int buf = blk & 1;
          if (blk + 1 < nblk) {
            stage_a((blk + 1) * TS, buf ^ 1);
            ab = load_ab((blk + 1) * TS, TS);
          }
          gdn_cp_commit();
          gdn_cp_wait<1>();
          __syncthreads();
          const T* sk = a_rows + buf * TS * DH;
          const float* sw = a_w + buf * TS * DH;
          const float* sa = a_ab + buf * TS;
          const int nt = min(TS, seg - blk * TS);
          for (int tt = 0; tt < nt; ++tt) {
            const int tl = blk * TS + tt;
            if (tl % K == 0) {
              float4* d = reinterpret_cast<float4*>(sub + (int64_t)(tl / K) * DH * DH) + tid;
#pragma unroll
              for (int c = 0; c < R / 4; ++c) d[c * NT] = make_float4(S[4 * c], S[4 * c + 1], S[4 * c + 2], S[4 * c + 3]);
            }
            float kr[R];
            gdn_load_rows<T, R>(sk + tt * DH + i0, kr);
            gdn_update(S, kr, sa[tt], sw[tt * DH + j]);
          }
          if (blk + 1 < nblk && tid < TS) a_ab[(buf ^ 1) * TS + tid] = ab;
          __syncthreads();  // this buffer is refilled next; sub-checkpoints visible to the block
        }
      }

      // ---- phase B: sub-blocks newest first, their inputs staged one sub-block ahead
      auto stage_b = [&](int sb, int bb) {
        gdn_stage_rows<T, DH, K, 3, NT>(b_rows + bb * 3 * K * DH, q, k, v, b, h, L, H, t0 + sb * K);
        float* dst = b_f32 + bb * 2 * K * DH;
        for (int c = tid; c < 2 * K * CHF; c += NT) {
          const int which = c / (K * CHF), rem = c % (K * CHF), tt = rem / CHF, ch = rem % CHF;
          const int tl = sb * K + tt;
          if (tl < seg) {
            const int64_t row = (b * L + t0 + tl) * H + h;
            const float* src = (which == 0 ? gy : wp) + row * DH;
            gdn_cp16(dst + (which * K + tt) * DH + ch * 4, src + ch * 4);
          }
        }
      };
      stage_b(nsb - 1, 0);
      gdn_cp_commit();
      float ab = load_ab((nsb - 1) * K, K);
      if (tid < 2 * K) b_ab[tid] = ab;
      for (int sb = nsb - 1; sb >= 0; --sb) {
        const int bb = (nsb - 1 - sb) & 1;
        if (sb > 0) {
          stage_b(sb - 1, bb ^ 1);
          ab = load_ab((sb - 1) * K, K);
        }
        gdn_cp_commit();
        gdn_cp_wait<1>();
        __syncthreads();
        const float* fgo = b_f32 + bb * 2 * K * DH;
        const float* fw = fgo + K * DH;
        const float* fab = b_ab + bb * 2 * K;
        {  // the sub-block's q, k, v rows as floats (threads 0 .. 3KDH/4 - 1, one 4-element
           // chunk each) and w.go per step (the last KDH/4 threads)
          constexpr int NCH = K * DH / 4;  // 4-element chunks of a [K][DH] block
          static_assert(4 * NCH == NT, "one chunk per thread");
          const int which = tid / NCH, m = (tid % NCH) / (DH / 4), c4 = (tid % (DH / 4)) * 4;
          if (which < 3) {
            *reinterpret_cast<float4*>(b_cvt + (which * K + m) * DH + c4) =
                gdn_ld4(b_rows + (bb * 3 + which) * K * DH + m * DH + c4);
          } else {
            const float4 ww = *reinterpret_cast<const float4*>(fw + m * DH + c4);
            const float4 gg = *reinterpret_cast<const float4*>(fgo + m * DH + c4);
            float part = fmaf(ww.x, gg.x, fmaf(ww.y, gg.y, fmaf(ww.z, gg.z, ww.w * gg.w)));
#pragma unroll
            for (int o = 1; o < DH / 4; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            if (c4 == 0) b_wgo[m] = part;
          }
        }
        __syncthreads();
        const float* rq_ = b_cvt;            // q rows
        const float* rk_ = b_cvt + K * DH;   // k rows
        const float* rv_ = b_cvt + 2 * K * DH;  // v rows
        const int tb = sb * K, nk = min(K, seg - tb);
        // The next (older) sub-block's sub-checkpoint is copied from L2 into slot K-1 of
        // this thread ahead of time: as soon as this sub-block no longer needs that slot.
        auto prefetch_sub = [&](int sbn) {
          const float4* src = reinterpret_cast<const float4*>(sub + (int64_t)sbn * DH * DH) + tid;
#pragma unroll
          for (int c = 0; c < R / 4; ++c) gdn_cp16(&slots4[((K - 1) * (R / 4) + c) * NT + tid], src + c * NT);
          gdn_cp_commit();
        };
        {
          float cur[R];
          // this sub-block's sub-checkpoint: prefetched into slot K-1 by the previous
          // (newer) sub-block, complete after the wait above; the newest one from L2
          const bool pre = sb < nsb - 1;
          const float4* src = pre ? &slots4[(K - 1) * (R / 4) * NT + tid]
                                  : reinterpret_cast<const float4*>(sub + (int64_t)sb * DH * DH) + tid;
#pragma unroll
          for (int c = 0; c < R / 4; ++c) {
            const float4 x = src[c * NT];
            cur[4 * c] = x.x, cur[4 * c + 1] = x.y, cur[4 * c + 2] = x.z, cur[4 * c + 3] = x.w;
            slots4[c * NT + tid] = x;
          }
          if (sb > 0 && nk < K) prefetch_sub(sb - 1);  // slot K-1 is not used by this sub-block
#pragma unroll 1
          for (int m = 1; m < nk; ++m) {
            float kr[R];
            gdn_ld_f32<R>(rk_ + (m - 1) * DH + i0, kr);
            gdn_update(cur, kr, fab[m - 1], fw[(m - 1) * DH + j]);
#pragma unroll
            for (int c = 0; c < R / 4; ++c)
              slots4[(m * (R / 4) + c) * NT + tid] = make_float4(cur[4 * c], cur[4 * c + 1], cur[4 * c + 2], cur[4 * c + 3]);
          }
        }
#pragma unroll 1
        for (int m = nk - 1; m >= 0; --m) {
          {
            const int64_t row = (b * L + t0 + tb + m) * H + h;
            float kr[R], Sp[R];
            gdn_ld_f32<R>(rk_ + m * DH + i0, kr);
            const float go = fgo[m * DH + j];
            {
              float qr[R];
              gdn_ld_f32<R>(rq_ + m * DH + i0, qr);
              const float2 go2 = gdn_bcast(go);
#pragma unroll
              for (int r = 0; r < R; r += 2) {  // output seed (B0): G += q go
                const float2 x = __ffma2_rn(gdn_pair(qr + r), go2, gdn_pair(G + r));
                G[r] = x.x, G[r + 1] = x.y;
              }
            }
#pragma unroll
            for (int c = 0; c < R / 4; ++c) {
              const float4 x = slots4[(m * (R / 4) + c) * NT + tid];
              Sp[4 * c] = x.x, Sp[4 * c + 1] = x.y, Sp[4 * c + 2] = x.z, Sp[4 * c + 3] = x.w;
            }
            const float vj = rv_[m * DH + j];
            const float a = fab[m], bt = fab[K + m];
            const float w = fw[m * DH + j];
            const float p = gdn_group_sum(gdn_dot(kr, Sp));  // S_{t-1}^T k, from the replayed state
            const float d = gdn_group_sum(gdn_dot(kr, G));
            const float gp = -a * bt * d;
            float gaP = gdn_dot(G, Sp), gbP = 0.f;
            if (m == K - 1 && sb > 0) prefetch_sub(sb - 1);  // slot K-1 has been read (gaP uses it)
            if (g == 0) {
              gaP = fmaf(-bt * d, p, gaP);
              gbP = d * fmaf(-a, p, vj);
              gv[row * DH + j] = from_f<T>(bt * d);
            }
            // this column's terms of grad_q and grad_k (G w + S_{t-1} gp), summed over the
            // warp's 8 columns through its transpose buffer; grad_q = S_t go = alpha
            // S_{t-1} go + k (w.go), alpha and the last term applied by the sub-block's reducer
            {
              float r1[R], r2[R];
              const float2 go2 = gdn_bcast(go), w2 = gdn_bcast(w), gp2 = gdn_bcast(gp);
#pragma unroll
              for (int r = 0; r < R; r += 2) {
                const float2 sp = gdn_pair(Sp + r);
                const float2 x1 = __fmul2_rn(sp, go2);
                const float2 x2 = __ffma2_rn(gdn_pair(G + r), w2, __fmul2_rn(sp, gp2));
                r1[r] = x1.x, r1[r + 1] = x1.y, r2[r] = x2.x, r2[r + 1] = x2.y;
              }
              float* pw = ppart + ((m * NW + warp) * 2) * DH;
              gdn_warp_colsum<R>(wbuf, r1, pw);
              gdn_warp_colsum<R>(wbuf, r2, pw + DH);
            }
            gdn_axpy_scaled(G, a, kr, gp);  // adjoint to t-1 (Bp'): G = a G + k gp
            // the scalar gradients of alpha and beta: over the row groups, then the warp's columns
            gaP = gdn_group_sum(gaP);
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
              gaP += __shfl_xor_sync(0xffffffffu, gaP, o);
              gbP += __shfl_xor_sync(0xffffffffu, gbP, o);
            }
            if (lane == 0) {
              psc[(m * NW + warp) * 2] = gaP;
              psc[(m * NW + warp) * 2 + 1] = gbP;
            }
          }
        }
        __syncthreads();  // the sub-block's per-warp partial sums are complete
        {  // reduce them over the warps: one float pair of grad_q or grad_k per thread
          const int m = tid / (NT / K), rem = tid % (NT / K), vq = rem / (DH / 2), i2 = (rem % (DH / 2)) * 2;
          if (m < nk) {
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int w2 = 0; w2 < NW; ++w2) {
              const float2 x = *reinterpret_cast<const float2*>(ppart + ((m * NW + w2) * 2 + vq) * DH + i2);
              acc.x += x.x, acc.y += x.y;
            }
            float out[2] = {acc.x, acc.y};
            const float a = fab[m];
            if (vq == 0) {  // grad_q = alpha (S_{t-1} go) + k (w.go)
              const float wg = b_wgo[m];
              out[0] = fmaf(a, out[0], rk_[m * DH + i2] * wg);
              out[1] = fmaf(a, out[1], rk_[m * DH + i2 + 1] * wg);
            }
            const int64_t row = (b * L + t0 + tb + m) * H + h;
            st_vec<T, 2>((vq == 0 ? gq : gk) + row * DH + i2, out);
          }
          if (tid < 2 * nk) {
            const int mm = tid >> 1, which = tid & 1;
            float sum = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < NW; ++w2) sum += psc[(mm * NW + w2) * 2 + which];
            const int64_t row = (b * L + t0 + tb + mm) * H + h;
            (which == 0 ? galpha : gbeta)[row] = from_f<T>(sum);
          }
        }
        if (sb > 0 && tid < 2 * K) b_ab[(bb ^ 1) * 2 * K + tid] = ab;
        __syncthreads();  // the staged buffer is refilled next
      }
    }
    // the adjoint carried past step 0 is the gradient of the initial state
    if (kH0 && gh0 != nullptr)
#pragma unroll
      for (int r = 0; r < R; ++r) gh0[sbase + r * DH] = G[r];
  }
}

// ============================================================================
// Chunkwise (WY) forward, bf16/fp16 inputs, Dh = 64, L a multiple of 128
// ============================================================================
//
// Within a chunk of Q = 128 steps entered with state S0, with gamma_r the
// cumulative decay from the chunk start (gamma_r / gamma_i <= 1 for i <= r):
//   w_r = beta_r (v_r - gamma_r S0^T k_r - sum_{i<r} (gamma_r / gamma_i)(k_r . k_i) w_i),
// i.e. (I + A) W = R with A[r, i] = beta_r (gamma_r / gamma_i) k_r . k_i (i < r)
// and R = diag(beta) (V - diag(gamma) K S0); then
//   S_end = gamma_last S0 + K^T diag(gamma_last / gamma) W
// (docs/DESIGN_gated_deltanet.md:139-270; pinned by oracle/ref_loops.gdn_chunked_forward).
// Given W, a chunk's outputs o_t = S_t^T q_t and its state update are exactly a
// GLA chunk with values W (S_t = gamma_t S0 + sum_{i<=t} (gamma_t/gamma_i) k_i w_i^T),
// so the forward runs in two kernels: this one, sequential over a unit's chunks,
// forms W (the unit triangular solve blocked by 16 rows: a panel update of the
// block's rows from the earlier rows, then a 16-step substitution per column)
// and the states at the checkpoints; the GLA chunk kernel (tcgen05) then
// computes the outputs from (q, k, W, alpha). W also fills the step cache the
// backward replays from. log(alpha) is taken of max(alpha, 1e-30) (an alpha of 0
// resets the state without a 0/0 in the decay ratios); a unit with an alpha above
// 1 (or NaN) is flagged and recomputed by the per-step forward.
namespace gdnc {
constexpr int Q = 128, DH = 64, NT = 256, BLK = 16;
constexpr int KS = DH + 4;   // row stride (floats) of the K, W and state buffers
constexpr int AS = BLK + 4;  // row stride of A's panel, stored transposed [i][row in block]
constexpr int TS2 = BLK + 1; // row stride of the diagonal blocks' inverses [blk][r][c]
constexpr size_t SMEM = (size_t)(2 * Q * KS + DH * KS + Q * AS + Q * TS2 + 6 * Q + 8) * sizeof(float);
}  // namespace gdnc

template <typename T, bool kH0>
__global__ void __launch_bounds__(gdnc::NT, 2)
gdn_wy_state_kernel(const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ alpha,
                    const T* __restrict__ beta, int L, int H, int seg, float* __restrict__ wcache,
                    T* __restrict__ wout, float* __restrict__ ckpt, int* __restrict__ flags,
                    const float* __restrict__ h0) {
  using namespace gdnc;
  extern __shared__ float4 gdnc_smem[];
  float* sK = reinterpret_cast<float*>(gdnc_smem);  // [Q][KS]
  float* sW = sK + Q * KS;                          // [Q][KS]: V, then R, then W
  float* sH = sW + Q * KS;                          // [DH][KS]: the state S[i][j]
  float* sA = sH + DH * KS;                         // [Q][AS]: A's panel [i][row - rb]; first the diagonal blocks
  float* sT = sA + Q * AS;                          // [Q][TS2]: the diagonal blocks' inverses [blk][r][c]
  float* sLg = sT + Q * TS2;                        // [Q] cumulative log decay
  float* sGam = sLg + Q;                            // [Q] gamma_r
  float* sDq = sGam + Q;                            // [Q] gamma_last / gamma_r
  float* sDm = sDq + Q;                             // [Q] gamma_63 / gamma_r (r < 64)
  float* sBeta = sDm + Q;                           // [Q]
  float* sWs = sBeta + Q;                           // [Q] scratch: log alpha, warp totals
  int* sFlag = reinterpret_cast<int*>(sWs + Q);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b = blockIdx.x / H;
  const int h = blockIdx.x % H;
  const int nck = L / Q, nseg = L / seg;

  if (tid == 0) *sFlag = 0;
  for (int e = tid; e < DH * DH; e += NT) {
    const int i = e / DH, j = e % DH;
    sH[i * KS + j] = kH0 ? h0[((b * H + h) * DH + i) * (int64_t)DH + j] : 0.f;
  }
  __syncthreads();

  for (int c = 0; c < nck; ++c) {
    const int64_t row0 = b * L + (int64_t)c * Q;  // [B,L] row of the chunk's first step
    // ---- (a) K, V rows as floats; alpha, beta
#pragma unroll
    for (int m = 0; m < Q * DH / 8 / NT; ++m) {
      const int idx = tid + NT * m, r = idx / 8, c8 = (idx % 8) * 8;
      const int64_t g = ((row0 + r) * H + h) * DH + c8;
      const Vec<T, 8> kv = ld_vec<T, 8>(k + g), vv = ld_vec<T, 8>(v + g);
#pragma unroll
      for (int e = 0; e < 8; e += 4) {
        *reinterpret_cast<float4*>(sK + r * KS + c8 + e) =
            make_float4(to_f(kv.v[e]), to_f(kv.v[e + 1]), to_f(kv.v[e + 2]), to_f(kv.v[e + 3]));
        *reinterpret_cast<float4*>(sW + r * KS + c8 + e) =
            make_float4(to_f(vv.v[e]), to_f(vv.v[e + 1]), to_f(vv.v[e + 2]), to_f(vv.v[e + 3]));
      }
    }
    if (tid < Q) {
      const int64_t g = (row0 + tid) * H + h;
      const float a = to_f(alpha[g]);
      if (!(a <= 1.f)) *sFlag = 1;
      sWs[tid] = logf(fmaxf(a, 1e-30f));
      sBeta[tid] = to_f(beta[g]);
    }
    __syncthreads();
    // ---- (b) cumulative log decay (warps 0-3 scan 32 steps each)
    if (warp < Q / 32) {
      float x = sWs[tid];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += n;
      }
      sLg[tid] = x;
    }
    __syncthreads();
    if (tid < Q) {
      float x = sLg[tid];
      for (int w2 = 0; w2 < tid / 32; ++w2) x += sLg[32 * w2 + 31];
      sWs[tid] = x;  // the scanned values, moved so the warp totals stay readable above
    }
    __syncthreads();
    if (tid < Q) {
      const float lg = sWs[tid];
      sLg[tid] = lg;
      sGam[tid] = expf(lg);
      sDq[tid] = expf(sWs[Q - 1] - lg);
      sDm[tid] = tid < 64 ? expf(sWs[63] - lg) : 0.f;
    }
    __syncthreads();
    // ---- (c) R = diag(beta) (V - diag(gamma) K S0): thread rows 8 rg.., columns 4 jg..
    {
      const int rg = tid / 16, jg = tid % 16;
      float acc[8][4];
#pragma unroll
      for (int rr = 0; rr < 8; ++rr)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[rr][jj] = 0.f;
      for (int i = 0; i < DH; i += 4) {
        float4 hr[4];
#pragma unroll
        for (int ii = 0; ii < 4; ++ii) hr[ii] = *reinterpret_cast<const float4*>(sH + (i + ii) * KS + 4 * jg);
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const float4 kk = *reinterpret_cast<const float4*>(sK + (8 * rg + rr) * KS + i);
          const float kx[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
          for (int ii = 0; ii < 4; ++ii) {
            acc[rr][0] = fmaf(kx[ii], hr[ii].x, acc[rr][0]);
            acc[rr][1] = fmaf(kx[ii], hr[ii].y, acc[rr][1]);
            acc[rr][2] = fmaf(kx[ii], hr[ii].z, acc[rr][2]);
            acc[rr][3] = fmaf(kx[ii], hr[ii].w, acc[rr][3]);
          }
        }
      }
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        const int r = 8 * rg + rr;
        const float bt = sBeta[r], gm = sGam[r];
        float4* wr = reinterpret_cast<float4*>(sW + r * KS + 4 * jg);
        const float4 vv = *wr;
        *wr = make_float4(bt * fmaf(-gm, acc[rr][0], vv.x), bt * fmaf(-gm, acc[rr][1], vv.y),
                          bt * fmaf(-gm, acc[rr][2], vv.z), bt * fmaf(-gm, acc[rr][3], vv.w));
      }
    }
    __syncthreads();
    // ---- (d) the unit lower triangular solve (I + A) W = R by blocks of 16 rows:
    // the diagonal blocks' inverses T_b = (I + A_bb)^-1 first (they need only K,
    // alpha, beta), then per block W_b = T_b (R_b - A_b,<b W_<b), two parallel products.
    // (d0) the eight diagonal blocks of A, [blk][r][i] in sA, 4 x 4 tiles
    if (tid < 8 * 16) {
      const int bb = tid / 16, rg = (tid % 16) % 4, ig = (tid % 16) / 4, rb = BLK * bb;
      float acc[4][4];
#pragma unroll
      for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
        for (int b2 = 0; b2 < 4; ++b2) acc[a2][b2] = 0.f;
      for (int d = 0; d < DH; d += 4) {
        float4 kr[4], ki[4];
#pragma unroll
        for (int a2 = 0; a2 < 4; ++a2) {
          kr[a2] = *reinterpret_cast<const float4*>(sK + (rb + 4 * rg + a2) * KS + d);
          ki[a2] = *reinterpret_cast<const float4*>(sK + (rb + 4 * ig + a2) * KS + d);
        }
#pragma unroll
        for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
          for (int b2 = 0; b2 < 4; ++b2)
            acc[a2][b2] = fmaf(kr[a2].x, ki[b2].x, fmaf(kr[a2].y, ki[b2].y,
                          fmaf(kr[a2].z, ki[b2].z, fmaf(kr[a2].w, ki[b2].w, acc[a2][b2]))));
      }
#pragma unroll
      for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
        for (int b2 = 0; b2 < 4; ++b2) {
          const int r = rb + 4 * rg + a2, i = rb + 4 * ig + b2;
          sA[(bb * BLK + 4 * rg + a2) * BLK + 4 * ig + b2] =
              i < r ? sBeta[r] * expf(sLg[r] - sLg[i]) * acc[a2][b2] : 0.f;
        }
    }
    __syncthreads();
    // (d0') column c of T_b by forward substitution, all blocks at once
    if (tid < 8 * 16) {
      const int bb = tid / 16, cc = tid % 16;
      const float* Ab = sA + bb * BLK * BLK;
      float x[BLK];
#pragma unroll
      for (int r = 0; r < BLK; ++r) {
        float v = r == cc ? 1.f : 0.f;
#pragma unroll
        for (int i = 0; i < r; ++i) v = fmaf(-Ab[r * BLK + i], x[i], v);
        x[r] = r < cc ? 0.f : v;
      }
#pragma unroll
      for (int r = 0; r < BLK; ++r) sT[(bb * BLK + r) * TS2 + cc] = x[r];
    }
    __syncthreads();
    for (int blk = 0; blk < Q / BLK; ++blk) {
      const int rb = BLK * blk;
      if (rb > 0) {
        // (d1) the panel A[rb.., 0..rb), stored transposed sA[i][row - rb]: 2 x 4 tiles
        if (tid < 2 * rb) {
          const int rg = tid % 8, ig = tid / 8;
          float acc[2][4];
#pragma unroll
          for (int a2 = 0; a2 < 2; ++a2)
#pragma unroll
            for (int b2 = 0; b2 < 4; ++b2) acc[a2][b2] = 0.f;
          for (int d = 0; d < DH; d += 4) {
            float4 kr[2], ki[4];
#pragma unroll
            for (int a2 = 0; a2 < 2; ++a2) kr[a2] = *reinterpret_cast<const float4*>(sK + (rb + 2 * rg + a2) * KS + d);
#pragma unroll
            for (int b2 = 0; b2 < 4; ++b2) ki[b2] = *reinterpret_cast<const float4*>(sK + (4 * ig + b2) * KS + d);
#pragma unroll
            for (int a2 = 0; a2 < 2; ++a2)
#pragma unroll
              for (int b2 = 0; b2 < 4; ++b2)
                acc[a2][b2] = fmaf(kr[a2].x, ki[b2].x, fmaf(kr[a2].y, ki[b2].y,
                              fmaf(kr[a2].z, ki[b2].z, fmaf(kr[a2].w, ki[b2].w, acc[a2][b2]))));
          }
#pragma unroll
          for (int b2 = 0; b2 < 4; ++b2) {
            const int i = 4 * ig + b2;
            const int r0 = rb + 2 * rg;
            *reinterpret_cast<float2*>(sA + i * AS + 2 * rg) =
                make_float2(sBeta[r0] * expf(sLg[r0] - sLg[i]) * acc[0][b2],
                            sBeta[r0 + 1] * expf(sLg[r0 + 1] - sLg[i]) * acc[1][b2]);
          }
        }
        __syncthreads();
        // (d2) R_b -= A_b,<b W_<b: 4 x 4 tiles, the rb earlier rows split over four
        // thread groups (lanes 8 and 16 apart) whose partial tiles are summed by shuffles
        {
          const int tile = (tid & 7) | ((tid >> 5) << 3), part = (lane >> 3) & 3;
          const int rg = tile % 4, jg = tile / 4, q4 = rb / 4;
          float acc[4][4];
#pragma unroll
          for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
            for (int b2 = 0; b2 < 4; ++b2) acc[a2][b2] = 0.f;
          for (int i = part * q4; i < (part + 1) * q4; ++i) {
            const float4 a = *reinterpret_cast<const float4*>(sA + i * AS + 4 * rg);
            const float4 w = *reinterpret_cast<const float4*>(sW + i * KS + 4 * jg);
            const float ax[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int a2 = 0; a2 < 4; ++a2) {
              acc[a2][0] = fmaf(ax[a2], w.x, acc[a2][0]);
              acc[a2][1] = fmaf(ax[a2], w.y, acc[a2][1]);
              acc[a2][2] = fmaf(ax[a2], w.z, acc[a2][2]);
              acc[a2][3] = fmaf(ax[a2], w.w, acc[a2][3]);
            }
          }
#pragma unroll
          for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
            for (int b2 = 0; b2 < 4; ++b2) {
              acc[a2][b2] += __shfl_xor_sync(0xffffffffu, acc[a2][b2], 8);
              acc[a2][b2] += __shfl_xor_sync(0xffffffffu, acc[a2][b2], 16);
            }
          if (part == 0) {
#pragma unroll
            for (int a2 = 0; a2 < 4; ++a2) {
              float4* rw = reinterpret_cast<float4*>(sW + (rb + 4 * rg + a2) * KS + 4 * jg);
              const float4 x = *rw;
              *rw = make_float4(x.x - acc[a2][0], x.y - acc[a2][1], x.z - acc[a2][2], x.w - acc[a2][3]);
            }
          }
        }
        __syncthreads();
      }
      // (d3) W_b = T_b R_b: one row and 4 columns per thread. The 16 threads of a
      // column group (the only ones that read and write the same words) form one
      // half-warp, so a warp barrier orders their reads of R_b before the writes.
      {
        const int rr = tid % 16, j4 = 4 * (tid / 16);
        const float* Tr = sT + (blk * BLK + rr) * TS2;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int cc = 0; cc < BLK; ++cc) {
          const float t = Tr[cc];
          const float4 x = *reinterpret_cast<const float4*>(sW + (rb + cc) * KS + j4);
          acc.x = fmaf(t, x.x, acc.x), acc.y = fmaf(t, x.y, acc.y), acc.z = fmaf(t, x.z, acc.z),
          acc.w = fmaf(t, x.w, acc.w);
        }
        __syncwarp();  // the half-warp has read its columns of R_b before they become W_b
        *reinterpret_cast<float4*>(sW + (rb + rr) * KS + j4) = acc;
      }
      // the next block's panel (d1) reads only K; its update (d2) reads this W after d1's barrier
    }
    __syncthreads();
    // ---- (e) W out: the step cache (float32) and the GLA kernel's values (T)
#pragma unroll
    for (int m = 0; m < Q * DH / 4 / NT; ++m) {
      const int idx = tid + NT * m, r = idx / 16, j4 = 4 * (idx % 16);
      const float4 w = *reinterpret_cast<const float4*>(sW + r * KS + j4);
      const int64_t g = ((row0 + r) * H + h) * DH + j4;
      if (wcache != nullptr) *reinterpret_cast<float4*>(wcache + g) = w;
      const float f[4] = {w.x, w.y, w.z, w.w};
      st_vec<T, 4>(wout + g, f);
    }
    // ---- (f) the state at the chunk's middle and end: thread rows 4 ig.., columns 4 jg..
    {
      const int ig = tid / 16, jg = tid % 16;
      float acc[4][4];
#pragma unroll
      for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
        for (int b2 = 0; b2 < 4; ++b2) acc[a2][b2] = 0.f;
      auto accumulate = [&](int r0, int r1, const float* scale) {
        for (int r = r0; r < r1; ++r) {
          const float sc = scale[r];
          const float4 kk = *reinterpret_cast<const float4*>(sK + r * KS + 4 * ig);
          const float4 ww = *reinterpret_cast<const float4*>(sW + r * KS + 4 * jg);
          const float kx[4] = {kk.x * sc, kk.y * sc, kk.z * sc, kk.w * sc};
#pragma unroll
          for (int a2 = 0; a2 < 4; ++a2) {
            acc[a2][0] = fmaf(kx[a2], ww.x, acc[a2][0]);
            acc[a2][1] = fmaf(kx[a2], ww.y, acc[a2][1]);
            acc[a2][2] = fmaf(kx[a2], ww.z, acc[a2][2]);
            acc[a2][3] = fmaf(kx[a2], ww.w, acc[a2][3]);
          }
        }
      };
      float hs[4][4];
      // middle: S_63 = gamma_63 S0 + sum_{r<64} (gamma_63/gamma_r) k_r w_r^T
      accumulate(0, Q / 2, sDm);
      const float g63 = sGam[Q / 2 - 1];
#pragma unroll
      for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
        for (int b2 = 0; b2 < 4; ++b2) hs[a2][b2] = fmaf(g63, sH[(4 * ig + a2) * KS + 4 * jg + b2], acc[a2][b2]);
      const int64_t tmid = (int64_t)c * Q + Q / 2;
      if (tmid % seg == 0) {
        float* ck = ckpt + ((b * nseg + tmid / seg - 1) * H + h) * (int64_t)DH * DH;
#pragma unroll
        for (int a2 = 0; a2 < 4; ++a2)
          *reinterpret_cast<float4*>(ck + (4 * ig + a2) * DH + 4 * jg) =
              make_float4(hs[a2][0], hs[a2][1], hs[a2][2], hs[a2][3]);
      }
      // end: S_127 = (gamma_127 / gamma_63) S_63 + sum_{r>=64} (gamma_127/gamma_r) k_r w_r^T
#pragma unroll
      for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
        for (int b2 = 0; b2 < 4; ++b2) acc[a2][b2] = 0.f;
      accumulate(Q / 2, Q, sDq);
      const float gq = sDq[Q / 2 - 1];  // gamma_127 / gamma_63
#pragma unroll
      for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
        for (int b2 = 0; b2 < 4; ++b2) {
          const float x = fmaf(gq, hs[a2][b2], acc[a2][b2]);
          hs[a2][b2] = x;
          sH[(4 * ig + a2) * KS + 4 * jg + b2] = x;  // this thread's own tile of the state
        }
      const int64_t tend = (int64_t)(c + 1) * Q;
      if (tend % seg == 0) {
        float* ck = ckpt + ((b * nseg + tend / seg - 1) * H + h) * (int64_t)DH * DH;
#pragma unroll
        for (int a2 = 0; a2 < 4; ++a2)
          *reinterpret_cast<float4*>(ck + (4 * ig + a2) * DH + 4 * jg) =
              make_float4(hs[a2][0], hs[a2][1], hs[a2][2], hs[a2][3]);
      }
    }
    __syncthreads();  // the next chunk overwrites K, W and the scalars
  }
  if (tid == 0) flags[blockIdx.x] = *sFlag;
}

// One-token decode step on a float32 state cache [B,H,Dh,Dh] (the final
// state's layout), advanced in place; y [B,H,Dh] float32. One step of the
// forward's recurrence, same layout (one CTA per (b, h)).
template <typename T, int DH>
__global__ void __launch_bounds__(DH * 4)
gdn_step_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                const T* __restrict__ alpha, const T* __restrict__ beta, float* __restrict__ state,
                float* __restrict__ y) {
  constexpr int R = DH / 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 3, j = warp * 8 + (lane & 7), i0 = g * R;
  const int64_t u = blockIdx.x;  // (b, h): one row of q, k, v and one alpha, beta
  float* sp = state + (u * DH + i0) * (int64_t)DH + j;
  float S[R], kr[R], qr[R];
#pragma unroll
  for (int r = 0; r < R; ++r) S[r] = sp[r * DH];
  gdn_load_rows<T, R>(k + u * DH + i0, kr);
  gdn_load_rows<T, R>(q + u * DH + i0, qr);
  const float vj = to_f(v[u * DH + j]), a = to_f(alpha[u]), bt = to_f(beta[u]);
  const float p = gdn_group_sum(gdn_dot(kr, S));
  const float sq = gdn_group_sum(gdn_dot(qr, S));
  const float kq = gdn_group_sum(gdn_dot(kr, qr));
  const float w = bt * fmaf(-a, p, vj);
  if (g == 0) y[u * DH + j] = fmaf(a, sq, kq * w);
  gdn_update(S, kr, a, w);
#pragma unroll
  for (int r = 0; r < R; ++r) sp[r * DH] = S[r];
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
                      int64_t H, int64_t seg, float* y, float* ckpt, float* wp, const float* h0, cudaStream_t st,
                      const int* only = nullptr) {
  const dim3 grid((unsigned)(batch * H));
  auto kern = h0 != nullptr ? gdn_fwd_kernel<T, DH, true> : gdn_fwd_kernel<T, DH, false>;
  kern<<<grid, DH * GdnFwdP<DH>::v, 0, st>>>(q, k, v, al, be, (int)L, (int)H, (int)seg, y, ckpt, wp, h0, only);
  return check_launch("gdn_fwd_kernel");
}

static size_t gdn_align(size_t n) { return (n + 255) / 256 * 256; }

// The chunkwise forward: 2-byte inputs, Dh = 64, L a multiple of the chunk,
// checkpoints at multiples of half a chunk, and fewer units than two per SM.
// Measured on B200 (L=2048, Dh=64, bf16; chunkwise against per step): 128 units
// 0.63 against 0.80 ms, 256 units 0.99 against 1.03, 512 units 1.95 against 1.83,
// 1024 units 3.50 against 3.15: with few units the chunk form's shorter per-unit
// path wins; from about two units per SM the per-step kernel (four CTAs per SM)
// keeps the SMs as busy and needs no second pass.
static bool gdn_chunked_ok(int elem_bytes, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return elem_bytes == 2 && Dh == gdnc::DH && L % gdnc::Q == 0 && seg % (gdnc::Q / 2) == 0 &&
         L <= (int64_t)INT32_MAX / 2 && batch * H < 2 * (int64_t)sms;
}

// workspace of the chunkwise forward: W as T [B,L,H,64], the GLA kernel's one
// checkpoint [B,1,H,64,64] float32, a flag per unit; 0 when the per-step forward runs
size_t gdn_fwd_ws_bytes(int elem_bytes, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg) {
  if (!gdn_chunked_ok(elem_bytes, batch, L, H, Dh, seg)) return 0;
  return gdn_align((size_t)batch * L * H * Dh * elem_bytes) + gdn_align((size_t)batch * H * Dh * Dh * 4) +
         gdn_align((size_t)batch * H * 4);
}

template <typename T>
int gdn_fwd_launch(const void* q, const void* k, const void* v, const void* alpha, const void* beta, int64_t batch,
                   int64_t L, int64_t H, int64_t Dh, int64_t seg, float* y, float* ckpt, float* wp,
                   const float* h0, void* ws, size_t ws_bytes, cudaStream_t st) {
  const T *q_ = (const T*)q, *k_ = (const T*)k, *v_ = (const T*)v, *a_ = (const T*)alpha, *b_ = (const T*)beta;
  const size_t need = gdn_fwd_ws_bytes((int)sizeof(T), batch, L, H, Dh, seg);
  if (need > 0 && ws != nullptr && ws_bytes >= need) {
    T* wbf = (T*)ws;
    float* gck = (float*)((char*)ws + gdn_align((size_t)batch * L * H * Dh * sizeof(T)));
    int* flags = (int*)((char*)gck + gdn_align((size_t)batch * H * Dh * Dh * 4));
    auto kern = h0 != nullptr ? gdn_wy_state_kernel<T, true> : gdn_wy_state_kernel<T, false>;
    if (int rc = gdn_set_smem(kern, gdnc::SMEM)) return rc;
    kern<<<(unsigned)(batch * H), gdnc::NT, gdnc::SMEM, st>>>(k_, v_, a_, b_, (int)L, (int)H, (int)seg, wp, wbf,
                                                              ckpt, flags, h0);
    if (int rc = check_launch("gdn_wy_state_kernel")) return rc;
    // the outputs: a GLA chunk with values W (its one checkpoint is scratch)
    const int code = sizeof(T) == 2 && std::is_same_v<T, __half> ? MR_F16 : MR_BF16;
    if (int rc = mr_gla_fwd_h0(q, k, wbf, alpha, code, batch, L, H, Dh, L, y, gck, h0, st)) return rc;
    // units with an alpha above 1: the per-step forward, for them only
    return gdn_fwd_dh<T, 64>(q_, k_, v_, a_, b_, batch, L, H, seg, y, ckpt, wp, h0, st, flags);
  }
  if (Dh == 32) return gdn_fwd_dh<T, 32>(q_, k_, v_, a_, b_, batch, L, H, seg, y, ckpt, wp, h0, st);
  return gdn_fwd_dh<T, 64>(q_, k_, v_, a_, b_, batch, L, H, seg, y, ckpt, wp, h0, st);
}

static int64_t gdn_bwd_grid(int64_t batch, int64_t H, int64_t Dh, int64_t seg) {
  const int64_t units = batch * H;
  const int64_t per_cta = gdn_scratch_floats(Dh, seg) * (int64_t)sizeof(float);
  int64_t grid = units < kGdnMaxCtas ? units : kGdnMaxCtas;
  const int64_t cap = kGdnScratchBudget / per_cta;
  if (grid > cap) grid = cap > 0 ? cap : 1;
  return grid;
}

size_t gdn_bwd_ws_bytes(int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg) {
  (void)L;
  return (size_t)gdn_bwd_grid(batch, H, Dh, seg) * gdn_scratch_floats(Dh, seg) * sizeof(float);
}

template <typename T, int DH>
static int gdn_bwd_dh(const float* gy, const float* gf, const float* ckpt, const float* wp, const T* q, const T* k, const T* v,
                      const T* al, const T* be, int64_t batch, int64_t L, int64_t H, int64_t seg, T* gq, T* gk,
                      T* gv, T* ga, T* gb, float* ws, const float* h0, float* gh0, cudaStream_t st) {
  constexpr size_t sm = GdnBwdSmem<T, DH>::bytes;
  auto kern = h0 != nullptr ? gdn_bwd_kernel<T, DH, true> : gdn_bwd_kernel<T, DH, false>;
  if (int rc = gdn_set_smem(kern, sm)) return rc;
  const dim3 grid((unsigned)gdn_bwd_grid(batch, H, DH, seg));
  kern<<<grid, DH * 4, sm, st>>>(gy, gf, ckpt, wp, q, k, v, al, be, (int)L, (int)H, (int)seg, (int)(batch * H), gq, gk,
                                 gv, ga, gb, ws, h0, gh0);
  return check_launch("gdn_bwd_kernel");
}

template <typename T>
int gdn_bwd_launch(const float* gy, const float* gf, const float* ckpt, const float* wp, const void* q, const void* k, const void* v,
                   const void* alpha, const void* beta, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg,
                   void* gq, void* gk, void* gv, void* galpha, void* gbeta, void* ws, const float* h0, float* gh0,
                   cudaStream_t st) {
  const T *q_ = (const T*)q, *k_ = (const T*)k, *v_ = (const T*)v, *a_ = (const T*)alpha, *b_ = (const T*)beta;
  T *gq_ = (T*)gq, *gk_ = (T*)gk, *gv_ = (T*)gv, *ga_ = (T*)galpha, *gb_ = (T*)gbeta;
  if (Dh == 32)
    return gdn_bwd_dh<T, 32>(gy, gf, ckpt, wp, q_, k_, v_, a_, b_, batch, L, H, seg, gq_, gk_, gv_, ga_, gb_,
                             (float*)ws, h0, gh0, st);
  return gdn_bwd_dh<T, 64>(gy, gf, ckpt, wp, q_, k_, v_, a_, b_, batch, L, H, seg, gq_, gk_, gv_, ga_, gb_, (float*)ws,
                           h0, gh0, st);
}

template <typename T>
int gdn_step_launch(const void* q, const void* k, const void* v, const void* alpha, const void* beta, int64_t batch,
                    int64_t H, int64_t Dh, float* state, float* y, cudaStream_t st) {
  const T *q_ = (const T*)q, *k_ = (const T*)k, *v_ = (const T*)v, *a_ = (const T*)alpha, *b_ = (const T*)beta;
  const dim3 grid((unsigned)(batch * H));
  if (Dh == 32)
    gdn_step_kernel<T, 32><<<grid, 128, 0, st>>>(q_, k_, v_, a_, b_, state, y);
  else
    gdn_step_kernel<T, 64><<<grid, 256, 0, st>>>(q_, k_, v_, a_, b_, state, y);
  return check_launch("gdn_step_kernel");
}

#define MR_INST(T)                                                                                              \
  template int gdn_step_launch<T>(const void*, const void*, const void*, const void*, const void*, int64_t,    \
                                  int64_t, int64_t, float*, float*, cudaStream_t);                             \
  template int gdn_fwd_launch<T>(const void*, const void*, const void*, const void*, const void*, int64_t,     \
                                 int64_t, int64_t, int64_t, int64_t, float*, float*, float*, const float*,     \
                                 void*, size_t, cudaStream_t);                                                \
  template int gdn_bwd_launch<T>(const float*, const float*, const float*, const float*, const void*,          \
                                 const void*,                                                                 \
                                 const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t,    \
                                 int64_t, void*, void*, void*, void*, void*, void*, const float*, float*,      \
                                 cudaStream_t);
MR_INST(float)
MR_INST(__nv_bfloat16)
MR_INST(__half)
#undef MR_INST

}  // namespace mr
