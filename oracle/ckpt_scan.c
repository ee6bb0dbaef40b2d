/*
 * CPU oracle (test infrastructure only): float32 C restatement of the
 * reference's checkpoint + recompute scans, used as the timed CPU baseline
 * (bench.py --impl reference and the cpu_baseline field) and as a fast
 * checker at sizes the float64 numpy oracle cannot reach. The library never
 * links or calls it.
 *
 * Algorithm and operation order follow the reference's Metal bodies:
 *   SSD    forward mlx_recurrence/ssd.py:85-111, backward ssd.py:174-268
 *   GLA    forward gla.py:78-100,  backward gla.py:158-235
 *   RG-LRU forward rglru.py:88-100, backward rglru.py:147-180
 *   rotLRU forward rotlru.py:93-124, backward rotlru.py:166-237
 *   Gated DeltaNet (a design only in the reference) docs/DESIGN_gated_deltanet.md
 *          sections 1 and 4
 * One OpenMP task per independent unit ((b,h) for SSD/GLA, b for the
 * diagonal scans, whose channels are looped inside). Cross-lane simd_sum
 * reductions become plain loops over the lane axis. The state at every
 * step of a segment is recomputed from the segment's checkpoint into a
 * per-unit scratch buffer, as in the reference. Optional final-state
 * cotangents (NULL allowed) seed the adjoint.
 *
 * Build: see oracle/build_oracle.py (gcc -O3 -fopenmp -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef int64_t i64;

/* ------------------------------------------------------------------ SSD -- */
void orc_ssd_fwd(const float* u, const float* delta, const float* Bm, const float* Cm,
                 const float* A, i64 Bt, i64 L, i64 H, i64 Dh, i64 N, i64 seg, float* y,
                 float* ckpt) {
  const i64 nseg = L / seg;
#pragma omp parallel for schedule(dynamic, 1)
  for (i64 bh = 0; bh < Bt * H; ++bh) {
    const i64 b = bh / H, h = bh % H;
    float* st = (float*)calloc((size_t)(Dh * N), sizeof(float));
    float* dec = (float*)malloc((size_t)N * sizeof(float));
    for (i64 t = 0; t < L; ++t) {
      const i64 row = (b * L + t) * H + h;
      const float dt = delta[row];
      for (i64 n = 0; n < N; ++n) dec[n] = expf(dt * A[h * N + n]);
      for (i64 d = 0; d < Dh; ++d) {
        const float uv = u[row * Dh + d];
        float yv = 0.f;
        float* s = st + d * N;
        for (i64 n = 0; n < N; ++n) {
          s[n] = dec[n] * s[n] + dt * Bm[row * N + n] * uv;
          yv += s[n] * Cm[row * N + n];
        }
        y[row * Dh + d] = yv;
      }
      if ((t + 1) % seg == 0) {
        float* ck = ckpt + ((b * nseg + t / seg) * H + h) * N * Dh;
        for (i64 d = 0; d < Dh; ++d)
          for (i64 n = 0; n < N; ++n) ck[n * Dh + d] = st[d * N + n];
      }
    }
    free(st);
    free(dec);
  }
}

/* grad_A_part: [Bt, H, N] per-batch partials (the caller sums over b). */
void orc_ssd_bwd(const float* gy, const float* gfinal, const float* ckpt, const float* u,
                 const float* delta, const float* Bm, const float* Cm, const float* A, i64 Bt,
                 i64 L, i64 H, i64 Dh, i64 N, i64 seg, float* gu, float* gdelta, float* gB,
                 float* gC, float* gA_part) {
  const i64 nseg = L / seg;
#pragma omp parallel for schedule(dynamic, 1)
  for (i64 bh = 0; bh < Bt * H; ++bh) {
    const i64 b = bh / H, h = bh % H;
    const i64 S = Dh * N;
    float* adj = (float*)calloc((size_t)S, sizeof(float));
    float* gA = (float*)calloc((size_t)N, sizeof(float));
    float* scr = (float*)malloc((size_t)((seg + 1) * S) * sizeof(float));
    float* dec = (float*)malloc((size_t)N * sizeof(float));
    if (gfinal)
      for (i64 i = 0; i < S; ++i) adj[i] = gfinal[bh * S + i]; /* [B,H,Dh,N] */
    for (i64 s = nseg - 1; s >= 0; --s) {
      float* st = scr; /* scr[tl] = state after step tl-1; scr[0] = segment start */
      if (s > 0) {
        const float* ck = ckpt + ((b * nseg + s - 1) * H + h) * N * Dh;
        for (i64 d = 0; d < Dh; ++d)
          for (i64 n = 0; n < N; ++n) st[d * N + n] = ck[n * Dh + d];
      } else {
        memset(st, 0, (size_t)S * sizeof(float));
      }
      for (i64 tl = 0; tl < seg; ++tl) {
        const i64 row = (b * L + s * seg + tl) * H + h;
        const float dt = delta[row];
        for (i64 n = 0; n < N; ++n) dec[n] = expf(dt * A[h * N + n]);
        const float* prev = scr + tl * S;
        float* cur = scr + (tl + 1) * S;
        for (i64 d = 0; d < Dh; ++d) {
          const float uv = u[row * Dh + d];
          for (i64 n = 0; n < N; ++n)
            cur[d * N + n] = dec[n] * prev[d * N + n] + dt * Bm[row * N + n] * uv;
        }
      }
      for (i64 tl = seg - 1; tl >= 0; --tl) {
        const i64 row = (b * L + s * seg + tl) * H + h;
        const float dt = delta[row];
        for (i64 n = 0; n < N; ++n) dec[n] = expf(dt * A[h * N + n]);
        const float* hc = scr + (tl + 1) * S;
        const float* hp = scr + tl * S;
        float gdt = 0.f;
        for (i64 n = 0; n < N; ++n) {
          gB[row * N + n] = 0.f;
          gC[row * N + n] = 0.f;
        }
        for (i64 d = 0; d < Dh; ++d) {
          const float uv = u[row * Dh + d];
          const float g = gy[row * Dh + d];
          float gud = 0.f;
          for (i64 n = 0; n < N; ++n) {
            const i64 i = d * N + n;
            const float bv = Bm[row * N + n], cv = Cm[row * N + n], a = A[h * N + n];
            adj[i] += g * cv;
            gud += adj[i] * dt * bv;
            gdt += adj[i] * (a * dec[n] * hp[i] + bv * uv);
            gA[n] += adj[i] * dt * dec[n] * hp[i];
            gB[row * N + n] += adj[i] * dt * uv;
            gC[row * N + n] += hc[i] * g;
            adj[i] *= dec[n];
          }
          gu[row * Dh + d] = gud;
        }
        gdelta[row] = gdt;
      }
    }
    for (i64 n = 0; n < N; ++n) gA_part[bh * N + n] = gA[n];
    free(adj);
    free(gA);
    free(scr);
    free(dec);
  }
}

/* ------------------------------------------------------------------ GLA -- */
void orc_gla_fwd(const float* q, const float* k, const float* v, const float* gates, i64 Bt,
                 i64 L, i64 H, i64 Dh, i64 seg, float* y, float* ckpt) {
  const i64 nseg = L / seg;
#pragma omp parallel for schedule(dynamic, 1)
  for (i64 bh = 0; bh < Bt * H; ++bh) {
    const i64 b = bh / H, h = bh % H;
    float* S = (float*)calloc((size_t)(Dh * Dh), sizeof(float)); /* [i][j] */
    for (i64 t = 0; t < L; ++t) {
      const i64 row = (b * L + t) * H + h;
      const float g = gates[row];
      const float* kr = k + row * Dh;
      const float* qr = q + row * Dh;
      const float* vr = v + row * Dh;
      float* yr = y + row * Dh;
      for (i64 j = 0; j < Dh; ++j) yr[j] = 0.f;
      for (i64 i = 0; i < Dh; ++i)
        for (i64 j = 0; j < Dh; ++j) {
          S[i * Dh + j] = g * S[i * Dh + j] + kr[i] * vr[j];
          yr[j] += qr[i] * S[i * Dh + j];
        }
      if ((t + 1) % seg == 0)
        memcpy(ckpt + ((b * nseg + t / seg) * H + h) * Dh * Dh, S, (size_t)(Dh * Dh) * sizeof(float));
    }
    free(S);
  }
}

void orc_gla_bwd(const float* gy, const float* gfinal, const float* ckpt, const float* q,
                 const float* k, const float* v, const float* gates, i64 Bt, i64 L, i64 H, i64 Dh,
                 i64 seg, float* gq, float* gk, float* gv, float* gg) {
  const i64 nseg = L / seg;
#pragma omp parallel for schedule(dynamic, 1)
  for (i64 bh = 0; bh < Bt * H; ++bh) {
    const i64 b = bh / H, h = bh % H;
    const i64 S2 = Dh * Dh;
    float* adj = (float*)calloc((size_t)S2, sizeof(float));
    float* scr = (float*)malloc((size_t)((seg + 1) * S2) * sizeof(float));
    if (gfinal)
      for (i64 i = 0; i < S2; ++i) adj[i] = gfinal[bh * S2 + i];
    for (i64 s = nseg - 1; s >= 0; --s) {
      if (s > 0)
        memcpy(scr, ckpt + ((b * nseg + s - 1) * H + h) * S2, (size_t)S2 * sizeof(float));
      else
        memset(scr, 0, (size_t)S2 * sizeof(float));
      for (i64 tl = 0; tl < seg; ++tl) {
        const i64 row = (b * L + s * seg + tl) * H + h;
        const float g = gates[row];
        const float* prev = scr + tl * S2;
        float* cur = scr + (tl + 1) * S2;
        for (i64 i = 0; i < Dh; ++i)
          for (i64 j = 0; j < Dh; ++j)
            cur[i * Dh + j] = g * prev[i * Dh + j] + k[row * Dh + i] * v[row * Dh + j];
      }
      for (i64 tl = seg - 1; tl >= 0; --tl) {
        const i64 row = (b * L + s * seg + tl) * H + h;
        const float g = gates[row];
        const float* hc = scr + (tl + 1) * S2;
        const float* hp = scr + tl * S2;
        const float* qr = q + row * Dh;
        const float* kr = k + row * Dh;
        const float* vr = v + row * Dh;
        const float* go = gy + row * Dh;
        float ggs = 0.f;
        for (i64 x = 0; x < Dh; ++x) {
          gv[row * Dh + x] = 0.f;
          gq[row * Dh + x] = 0.f;
          gk[row * Dh + x] = 0.f;
        }
        for (i64 i = 0; i < Dh; ++i)
          for (i64 j = 0; j < Dh; ++j) {
            const i64 e = i * Dh + j;
            adj[e] += qr[i] * go[j];
            gv[row * Dh + j] += adj[e] * kr[i];
            ggs += adj[e] * hp[e];
            gq[row * Dh + i] += go[j] * hc[e];
            gk[row * Dh + i] += adj[e] * vr[j];
            adj[e] *= g;
          }
        gg[row] = ggs;
      }
    }
    free(adj);
    free(scr);
  }
}

/* --------------------------------------------------------------- RG-LRU -- */
void orc_rglru_fwd(const float* a, const float* x, i64 Bt, i64 L, i64 D, i64 seg, float* y,
                   float* ckpt) {
  const i64 nseg = L / seg;
#pragma omp parallel for schedule(static)
  for (i64 b = 0; b < Bt; ++b) {
    float* h = (float*)calloc((size_t)D, sizeof(float));
    for (i64 t = 0; t < L; ++t) {
      const i64 o = (b * L + t) * D;
      for (i64 d = 0; d < D; ++d) {
        h[d] = a[o + d] * h[d] + x[o + d];
        y[o + d] = h[d];
      }
      if ((t + 1) % seg == 0) memcpy(ckpt + (b * nseg + t / seg) * D, h, (size_t)D * sizeof(float));
    }
    free(h);
  }
}

void orc_rglru_bwd(const float* gy, const float* gfinal, const float* ckpt, const float* a,
                   const float* x, i64 Bt, i64 L, i64 D, i64 seg, float* ga, float* gx) {
  const i64 nseg = L / seg;
#pragma omp parallel for schedule(static)
  for (i64 b = 0; b < Bt; ++b) {
    float* adj = (float*)calloc((size_t)D, sizeof(float));
    float* hs = (float*)malloc((size_t)((seg + 1) * D) * sizeof(float));
    if (gfinal) memcpy(adj, gfinal + b * D, (size_t)D * sizeof(float));
    for (i64 s = nseg - 1; s >= 0; --s) {
      if (s > 0)
        memcpy(hs, ckpt + (b * nseg + s - 1) * D, (size_t)D * sizeof(float));
      else
        memset(hs, 0, (size_t)D * sizeof(float));
      for (i64 tl = 0; tl < seg; ++tl) {
        const i64 o = (b * L + s * seg + tl) * D;
        for (i64 d = 0; d < D; ++d) hs[(tl + 1) * D + d] = a[o + d] * hs[tl * D + d] + x[o + d];
      }
      for (i64 tl = seg - 1; tl >= 0; --tl) {
        const i64 o = (b * L + s * seg + tl) * D;
        for (i64 d = 0; d < D; ++d) {
          adj[d] += gy[o + d];
          gx[o + d] = adj[d];
          ga[o + d] = adj[d] * hs[tl * D + d];
          adj[d] *= a[o + d];
        }
      }
    }
    free(adj);
    free(hs);
  }
}

/* --------------------------------------------------------------- rotLRU -- */
void orc_rotlru_fwd(const float* a, const float* cs, const float* sn, const float* x, i64 Bt,
                    i64 L, i64 Dp, i64 seg, float* y, float* ckpt) {
  const i64 nseg = L / seg, D = 2 * Dp;
#pragma omp parallel for schedule(static)
  for (i64 b = 0; b < Bt; ++b) {
    float* st = (float*)calloc((size_t)D, sizeof(float));
    for (i64 t = 0; t < L; ++t) {
      const i64 op = (b * L + t) * Dp, ox = (b * L + t) * D;
      for (i64 p = 0; p < Dp; ++p) {
        const float av = a[op + p], c = cs[op + p], s = sn[op + p];
        const float u = st[2 * p], w = st[2 * p + 1];
        const float un = av * (c * u - s * w) + x[ox + 2 * p];
        const float wn = av * (s * u + c * w) + x[ox + 2 * p + 1];
        st[2 * p] = un;
        st[2 * p + 1] = wn;
        y[ox + 2 * p] = un;
        y[ox + 2 * p + 1] = wn;
      }
      if ((t + 1) % seg == 0) memcpy(ckpt + (b * nseg + t / seg) * D, st, (size_t)D * sizeof(float));
    }
    free(st);
  }
}

void orc_rotlru_bwd(const float* gy, const float* gfinal, const float* ckpt, const float* a,
                    const float* cs, const float* sn, const float* x, i64 Bt, i64 L, i64 Dp,
                    i64 seg, float* ga, float* gcs, float* gsn, float* gx) {
  const i64 nseg = L / seg, D = 2 * Dp;
#pragma omp parallel for schedule(static)
  for (i64 b = 0; b < Bt; ++b) {
    float* adj = (float*)calloc((size_t)D, sizeof(float));
    float* hs = (float*)malloc((size_t)((seg + 1) * D) * sizeof(float));
    if (gfinal) memcpy(adj, gfinal + b * D, (size_t)D * sizeof(float));
    for (i64 s = nseg - 1; s >= 0; --s) {
      if (s > 0)
        memcpy(hs, ckpt + (b * nseg + s - 1) * D, (size_t)D * sizeof(float));
      else
        memset(hs, 0, (size_t)D * sizeof(float));
      for (i64 tl = 0; tl < seg; ++tl) {
        const i64 op = (b * L + s * seg + tl) * Dp, ox = (b * L + s * seg + tl) * D;
        const float* pv = hs + tl * D;
        float* cu = hs + (tl + 1) * D;
        for (i64 p = 0; p < Dp; ++p) {
          const float av = a[op + p], c = cs[op + p], sv = sn[op + p];
          const float u = pv[2 * p], w = pv[2 * p + 1];
          cu[2 * p] = av * (c * u - sv * w) + x[ox + 2 * p];
          cu[2 * p + 1] = av * (sv * u + c * w) + x[ox + 2 * p + 1];
        }
      }
      for (i64 tl = seg - 1; tl >= 0; --tl) {
        const i64 op = (b * L + s * seg + tl) * Dp, ox = (b * L + s * seg + tl) * D;
        const float* pv = hs + tl * D;
        for (i64 p = 0; p < Dp; ++p) {
          const float av = a[op + p], c = cs[op + p], sv = sn[op + p];
          const float up = pv[2 * p], wp = pv[2 * p + 1];
          float aU = adj[2 * p] + gy[ox + 2 * p];
          float aW = adj[2 * p + 1] + gy[ox + 2 * p + 1];
          gx[ox + 2 * p] = aU;
          gx[ox + 2 * p + 1] = aW;
          const float ru = c * up - sv * wp, rw = sv * up + c * wp;
          ga[op + p] = aU * ru + aW * rw;
          gcs[op + p] = av * (aU * up + aW * wp);
          gsn[op + p] = av * (aW * up - aU * wp);
          adj[2 * p] = av * (c * aU + sv * aW);
          adj[2 * p + 1] = av * (-sv * aU + c * aW);
        }
      }
    }
    free(adj);
    free(hs);
  }
}

/* ------------------------------------------------------- Gated DeltaNet -- */
/* The reference carries this recurrence as a design only
 * (docs/DESIGN_gated_deltanet.md): S_t = alpha (I - beta k k^T) S_{t-1} +
 * beta k v^T, o_t = S_t^T q (section 1, R1''/R2'), S[i][j] with i the key axis;
 * the adjoint of its section 4. Checkpoint + recompute as the other scans. */
static void gdn_advance(float* S, const float* kr, const float* vr, float a, float bt, i64 Dh, float* p,
                        float* w) {
  for (i64 j = 0; j < Dh; ++j) p[j] = 0.f;
  for (i64 i = 0; i < Dh; ++i)
    for (i64 j = 0; j < Dh; ++j) p[j] += kr[i] * S[i * Dh + j];
  for (i64 j = 0; j < Dh; ++j) w[j] = bt * (vr[j] - a * p[j]);
  for (i64 i = 0; i < Dh; ++i)
    for (i64 j = 0; j < Dh; ++j) S[i * Dh + j] = a * S[i * Dh + j] + kr[i] * w[j];
}

void orc_gdn_fwd(const float* q, const float* k, const float* v, const float* alpha, const float* beta, i64 Bt,
                 i64 L, i64 H, i64 Dh, i64 seg, float* y, float* ckpt) {
  const i64 nseg = L / seg;
#pragma omp parallel for schedule(dynamic, 1)
  for (i64 bh = 0; bh < Bt * H; ++bh) {
    const i64 b = bh / H, h = bh % H;
    float* S = (float*)calloc((size_t)(Dh * Dh + 2 * Dh), sizeof(float));
    float *p = S + Dh * Dh, *w = p + Dh;
    for (i64 t = 0; t < L; ++t) {
      const i64 row = (b * L + t) * H + h;
      gdn_advance(S, k + row * Dh, v + row * Dh, alpha[row], beta[row], Dh, p, w);
      float* yr = y + row * Dh;
      for (i64 j = 0; j < Dh; ++j) yr[j] = 0.f;
      for (i64 i = 0; i < Dh; ++i)
        for (i64 j = 0; j < Dh; ++j) yr[j] += q[row * Dh + i] * S[i * Dh + j];
      if ((t + 1) % seg == 0)
        memcpy(ckpt + ((b * nseg + t / seg) * H + h) * Dh * Dh, S, (size_t)(Dh * Dh) * sizeof(float));
    }
    free(S);
  }
}

void orc_gdn_bwd(const float* gy, const float* gfinal, const float* ckpt, const float* q, const float* k,
                 const float* v, const float* alpha, const float* beta, i64 Bt, i64 L, i64 H, i64 Dh, i64 seg,
                 float* gq, float* gk, float* gv, float* ga, float* gb) {
  const i64 nseg = L / seg;
#pragma omp parallel for schedule(dynamic, 1)
  for (i64 bh = 0; bh < Bt * H; ++bh) {
    const i64 b = bh / H, h = bh % H;
    const i64 S2 = Dh * Dh;
    float* G = (float*)calloc((size_t)S2, sizeof(float));
    float* scr = (float*)malloc((size_t)((seg + 1) * S2 + 4 * Dh) * sizeof(float));
    float *p = scr + (seg + 1) * S2, *w = p + Dh, *d = w + Dh, *tmp = d + Dh;
    if (gfinal)
      for (i64 i = 0; i < S2; ++i) G[i] = gfinal[bh * S2 + i];
    for (i64 s = nseg - 1; s >= 0; --s) {
      if (s > 0)
        memcpy(scr, ckpt + ((b * nseg + s - 1) * H + h) * S2, (size_t)S2 * sizeof(float));
      else
        memset(scr, 0, (size_t)S2 * sizeof(float));
      for (i64 tl = 0; tl < seg; ++tl) {
        const i64 row = (b * L + s * seg + tl) * H + h;
        memcpy(scr + (tl + 1) * S2, scr + tl * S2, (size_t)S2 * sizeof(float));
        gdn_advance(scr + (tl + 1) * S2, k + row * Dh, v + row * Dh, alpha[row], beta[row], Dh, p, w);
      }
      for (i64 tl = seg - 1; tl >= 0; --tl) {
        const i64 row = (b * L + s * seg + tl) * H + h;
        const float a = alpha[row], bt = beta[row];
        const float* Sp = scr + tl * S2;
        const float* St = scr + (tl + 1) * S2;
        const float *qr = q + row * Dh, *kr = k + row * Dh, *vr = v + row * Dh, *go = gy + row * Dh;
        for (i64 j = 0; j < Dh; ++j) p[j] = 0.f;
        for (i64 i = 0; i < Dh; ++i)
          for (i64 j = 0; j < Dh; ++j) p[j] += kr[i] * Sp[i * Dh + j];
        for (i64 j = 0; j < Dh; ++j) w[j] = bt * (vr[j] - a * p[j]);
        for (i64 i = 0; i < Dh; ++i)
          for (i64 j = 0; j < Dh; ++j) G[i * Dh + j] += qr[i] * go[j];
        for (i64 j = 0; j < Dh; ++j) d[j] = 0.f;
        for (i64 i = 0; i < Dh; ++i)
          for (i64 j = 0; j < Dh; ++j) d[j] += kr[i] * G[i * Dh + j];
        float gas = 0.f, gbs = 0.f;
        for (i64 i = 0; i < Dh; ++i) {
          float sq = 0.f, sk = 0.f, sd = 0.f;
          for (i64 j = 0; j < Dh; ++j) {
            const i64 e = i * Dh + j;
            sq += St[e] * go[j];
            sk += G[e] * w[j];
            sd += Sp[e] * d[j];
            gas += G[e] * Sp[e];
          }
          gq[row * Dh + i] = sq;
          tmp[i] = sk - a * bt * sd;
        }
        for (i64 i = 0; i < Dh; ++i) gk[row * Dh + i] = tmp[i];
        for (i64 j = 0; j < Dh; ++j) {
          gv[row * Dh + j] = bt * d[j];
          gas -= bt * d[j] * p[j];
          gbs += d[j] * (vr[j] - a * p[j]);
        }
        ga[row] = gas;
        gb[row] = gbs;
        for (i64 i = 0; i < Dh; ++i)
          for (i64 j = 0; j < Dh; ++j) G[i * Dh + j] = a * G[i * Dh + j] - a * bt * kr[i] * d[j];
      }
    }
    free(G);
    free(scr);
  }
}
