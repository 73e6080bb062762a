/*
 * TEST INFRASTRUCTURE ONLY -- the timed CPU baseline of the quantized MoE path.
 *
 * The reference has no CPU implementation of this path (it is Metal-only) and
 * the MLX CPU backend BASELINE.json names is not in the reference tree, so
 * the CPU baseline is this port of the same arithmetic (oracle/mc_oracle.c),
 * written for speed: OpenMP over output rows, vectorisable inner loops,
 * -O3 -ffast-math (sums may be reassociated, so results agree with the exact
 * oracle only within tolerance). Only bench.py's cpu_baseline and
 * --impl reference legs call it.
 *
 * Algorithm per Q4 row (dot_word_q4 / GEMV_Q4_BODY, lfm.metal:102-139):
 *   y = sum_g s_g * (sum_{k in g} q_k x_k) + b_g * (sum_{k in g} x_k).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf(uint16_t h) {
  union { uint32_t u; float f; } v; v.u = (uint32_t)h << 16; return v.f;
}
static inline uint16_t tobf(float f) {
  union { uint32_t u; float f; } v; v.f = f;
  uint32_t u = v.u;
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float rbf(float f) { return bf(tobf(f)); }

int of_threads(void) { return omp_get_max_threads(); }
void of_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }

/* one Q4 row against x (float, K), xg (group sums) */
static inline float q4_row(const uint32_t* codes, const uint16_t* s, const uint16_t* b, int K,
                           const float* x, const float* xg) {
  const int G = K / 64;
  float acc = 0.0f;
  for (int g = 0; g < G; ++g) {
    const uint32_t* w = codes + 8 * g;
    const float* xx = x + 64 * g;
    float qx = 0.0f;
    for (int i = 0; i < 8; ++i) {
      uint32_t v = w[i];
      for (int j = 0; j < 8; ++j) qx += (float)((v >> (4 * j)) & 15u) * xx[8 * i + j];
    }
    acc += bf(s[g]) * qx + bf(b[g]) * xg[g];
  }
  return acc;
}

static void prep_x(const uint16_t* xb, int K, float* x, float* xg) {
  for (int k = 0; k < K; ++k) x[k] = bf(xb[k]);
  for (int g = 0; g < K / 64; ++g) {
    float s = 0.0f;
    for (int i = 0; i < 64; ++i) s += x[64 * g + i];
    xg[g] = s;
  }
}

void of_gemv_q4(const uint32_t* codes, const uint16_t* s, const uint16_t* b, int N, int K,
                const uint16_t* xb, uint16_t* y) {
  float* x = (float*)malloc(sizeof(float) * K);
  float* xg = (float*)malloc(sizeof(float) * (K / 64));
  prep_x(xb, K, x, xg);
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n)
    y[n] = tobf(q4_row(codes + (size_t)n * (K / 8), s + (size_t)n * (K / 64),
                       b + (size_t)n * (K / 64), K, x, xg));
  free(x); free(xg);
}

/* One BASELINE cfg1 decode layer for one token: add + RMSNorm, bf16 router,
 * softmax-renorm top-4, gate/up/SiLU, down + combine. */
void of_moe_decode_layer(const uint16_t* h, const uint16_t* badd, const uint16_t* norm_w,
                         const uint16_t* router, const uint32_t* gc, const uint16_t* gs,
                         const uint16_t* gb, const uint32_t* uc, const uint16_t* us,
                         const uint16_t* ub, const uint32_t* dc, const uint16_t* ds,
                         const uint16_t* db, int E, int H, int I, float eps,
                         uint16_t* hout, uint32_t* ids, uint16_t* wts, uint16_t* out) {
  float* n = (float*)malloc(sizeof(float) * H);
  float* ng = (float*)malloc(sizeof(float) * (H / 64));
  float* z = (float*)malloc(sizeof(float) * E);
  float* act = (float*)malloc(sizeof(float) * 4 * I);
  float* ag = (float*)malloc(sizeof(float) * 4 * (I / 64));
  float ss = 0.0f;
  for (int k = 0; k < H; ++k) {
    float v = rbf(bf(h[k]) + (badd ? bf(badd[k]) : 0.0f));
    hout[k] = tobf(v);
    n[k] = v;
    ss += v * v;
  }
  float inv = 1.0f / sqrtf(ss / (float)H + eps);
  for (int k = 0; k < H; ++k) n[k] = rbf(n[k] * inv * bf(norm_w[k]));
  for (int g = 0; g < H / 64; ++g) {
    float s = 0.0f;
    for (int i = 0; i < 64; ++i) s += n[64 * g + i];
    ng[g] = s;
  }
#pragma omp parallel for schedule(static)
  for (int e = 0; e < E; ++e) {
    float a = 0.0f;
    const uint16_t* r = router + (size_t)e * H;
    for (int k = 0; k < H; ++k) a += bf(r[k]) * n[k];
    z[e] = a;
  }
  int used[256] = {0};
  uint32_t ch[4];
  for (int r = 0; r < 4; ++r) {
    float bv = -INFINITY; int bi = 0;
    for (int e = 0; e < E; ++e)
      if (!used[e] && z[e] > bv) { bv = z[e]; bi = e; }
    ch[r] = (uint32_t)bi; used[bi] = 1;
  }
  float ex[4], den = 0.0f;
  for (int r = 0; r < 4; ++r) { ex[r] = expf(z[ch[r]] - z[ch[0]]); den += ex[r]; }
  for (int r = 0; r < 4; ++r) { ids[r] = ch[r]; wts[r] = tobf(ex[r] / den); }
  const int Gh = H / 64, Gi = I / 64;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < 4 * I; ++t) {
    const int r = t / I, i = t % I;
    const size_t row = (size_t)ch[r] * I + i;
    float g = rbf(q4_row(gc + row * (H / 8), gs + row * Gh, gb + row * Gh, H, n, ng));
    float u = rbf(q4_row(uc + row * (H / 8), us + row * Gh, ub + row * Gh, H, n, ng));
    act[t] = rbf(rbf(g / (1.0f + expf(-g))) * u);
  }
  for (int r = 0; r < 4; ++r)
    for (int g = 0; g < Gi; ++g) {
      float s = 0.0f;
      for (int i = 0; i < 64; ++i) s += act[r * I + 64 * g + i];
      ag[r * Gi + g] = s;
    }
#pragma omp parallel for schedule(static)
  for (int i = 0; i < H; ++i) {
    float tot = 0.0f;
    for (int r = 0; r < 4; ++r) {
      const size_t row = (size_t)ch[r] * H + i;
      float p = rbf(q4_row(dc + row * (I / 8), ds + row * Gi, db + row * Gi, I, act + r * I,
                           ag + r * Gi));
      tot += rbf(bf(wts[r]) * p);
    }
    out[i] = tobf(tot);
  }
  free(n); free(ng); free(z); free(act); free(ag);
}

/* Grouped Q4 GEMM over sorted rows (prefill baseline): C[i] = A[i] . Wdeq[e]^T,
 * dequantising each expert once into a float panel. */
void of_gemm_q4_grouped(const uint16_t* A, int K, const uint32_t* codes, const uint16_t* scales,
                        const uint16_t* biases, int N, const uint32_t* counts,
                        const uint32_t* offsets, int E, uint16_t* C) {
  float* wd = (float*)malloc(sizeof(float) * (size_t)N * K);
  const int G = K / 64;
  for (int e = 0; e < E; ++e) {
    if (!counts[e]) continue;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
      const size_t row = (size_t)e * N + n;
      for (int k = 0; k < K; ++k) {
        uint32_t w = codes[row * (K / 8) + k / 8];
        float q = (float)((w >> (4 * (k & 7))) & 15u);
        wd[(size_t)n * K + k] = rbf(bf(scales[row * G + k / 64]) * q + bf(biases[row * G + k / 64]));
      }
    }
#pragma omp parallel for schedule(static)
    for (uint32_t i = offsets[e]; i < offsets[e] + counts[e]; ++i) {
      float a[4096];
      for (int k = 0; k < K; ++k) a[k] = bf(A[(size_t)i * K + k]);
      for (int n = 0; n < N; ++n) {
        const float* w = wd + (size_t)n * K;
        float s = 0.0f;
        for (int k = 0; k < K; ++k) s += a[k] * w[k];
        C[(size_t)i * N + n] = tobf(s);
      }
    }
  }
  free(wd);
}

/* Whole prefill MoE FFN (softmax-renorm top-4, sort, grouped gate/up/SwiGLU,
 * grouped down, combine) for m tokens: the CPU baseline of BASELINE cfg3. */
void of_moe_prefill(const uint16_t* x, const float* logits, int m, int E, int H, int I,
                    const uint32_t* gc, const uint16_t* gs, const uint16_t* gb,
                    const uint32_t* uc, const uint16_t* us, const uint16_t* ub,
                    const uint32_t* dc, const uint16_t* ds, const uint16_t* db, uint16_t* out) {
  const int S = 4 * m;
  uint32_t* ids = (uint32_t*)malloc(sizeof(uint32_t) * S);
  float* w = (float*)malloc(sizeof(float) * S);
  uint32_t* counts = (uint32_t*)calloc(E, sizeof(uint32_t));
  uint32_t* offsets = (uint32_t*)malloc(sizeof(uint32_t) * E);
  uint32_t* sorted = (uint32_t*)malloc(sizeof(uint32_t) * S);
  uint32_t* slot = (uint32_t*)malloc(sizeof(uint32_t) * S);
  uint16_t* gx = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)S * H);
  uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)S * I);
  uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)S * I);
  uint16_t* ed = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)S * H);
  for (int t = 0; t < m; ++t) {
    const float* z = logits + (size_t)t * E;
    int used[256] = {0};
    float ex[4], den = 0.0f;
    for (int r = 0; r < 4; ++r) {
      float bv = -INFINITY; int bi = 0;
      for (int e = 0; e < E; ++e) if (!used[e] && z[e] > bv) { bv = z[e]; bi = e; }
      used[bi] = 1; ids[4 * t + r] = (uint32_t)bi;
      ex[r] = expf(z[bi] - z[ids[4 * t]]); den += ex[r];
    }
    for (int r = 0; r < 4; ++r) w[4 * t + r] = rbf(ex[r] / den);
  }
  for (int i = 0; i < S; ++i) counts[ids[i]]++;
  uint32_t acc = 0;
  for (int e = 0; e < E; ++e) { offsets[e] = acc; acc += counts[e]; }
  uint32_t* pos = (uint32_t*)malloc(sizeof(uint32_t) * E);
  memcpy(pos, offsets, sizeof(uint32_t) * E);
  for (int i = 0; i < S; ++i) { uint32_t p = pos[ids[i]]++; sorted[p] = (uint32_t)(i / 4); slot[i] = p; }
#pragma omp parallel for schedule(static)
  for (int i = 0; i < S; ++i) memcpy(gx + (size_t)i * H, x + (size_t)sorted[i] * H, 2 * (size_t)H);
  of_gemm_q4_grouped(gx, H, gc, gs, gb, I, counts, offsets, E, g);
  of_gemm_q4_grouped(gx, H, uc, us, ub, I, counts, offsets, E, u);
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < (size_t)S * I; ++i) {
    float gv = bf(g[i]);
    g[i] = tobf(rbf(gv / (1.0f + expf(-gv))) * bf(u[i]));
  }
  of_gemm_q4_grouped(g, I, dc, ds, db, H, counts, offsets, E, ed);
#pragma omp parallel for schedule(static)
  for (int t = 0; t < m; ++t)
    for (int h = 0; h < H; ++h) {
      float s = 0.0f;
      for (int r = 0; r < 4; ++r) s += rbf(w[4 * t + r] * bf(ed[(size_t)slot[4 * t + r] * H + h]));
      out[(size_t)t * H + h] = tobf(s);
    }
  free(ids); free(w); free(counts); free(offsets); free(sorted); free(slot); free(gx);
  free(g); free(u); free(ed); free(pos);
}

/* Q6 LM head GEMV + argmax over bf16-rounded logits, lowest index on ties
 * (lfm.metal:1200-1282): the CPU baseline's head for BASELINE cfg4. Codes are
 * 4 per 3 bytes, little-endian, K*6/8 bytes per row. */
uint32_t of_head_q6_argmax(const uint8_t* codes, const uint16_t* s, const uint16_t* b, int N, int K,
                           const uint16_t* xb) {
  float* x = (float*)malloc(sizeof(float) * K);
  float* xg = (float*)malloc(sizeof(float) * (K / 64));
  prep_x(xb, K, x, xg);
  const int G = K / 64, rb = K * 6 / 8;
  float best_v = -INFINITY;
  int best_i = 0;
#pragma omp parallel
  {
    float bv = -INFINITY;
    int bi = 0;
#pragma omp for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint8_t* r = codes + (size_t)n * rb;
      float acc = 0.0f;
      for (int g = 0; g < G; ++g) {
        const uint8_t* p = r + 48 * g;
        const float* xx = x + 64 * g;
        float qx = 0.0f;
        for (int t = 0; t < 16; ++t) {
          const uint32_t b0 = p[3 * t], b1 = p[3 * t + 1], b2 = p[3 * t + 2];
          qx += (float)(b0 & 63u) * xx[4 * t] + (float)((b0 >> 6) | ((b1 & 15u) << 2)) * xx[4 * t + 1] +
                (float)((b1 >> 4) | ((b2 & 3u) << 4)) * xx[4 * t + 2] + (float)(b2 >> 2) * xx[4 * t + 3];
        }
        acc += bf(s[(size_t)n * G + g]) * qx + bf(b[(size_t)n * G + g]) * xg[g];
      }
      const float v = rbf(acc);
      if (v > bv || (v == bv && n < bi)) { bv = v; bi = n; }
    }
#pragma omp critical
    {
      if (bv > best_v || (bv == best_v && bi < best_i)) { best_v = bv; best_i = bi; }
    }
  }
  free(x); free(xg);
  return (uint32_t)best_i;
}
