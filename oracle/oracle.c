/*
 * CPU oracle for the maple-b200 decode path.  TEST INFRASTRUCTURE ONLY: it is
 * loaded by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * as the checker, never by the product path.
 *
 * It restates the reference's algorithms (cloud-000/maple-flash-dgx-spark,
 * src/maple_run/...) on the CPU, following the reference's rounding points
 * (bf16 stores between operators, fp32 math inside them) and the canonical
 * numerics the CUDA kernels define (fixed reduction orders, exp by
 * Cody-Waite + Taylor, IEEE div/sqrt, exact integer packed contractions), so
 * that a GPU result can be compared bit for bit.
 *
 * Build: oracle/build.py (gcc -O2 -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ scalars --- */
static inline float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t u_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* fp32 -> bf16 round-to-nearest-even, NaN -> 0x7FC0 (torch's convention). */
uint16_t orc_f32_to_bf16(float f) {
  uint32_t u = u_of(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float bf(float f) { return f_of((uint32_t)orc_f32_to_bf16(f) << 16); }

/* exp(x): x = n*ln2 + r with ln2 split hi/lo (Cody & Waite), e^r by its
 * Taylor series to degree 7 (Horner, fused multiply-add), 2^n applied as two
 * exact power-of-two factors. */
float orc_exp(float x) {
  if (x != x) return x;
  if (x < -104.0f) return 0.0f;
  if (x > 88.7228393554688f) return INFINITY;
  const float n = rintf(x * 1.44269504088896341f);
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.42860676533018704e-06f, r);
  float p = 1.98412698412698413e-04f;
  p = fmaf(p, r, 1.38888888888888889e-03f);
  p = fmaf(p, r, 8.33333333333333333e-03f);
  p = fmaf(p, r, 4.16666666666666667e-02f);
  p = fmaf(p, r, 1.66666666666666667e-01f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ni = (int)n;
  const int n1 = ni / 2, n2 = ni - n1;
  p = p * f_of((uint32_t)(n1 + 127) << 23);
  return p * f_of((uint32_t)(n2 + 127) << 23);
}

static inline float sigmoid_(float x) { return 1.0f / (1.0f + orc_exp(-x)); }

static inline float rstd_of(float sumsq, int n, float eps) {
  const float var = sumsq / (float)n;
  return 1.0f / sqrtf(var + eps);
}

/* R128 order: partial p_j (j < 128) accumulates elements j, j+128, ...
 * sequentially from 0; q_l = ((p_l + p_{l+32}) + p_{l+64}) + p_{l+96};
 * then an xor butterfly over the 32 q_l (16, 8, 4, 2, 1). */
static float r128_finish(const float p[128]) {
  float q[32];
  for (int l = 0; l < 32; ++l) q[l] = ((p[l] + p[l + 32]) + p[l + 64]) + p[l + 96];
  for (int m = 16; m >= 1; m >>= 1) {
    float nx[32];
    for (int l = 0; l < 32; ++l) nx[l] = q[l] + q[l ^ m];
    memcpy(q, nx, sizeof(nx));
  }
  return q[0];
}

float orc_r128_sum(const float* v, int64_t n) {
  float p[128] = {0};
  for (int64_t i = 0; i < n; ++i) p[i & 127] = p[i & 127] + v[i];
  return r128_finish(p);
}

float orc_r128_sumsq(const float* v, int64_t n) {
  float p[128] = {0};
  for (int64_t i = 0; i < n; ++i) p[i & 127] = fmaf(v[i], v[i], p[i & 127]);
  return r128_finish(p);
}

float orc_r128_dot(const float* a, const float* b, int64_t n) {
  float p[128] = {0};
  for (int64_t i = 0; i < n; ++i) p[i & 127] = fmaf(a[i], b[i], p[i & 127]);
  return r128_finish(p);
}

/* --------------------------------------------------------------- FXA ---- */
#define FXA_NONFINITE (1 << 20)

int orc_fxa_shift(const float* v, int64_t n) {
  uint32_t amax = 0;
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t a = u_of(v[i]) & 0x7fffffffu;
    if (a > amax) amax = a;
  }
  if (amax == 0) return 0;
  const int ef = (int)(amax >> 23);
  if (ef == 0xff) return FXA_NONFINITE;
  return 25 - (ef - 127);
}

static inline double pow2d(int s) { return ldexp(1.0, s); }

static inline int64_t fxa_encode(float v, int s) { return (int64_t)rint((double)v * pow2d(s)); }

static inline float fxa_value(int64_t S, int s) { return (float)((double)S * pow2d(-s)); }

/* Byte lookup table of an FXA vector for 2-bit codes: entry [q][b] =
 * sum_{i<4} (((b >> 2i) & 3) - 1) * X[4q + i], so a code byte costs one
 * lookup.  The sums are exact integers, identical to the direct loop. */
static int64_t* tern_lut(const int64_t* X, int64_t k) {
  int64_t* lut = (int64_t*)malloc(sizeof(int64_t) * (k / 4) * 256);
  for (int64_t q = 0; q < k / 4; ++q)
    for (int b = 0; b < 256; ++b) {
      int64_t v = 0;
      for (int i = 0; i < 4; ++i) v += ((int64_t)((b >> (2 * i)) & 3) - 1) * X[4 * q + i];
      lut[q * 256 + b] = v;
    }
  return lut;
}

/* Exact sum_k (c_k - 1) * X_k over a ternary code row. */
static int64_t tern_dot(const uint32_t* row, int64_t nwords, const int64_t* lut) {
  int64_t S = 0;
  for (int64_t w = 0; w < nwords; ++w) {
    const uint32_t word = row[w];
    const int64_t* l = lut + w * 4 * 256;
    S += l[word & 0xff] + l[256 + ((word >> 8) & 0xff)] + l[512 + ((word >> 16) & 0xff)] + l[768 + (word >> 24)];
  }
  return S;
}

/* ------------------------------------------------------ ternary GEMV ---- */
/* Reference: kernels/ternary_gemv.py:76-153.  y[b,n] = alpha[n] * rstd *
 * sum_k (c-1) * x[b,k]*w[k].  The sum is the exact integer contraction of the
 * codes with the FXA encoding of x*w, rounded once to fp32. */
void orc_ternary_gemv(const float* x, int64_t batch, int64_t k, const uint32_t* codes, int64_t n,
                      const float* alpha, const float* rms_w, float eps, int out_bf16, float* y) {
  const int64_t nwords = k / 16;
  float* xh = (float*)malloc(sizeof(float) * k);
  int64_t* X = (int64_t*)malloc(sizeof(int64_t) * k);
  for (int64_t b = 0; b < batch; ++b) {
    const float* xr = x + b * k;
    float rstd = 1.0f;
    for (int64_t i = 0; i < k; ++i) xh[i] = rms_w ? xr[i] * rms_w[i] : xr[i];
    if (rms_w) rstd = rstd_of(orc_r128_sumsq(xr, k), (int)k, eps);
    const int s = orc_fxa_shift(xh, k);
    for (int64_t i = 0; i < k; ++i) X[i] = (s == FXA_NONFINITE) ? 0 : fxa_encode(xh[i], s);
    int64_t* lut = tern_lut(X, k);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
      const int64_t S = tern_dot(codes + r * nwords, nwords, lut);
      float v = (s == FXA_NONFINITE) ? f_of(0x7fc00000u) : fxa_value(S, s);
      if (rms_w) v = v * rstd;
      v = v * alpha[r];
      y[b * n + r] = out_bf16 ? bf(v) : v;
    }
    free(lut);
  }
  free(xh);
  free(X);
}

/* ---------------------------------------------------------- helpers ---- */
/* FXA encoding of one activation row (no RMS). Returns the shift. */
static int fxa_row(const float* v, int64_t k, int64_t* X) {
  const int s = orc_fxa_shift(v, k);
  for (int64_t i = 0; i < k; ++i) X[i] = (s == FXA_NONFINITE) ? 0 : fxa_encode(v[i], s);
  return s;
}

static inline float fxa_val_or_nan(int64_t S, int s) {
  return (s == FXA_NONFINITE) ? f_of(0x7fc00000u) : fxa_value(S, s);
}

/* ------------------------------------------------------------ norms ---- */
/* Reference: kernels/fused_norm.py:11-29 (rms_norm). */
void orc_rms_norm(const float* x, int64_t rows, int64_t n, const float* w, float eps, int out_bf16,
                  float* y) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * n;
    const float rstd = rstd_of(orc_r128_sumsq(xr, n), (int)n, eps);
    for (int64_t k = 0; k < n; ++k) {
      const float v = (xr[k] * rstd) * w[k];
      y[r * n + k] = out_bf16 ? bf(v) : v;
    }
  }
}

/* Reference: kernels/fused_norm.py:32-57 (add_rms_norm): residual = x + y,
 * the norm is taken of the unrounded fp32 sum. */
void orc_add_rms_norm(const float* x, const float* y, int64_t rows, int64_t n, const float* w, float eps,
                      int out_bf16, float* residual, float* normed) {
  float* s = (float*)malloc(sizeof(float) * n);
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t k = 0; k < n; ++k) {
      s[k] = x[r * n + k] + y[r * n + k];
      residual[r * n + k] = out_bf16 ? bf(s[k]) : s[k];
    }
    const float rstd = rstd_of(orc_r128_sumsq(s, n), (int)n, eps);
    for (int64_t k = 0; k < n; ++k) {
      const float v = (s[k] * rstd) * w[k];
      normed[r * n + k] = out_bf16 ? bf(v) : v;
    }
  }
  free(s);
}

/* ----------------------------------------------------------- router ---- */
/* Reference: kernels/router.py:20-126.  logits = R128 dot; softmax with the
 * R128 sum; top-k by repeated argmax (ties -> lowest index); w = p/(sum+1e-20). */
void orc_router_topk(const float* x, int64_t T, int64_t K, const float* G, int64_t E, int64_t topk,
                     int32_t* idx, float* wt) {
  float* p = (float*)malloc(sizeof(float) * E);
  for (int64_t t = 0; t < T; ++t) {
    float m = -INFINITY;
    for (int64_t e = 0; e < E; ++e) {
      p[e] = orc_r128_dot(x + t * K, G + e * K, K);
      if (p[e] > m) m = p[e];
    }
    for (int64_t e = 0; e < E; ++e) p[e] = orc_exp(p[e] - m);
    const float sum = orc_r128_sum(p, E);
    for (int64_t e = 0; e < E; ++e) p[e] = p[e] / sum;
    float total = 0.0f;
    for (int64_t r = 0; r < topk; ++r) {
      int64_t bi = -1;
      float bv = -INFINITY;
      for (int64_t e = 0; e < E; ++e)
        if (bi < 0 || p[e] > bv) { bv = p[e]; bi = e; }
      total = total + bv;
      idx[t * topk + r] = (int32_t)bi;
      wt[t * topk + r] = bv;
      p[bi] = -INFINITY;
    }
    const float inv = 1.0f / (total + 1e-20f);
    for (int64_t r = 0; r < topk; ++r) wt[t * topk + r] = wt[t * topk + r] * inv;
  }
  free(p);
}

/* --------------------------------------------------------- experts ---- */
/* Reference: kernels/ternary_expert.py:58-122 (indexed GEMV). x row of slot
 * z is z / x_div. */
void orc_expert_gemv(const float* x, int64_t x_div, const int32_t* ids, int64_t slots, int64_t K,
                     const uint32_t* codes, int64_t E, int64_t N, const float* alpha, int out_bf16, float* y) {
  const int64_t nwords = K / 16;
  int64_t* X = (int64_t*)malloc(sizeof(int64_t) * K);
  for (int64_t z = 0; z < slots; ++z) {
    const int s = fxa_row(x + (z / x_div) * K, K, X);
    int64_t* lut = tern_lut(X, K);
    const int32_t e = ids[z];
    const int ok = e >= 0 && e < E;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      float v = f_of(0x7fc00000u);
      if (ok) v = fxa_val_or_nan(tern_dot(codes + ((int64_t)e * N + n) * nwords, nwords, lut), s) * alpha[e * N + n];
      y[z * N + n] = out_bf16 ? bf(v) : v;
    }
    free(lut);
  }
  free(X);
}

/* Reference: kernels/ternary_expert.py:240-319 (fused up+gate, clamp, SiLU):
 * up rows [0, I), gate rows [I, 2I) of the selected expert. */
void orc_expert_swiglu(const float* x, int64_t T, int64_t topk, int64_t K, const uint32_t* codes, int64_t E,
                       int64_t I, const float* alpha, const int32_t* ids, int out_bf16, float* h) {
  const int64_t nwords = K / 16;
  int64_t* X = (int64_t*)malloc(sizeof(int64_t) * K);
  for (int64_t t = 0; t < T; ++t) {
    const int s = fxa_row(x + t * K, K, X);
    int64_t* lut = tern_lut(X, K);
    for (int64_t j = 0; j < topk; ++j) {
      const int32_t e = ids[t * topk + j];
      const int ok = e >= 0 && e < E;
#pragma omp parallel for schedule(static)
      for (int64_t n = 0; n < I; ++n) {
        float out = f_of(0x7fc00000u);
        if (ok) {
          const uint32_t* base = codes + (int64_t)e * 2 * I * nwords;
          float up = fxa_val_or_nan(tern_dot(base + n * nwords, nwords, lut), s) * alpha[e * 2 * I + n];
          float gate = fxa_val_or_nan(tern_dot(base + (I + n) * nwords, nwords, lut), s) * alpha[e * 2 * I + I + n];
          up = fminf(fmaxf(up, -7.0f), 7.0f);
          gate = fminf(gate, 7.0f);
          out = (up * gate) * sigmoid_(gate);
        }
        h[(t * topk + j) * I + n] = out_bf16 ? bf(out) : out;
      }
    }
    free(lut);
  }
  free(X);
}

/* Down projection of every top-k slot and the weighted combine.
 * mode 0 (reference model path: ternary_expert_gemv then moe_reduce_add,
 *   kernels/fused_norm.py:60-97): y_s = round(alpha*S_s), acc = fmaf(w_s, y_s, acc).
 * mode 1 (reference ternary_expert_down_sum, ternary_expert.py:322-400):
 *   acc = fmaf(w_s * S_s, alpha, acc).
 * out = round(acc + residual). */
void orc_expert_down_reduce(const float* h, int64_t T, int64_t topk, int64_t K, const int32_t* ids,
                            const float* wt, const uint32_t* codes, int64_t E, int64_t N, const float* alpha,
                            const float* residual, int mode, int out_bf16, float* out) {
  const int64_t nwords = K / 16;
  int64_t* X = (int64_t*)malloc(sizeof(int64_t) * K * topk);
  int64_t** luts = (int64_t**)malloc(sizeof(int64_t*) * topk);
  int* sh = (int*)malloc(sizeof(int) * topk);
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t j = 0; j < topk; ++j) {
      sh[j] = fxa_row(h + (t * topk + j) * K, K, X + j * K);
      luts[j] = tern_lut(X + j * K, K);
    }
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int64_t j = 0; j < topk; ++j) {
        int32_t e = ids[t * topk + j];
        const int ok = e >= 0 && e < E;
        if (!ok) e = 0;
        float v = ok ? fxa_val_or_nan(tern_dot(codes + ((int64_t)e * N + n) * nwords, nwords, luts[j]), sh[j])
                     : f_of(0x7fc00000u);
        const float w = wt[t * topk + j];
        if (mode == 0) {
          float y = v * alpha[e * N + n];
          if (out_bf16) y = bf(y);
          acc = fmaf(w, y, acc);
        } else {
          acc = fmaf(w * v, alpha[e * N + n], acc);
        }
      }
      if (residual) acc = acc + residual[t * N + n];
      out[t * N + n] = out_bf16 ? bf(acc) : acc;
    }
    for (int64_t j = 0; j < topk; ++j) free(luts[j]);
  }
  free(X);
  free(sh);
  free(luts);
}

/* Reference: kernels/fused_norm.py:60-97. */
void orc_moe_reduce_add(const float* x, const float* w, const float* residual, int64_t T, int64_t topk,
                        int64_t N, int out_bf16, float* y) {
  for (int64_t t = 0; t < T; ++t)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int64_t j = 0; j < topk; ++j) acc = fmaf(w[t * topk + j], x[(t * topk + j) * N + n], acc);
      if (residual) acc = acc + residual[t * N + n];
      y[t * N + n] = out_bf16 ? bf(acc) : acc;
    }
}

/* -------------------------------------------------------- attention ---- */
/* Reference: kernels/decode_attn.py:64-163.  Caches are fp32 arrays holding
 * the (bf16) cache values, [Bc, Hkv, T, D]. */
void orc_apply_qkv_decode(const float* qkv, int64_t B, const float* qw, const float* kw, const float* cos,
                          const float* sin, int64_t R, float* q_out, float* kc, float* vc, int64_t Bc,
                          int64_t T, const int64_t* seqlen, const int32_t* row_map, int64_t Hq, int64_t Hkv,
                          int64_t D, int use_rope, float eps, int out_bf16) {
  const int64_t W = (Hq + 2 * Hkv) * D;
  float* xh = (float*)malloc(sizeof(float) * D);
  for (int64_t b = 0; b < B; ++b) {
    const float* row = qkv + b * W;
    const int64_t pos = seqlen[b];
    const int64_t cb = row_map ? row_map[b] : b;
    const int store_ok = pos >= 0 && pos < T && cb >= 0 && cb < Bc;
    for (int64_t hd = 0; hd < Hq + 2 * Hkv; ++hd) {
      const float* x = row + hd * D;
      if (hd >= Hq + Hkv) {
        if (!store_ok) continue;
        float* dst = vc + ((cb * Hkv + (hd - Hq - Hkv)) * T + pos) * D;
        for (int64_t d = 0; d < D; ++d) dst[d] = out_bf16 ? bf(x[d]) : x[d];
        continue;
      }
      const int is_q = hd < Hq;
      if (!is_q && !store_ok) continue;
      const float* w = is_q ? qw : kw;
      const float rstd = rstd_of(orc_r128_sumsq(x, D), (int)D, eps);
      for (int64_t d = 0; d < D; ++d) xh[d] = (x[d] * rstd) * w[d];
      float* dst = is_q ? q_out + (b * Hq + hd) * D : kc + ((cb * Hkv + (hd - Hq)) * T + pos) * D;
      const float* cs = cos + b * R;
      const float* sn = sin + b * R;
      const int64_t half = R / 2;
      for (int64_t d = 0; d < D; ++d) {
        float o = xh[d];
        if (use_rope && d < R) {
          if (d < half) o = xh[d] * cs[d] + (-xh[d + half]) * sn[d];
          else o = xh[d] * cs[d] + xh[d - half] * sn[d];
        }
        dst[d] = out_bf16 ? bf(o) : o;
      }
    }
  }
  free(xh);
}

/* Reference: kernels/decode_attn.py:166-359 with split length P (canonical
 * split/merge arithmetic of the CUDA kernel). */
void orc_decode_gqa(const float* q, int64_t B, int64_t Hq, const float* kc, const float* vc, int64_t Bc,
                    int64_t Hkv, int64_t T, int64_t D, const int64_t* seqlen, const int32_t* row_map,
                    float scale, int64_t window, int64_t P, int out_bf16, float* out) {
  const int64_t G = Hq / Hkv;
  float* sc = (float*)malloc(sizeof(float) * P);
  float* pb = (float*)malloc(sizeof(float) * P);
  const int64_t nsmax = (T + P - 1) / P;
  float* accs = (float*)malloc(sizeof(float) * nsmax * D);
  float* ms = (float*)malloc(sizeof(float) * nsmax);
  float* ls = (float*)malloc(sizeof(float) * nsmax);
  for (int64_t b = 0; b < B; ++b) {
    const int64_t pos = seqlen[b];
    const int64_t kv_len = pos + 1 < T ? pos + 1 : T;
    const int64_t start = window > 0 ? (kv_len - window > 0 ? kv_len - window : 0) : 0;
    const int64_t ns = kv_len > start ? (kv_len - start + P - 1) / P : 0;
    int64_t cb = row_map ? row_map[b] : b;
    if (cb < 0 || cb >= Bc) cb = 0;
    for (int64_t h = 0; h < Hkv; ++h)
      for (int64_t g = 0; g < G; ++g) {
        const int64_t hq = h * G + g;
        const float* qv = q + (b * Hq + hq) * D;
        for (int64_t s = 0; s < ns; ++s) {
          const int64_t t0 = start + s * P;
          const int64_t n = (kv_len - t0) < P ? (kv_len - t0) : P;
          float m = -INFINITY;
          for (int64_t t = 0; t < n; ++t) {
            sc[t] = orc_r128_dot(qv, kc + ((cb * Hkv + h) * T + t0 + t) * D, D) * scale;
            if (sc[t] > m) m = sc[t];
          }
          for (int64_t t = 0; t < n; ++t) sc[t] = orc_exp(sc[t] - m);
          ls[s] = orc_r128_sum(sc, n);
          ms[s] = m;
          /* P rounds to the cache dtype before P.V (decode_attn.py:284-289); an
           * fp32 cache (out_bf16 == 0) keeps it in fp32 (the IEEE path). */
          for (int64_t t = 0; t < n; ++t) pb[t] = out_bf16 ? bf(sc[t]) : sc[t];
          for (int64_t d = 0; d < D; ++d) {
            float a = 0.0f;
            for (int64_t t = 0; t < n; ++t) a = fmaf(pb[t], vc[((cb * Hkv + h) * T + t0 + t) * D + d], a);
            accs[s * D + d] = a;
          }
        }
        float* o = out + (b * Hq + hq) * D;
        if (ns == 1) {
          for (int64_t d = 0; d < D; ++d) { const float v = accs[d] / ls[0]; o[d] = out_bf16 ? bf(v) : v; }
        } else {
          float M = -INFINITY;
          for (int64_t s = 0; s < ns; ++s) if (ms[s] > M) M = ms[s];
          for (int64_t d = 0; d < D; ++d) {
            float num = 0.0f, den = 0.0f;
            for (int64_t s = 0; s < ns; ++s) {
              const float w = orc_exp(ms[s] - M);
              num = fmaf(w, accs[s * D + d], num);
              den = fmaf(w, ls[s], den);
            }
            const float v = num / den;
            o[d] = out_bf16 ? bf(v) : v;
          }
        }
      }
  }
  free(sc); free(pb); free(accs); free(ms); free(ls);
}

/* ------------------------------------------------------------- head ---- */
/* Reference: kernels/rtn4.py:84-167 / :418-511.  y = sum_g [s_g*C_g + b_g*X_g]
 * in double (group order), C_g = sum c*X, X_g = sum X (exact); biases == NULL
 * means symmetric b_g = -8*s_g.  row_index (nullable) maps output row ->
 * physical head row (FlashHead probes). */
void orc_rtn4_gemv(const float* x, int64_t B, int64_t K, const uint32_t* codes, int64_t N, const float* scales,
                   const float* biases, int64_t G, const int64_t* row_index, int out_bf16, float* y) {
  const int64_t nwords = K / 8, ng = K / G;
  int64_t* X = (int64_t*)malloc(sizeof(int64_t) * K);
  int64_t* Xg = (int64_t*)malloc(sizeof(int64_t) * ng);
  for (int64_t b = 0; b < B; ++b) {
    const int s = fxa_row(x + b * K, K, X);
    for (int64_t g = 0; g < ng; ++g) {
      Xg[g] = 0;
      for (int64_t k = g * G; k < (g + 1) * G; ++k) Xg[g] += X[k];
    }
    /* byte LUT: entry [q][b] = (b & 15) * X[2q] + (b >> 4) * X[2q + 1] */
    int64_t* lut = (int64_t*)malloc(sizeof(int64_t) * (K / 2) * 256);
    for (int64_t q = 0; q < K / 2; ++q)
      for (int bb = 0; bb < 256; ++bb) lut[q * 256 + bb] = (int64_t)(bb & 15) * X[2 * q] + (int64_t)(bb >> 4) * X[2 * q + 1];
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < N; ++r) {
      const int64_t pr = row_index ? row_index[r] : r;
      const uint32_t* row = codes + pr * nwords;
      double acc = 0.0;
      for (int64_t g = 0; g < ng; ++g) {
        int64_t C = 0;
        for (int64_t w = g * G / 8; w < (g + 1) * G / 8; ++w) {
          const uint32_t word = row[w];
          const int64_t* l = lut + w * 4 * 256;
          C += l[word & 0xff] + l[256 + ((word >> 8) & 0xff)] + l[512 + ((word >> 16) & 0xff)] + l[768 + (word >> 24)];
        }
        const float sg = scales[pr * ng + g];
        const float bg = biases ? biases[pr * ng + g] : -8.0f * sg;
        acc = (acc + (double)sg * (double)C) + (double)bg * (double)Xg[g];
      }
      const float v = (s == FXA_NONFINITE) ? f_of(0x7fc00000u) : (float)(acc * pow2d(-s));
      y[b * N + r] = out_bf16 ? bf(v) : v;
    }
    free(lut);
  }
  free(X);
  free(Xg);
}

/* torch.argmax semantics: first index of the maximum, NaN counts as maximum. */
void orc_argmax(const float* logits, int64_t B, int64_t V, int64_t* out) {
  for (int64_t b = 0; b < B; ++b) {
    const float* r = logits + b * V;
    int64_t bi = 0;
    for (int64_t i = 1; i < V; ++i) {
      const float a = r[i], c = r[bi];
      if (c != c) break;
      if (a != a || a > c) bi = i;
    }
    out[b] = bi;
  }
}

/* Reference: kernels/sampler.py:24-103 (top-k, temperature softmax, nucleus,
 * inverse CDF with the caller's uniform). */
void orc_fused_sample(const float* logits, int64_t B, int64_t V, const float* u, float temperature, float top_p,
                      int64_t K, int64_t* out) {
  const float inv_t = (float)(1.0 / (double)temperature);
  float* kv = (float*)malloc(sizeof(float) * K);
  int64_t* ki = (int64_t*)malloc(sizeof(int64_t) * K);
  unsigned char* used = (unsigned char*)malloc(V);
  float* p = (float*)malloc(sizeof(float) * K);
  for (int64_t b = 0; b < B; ++b) {
    const float* r = logits + b * V;
    memset(used, 0, V);
    for (int64_t j = 0; j < K; ++j) {
      int64_t bi = -1;
      for (int64_t i = 0; i < V; ++i)
        if (!used[i] && (bi < 0 || r[i] > r[bi])) bi = i;
      used[bi] = 1;
      kv[j] = r[bi];
      ki[j] = bi;
    }
    for (int64_t j = 0; j < K; ++j) p[j] = orc_exp((kv[j] - kv[0]) * inv_t);
    const float sum = orc_r128_sum(p, K);
    for (int64_t j = 0; j < K; ++j) p[j] = p[j] / sum;
    float cum = 0.0f;
    for (int64_t j = 0; j < K; ++j) {
      const float pj = p[j];
      cum = cum + pj;
      p[j] = (cum - pj <= top_p) ? pj : 0.0f;
    }
    const float total = orc_r128_sum(p, K);
    const float uu = u[b] * total;
    cum = 0.0f;
    int64_t pick = 0;
    for (int64_t j = 0; j < K; ++j) {
      cum = cum + p[j];
      if (cum <= uu) ++pick;
    }
    if (pick > K - 1) pick = K - 1;
    out[b] = ki[pick];
  }
  free(kv); free(ki); free(used); free(p);
}

/* Reference: kernels/rtn4.py:27-47 (gather + dequant c*s + b in fp32). */
void orc_rtn4_embedding(const int64_t* ids, int64_t B, const uint32_t* codes, const float* scales,
                        const float* biases, int64_t V, int64_t H, int64_t G, int out_bf16, float* out) {
  const int64_t ng = H / G;
  for (int64_t b = 0; b < B; ++b) {
    const int64_t id = ids[b];
    for (int64_t k = 0; k < H; ++k) {
      float v = 0.0f;
      if (id >= 0 && id < V) {
        const float c = (float)((codes[id * (H / 8) + k / 8] >> (4 * (k & 7))) & 15u);
        const float s = scales[id * ng + k / G];
        const float bb = biases ? biases[id * ng + k / G] : -8.0f * s;
        v = c * s + bb;
      }
      out[b * H + k] = out_bf16 ? bf(v) : v;
    }
  }
}

/* ------------------------------------------------------- synthetic ---- */
/* Same generator as the CUDA library's maple_synth_* (integer hashing, one
 * fp32 multiply-add, one rounding), written independently. */
static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
static inline uint64_t skey(uint64_t seed, uint64_t stream) { return mix64(mix64(seed) ^ (stream * 0x9E3779B97F4A7C15ULL)); }
static inline uint64_t hat(uint64_t key, uint64_t i) { return mix64(key ^ (i * 0xD1B54A32D192ED03ULL)); }
static inline float ncst(double scale) { return (float)(scale / sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0)); }
static inline float nat(uint64_t key, uint64_t i, float c) {
  const uint64_t h = hat(key, i);
  const int s = (int)(h & 0xffff) + (int)((h >> 16) & 0xffff) + (int)((h >> 32) & 0xffff) + (int)(h >> 48);
  return (float)(s - 131070) * c;
}

void orc_synth_ternary(uint64_t seed, uint64_t stream, int64_t n_words, uint32_t* out) {
  const uint64_t key = skey(seed, stream);
#pragma omp parallel for schedule(static)
  for (int64_t w = 0; w < n_words; ++w) {
    uint32_t word = 0;
    for (int q = 0; q < 4; ++q) {
      const uint64_t h = hat(key, 4 * (uint64_t)w + q);
      for (int j = 0; j < 4; ++j) {
        const uint32_t u = (uint32_t)((h >> (16 * j)) & 0xffffu);
        const uint32_t code = u < 26214u ? 1u : (u < 45875u ? 0u : 2u);
        word |= code << (2 * (4 * q + j));
      }
    }
    out[w] = word;
  }
}

/* out_bf16: round each value to bf16 (stored as fp32). */
void orc_synth_normal(uint64_t seed, uint64_t stream, int64_t n, double scale, float offset, int use_abs,
                      int out_bf16, float* out) {
  const uint64_t key = skey(seed, stream);
  const float c = ncst(scale);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float v = nat(key, (uint64_t)i, c);
    if (use_abs) v = fabsf(v);
    v = v + offset;
    out[i] = out_bf16 ? bf(v) : v;
  }
}

void orc_synth_rtn4_sym(uint64_t seed, uint64_t stream, int64_t rows, int64_t k, int64_t group, double scale,
                        uint32_t* codes, float* scales) {
  const uint64_t key = skey(seed, stream);
  const float c = ncst(scale);
  const int64_t ng = k / group;
#pragma omp parallel for schedule(static)
  for (int64_t rg = 0; rg < rows * ng; ++rg) {
    const int64_t r = rg / ng, g = rg % ng;
    const int64_t base = r * k + g * group;
    float amax = 0.0f;
    for (int64_t i = 0; i < group; ++i) amax = fmaxf(amax, fabsf(nat(key, (uint64_t)(base + i), c)));
    const float sc = amax / 7.0f;
    for (int64_t w = 0; w < group / 8; ++w) {
      uint32_t word = 0;
      for (int j = 0; j < 8; ++j) {
        float q = 0.0f;
        if (sc > 0.0f) q = fminf(fmaxf(rintf(nat(key, (uint64_t)(base + 8 * w + j), c) / sc), -8.0f), 7.0f);
        word |= (uint32_t)((int)q + 8) << (4 * j);
      }
      codes[(base >> 3) + w] = word;
    }
    scales[rg] = bf(sc);
  }
}

void orc_synth_tokens(uint64_t seed, uint64_t stream, int64_t n, int64_t vocab, int64_t* out) {
  const uint64_t key = skey(seed, stream);
  for (int64_t i = 0; i < n; ++i) out[i] = (int64_t)(hat(key, (uint64_t)i) % (uint64_t)vocab);
}

/* ------------------------------------------------ balanced k-means ---- */
/* Reference: src/maple_run/flash_head.py:30-110 (_balanced_spherical_kmeans),
 * restated in the canonical arithmetic of the CUDA k-means
 * (maple_flash_dgx_spark_b200/csrc/kmeans.cu): a similarity is the fp32 dot
 * accumulated over k = 0..d-1 in order from 0.0f with fmaf; a centroid is the
 * fp32 sum of its members' rows in ascending row order (plain adds), divided
 * by the member count (at least 1), then divided by (sqrt(R128 sum of
 * squares) + 1e-8); the objective is the mean of the members' similarities
 * to their centroids, summed in double within blocks of 1024 rows in order
 * and then over the blocks in order. */
void orc_km_dots(const float* a, int64_t na, const float* b, int64_t nb, int64_t d, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < na; ++i) {
    const float* ar = a + i * d;
    for (int64_t j = 0; j < nb; ++j) {
      const float* br = b + j * d;
      float acc = 0.0f;
      for (int64_t k = 0; k < d; ++k) acc = fmaf(ar[k], br[k], acc);
      out[i * nb + j] = acc;
    }
  }
}

void orc_km_normalize(float* v, int64_t rows, int64_t d) {
  for (int64_t j = 0; j < rows; ++j) {
    float* r = v + j * d;
    const float nrm = sqrtf(orc_r128_sumsq(r, d)) + 1e-8f;
    for (int64_t k = 0; k < d; ++k) r[k] = r[k] / nrm;
  }
}

void orc_km_update(const float* w, int64_t n, int64_t d, const int32_t* labels, int64_t c, float* cent) {
  int64_t* cnt = (int64_t*)calloc((size_t)c, sizeof(int64_t));
  memset(cent, 0, (size_t)(c * d) * sizeof(float));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t l = labels[i];
    cnt[l] += 1;
    float* cr = cent + l * d;
    const float* wr = w + i * d;
    for (int64_t k = 0; k < d; ++k) cr[k] = cr[k] + wr[k];
  }
  for (int64_t j = 0; j < c; ++j) {
    const float cf = (float)(cnt[j] > 0 ? cnt[j] : 1);
    float* cr = cent + j * d;
    for (int64_t k = 0; k < d; ++k) cr[k] = cr[k] / cf;
  }
  orc_km_normalize(cent, c, d);
  free(cnt);
}

double orc_km_objective(const float* w, int64_t n, int64_t d, const int32_t* labels, const float* cent) {
  double total = 0.0;
  for (int64_t b0 = 0; b0 < n; b0 += 1024) {
    double part = 0.0;
    const int64_t b1 = b0 + 1024 < n ? b0 + 1024 : n;
    for (int64_t i = b0; i < b1; ++i) {
      const float* wr = w + i * d;
      const float* cr = cent + (int64_t)labels[i] * d;
      float acc = 0.0f;
      for (int64_t k = 0; k < d; ++k) acc = fmaf(wr[k], cr[k], acc);
      part += (double)acc;
    }
    total += part;
  }
  return total / (double)n;
}
