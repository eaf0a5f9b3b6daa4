/* CPU oracle (TEST INFRASTRUCTURE ONLY): scalar restatement of the reference engine's
 * arithmetic for the speculative greedy-decode hot path.  Every loop keeps the reference's
 * fp32 operation order; "fused" below marks a place where the reference, as compiled by its
 * own build flags (g++ -O3 -march=native, default -ffp-contract=fast), turns a*b+c into one
 * FMA, which this file states explicitly with fmaf()/fma().  Build with -ffp-contract=off.
 *
 * Reference files are cited by their path inside the reference project.
 */
#include "g4_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- bf16 helpers: gemma4_engine.cpp:33-35 (f2bf RNE with NaN quieting), :37-42 (rbf8) ---- */
float or_bf2f(uint16_t b) { uint32_t u = (uint32_t)b << 16; float f; memcpy(&f, &u, 4); return f; }
uint16_t or_f2bf(float f) {
  uint32_t u; memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float or_r16(float f) { return or_bf2f(or_f2bf(f)); }

/* horizontal sum of 8 lanes in the order of w4g32_avx2.h:41-44 (hsum) and
 * bf16_exp3_head.h:78-81 (hsum8): ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)). */
static float hsum8(const float v[8]) {
  float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
  return (a0 + a1) + (a2 + a3);
}

/* ---- W4G32 float GEMM ----
 * w4g32_avx2.h:20-23 (prep_x: even/odd split, sequential group sums),
 * :65-96 (gemm_rows_tile<MT>): lane j of group g multiplies element 2j (low nibble of byte j),
 * then fma 16+2j (low nibble of byte 8+j), 2j+1 (high nibble of byte j), 17+2j (high nibble of
 * byte 8+j); row_j = fma(a_j, scale, row_j); off = fma(scale, gsum, off) (fused by the
 * reference build); y = hsum(row) - 8*off.  Used by lin_task (gemma4_engine.cpp:243-255). */
void or_w4g32_gemm(const uint8_t* W, const uint16_t* S, const float* X, int M, int N, int K, float* Y) {
  const int G = K / 32;
  float* gs = (float*)malloc(sizeof(float) * (size_t)M * G);
  for (int m = 0; m < M; ++m)
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
      for (int i = 0; i < 32; ++i) s += X[(size_t)m * K + g * 32 + i];
      gs[(size_t)m * G + g] = s;
    }
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    const uint8_t* w = W + (size_t)n * (K / 2);
    const uint16_t* s = S + (size_t)n * G;
    for (int m = 0; m < M; ++m) {
      const float* x = X + (size_t)m * K;
      float row[8] = {0, 0, 0, 0, 0, 0, 0, 0}, off = 0.f;
      for (int g = 0; g < G; ++g) {
        const uint8_t* p = w + (size_t)g * 16;
        const float* xg = x + g * 32;
        const float sc = or_bf2f(s[g]);
        for (int j = 0; j < 8; ++j) {
          float a = (float)(p[j] & 15) * xg[2 * j];
          a = fmaf((float)(p[8 + j] & 15), xg[16 + 2 * j], a);
          a = fmaf((float)(p[j] >> 4), xg[2 * j + 1], a);
          a = fmaf((float)(p[8 + j] >> 4), xg[17 + 2 * j], a);
          row[j] = fmaf(a, sc, row[j]);
        }
        off = fmaf(sc, gs[(size_t)m * G + g], off); /* fused */
      }
      Y[(size_t)m * N + n] = hsum8(row) - 8.f * off;
    }
  }
  free(gs);
}

/* ---- W4A8 ----
 * w4a8_avx2.h:30-42 (quant): amax over the 32-group, sx = amax/127, inv = sx>0 ? 1/sx : 0,
 * q = RNE(x*inv) saturated to int16 then int8, sum = sum of the unsaturated int32 values. */
static int32_t cvt_rne(float v) {
  if (!(v > -2147483648.f && v < 2147483648.f)) return INT32_MIN; /* cvtps_epi32 "indefinite" */
  return (int32_t)nearbyintf(v);
}
void or_w4a8_quant(const float* X, int M, int K, int8_t* q, float* sx, int32_t* sum) {
  const int G = K / 32;
  for (int m = 0; m < M; ++m)
    for (int g = 0; g < G; ++g) {
      const float* p = X + (size_t)m * K + g * 32;
      float amax = 0.f;
      for (int i = 0; i < 32; ++i) { float a = fabsf(p[i]); amax = a > amax ? a : amax; }
      const float s = amax / 127.0f, inv = s > 0 ? 1.0f / s : 0.0f;
      int32_t tot = 0;
      for (int i = 0; i < 32; ++i) {
        int32_t r = cvt_rne(p[i] * inv);
        tot += r;
        int32_t r16 = r < -32768 ? -32768 : (r > 32767 ? 32767 : r);
        q[(size_t)m * K + g * 32 + i] = (int8_t)(r16 < -128 ? -128 : (r16 > 127 ? 127 : r16));
      }
      sx[(size_t)m * G + g] = s;
      sum[(size_t)m * G + g] = tot;
    }
}
/* w4a8_avx2.h:46-60 (tile<MT>): exact integer group dot minus 8*sum, then
 * row = fma(float(a32), sw*sx, row) over groups in order (repack_tiles :20-27 only moves bytes). */
void or_w4a8_gemm(const uint8_t* W, const uint16_t* S, const int8_t* q, const float* sx,
                  const int32_t* sum, int M, int N, int K, float* Y) {
  const int G = K / 32;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    const uint8_t* w = W + (size_t)n * (K / 2);
    for (int m = 0; m < M; ++m) {
      float row = 0.f;
      for (int g = 0; g < G; ++g) {
        int32_t a = 0;
        for (int i = 0; i < 16; ++i) {
          const uint8_t b = w[g * 16 + i];
          a += (int32_t)(b & 15) * q[(size_t)m * K + g * 32 + 2 * i];
          a += (int32_t)(b >> 4) * q[(size_t)m * K + g * 32 + 2 * i + 1];
        }
        a -= 8 * sum[(size_t)m * G + g];
        const float sc = or_bf2f(S[(size_t)n * G + g]) * sx[(size_t)m * G + g];
        row = fmaf((float)a, sc, row);
      }
      Y[(size_t)m * N + n] = row;
    }
  }
}

/* ---- bf16-exp3 packed head ----
 * codebook: gemma4_engine.cpp:1232-1234 (exponent histogram, stable sort by count, top 8);
 * pack: bf16_exp3_head.h:26-49; dot: rows_tile :84-107 (lane j takes weights j, 16+j, 8+j, 24+j
 * of each group in that order, then hsum8, then the CSR exception patches). */
void or_bf16p_codebook(const uint16_t* E, int64_t count, uint8_t cb8[8]) {
  int64_t hist[256]; memset(hist, 0, sizeof hist);
  for (int64_t i = 0; i < count; ++i) hist[(E[i] >> 7) & 0xFF]++;
  int ord[256]; for (int i = 0; i < 256; ++i) ord[i] = i;
  for (int i = 1; i < 256; ++i) { /* stable insertion sort, descending count */
    int v = ord[i], j = i - 1;
    while (j >= 0 && hist[ord[j]] < hist[v]) { ord[j + 1] = ord[j]; --j; }
    ord[j + 1] = v;
  }
  for (int i = 0; i < 8; ++i) cb8[i] = (uint8_t)ord[i];
}
static int cb_index(const uint8_t cb8[8], int e, int* exc) {
  for (int i = 0; i < 8; ++i) if (cb8[i] == e) { *exc = 0; return i; }
  int best = 0, bd = 1 << 30;
  for (int i = 0; i < 8; ++i) { int dd = abs((int)cb8[i] - e); if (dd < bd) { bd = dd; best = i; } }
  *exc = 1; return best;
}
int64_t or_bf16p_count(const uint16_t* E, int N, int K, const uint8_t cb8[8], int64_t* exc_ptr) {
  exc_ptr[0] = 0;
  for (int n = 0; n < N; ++n) {
    int64_t c = 0;
    for (int k = 0; k < K; ++k) { int exc; cb_index(cb8, (E[(size_t)n * K + k] >> 7) & 0xFF, &exc); c += exc; }
    exc_ptr[n + 1] = exc_ptr[n] + c;
  }
  return exc_ptr[N];
}
void or_bf16p_pack(const uint16_t* E, int N, int K, const uint8_t cb8[8], uint8_t* data,
                   const int64_t* exc_ptr, uint16_t* exc_col, float* exc_delta) {
  const int G = K / 32;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    int64_t e_out = exc_ptr[n];
    for (int g = 0; g < G; ++g) {
      uint8_t* d = data + ((size_t)n * G + g) * 44;
      uint32_t pl[3] = {0, 0, 0};
      for (int j = 0; j < 32; ++j) {
        const uint16_t w = E[(size_t)n * K + g * 32 + j];
        const int sign = w >> 15, e = (w >> 7) & 0xFF, m = w & 0x7F;
        int exc; const int idx = cb_index(cb8, e, &exc);
        if (exc) {
          const uint16_t dec = (uint16_t)((sign << 15) | (cb8[idx] << 7) | m);
          exc_col[e_out] = (uint16_t)(g * 32 + j);
          exc_delta[e_out] = or_bf2f(w) - or_bf2f(dec);
          ++e_out;
        }
        d[j] = (uint8_t)((sign << 7) | m);
        for (int k = 0; k < 3; ++k) pl[k] |= (uint32_t)((idx >> k) & 1) << j;
      }
      memcpy(d + 32, pl, 12);
    }
  }
}
static float bf16p_weight(const uint8_t* d, const uint8_t cb8[8], int j) {
  uint32_t pl[3]; memcpy(pl, d + 32, 12);
  const int idx = (int)((pl[0] >> j) & 1) | (int)(((pl[1] >> j) & 1) << 1) | (int)(((pl[2] >> j) & 1) << 2);
  const uint16_t b = (uint16_t)(((d[j] & 0x80) << 8) | (cb8[idx] << 7) | (d[j] & 0x7F));
  return or_bf2f(b);
}
void or_bf16p_gemm(const uint8_t* data, const uint8_t cb8[8], const int64_t* exc_ptr,
                   const uint16_t* exc_col, const float* exc_delta, int N, int K,
                   const float* X, int M, float* Y) {
  const int G = K / 32;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    for (int m = 0; m < M; ++m) {
      const float* x = X + (size_t)m * K;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int g = 0; g < G; ++g) {
        const uint8_t* d = data + ((size_t)n * G + g) * 44;
        const float* xg = x + g * 32;
        for (int j = 0; j < 8; ++j) {
          acc[j] = fmaf(bf16p_weight(d, cb8, j), xg[j], acc[j]);
          acc[j] = fmaf(bf16p_weight(d, cb8, 16 + j), xg[16 + j], acc[j]);
          acc[j] = fmaf(bf16p_weight(d, cb8, 8 + j), xg[8 + j], acc[j]);
          acc[j] = fmaf(bf16p_weight(d, cb8, 24 + j), xg[24 + j], acc[j]);
        }
      }
      float y = hsum8(acc);
      for (int64_t e = exc_ptr[n]; e < exc_ptr[n + 1]; ++e) y += exc_delta[e] * x[exc_col[e]]; /* not fused under Zen 3 tuning */
      Y[(size_t)m * N + n] = y;
    }
  }
}

/* ---- softcap, threshold, argmax rule ----
 * cap: gemma4_engine.cpp:1410 (r16(30*tanhf(s/30))); calc_thr: :1455-1459 (= calc_thr_fast :454-459
 * without its -1e-4); pick: full-head argmax :1491-1497 and eval_row's rule :1469-1471, with ties
 * resolved to the lowest index. */
float or_cap(float s) { return or_r16(30.0f * tanhf(s / 30.0f)); }
float or_calc_thr(float L) {
  const float Lr = or_r16(L), cmL = or_cap(Lr);
  float lo = Lr - 64.0f, hi = Lr;
  for (int it = 0; it < 40; ++it) { const float mid = 0.5f * (lo + hi); if (or_cap(or_r16(mid)) == cmL) hi = mid; else lo = mid; }
  return hi - 0.25f;
}
int or_head_pick(const float* raw, int N) {
  float mx = -1e30f;
  for (int i = 0; i < N; ++i) { const float v = or_r16(raw[i]); mx = v > mx ? v : mx; }
  const float cm = or_cap(mx);
  for (int i = 0; i < N; ++i) { const float v = or_r16(raw[i]); if (v >= mx - 2.0f && or_cap(v) == cm) return i; }
  return -1;
}

/* ---- certified int4 head screen ----
 * build: gemma4_engine.cpp:1235-1244 (bf16 scale f2bf(amax/7), q = clamp(nearbyint(w/sc), -8, 7),
 * coef = sqrt(sum e^2) + 1e-4*sqrt(sum w^2) in double, fused).  The reference hard-codes K=1536;
 * this is the same procedure for any K. */
void or_screen_build(const uint16_t* E, int N, int K, uint8_t* W4, uint16_t* S4, float* coef) {
  const int G = K / 32;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    double e2 = 0, w2 = 0;
    for (int g = 0; g < G; ++g) {
      float amax = 0, w[32];
      for (int i = 0; i < 32; ++i) { w[i] = or_bf2f(E[(size_t)n * K + g * 32 + i]); const float a = fabsf(w[i]); amax = amax > a ? amax : a; }
      const uint16_t sb = or_f2bf(amax / 7.0f);
      const float sc = or_bf2f(sb);
      S4[(size_t)n * G + g] = sb;
      int qv[32];
      for (int i = 0; i < 32; ++i) {
        int v = sc > 0 ? (int)nearbyintf(w[i] / sc) : 0;
        v = v < -8 ? -8 : (v > 7 ? 7 : v);
        qv[i] = v + 8;
        const double d = (double)w[i] - (double)v * sc;
        e2 += d * d; w2 += (double)w[i] * w[i];
      }
      for (int i = 0; i < 16; ++i) W4[(size_t)n * (K / 2) + g * 16 + i] = (uint8_t)(qv[2 * i] | (qv[2 * i + 1] << 4));
    }
    coef[n] = (float)fma(1e-4, sqrt(w2), sqrt(e2)); /* fused */
  }
}
/* double sum of squares in the order of ss_avx2 (gemma4_engine.cpp:326-343): 16 partial sums
 * (4 accumulators x 4 lanes, stride 16), combined (s0+s1)+(s2+s3), then lanes (0+2)+(1+3). */
static double ss16(const float* x, int n) {
  double s[4][4] = {{0}};
  for (int i = 0; i < n; i += 16)
    for (int a = 0; a < 4; ++a)
      for (int b = 0; b < 4; ++b) { const double d = x[i + 4 * a + b]; s[a][b] = fma(d, d, s[a][b]); }
  double t[4];
  for (int b = 0; b < 4; ++b) t[b] = (s[0][b] + s[1][b]) + (s[2][b] + s[3][b]);
  return (t[0] + t[2]) + (t[1] + t[3]);
}
/* One verify row through the screen, stated without thread scheduling: hn = |h| (double), s = the
 * W4G32 screen dot (same arithmetic as gemm_rows_tile), lower = s - c*hn and upper = s + c*hn
 * (fused, screen_task :484-486), L = max lower, survivors = {n : upper >= calc_thr(L)} in index
 * order (eval_row :1453-1467).  Seeds (:1418-1449) can only raise the running bound early and do
 * not change L or the final survivor set.  More than lim survivors means fallback (-1). */
float or_hnorm(const float* h, int K) { return (float)sqrt(ss16(h, K)); }
/* seed lower bound (:1418-1449): max over seed rows of s - c*hn (fused). */
float or_seed_bound(const uint8_t* W4, const uint16_t* S4, const float* coef, int K, const float* h,
                    const int* seeds, int nseeds) {
  const float hn = or_hnorm(h, K);
  float L = -1e30f;
  for (int i = 0; i < nseeds; ++i) {
    const int n = seeds[i];
    float s;
    or_w4g32_gemm(W4 + (size_t)n * (K / 2), S4 + (size_t)n * (K / 32), h, 1, 1, K, &s);
    const float lw = fmaf(-coef[n], hn, s);
    L = lw > L ? lw : L;
  }
  return L;
}
int or_screen_row(const uint8_t* W4, const uint16_t* S4, const float* coef, int N, int K,
                  const float* h, const int* seeds, int nseeds, int lim, int* surv, float* L_out) {
  (void)seeds; (void)nseeds;
  const float hn = or_hnorm(h, K);
  float* s = (float*)malloc(sizeof(float) * (size_t)N);
  or_w4g32_gemm(W4, S4, h, 1, N, K, s);
  float L = -1e30f;
  for (int n = 0; n < N; ++n) { const float lw = fmaf(-coef[n], hn, s[n]); L = lw > L ? lw : L; }
  const float thr = or_calc_thr(L);
  int cnt = 0;
  for (int n = 0; n < N; ++n) {
    const float u = fmaf(coef[n], hn, s[n]);
    if (u >= thr) { if (cnt >= lim) { free(s); *L_out = L; return -1; } surv[cnt++] = n; }
  }
  free(s);
  *L_out = L;
  return cnt;
}

/* ---- split-KV decode attention ----
 * exp8: gemma4_engine.cpp:43-53 (Cephes-style expf, the reference's own polynomial).
 * attn_task :743-877 with T key chunks [kmin + t*len/T, kmin + (t+1)*len/T): scores are
 * hsum(s0+s1) of two 8-lane fma chains with stride 16 (:786-797); per-chunk max; weights
 * exp8(s - max) summed in key order; O = fma(w, v, O) in key order.  attn_merge :1019-1059:
 * M0 = max of the chunk maxima with L>0, l = sum L_t*expf(M_t-M0) in double, out =
 * r16((sum_t fma(O_t, sc_t)) * (float)(1/l)).  No softmax scale (q carries it). */
float or_exp8(float x) {
  x = fminf(fmaxf(x, -87.3f), 88.3f);
  const float fx = floorf(fmaf(x, 1.44269504088896341f, 0.5f));
  x = fmaf(-fx, 0.693359375f, x);
  x = fmaf(-fx, -2.12194440e-4f, x);
  const float z = x * x;
  float y = 1.9875691500E-4f;
  y = fmaf(y, x, 1.3981999507E-3f);
  y = fmaf(y, x, 8.3334519073E-3f);
  y = fmaf(y, x, 4.1665795894E-2f);
  y = fmaf(y, x, 1.6666665459E-1f);
  y = fmaf(y, x, 5.0000001201E-1f);
  y = fmaf(y, z, x + 1.0f);
  const uint32_t n = (uint32_t)(((int32_t)fx + 127) << 23);
  float p; memcpy(&p, &n, 4);
  return y * p;
}
/* gemma4_engine.cpp:54-60 (gelu8: tanh-GELU through exp8). */
float or_gelu(float x) {
  const float x3 = (x * x) * x;
  const float u = 0.7978845608028654f * fmaf(0.044715f, x3, x);
  const float e = or_exp8(2.0f * u);
  const float th = 1.0f - 2.0f / (e + 1.0f);
  return (0.5f * x) * (1.0f + th);
}
static float dot16(const float* q, const uint16_t* k, int hd) {
  float s0[8] = {0}, s1[8] = {0}, t[8];
  for (int i = 0; i < hd; i += 16)
    for (int l = 0; l < 8; ++l) {
      s0[l] = fmaf(q[i + l], or_bf2f(k[i + l]), s0[l]);
      s1[l] = fmaf(q[i + 8 + l], or_bf2f(k[i + 8 + l]), s1[l]);
    }
  for (int l = 0; l < 8; ++l) t[l] = s0[l] + s1[l];
  return hsum8(t);
}
void or_attn_splitkv(const uint16_t* Kc, const uint16_t* Vc, int hd, int nh, int M,
                     const float* q, const int* pos, const int* lo, int kmin, int kmax,
                     int T, float* out) {
  const int len = kmax - kmin + 1;
  float* AM = (float*)malloc(sizeof(float) * (size_t)T * M * nh);
  float* AL = (float*)malloc(sizeof(float) * (size_t)T * M * nh);
  float* AO = (float*)calloc((size_t)T * M * nh * hd, sizeof(float));
  float* S = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1) * M * nh);
  for (int t = 0; t < T; ++t) {
    const int c0 = kmin + (int)((long)t * len / T), c1 = kmin + (int)((long)(t + 1) * len / T);
    for (int i = 0; i < M * nh; ++i) { AM[(size_t)t * M * nh + i] = -1e30f; }
    for (int p = c0; p < c1; ++p)
      for (int m = 0; m < M; ++m) {
        if (!(p >= lo[m] && p <= pos[m])) continue;
        for (int h = 0; h < nh; ++h) {
          const float sc = dot16(q + ((size_t)m * nh + h) * hd, Kc + (size_t)p * hd, hd);
          S[((size_t)(p - kmin) * M + m) * nh + h] = sc;
          float* am = &AM[((size_t)t * M + m) * nh + h];
          *am = (*am < sc) ? sc : *am;
        }
      }
    for (int m = 0; m < M; ++m)
      for (int h = 0; h < nh; ++h) {
        float l8 = 0.f;
        float* o = AO + (((size_t)t * M + m) * nh + h) * hd;
        const float mx = AM[((size_t)t * M + m) * nh + h];
        for (int p = c0; p < c1; ++p) {
          if (!(p >= lo[m] && p <= pos[m])) continue;
          const float w = or_exp8(S[((size_t)(p - kmin) * M + m) * nh + h] - mx);
          l8 += w;
          for (int i = 0; i < hd; ++i) o[i] = fmaf(w, or_bf2f(Vc[(size_t)p * hd + i]), o[i]);
        }
        AL[((size_t)t * M + m) * nh + h] = (lo[m] > pos[m]) ? 0.0f : l8;
      }
  }
  for (int m = 0; m < M; ++m)
    for (int h = 0; h < nh; ++h) {
      float M0 = -1e30f;
      for (int t = 0; t < T; ++t) {
        const size_t ix = ((size_t)t * M + m) * nh + h;
        if (AL[ix] > 0) M0 = M0 < AM[ix] ? AM[ix] : M0;
      }
      double l = 0; float scs[64]; int act[64], na = 0;
      for (int t = 0; t < T; ++t) {
        const size_t ix = ((size_t)t * M + m) * nh + h;
        if (!(AL[ix] > 0)) continue;
        const float sc = expf(AM[ix] - M0);
        l += (double)AL[ix] * sc;
        scs[na] = sc; act[na] = t; ++na;
      }
      const float inv = (float)(1.0 / l);
      for (int i = 0; i < hd; ++i) {
        float acc = 0.f;
        for (int k = 0; k < na; ++k) acc = fmaf(AO[(((size_t)act[k] * M + m) * nh + h) * hd + i], scs[k], acc);
        out[((size_t)m * nh + h) * hd + i] = or_r16(acc * inv);
      }
    }
  free(AM); free(AL); free(AO); free(S);
}

/* OpenMP threads of the restatement's parallel loops (the process's OMP_NUM_THREADS may be fixed by
 * a launcher). */
#include <omp.h>
void or_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
int or_get_threads(void) { return omp_get_max_threads(); }
