/* CPU oracle, end to end (TEST INFRASTRUCTURE ONLY): the synthetic Gemma-style E2B model of
 * BASELINE.json configs[4] with its MTP drafter and the chain-mode speculative loop, restated in
 * plain C on top of the kernel restatements of g4_oracle.c.  The model and its seeded weights are
 * defined in gemma4-e2b-laptop-cpu_b200/csrc/g4_model.cuh ("g4-e2b-synth v1"); the layer is the
 * reference's fwd (gemma4_engine.cpp:1256-1502) without PLE, the draft step its draft_step
 * (:1534-1563) at the target's width, the loop its run_req (:1582-1663) in chain mode.
 *
 * The head is evaluated over the full exact head: the certified screen provably keeps every row
 * that can win, so the screened pick equals the full pick (tested separately).
 */
#include "g4_oracle.h"
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---- weight generator (g4_model.cuh) */
static uint64_t smix(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static uint64_t wh(uint64_t seed, uint64_t id, uint64_t i) { return smix((seed * 0x100000001B3ull) ^ (id << 40) ^ i); }
static float wnorm(uint64_t h) {
  const int s = (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48) - 131070;
  return (float)s * 2.642868e-5f;
}
/* int4 byte: both nibbles uniform in [0, 15], i.e. q = t - 8 uniform in [-8, 7] */
static uint8_t w4_byte(uint64_t h) { return (uint8_t)(h & 0xFF); }
static uint32_t perm_token(uint32_t i, uint32_t vocab) { return (uint32_t)(((uint64_t)i * 0x9E3779B1ull + 12345ull) & (uint64_t)(vocab - 1)); }
enum { T_Q = 0, T_K = 1, T_V = 2, T_O = 3, T_GATE = 4, T_UP = 5, T_DOWN = 6, T_IN_LN = 8, T_POST_ATTN = 9, T_PRE_FF = 10,
       T_POST_FF = 11, T_QN = 12, T_KN = 13, T_PG = 7, T_PP = 14, T_POST_PLE = 15 };
#define T_PLE 1002ull
#define T_PLPROJ 1003ull
#define T_PLNORM 1004ull
#define PLE_D 256 /* per-layer input width (PD, gemma4_engine.cpp:1222) */
#define T_SCALES 0x100000ull
#define T_EMBED 1000ull
#define T_FNORM 1001ull
#define T_DPRE 2000ull
#define T_DPOST 2001ull
#define T_DCENT 2002ull
#define T_DNORM 2003ull
static uint64_t layer_id(int l, uint64_t w) { return 16ull * (uint64_t)l + w; }
static uint64_t dlayer_id(int l, uint64_t w) { return 2100ull + 16ull * (uint64_t)l + w; }

typedef struct { uint8_t* w; uint16_t* s; int N, K; void* ref; } Lin;
/* Kernel hooks: when set, the linears, the split-KV attention and the exact head run through these
 * (bench.py points them at the reference's own AVX2 kernels in oracle/_ref/libg4ref.so, driven by
 * the reference's thread pool), the rest of the restatement stays as it is. */
typedef struct {
  void* (*lin_prepare)(const uint8_t* W, const uint16_t* S, int N, int K);
  void (*lin_run)(void* h, const float* X, int M, float* Y, int i8);
  void (*attn)(const uint16_t* Kc, const uint16_t* Vc, int hd, int nh, int M, const float* q, const int* pos,
               const int* lo, int kmin, int kmax, float* out);
  void* (*head_prepare)(const uint16_t* E, int N, int K, const uint8_t* cb8);
  void (*head_run)(void* h, const float* X, int M, float* Y);
  /* the tiled prefill attention (variant 0) of a whole block; may be NULL */
  void (*attn_tile)(const uint16_t* Kc, const uint16_t* Vc, int hd, int sliding, const float* q, int qstride, int pos0,
                    int M, float* att);
} or_e2e_hooks;
typedef struct {
  Lin qkv, o, gu, down;
  float *in_ln, *post_attn, *pre_ff, *post_ff, *qn, *kn;
  int global;
  float scalar;
  Lin pg, pp;      /* per-layer input gate [PD][H] and projection [H][PD] (PLE) */
  float* post_ple; /* post_per_layer_input_norm (PLE) */
} TLayer;
typedef struct { Lin q, o, gu, down; float *in_ln, *post_attn, *pre_ff, *post_ff, *qn; int global; } DLayer;

typedef struct {
  int H, NL, I, V, NQ, HD, WINDOW, DL, DCENT, DTOP, DPER;
  int OWN; /* KV owners: layers [0, OWN) own a cache (0 = all) */
  int IS;  /* MLP width of the KV-shared layers (0 = I) */
  int ple; /* per-layer embeddings */
  int HDG;    /* head dim of the global layers (0 = HD; the E2B model: 512) */
  int HDM;    /* the larger of HD and HDG: the KV cache's slot width */
  int rope_q; /* global layers rotate the first quarter of their pair indices only (proportional RoPE) */
  uint16_t* PLEt; /* [V][NL * PD] bf16 */
  Lin plproj;     /* per_layer_model_projection [NL * PD][H] */
  float* plnorm;  /* per_layer_projection_norm [PD] */
  int ctx_max, prefill_block, k_draft, ngram, ngram_len, prefill_int8, decode_int8, attn_chunks, att_par, drafter;
  uint64_t seed;
  TLayer* L;
  DLayer* D;
  Lin dpre, dpost, dcent;
  float *fnorm, *dnorm;
  uint16_t* E;
  uint8_t cb[8];
  uint8_t* hdata;
  int64_t* exc_ptr;
  uint16_t* exc_col;
  float* exc_delta;
  uint16_t *Kc, *Vc;
  float *rc[2], *rs[2];
  int i8;
  int fake_n; /* ENGINE_FAKE_CTX positions before the prompt */
  /* decode state between or_e2e_decode calls */
  int* seq;
  int seq_len, seq_cap, P, conf, stopped;
  float* hprev;
  int st[4];
  /* optional kernel hooks (or_e2e_set_hooks): the reference's own compiled kernels */
  or_e2e_hooks hk;
  void* head_ref;
} Model;

/* owner_of (gemma4_engine.cpp:1251): the layer whose KV cache layer l reads - itself when it owns
 * one, else the last owner of its type (l % 5 == 4: global). */
static int owns(const Model* m, int l) { return m->OWN <= 0 || l < m->OWN; }
static int mlp_of(const Model* m, int l) { return (!owns(m, l) && m->IS > 0) ? m->IS : m->I; }
/* layer l's head dim (a.hd, gemma4_engine.cpp:1224: 256 sliding, 512 global in the E2B model) */
static int hd_of(const Model* m, int l) { return (l % 5 == 4 && m->HDG > 0) ? m->HDG : m->HD; }
static int owner_of(const Model* m, int l) {
  if (owns(m, l)) return l;
  for (int j = m->OWN - 1; j >= 0; --j)
    if ((j % 5 == 4) == (l % 5 == 4)) return j;
  return -1;
}

static void gen_lin(Model* m, Lin* lin, const uint64_t* ids, const int* rows, int parts, int K) {
  int N = 0;
  for (int p = 0; p < parts; ++p) N += rows[p];
  lin->N = N; lin->K = K;
  lin->w = (uint8_t*)malloc((size_t)N * K / 2);
  lin->s = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)N * K / 32);
  size_t ro = 0, so = 0;
  for (int p = 0; p < parts; ++p) {
    const long long nb = (long long)rows[p] * K / 2, ns = (long long)rows[p] * K / 32;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < nb; ++i) lin->w[ro + i] = w4_byte(wh(m->seed, ids[p], (uint64_t)i));
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < ns; ++i)
      lin->s[so + i] = or_f2bf(fabsf(wnorm(wh(m->seed, ids[p] | T_SCALES, (uint64_t)i))) * 0.01f);
    ro += nb; so += ns;
  }
}
static float* gen_norm(Model* m, uint64_t id, int n, float mul) {
  float* p = (float*)malloc(sizeof(float) * n);
  for (int i = 0; i < n; ++i) p[i] = or_bf2f(or_f2bf((1.0f + 0.1f * wnorm(wh(m->seed, id, (uint64_t)i))) * mul));
  return p;
}

typedef struct {
  int hidden, n_layers, mlp, vocab, ctx_max, prefill_block, k_draft, ngram, ngram_len, prefill_int8, decode_int8;
  int head_screen, screen_lim, attn_chunks, att_par, drafter;
  unsigned long long seed;
  int kv_owners; /* layers [0, kv_owners) own a KV cache (0 = all), g4_engine_config's field */
  int mlp_shared; /* MLP width of the KV-shared layers (0 = mlp) */
  int ple;        /* per-layer embeddings (PD = 256 per layer) */
  int hd_global;  /* head dim of the global layers (0 = 256) */
  int rope_global_quarter; /* proportional RoPE in the global layers (partial_rotary_factor 0.25) */
} or_e2e_config;  /* g4_engine_config's first fields, then kv_owners, mlp_shared and ple */

void* or_e2e_create(const or_e2e_config* c) {
  Model* m = (Model*)calloc(1, sizeof(Model));
  m->H = c->hidden; m->NL = c->n_layers; m->I = c->mlp; m->V = c->vocab; m->NQ = 8; m->HD = 256; m->WINDOW = 512;
  m->DL = 4; m->DPER = 128; m->DCENT = c->vocab / 128; m->DTOP = m->DCENT < 32 ? m->DCENT : 32;
  m->ctx_max = c->ctx_max; m->prefill_block = c->prefill_block; m->k_draft = c->k_draft; m->ngram = c->ngram;
  m->ngram_len = c->ngram_len; m->prefill_int8 = c->prefill_int8; m->decode_int8 = c->decode_int8;
  m->attn_chunks = c->attn_chunks; m->att_par = c->att_par; m->drafter = c->drafter; m->seed = c->seed;
  m->OWN = c->kv_owners;
  m->IS = c->mlp_shared;
  m->ple = c->ple;
  m->HDG = c->hd_global > 0 ? c->hd_global : m->HD;
  m->HDM = m->HDG > m->HD ? m->HDG : m->HD;
  m->rope_q = c->rope_global_quarter;
  if (m->HDG != m->HD) m->drafter = 0; /* the drafter is built for one head size; off with wider global heads */
  const int H = m->H, QD = m->NQ * m->HD, I = m->I;
  m->L = (TLayer*)calloc(m->NL, sizeof(TLayer));
  for (int l = 0; l < m->NL; ++l) {
    TLayer* t = &m->L[l];
    t->global = (l % 5 == 4);
    t->scalar = 1.0f;
    /* a KV-shared layer has the q projection only (no k/v projections, no k_norm) */
    const int hdl = hd_of(m, l), QDl = m->NQ * hdl;
    { uint64_t ids[3] = {layer_id(l, T_Q), layer_id(l, T_K), layer_id(l, T_V)}; int rows[3] = {QDl, hdl, hdl}; gen_lin(m, &t->qkv, ids, rows, owns(m, l) ? 3 : 1, H); }
    { uint64_t ids[1] = {layer_id(l, T_O)}; int rows[1] = {H}; gen_lin(m, &t->o, ids, rows, 1, QDl); }
    { const int Il = mlp_of(m, l); uint64_t ids[2] = {layer_id(l, T_GATE), layer_id(l, T_UP)}; int rows[2] = {Il, Il}; gen_lin(m, &t->gu, ids, rows, 2, H); }
    { uint64_t ids[1] = {layer_id(l, T_DOWN)}; int rows[1] = {H}; gen_lin(m, &t->down, ids, rows, 1, mlp_of(m, l)); }
    t->in_ln = gen_norm(m, layer_id(l, T_IN_LN), H, 1.f);
    t->post_attn = gen_norm(m, layer_id(l, T_POST_ATTN), H, 1.f);
    t->pre_ff = gen_norm(m, layer_id(l, T_PRE_FF), H, 1.f);
    t->post_ff = gen_norm(m, layer_id(l, T_POST_FF), H, 1.f);
    t->qn = gen_norm(m, layer_id(l, T_QN), hdl, 0.0625f);
    t->kn = owns(m, l) ? gen_norm(m, layer_id(l, T_KN), hdl, 1.f) : NULL;
    if (m->ple) {
      { uint64_t ids[1] = {layer_id(l, T_PG)}; int rows[1] = {PLE_D}; gen_lin(m, &t->pg, ids, rows, 1, H); }
      { uint64_t ids[1] = {layer_id(l, T_PP)}; int rows[1] = {H}; gen_lin(m, &t->pp, ids, rows, 1, PLE_D); }
      t->post_ple = gen_norm(m, layer_id(l, T_POST_PLE), H, 1.f);
    }
  }
  if (m->ple) {
    const long long NP = (long long)m->NL * PLE_D, PV = (long long)m->V * NP;
    { uint64_t ids[1] = {T_PLPROJ}; int rows[1] = {(int)NP}; gen_lin(m, &m->plproj, ids, rows, 1, H); }
    m->plnorm = gen_norm(m, T_PLNORM, PLE_D, 1.f);
    m->PLEt = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)PV);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < PV; ++i) m->PLEt[i] = or_f2bf(0.02f * wnorm(wh(m->seed, T_PLE, (uint64_t)i)));
  }
  m->fnorm = gen_norm(m, T_FNORM, H, 1.f);
  const long long EV = (long long)m->V * H;
  m->E = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)EV);
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < EV; ++i) m->E[i] = or_f2bf(0.02f * wnorm(wh(m->seed, T_EMBED, (uint64_t)i)));
  or_bf16p_codebook(m->E, EV, m->cb);
  m->exc_ptr = (int64_t*)malloc(sizeof(int64_t) * (m->V + 1));
  const int64_t ne = or_bf16p_count(m->E, m->V, H, m->cb, m->exc_ptr);
  m->hdata = (uint8_t*)malloc((size_t)m->V * (H / 32) * 44);
  m->exc_col = (uint16_t*)malloc(sizeof(uint16_t) * (ne > 0 ? ne : 1));
  m->exc_delta = (float*)malloc(sizeof(float) * (ne > 0 ? ne : 1));
  or_bf16p_pack(m->E, m->V, H, m->cb, m->hdata, m->exc_ptr, m->exc_col, m->exc_delta);
  if (m->drafter) {
    { uint64_t ids[1] = {T_DPRE}; int rows[1] = {H}; gen_lin(m, &m->dpre, ids, rows, 1, 2 * H); }
    { uint64_t ids[1] = {T_DPOST}; int rows[1] = {H}; gen_lin(m, &m->dpost, ids, rows, 1, H); }
    { uint64_t ids[1] = {T_DCENT}; int rows[1] = {m->DCENT}; gen_lin(m, &m->dcent, ids, rows, 1, H); }
    m->dnorm = gen_norm(m, T_DNORM, H, 1.f);
    m->D = (DLayer*)calloc(m->DL, sizeof(DLayer));
    for (int l = 0; l < m->DL; ++l) {
      DLayer* t = &m->D[l];
      t->global = (l == m->DL - 1);
      { uint64_t ids[1] = {dlayer_id(l, T_Q)}; int rows[1] = {QD}; gen_lin(m, &t->q, ids, rows, 1, H); }
      { uint64_t ids[1] = {dlayer_id(l, T_O)}; int rows[1] = {H}; gen_lin(m, &t->o, ids, rows, 1, QD); }
      { uint64_t ids[2] = {dlayer_id(l, T_GATE), dlayer_id(l, T_UP)}; int rows[2] = {I, I}; gen_lin(m, &t->gu, ids, rows, 2, H); }
      { uint64_t ids[1] = {dlayer_id(l, T_DOWN)}; int rows[1] = {H}; gen_lin(m, &t->down, ids, rows, 1, I); }
      t->in_ln = gen_norm(m, dlayer_id(l, T_IN_LN), H, 1.f);
      t->post_attn = gen_norm(m, dlayer_id(l, T_POST_ATTN), H, 1.f);
      t->pre_ff = gen_norm(m, dlayer_id(l, T_PRE_FF), H, 1.f);
      t->post_ff = gen_norm(m, dlayer_id(l, T_POST_FF), H, 1.f);
      t->qn = gen_norm(m, dlayer_id(l, T_QN), m->HD, 0.0625f);
    }
  }
  /* KV cache: one slot of ctx_max x HDM per layer, rows of the layer's head dim */
  const size_t kvn = (size_t)m->NL * m->ctx_max * m->HDM;
  m->Kc = (uint16_t*)calloc(kvn, sizeof(uint16_t));
  m->Vc = (uint16_t*)calloc(kvn, sizeof(uint16_t));
  /* RoPE tables per layer type (:1246-1247): pair index j < ra rotates at theta^(-2j/hd), the rest
   * not at all; ra = hd/2, or hd/8 for proportional RoPE in the global layers */
  for (int ty = 0; ty < 2; ++ty) {
    const double theta = ty ? 1e6 : 1e4;
    const int hdt = ty ? m->HDG : m->HD, hh = hdt / 2;
    const int ra = (int)(hdt * ((ty && m->rope_q) ? 0.25 : 1.0)) / 2;
    m->rc[ty] = (float*)malloc(sizeof(float) * (size_t)m->ctx_max * hh);
    m->rs[ty] = (float*)malloc(sizeof(float) * (size_t)m->ctx_max * hh);
    for (int p = 0; p < m->ctx_max; ++p)
      for (int j = 0; j < hh; ++j) {
        const double inv = j < ra ? 1.0 / pow(theta, (2.0 * j) / hdt) : 0.0;
        const double ang = p * inv;
        m->rc[ty][(size_t)p * hh + j] = (float)cos(ang);
        m->rs[ty][(size_t)p * hh + j] = (float)sin(ang);
      }
  }
  return m;
}

static void free_lin(Lin* l) { free(l->w); free(l->s); }
void or_e2e_destroy(void* mp) {
  Model* m = (Model*)mp;
  if (!m) return;
  for (int l = 0; l < m->NL; ++l) {
    TLayer* t = &m->L[l];
    free_lin(&t->qkv); free_lin(&t->o); free_lin(&t->gu); free_lin(&t->down);
    free(t->in_ln); free(t->post_attn); free(t->pre_ff); free(t->post_ff); free(t->qn); free(t->kn);
    free_lin(&t->pg); free_lin(&t->pp); free(t->post_ple);
  }
  free(m->L);
  free_lin(&m->plproj); free(m->plnorm); free(m->PLEt);
  if (m->D) {
    for (int l = 0; l < m->DL; ++l) {
      DLayer* t = &m->D[l];
      free_lin(&t->q); free_lin(&t->o); free_lin(&t->gu); free_lin(&t->down);
      free(t->in_ln); free(t->post_attn); free(t->pre_ff); free(t->post_ff); free(t->qn);
    }
    free(m->D);
    free_lin(&m->dpre); free_lin(&m->dpost); free_lin(&m->dcent); free(m->dnorm);
  }
  free(m->fnorm); free(m->E); free(m->hdata); free(m->exc_ptr); free(m->exc_col); free(m->exc_delta);
  free(m->Kc); free(m->Vc); free(m->seq); free(m->hprev);
  for (int t = 0; t < 2; ++t) { free(m->rc[t]); free(m->rs[t]); }
  free(m);
}

/* ---- row operations (gemma4_engine.cpp:326-402) */
static float rms_scale(const float* x, int n) {
  double s[4][4] = {{0}};
  for (int i = 0; i < n; i += 16)
    for (int a = 0; a < 4; ++a)
      for (int b = 0; b < 4; ++b) { const double d = x[i + 4 * a + b]; s[a][b] = fma(d, d, s[a][b]); }
  double t[4];
  for (int b = 0; b < 4; ++b) t[b] = (s[0][b] + s[1][b]) + (s[2][b] + s[3][b]);
  const double ss = (t[0] + t[2]) + (t[1] + t[3]);
  return 1.0f / sqrtf((float)(ss / n) + 1e-6f);
}
static void rmsnorm(const float* x, const float* w, int n, float* y, int round) {
  const float r = rms_scale(x, n);
  for (int i = 0; i < n; ++i) { const float v = (x[i] * r) * w[i]; y[i] = round ? or_r16(v) : v; }
}
/* M rows of rmsnorm (the checker of g4_rmsnorm). */
void or_rmsnorm(const float* x, const float* w, int M, int n, float* y, int round) {
  for (int m = 0; m < M; ++m) rmsnorm(x + (size_t)m * n, w, n, y + (size_t)m * n, round);
}
static void rope(float* h, const float* cs, const float* sn, int hd) {
  const int hh = hd / 2;
  for (int j = 0; j < hh; ++j) {
    const float u = h[j], w = h[j + hh];
    h[j] = fmaf(u, cs[j], -(w * sn[j]));
    h[j + hh] = fmaf(w, cs[j], u * sn[j]);
  }
}
static void rms_r16_w(float* x, const float* w, int n) {
  const float r = rms_scale(x, n);
  for (int i = 0; i < n; ++i) x[i] = or_r16(w ? (x[i] * r) * w[i] : x[i] * r);
}

static void lin(Model* m, const Lin* w, const float* X, int M, float* Y, int force_i8) {
  if (m->hk.lin_run && w->ref) {
    m->hk.lin_run(w->ref, X, M, Y, (m->i8 && M >= 2) || force_i8);
    return;
  }
  if ((m->i8 && M >= 2) || force_i8) {
    int8_t* q = (int8_t*)malloc((size_t)M * w->K);
    float* sx = (float*)malloc(sizeof(float) * (size_t)M * (w->K / 32));
    int32_t* sm = (int32_t*)malloc(sizeof(int32_t) * (size_t)M * (w->K / 32));
    or_w4a8_quant(X, M, w->K, q, sx, sm);
    or_w4a8_gemm(w->w, w->s, q, sx, sm, M, w->N, w->K, Y);
    free(q); free(sx); free(sm);
  } else {
    or_w4g32_gemm(w->w, w->s, X, M, w->N, w->K, Y);
  }
}

/* non-split attention for row m: variant 0 = attn_tile (:1061-1083), 1 = per-(m,h) (:1337-1355) */
static void attn_row(const Model* m, const uint16_t* Kc, const uint16_t* Vc, int hd, const float* q, int lo, int pos,
                     int variant, float* out) {
  const int len = pos - lo + 1;
  float* sc = (float*)malloc(sizeof(float) * len);
  for (int h = 0; h < m->NQ; ++h) {
    const float* qh = q + (size_t)h * hd;
    float mx = -1e30f;
    for (int p = lo; p <= pos; ++p) {
      const uint16_t* kr = Kc + (size_t)p * hd;
      float s;
      if (variant == 0) {
        float s0[8] = {0}, s1[8] = {0}, t[8];
        for (int i = 0; i < hd; i += 16)
          for (int l = 0; l < 8; ++l) { s0[l] = fmaf(qh[i + l], or_bf2f(kr[i + l]), s0[l]); s1[l] = fmaf(qh[i + 8 + l], or_bf2f(kr[i + 8 + l]), s1[l]); }
        for (int l = 0; l < 8; ++l) t[l] = s0[l] + s1[l];
        s = ((t[0] + t[4]) + (t[1] + t[5])) + ((t[2] + t[6]) + (t[3] + t[7]));
      } else {
        float sv[8] = {0};
        for (int i = 0; i < hd; i += 8)
          for (int l = 0; l < 8; ++l) sv[l] = fmaf(qh[i + l], or_bf2f(kr[i + l]), sv[l]);
        s = ((sv[0] + sv[4]) + (sv[1] + sv[5])) + ((sv[2] + sv[6]) + (sv[3] + sv[7]));
      }
      sc[p - lo] = s;
      mx = mx < s ? s : mx;
    }
    float den = 0.f;
    for (int p = 0; p < len; ++p) { sc[p] = variant == 0 ? or_exp8(sc[p] - mx) : expf(sc[p] - mx); den += sc[p]; }
    float* o = out + (size_t)h * hd;
    for (int i = 0; i < hd; ++i) o[i] = 0.f;
    if (variant == 0) {
      for (int p = 0; p < len; ++p)
        for (int i = 0; i < hd; ++i) o[i] = fmaf(sc[p], or_bf2f(Vc[(size_t)(lo + p) * hd + i]), o[i]);
      const float inv = 1.0f / den;
      for (int i = 0; i < hd; ++i) o[i] = or_r16(o[i] * inv);
    } else {
      for (int p = 0; p < len; ++p) {
        const float w = sc[p] / den;
        for (int i = 0; i < hd; ++i) o[i] = fmaf(w, or_bf2f(Vc[(size_t)(lo + p) * hd + i]), o[i]);
      }
      for (int i = 0; i < hd; ++i) o[i] = or_r16(o[i]);
    }
  }
  free(sc);
}

/* One target forward over M tokens at pos0 (fwd).  G[hf..] = greedy tokens, hbuf[hf..] = hidden. */
static void forward(Model* m, const int* toks, int M, int pos0, int want, int hf, int* G, float* hbuf) {
  const int H = m->H, QDM = m->NQ * m->HDM, ldmax = QDM + 2 * m->HDM;
  const int I = m->IS > m->I ? m->IS : m->I; /* buffer width: the widest MLP */
  float* x = (float*)malloc(sizeof(float) * (size_t)M * H);
  float* a = (float*)malloc(sizeof(float) * (size_t)M * H);
  float* qkv = (float*)malloc(sizeof(float) * (size_t)M * ldmax);
  float* att = (float*)malloc(sizeof(float) * (size_t)M * QDM);
  float* o = (float*)malloc(sizeof(float) * (size_t)M * H);
  float* gu = (float*)malloc(sizeof(float) * (size_t)M * 2 * I);
  float* act = (float*)malloc(sizeof(float) * (size_t)M * I);
  float* mlp_in = (float*)malloc(sizeof(float) * (size_t)M * H);
  const float sqrtH = sqrtf((float)H);
  for (int r = 0; r < M; ++r)
    for (int i = 0; i < H; ++i) x[(size_t)r * H + i] = or_r16(or_bf2f(m->E[(size_t)toks[r] * H + i]) * sqrtH);
  /* per-layer inputs (the int8 branch of :1270-1288): pr = per_layer_model_projection(x), then per
   * (row, layer) r16(pr / sqrt(H)), its RMS norm with per_layer_projection_norm, plus the table row
   * scaled by sqrt(256) = 16 and rounded, times 2^-0.5 */
  const int NP = m->NL * PLE_D;
  float* pli = NULL;
  float* pgv = NULL;
  float* g2 = NULL;
  if (m->ple) {
    float* pr = (float*)malloc(sizeof(float) * (size_t)M * NP);
    pli = (float*)malloc(sizeof(float) * (size_t)M * NP);
    pgv = (float*)malloc(sizeof(float) * (size_t)M * PLE_D);
    g2 = (float*)malloc(sizeof(float) * (size_t)M * PLE_D);
    lin(m, &m->plproj, x, M, pr, 0);
    const float s1 = 1.0f / sqrtf((float)H);
    float pj[PLE_D];
    for (int r = 0; r < M; ++r)
      for (int l = 0; l < m->NL; ++l) {
        float* prl = pr + (size_t)r * NP + (size_t)l * PLE_D;
        for (int i = 0; i < PLE_D; ++i) prl[i] = or_r16(prl[i] * s1);
        rmsnorm(prl, m->plnorm, PLE_D, pj, 0);
        const uint16_t* pel = m->PLEt + (size_t)toks[r] * NP + (size_t)l * PLE_D;
        for (int i = 0; i < PLE_D; ++i)
          pli[(size_t)r * NP + (size_t)l * PLE_D + i] = (pj[i] + or_r16(or_bf2f(pel[i]) * 16.0f)) * 0.70710678118f;
      }
    free(pr);
  }
  for (int l = 0; l < m->NL; ++l) {
    TLayer* t = &m->L[l];
    const int ty = t->global ? 1 : 0;
    const int ld = t->qkv.N; /* QD + 2 hd, or QD for a KV-shared layer */
    const int hd = hd_of(m, l), QD = m->NQ * hd;
    for (int r = 0; r < M; ++r) rmsnorm(x + (size_t)r * H, t->in_ln, H, a + (size_t)r * H, 0);
    lin(m, &t->qkv, a, M, qkv, 0);
    uint16_t* Kc = m->Kc + (size_t)owner_of(m, l) * m->ctx_max * m->HDM;
    uint16_t* Vc = m->Vc + (size_t)owner_of(m, l) * m->ctx_max * m->HDM;
    for (int r = 0; r < M; ++r) {
      const int pos = pos0 + r;
      const float* cs = m->rc[ty] + (size_t)pos * (hd / 2);
      const float* sn = m->rs[ty] + (size_t)pos * (hd / 2);
      float* qr = qkv + (size_t)r * ld;
      for (int h = 0; h < m->NQ; ++h) { rms_r16_w(qr + (size_t)h * hd, t->qn, hd); rope(qr + (size_t)h * hd, cs, sn, hd); }
      if (!owns(m, l)) continue; /* K and V come from the owner's cache */
      float* kr = qr + QD;
      float* vr = qr + QD + hd;
      rms_r16_w(kr, t->kn, hd); rope(kr, cs, sn, hd);
      rms_r16_w(vr, NULL, hd);
      for (int i = 0; i < hd; ++i) { Kc[(size_t)pos * hd + i] = or_f2bf(kr[i]); Vc[(size_t)pos * hd + i] = or_f2bf(vr[i]); }
    }
    if (M <= 4 && pos0 + M > m->att_par) {
      int pos[4], lo[4], kmin = 1 << 30;
      float* q = (float*)malloc(sizeof(float) * (size_t)M * QD);
      for (int r = 0; r < M; ++r) {
        pos[r] = pos0 + r;
        lo[r] = t->global ? 0 : (pos[r] - 511 > 0 ? pos[r] - 511 : 0);
        kmin = lo[r] < kmin ? lo[r] : kmin;
        memcpy(q + (size_t)r * QD, qkv + (size_t)r * ld, sizeof(float) * QD);
      }
      if (m->hk.attn) m->hk.attn(Kc, Vc, hd, m->NQ, M, q, pos, lo, kmin, pos0 + M - 1, att);
      else or_attn_splitkv(Kc, Vc, hd, m->NQ, M, q, pos, lo, kmin, pos0 + M - 1, m->attn_chunks, att);
      free(q);
    } else {
      const int variant = (M >= 4 && pos0 + M > 64) ? 0 : 1;
      if (variant == 0 && m->hk.attn_tile) {
        m->hk.attn_tile(Kc, Vc, hd, t->global ? 0 : 1, qkv, ld, pos0, M, att);
      } else
#pragma omp parallel for schedule(dynamic)
      for (int r = 0; r < M; ++r) {
        const int pos = pos0 + r, lo = t->global ? 0 : (pos - 511 > 0 ? pos - 511 : 0);
        attn_row(m, Kc, Vc, hd, qkv + (size_t)r * ld, lo, pos, variant, att + (size_t)r * QD);
      }
    }
    lin(m, &t->o, att, M, o, 0);
    for (int r = 0; r < M; ++r) {
      float* om = o + (size_t)r * H;
      float* xm = x + (size_t)r * H;
      for (int i = 0; i < H; ++i) om[i] = or_r16(om[i]);
      const float rr = rms_scale(om, H);
      for (int i = 0; i < H; ++i) xm[i] = or_r16(xm[i] + or_r16((om[i] * rr) * t->post_attn[i]));
      rmsnorm(xm, t->pre_ff, H, mlp_in + (size_t)r * H, 1);
    }
    lin(m, &t->gu, mlp_in, M, gu, 0);
    const int Il = t->down.K; /* this layer's MLP width */
    for (int r = 0; r < M; ++r)
      for (int i = 0; i < Il; ++i) {
        const float g = or_r16(gu[(size_t)r * 2 * Il + i]), u = or_r16(gu[(size_t)r * 2 * Il + Il + i]);
        act[(size_t)r * Il + i] = or_r16(or_r16(or_gelu(g)) * u);
      }
    lin(m, &t->down, act, M, o, 0);
    for (int r = 0; r < M; ++r) {
      float* om = o + (size_t)r * H;
      float* xm = x + (size_t)r * H;
      for (int i = 0; i < H; ++i) om[i] = or_r16(om[i]);
      const float rr = rms_scale(om, H);
      if (m->ple) /* add_res_prep_x (:1376): the layer scalar comes after the per-layer input */
        for (int i = 0; i < H; ++i) xm[i] = or_r16(xm[i] + or_r16((om[i] * rr) * t->post_ff[i]));
      else
        for (int i = 0; i < H; ++i) xm[i] = or_r16(or_r16(xm[i] + or_r16((om[i] * rr) * t->post_ff[i])) * t->scalar);
    }
    if (m->ple) { /* the per-layer input (:1379-1388, int8 branch) */
      lin(m, &t->pg, x, M, pgv, 0);
      for (int r = 0; r < M; ++r)
        for (int i = 0; i < PLE_D; ++i)
          g2[(size_t)r * PLE_D + i] = or_r16(or_r16(or_gelu(or_r16(pgv[(size_t)r * PLE_D + i]))) *
                                             or_r16(pli[(size_t)r * NP + (size_t)l * PLE_D + i]));
      lin(m, &t->pp, g2, M, o, 0);
      for (int r = 0; r < M; ++r) {
        float* om = o + (size_t)r * H;
        float* xm = x + (size_t)r * H;
        for (int i = 0; i < H; ++i) om[i] = or_r16(om[i]);
        const float rr = rms_scale(om, H);
        for (int i = 0; i < H; ++i) xm[i] = or_r16(or_r16(xm[i] + or_r16((om[i] * rr) * t->post_ple[i])) * t->scalar);
      }
    }
  }
  free(pli); free(pgv); free(g2);
  if (want) {
    float* logits = (float*)malloc(sizeof(float) * (size_t)m->V * 4);
    for (int r = hf; r < M; ++r) rmsnorm(x + (size_t)r * H, m->fnorm, H, hbuf + (size_t)r * H, 1);
    for (int r0 = hf; r0 < M; r0 += 4) { /* rows in groups of 4 (:1500) */
      const int mh = M - r0 < 4 ? M - r0 : 4;
      if (m->hk.head_run && m->head_ref)
        m->hk.head_run(m->head_ref, hbuf + (size_t)r0 * H, mh, logits);
      else
        or_bf16p_gemm(m->hdata, m->cb, m->exc_ptr, m->exc_col, m->exc_delta, m->V, H, hbuf + (size_t)r0 * H, mh, logits);
      for (int r = 0; r < mh; ++r) G[r0 + r] = or_head_pick(logits + (size_t)r * m->V, m->V);
    }
    free(logits);
  }
  free(x); free(a); free(qkv); free(att); free(o); free(gu); free(act); free(mlp_in);
}

/* One draft step (draft_step :1534-1563): returns the drafted token; next hidden into h_next. */
static int draft(Model* m, int tok, const float* h, int pos, int P, float* h_next) {
  const int H = m->H, QD = m->NQ * m->HD, I = m->I, hd = m->HD;
  float* comb = (float*)malloc(sizeof(float) * 2 * H);
  float* dx = (float*)malloc(sizeof(float) * H);
  float* da = (float*)malloc(sizeof(float) * (H > I ? H : I));
  float* dq = (float*)malloc(sizeof(float) * QD);
  float* dopt = (float*)malloc(sizeof(float) * QD);
  float* dgu = (float*)malloc(sizeof(float) * 2 * I);
  float* dact = (float*)malloc(sizeof(float) * I);
  float* dh = (float*)malloc(sizeof(float) * H);
  float* score = (float*)malloc(sizeof(float) * m->DCENT);
  const float sqrtH = sqrtf((float)H);
  for (int i = 0; i < H; ++i) { comb[i] = or_r16(or_bf2f(m->E[(size_t)tok * H + i]) * sqrtH); comb[H + i] = h[i]; }
  lin(m, &m->dpre, comb, 1, dx, 1);
  for (int i = 0; i < H; ++i) dx[i] = or_r16(dx[i]);
  for (int l = 0; l < m->DL; ++l) {
    DLayer* t = &m->D[l];
    const int ty = t->global ? 1 : 0;
    int tl = -1;
    for (int l2 = m->NL - 1; l2 >= 0; --l2)
      if ((l2 % 5 == 4) == t->global) { tl = owner_of(m, l2); break; }
    rmsnorm(dx, t->in_ln, H, da, 0);
    lin(m, &t->q, da, 1, dq, 1);
    const float* cs = m->rc[ty] + (size_t)pos * (hd / 2);
    const float* sn = m->rs[ty] + (size_t)pos * (hd / 2);
    for (int hh = 0; hh < m->NQ; ++hh) { rms_r16_w(dq + (size_t)hh * hd, t->qn, hd); rope(dq + (size_t)hh * hd, cs, sn, hd); }
    const int lo = t->global ? 0 : (pos - 511 > 0 ? pos - 511 : 0);
    int pp = P, ll = lo;
    if (m->hk.attn)
      m->hk.attn(m->Kc + (size_t)tl * m->ctx_max * m->HDM, m->Vc + (size_t)tl * m->ctx_max * m->HDM, hd, m->NQ, 1, dq, &pp, &ll, lo, P,
                 dopt);
    else
      or_attn_splitkv(m->Kc + (size_t)tl * m->ctx_max * m->HDM, m->Vc + (size_t)tl * m->ctx_max * m->HDM, hd, m->NQ, 1, dq, &pp, &ll,
                      lo, P, m->attn_chunks, dopt);
    lin(m, &t->o, dopt, 1, da, 1);
    for (int i = 0; i < H; ++i) da[i] = or_r16(da[i]);
    { const float r = rms_scale(da, H); for (int i = 0; i < H; ++i) dx[i] = or_r16(dx[i] + or_r16((da[i] * r) * t->post_attn[i])); }
    rmsnorm(dx, t->pre_ff, H, da, 1);
    lin(m, &t->gu, da, 1, dgu, 1);
    for (int i = 0; i < I; ++i) dact[i] = or_r16(or_r16(or_gelu(or_r16(dgu[i]))) * or_r16(dgu[I + i]));
    lin(m, &t->down, dact, 1, da, 1);
    for (int i = 0; i < H; ++i) da[i] = or_r16(da[i]);
    { const float r = rms_scale(da, H); for (int i = 0; i < H; ++i) dx[i] = or_r16(dx[i] + or_r16((da[i] * r) * t->post_ff[i])); }
    for (int i = 0; i < H; ++i) dx[i] = or_r16(dx[i] * 1.0f);
  }
  rmsnorm(dx, m->dnorm, H, dh, 1);
  lin(m, &m->dpost, dh, 1, h_next, 1);
  lin(m, &m->dcent, dh, 1, score, 1);
  for (int i = 0; i < H; ++i) h_next[i] = or_r16(h_next[i]);
  /* top DTOP centroids (insertion sort, :1554-1555), candidates, scores, first max */
  int top[32];
  float thr[32];
  int cnt = 0;
  for (int c = 0; c < m->DCENT; ++c) {
    const float s = score[c];
    if (cnt < m->DTOP) { int j = cnt++; while (j > 0 && thr[j - 1] < s) { thr[j] = thr[j - 1]; top[j] = top[j - 1]; --j; } thr[j] = s; top[j] = c; }
    else if (s > thr[m->DTOP - 1]) { int j = m->DTOP - 1; while (j > 0 && thr[j - 1] < s) { thr[j] = thr[j - 1]; top[j] = top[j - 1]; --j; } thr[j] = s; top[j] = c; }
  }
  int best = -1;
  float bs = -1e30f;
  for (int t = 0; t < m->DTOP; ++t)
    for (int j = 0; j < m->DPER; ++j) {
      const int c = (int)perm_token((uint32_t)(top[t] * m->DPER + j), (uint32_t)m->V);
      const uint16_t* er = m->E + (size_t)c * H;
      float a0[8] = {0}, b0[8] = {0}, tt[8];
      for (int k = 0; k < H; k += 16)
        for (int l = 0; l < 8; ++l) { a0[l] = fmaf(or_bf2f(er[k + l]), dh[k + l], a0[l]); b0[l] = fmaf(or_bf2f(er[k + 8 + l]), dh[k + 8 + l], b0[l]); }
      for (int l = 0; l < 8; ++l) tt[l] = a0[l] + b0[l];
      const float s = ((tt[0] + tt[4]) + (tt[1] + tt[5])) + ((tt[2] + tt[6]) + (tt[3] + tt[7]));
      if (best < 0 || s > bs) { bs = s; best = c; }
    }
  free(comb); free(dx); free(da); free(dq); free(dopt); free(dgu); free(dact); free(dh); free(score);
  return best;
}

int or_e2e_forward(void* mp, const int32_t* toks, int M, int pos0, int want, int hf, int int8, int32_t* G, float* hbuf) {
  Model* m = (Model*)mp;
  m->i8 = int8;
  float* hb = hbuf ? hbuf : (float*)malloc(sizeof(float) * (size_t)M * m->H);
  forward(m, toks, M, pos0, want, hf, G, hb);
  if (!hbuf) free(hb);
  return 0;
}
int or_e2e_draft(void* mp, int32_t tok, const float* h, int pos, int P, int32_t* out_tok, float* h_next) {
  Model* m = (Model*)mp;
  float* hn = h_next ? h_next : (float*)malloc(sizeof(float) * m->H);
  *out_tok = draft(m, tok, h, pos, P, hn);
  if (!h_next) free(hn);
  return 0;
}

static int is_stop(int t) { return t == 106 || t == 1; }

/* ENGINE_FAKE_CTX (gemma4_engine.cpp:1249-1250): fill positions [0, n) of every layer's K and V with
 * the reference's seeded LCG values, so that decode can be timed at a long context without a long
 * prefill; the prompt then starts at position n. */
void or_e2e_fake_ctx(void* mp, int n) {
  Model* m = (Model*)mp;
  uint32_t rs = 12345;
  for (int l = 0; l < m->NL && owns(m, l); ++l) /* the owners' caches, one stream (:1249-1250) */
    for (size_t i = 0; i < (size_t)n * hd_of(m, l); ++i) {
      rs = rs * 1664525u + 1013904223u;
      m->Kc[(size_t)l * m->ctx_max * m->HDM + i] = or_f2bf(((int)(rs >> 9) % 2001 - 1000) / 700.0f);
      rs = rs * 1664525u + 1013904223u;
      m->Vc[(size_t)l * m->ctx_max * m->HDM + i] = or_f2bf(((int)(rs >> 9) % 2001 - 1000) / 700.0f);
    }
  m->fake_n = n;
}

/* run_req (:1582-1663), split like the engine's API into a prefill (blocks of prefill_block, int8 per
 * ENGINE_PREFILL_INT8, :1595) and resumable chain-mode decode rounds (prompt lookup or k MTP drafts
 * -> one verify forward -> greedy acceptance).  The decode state lives in the model. */
/* run_req's prefill (:1598-1600) from prompt position start: the K/V rows of positions < start are
 * kept (they hold an earlier request's prefix of this prompt, the prefix cache), the blocks of
 * prefill_block rows start at start. */
int or_e2e_prefill_from(void* mp, const int32_t* prompt, int n, int start, int32_t* first) {
  Model* m = (Model*)mp;
  const int FN = m->fake_n, H = m->H;
  if (start < 0 || start >= n) return -1;
  int G[64];
  float* hbuf = (float*)malloc(sizeof(float) * 64 * H);
  m->i8 = m->prefill_int8;
  int done = start, lastM = 0;
  while (done < n) {
    const int M = m->prefill_block < n - done ? m->prefill_block : n - done;
    const int last = done + M == n;
    forward(m, prompt + done, M, FN + done, last, last ? M - 1 : 0, G, hbuf);
    done += M; lastM = M;
  }
  free(m->seq);
  m->seq_cap = n + 4096;
  m->seq = (int*)malloc(sizeof(int) * (size_t)m->seq_cap);
  memcpy(m->seq, prompt, sizeof(int) * n);
  m->seq_len = n;
  m->seq[m->seq_len++] = G[lastM - 1];
  if (!m->hprev) m->hprev = (float*)malloc(sizeof(float) * H);
  memcpy(m->hprev, hbuf + (size_t)(lastM - 1) * H, sizeof(float) * H);
  m->P = FN + n - 1;
  m->conf = G[lastM - 1];
  m->stopped = is_stop(m->conf);
  memset(m->st, 0, sizeof m->st);
  if (first) *first = G[lastM - 1];
  free(hbuf);
  return 0;
}
int or_e2e_prefill(void* mp, const int32_t* prompt, int n, int32_t* first) { return or_e2e_prefill_from(mp, prompt, n, 0, first); }

/* Drafts per round (BENCH_MODE's k). */
void or_e2e_set_k(void* mp, int k) { ((Model*)mp)->k_draft = k; }

/* The committed history (prompt and every committed token) and the last committed position P. */
int or_e2e_history(void* mp, int32_t* out, int cap, int* len, int* P) {
  Model* m = (Model*)mp;
  const int k = m->seq_len < cap ? m->seq_len : cap;
  if (out && m->seq) memcpy(out, m->seq, sizeof(int32_t) * (size_t)k);
  *len = m->seq_len;
  *P = m->P;
  return 0;
}

/* Decode state from elsewhere (a prefill of the same prompt on another implementation): the K and V
 * rows of positions [0, npos) of every layer ([NL][npos][HD] bf16), the committed history, the hidden
 * state of the last committed row and its position P; conf = the last history entry. */
int or_e2e_set_state(void* mp, const uint16_t* Kc, const uint16_t* Vc, int npos, const int32_t* seq, int seq_len,
                     const float* hprev, int P) {
  Model* m = (Model*)mp;
  if (npos > m->ctx_max || seq_len < 1 || P + 1 > npos || m->HDM != m->HD) return -1; /* one head size only */
  for (int l = 0; l < m->NL; ++l) {
    memcpy(m->Kc + (size_t)l * m->ctx_max * m->HD, Kc + (size_t)l * npos * m->HD, sizeof(uint16_t) * (size_t)npos * m->HD);
    memcpy(m->Vc + (size_t)l * m->ctx_max * m->HD, Vc + (size_t)l * npos * m->HD, sizeof(uint16_t) * (size_t)npos * m->HD);
  }
  free(m->seq);
  m->seq_cap = seq_len + 4096;
  m->seq = (int*)malloc(sizeof(int) * (size_t)m->seq_cap);
  memcpy(m->seq, seq, sizeof(int) * seq_len);
  m->seq_len = seq_len;
  if (!m->hprev) m->hprev = (float*)malloc(sizeof(float) * m->H);
  memcpy(m->hprev, hprev, sizeof(float) * m->H);
  m->P = P;
  m->conf = seq[seq_len - 1];
  m->stopped = is_stop(m->conf);
  memset(m->st, 0, sizeof m->st);
  return 0;
}

/* Up to max_rounds rounds or max_tokens committed tokens (or a stop token).  stats (may be NULL)
 * [0..3] = rounds, ngram_rounds, drafted, accepted since the prefill.  trace (may be NULL): per
 * round 6 ints {nd, prompt lookup used, drafts[3] (-1 padded), nacc}, at most trace_cap rounds. */
int or_e2e_decode(void* mp, int max_rounds, int max_tokens, int32_t* out, int* n_out, int* stats, int32_t* trace,
                  int trace_cap) {
  Model* m = (Model*)mp;
  const int H = m->H;
  int G[8];
  float* hbuf = (float*)malloc(sizeof(float) * 8 * H);
  float* hcur = (float*)malloc(sizeof(float) * H);
  float* hnext = (float*)malloc(sizeof(float) * H);
  m->i8 = m->decode_int8 && m->prefill_int8; /* (:1600) */
  int produced = 0, rounds = 0;
  while (rounds < max_rounds && produced < max_tokens && !m->stopped) {
    if (m->seq_len + 8 > m->seq_cap) {
      m->seq_cap *= 2;
      m->seq = (int*)realloc(m->seq, sizeof(int) * (size_t)m->seq_cap);
    }
    const int* seq = m->seq;
    const int L = m->seq_len;
    int block[8], nd = 0, used_ng = 0;
    block[0] = m->conf;
    if (m->ngram > 0 && L > m->ngram) { /* prompt lookup (:1624-1628) */
      for (int i = L - m->ngram - 1; i >= 0; --i) {
        int eq = 1;
        for (int t = 0; t < m->ngram; ++t) if (seq[i + t] != seq[L - m->ngram + t]) { eq = 0; break; }
        if (eq) { for (int j = 0; j < m->ngram_len && j < 7 && i + m->ngram + j < L; ++j) block[1 + nd++] = seq[i + m->ngram + j]; break; }
      }
      if (nd > 0) { used_ng = 1; m->st[1]++; }
    }
    if (!used_ng && m->drafter && m->k_draft > 0) {
      int cur = m->conf;
      memcpy(hcur, m->hprev, sizeof(float) * H);
      for (int j = 0; j < m->k_draft; ++j) {
        const int dtok = draft(m, cur, hcur, m->P + 1 + j, m->P, hnext);
        block[1 + nd++] = dtok;
        cur = dtok;
        memcpy(hcur, hnext, sizeof(float) * H);
      }
      m->st[2] += nd;
    }
    forward(m, block, nd + 1, m->P + 1, 1, 0, G, hbuf);
    m->st[0]++;
    rounds++;
    int nacc = 0;
    while (nacc < nd && block[nacc + 1] == G[nacc]) ++nacc;
    m->st[3] += nacc;
    if (trace && m->st[0] <= trace_cap) {
      int32_t* t = trace + 6 * (size_t)(m->st[0] - 1);
      t[0] = nd; t[1] = used_ng;
      for (int j = 0; j < 3; ++j) t[2 + j] = (!used_ng && j < nd) ? block[1 + j] : -1;
      t[5] = nacc;
    }
    for (int i = 0; i <= nacc; ++i) {
      m->seq[m->seq_len++] = G[i];
      if (out && produced < max_tokens) out[produced] = G[i];
      ++produced;
      if (is_stop(G[i])) { m->stopped = 1; break; }
    }
    m->conf = G[nacc];
    memcpy(m->hprev, hbuf + (size_t)nacc * H, sizeof(float) * H);
    m->P += nacc + 1;
  }
  *n_out = produced < max_tokens ? produced : max_tokens;
  if (stats) for (int i = 0; i < 4; ++i) stats[i] = m->st[i];
  free(hbuf); free(hcur); free(hnext);
  return 0;
}

/* run_req: prefill, then decode until n_new tokens (the first from the prefill) or a stop token. */
int or_e2e_generate_trace(void* mp, const int32_t* prompt, int n, int n_new, int32_t* out, int* n_out, int* stats,
                          int32_t* trace, int trace_cap) {
  Model* m = (Model*)mp;
  int first = 0, got = 0;
  or_e2e_prefill(mp, prompt, n, &first);
  out[0] = first;
  if (n_new > 1 && !m->stopped) or_e2e_decode(mp, 1 << 30, n_new - 1, out + 1, &got, NULL, trace, trace_cap);
  int total = 1 + got;
  for (int i = 0; i < total; ++i) if (is_stop(out[i])) { total = i + 1; break; }
  *n_out = total;
  if (stats) for (int i = 0; i < 4; ++i) stats[i] = m->st[i];
  return 0;
}
int or_e2e_generate(void* mp, const int32_t* prompt, int n, int n_new, int32_t* out, int* n_out, int* stats) {
  return or_e2e_generate_trace(mp, prompt, n, n_new, out, n_out, stats, NULL, 0);
}

/* Route the linears, the split-KV attention and the exact head through h (prepared once per matrix). */
static void hook_lin(Model* m, Lin* l) { if (l->w) l->ref = m->hk.lin_prepare(l->w, l->s, l->N, l->K); }
int or_e2e_set_hooks(void* mp, const or_e2e_hooks* h) {
  Model* m = (Model*)mp;
  m->hk = *h;
  if (!h->lin_prepare || !h->head_prepare) return -1;
  for (int l = 0; l < m->NL; ++l) {
    TLayer* t = &m->L[l];
    hook_lin(m, &t->qkv); hook_lin(m, &t->o); hook_lin(m, &t->gu); hook_lin(m, &t->down);
    if (m->ple) { hook_lin(m, &t->pg); hook_lin(m, &t->pp); }
  }
  if (m->ple) hook_lin(m, &m->plproj);
  if (m->D) {
    for (int l = 0; l < m->DL; ++l) {
      DLayer* t = &m->D[l];
      hook_lin(m, &t->q); hook_lin(m, &t->o); hook_lin(m, &t->gu); hook_lin(m, &t->down);
    }
    hook_lin(m, &m->dpre); hook_lin(m, &m->dpost); hook_lin(m, &m->dcent);
  }
  m->head_ref = h->head_prepare(m->E, m->V, m->H, m->cb);
  return 0;
}

/* raw weight bytes for cross-checking the generator: tensor `id`, first n bytes (reference layout) */
void or_e2e_gen_bytes(unsigned long long seed, unsigned long long id, long long n, uint8_t* out) {
  for (long long i = 0; i < n; ++i) out[i] = (uint8_t)(wh(seed, id, (uint64_t)i) & 0xFF);
}

/* layer_scalar of target layer l (gemma4_engine.cpp:1389-1404; 1 unless set): x = r16(x * s) after
 * the MLP residual, as the library applies it (s is used as given; pass a bf16 value). */
void or_e2e_set_layer_scalar(void* mp, int l, float s) {
  Model* m = (Model*)mp;
  if (l >= 0 && l < m->NL) m->L[l].scalar = s;
}

/* The target model written as a checkpoint in the reference's format (test fixture writer): a
 * safetensors file with the names the reference loads (gemma4_engine.cpp:1222-1231) - per layer
 * the q/k/v/o and gate/up/down matrices as weight_packed (I32 [N][K/8], or U8 [N][K/2] when
 * packed_u8) plus weight_scale (BF16 [N][K/32]), the six norms and layer_scalar (BF16), then
 * norm.weight and embed_tokens.weight.  Returns 0, or -1 when the file cannot be written. */
typedef struct { char name[96]; const char* dtype; long long shape[2]; int nd; const void* data; size_t nbytes; } CkOut;
static void ck_add(CkOut* o, int* n, const char* name, const char* dtype, long long a, long long b, int nd, const void* data,
                   size_t nbytes) {
  CkOut* t = &o[(*n)++];
  snprintf(t->name, sizeof t->name, "%s", name);
  t->dtype = dtype; t->shape[0] = a; t->shape[1] = b; t->nd = nd; t->data = data; t->nbytes = nbytes;
}
int or_e2e_write_checkpoint(void* mp, const char* path, int packed_u8) {
  Model* m = (Model*)mp;
  const int H = m->H;
  const int per = 7 * 2 + 7 + 5;
  CkOut* o = (CkOut*)calloc((size_t)m->NL * per + 8, sizeof(CkOut));
  uint16_t* bf = (uint16_t*)malloc(sizeof(uint16_t) * ((size_t)m->NL * (5 * H + 2 * m->HDM + 1) + H + PLE_D));
  size_t bo = 0;
  int n = 0;
  char nm[96];
  for (int l = 0; l < m->NL; ++l) {
    const TLayer* t = &m->L[l];
    const int I = t->down.K;                     /* this layer's MLP width */
    const int HD = hd_of(m, l), QD = m->NQ * HD; /* and head dim */
    struct { const char* name; const Lin* lin; int row0, rows; } lins[7] = {
        {"self_attn.q_proj", &t->qkv, 0, QD}, {"self_attn.k_proj", &t->qkv, QD, HD}, {"self_attn.v_proj", &t->qkv, QD + HD, HD},
        {"self_attn.o_proj", &t->o, 0, H},    {"mlp.gate_proj", &t->gu, 0, I},       {"mlp.up_proj", &t->gu, I, I},
        {"mlp.down_proj", &t->down, 0, H}};
    for (int k = 0; k < 7; ++k) {
      if (!owns(m, l) && (k == 1 || k == 2)) continue; /* a KV-shared layer has no k/v projections */
      const Lin* L = lins[k].lin;
      const int K = L->K, rows = lins[k].rows;
      snprintf(nm, sizeof nm, "layers.%d.%s.weight_packed", l, lins[k].name);
      if (packed_u8) ck_add(o, &n, nm, "U8", rows, K / 2, 2, L->w + (size_t)lins[k].row0 * K / 2, (size_t)rows * K / 2);
      else ck_add(o, &n, nm, "I32", rows, K / 8, 2, L->w + (size_t)lins[k].row0 * K / 2, (size_t)rows * K / 2);
      snprintf(nm, sizeof nm, "layers.%d.%s.weight_scale", l, lins[k].name);
      ck_add(o, &n, nm, "BF16", rows, K / 32, 2, L->s + (size_t)lins[k].row0 * K / 32, sizeof(uint16_t) * (size_t)rows * K / 32);
    }
    struct { const char* name; const float* v; int len; } vecs[6] = {
        {"input_layernorm.weight", t->in_ln, H}, {"post_attention_layernorm.weight", t->post_attn, H},
        {"pre_feedforward_layernorm.weight", t->pre_ff, H}, {"post_feedforward_layernorm.weight", t->post_ff, H},
        {"self_attn.q_norm.weight", t->qn, HD}, {"self_attn.k_norm.weight", t->kn, HD}};
    for (int k = 0; k < 6; ++k) {
      if (!vecs[k].v) continue; /* k_norm of a KV-shared layer */
      uint16_t* dst = bf + bo;
      for (int i = 0; i < vecs[k].len; ++i) dst[i] = or_f2bf(vecs[k].v[i]);
      bo += (size_t)vecs[k].len;
      snprintf(nm, sizeof nm, "layers.%d.%s", l, vecs[k].name);
      ck_add(o, &n, nm, "BF16", vecs[k].len, 0, 1, dst, sizeof(uint16_t) * (size_t)vecs[k].len);
    }
    if (m->ple) { /* per_layer_input_gate, per_layer_projection, post_per_layer_input_norm (:1226-1229) */
      const struct { const char* name; const Lin* lin; } pl[2] = {{"per_layer_input_gate", &t->pg}, {"per_layer_projection", &t->pp}};
      for (int k = 0; k < 2; ++k) {
        const Lin* L = pl[k].lin;
        snprintf(nm, sizeof nm, "layers.%d.%s.weight_packed", l, pl[k].name);
        if (packed_u8) ck_add(o, &n, nm, "U8", L->N, L->K / 2, 2, L->w, (size_t)L->N * L->K / 2);
        else ck_add(o, &n, nm, "I32", L->N, L->K / 8, 2, L->w, (size_t)L->N * L->K / 2);
        snprintf(nm, sizeof nm, "layers.%d.%s.weight_scale", l, pl[k].name);
        ck_add(o, &n, nm, "BF16", L->N, L->K / 32, 2, L->s, sizeof(uint16_t) * (size_t)L->N * L->K / 32);
      }
      uint16_t* dst = bf + bo;
      for (int i = 0; i < H; ++i) dst[i] = or_f2bf(t->post_ple[i]);
      bo += (size_t)H;
      snprintf(nm, sizeof nm, "layers.%d.post_per_layer_input_norm.weight", l);
      ck_add(o, &n, nm, "BF16", H, 0, 1, dst, sizeof(uint16_t) * (size_t)H);
    }
    bf[bo] = or_f2bf(t->scalar);
    snprintf(nm, sizeof nm, "layers.%d.layer_scalar", l);
    ck_add(o, &n, nm, "BF16", 1, 0, 1, bf + bo, 2);
    bo += 1;
  }
  {
    uint16_t* dst = bf + bo;
    for (int i = 0; i < H; ++i) dst[i] = or_f2bf(m->fnorm[i]);
    bo += H; /* the per-layer projection norm below goes after it */
    ck_add(o, &n, "norm.weight", "BF16", H, 0, 1, dst, sizeof(uint16_t) * (size_t)H);
  }
  ck_add(o, &n, "embed_tokens.weight", "BF16", m->V, H, 2, m->E, sizeof(uint16_t) * (size_t)m->V * H);
  if (m->ple) { /* embed_tokens_per_layer, per_layer_model_projection, per_layer_projection_norm (:1230-1231) */
    const long long NP = (long long)m->NL * PLE_D;
    ck_add(o, &n, "embed_tokens_per_layer.weight", "BF16", m->V, NP, 2, m->PLEt, sizeof(uint16_t) * (size_t)m->V * NP);
    const Lin* L = &m->plproj;
    if (packed_u8) ck_add(o, &n, "per_layer_model_projection.weight_packed", "U8", L->N, L->K / 2, 2, L->w, (size_t)L->N * L->K / 2);
    else ck_add(o, &n, "per_layer_model_projection.weight_packed", "I32", L->N, L->K / 8, 2, L->w, (size_t)L->N * L->K / 2);
    ck_add(o, &n, "per_layer_model_projection.weight_scale", "BF16", L->N, L->K / 32, 2, L->s, sizeof(uint16_t) * (size_t)L->N * L->K / 32);
    uint16_t* dst = bf + bo;
    for (int i = 0; i < PLE_D; ++i) dst[i] = or_f2bf(m->plnorm[i]);
    bo += PLE_D;
    ck_add(o, &n, "per_layer_projection_norm.weight", "BF16", PLE_D, 0, 1, dst, sizeof(uint16_t) * PLE_D);
  }
  /* header: JSON, padded with spaces to a multiple of 8 bytes */
  size_t cap = 256 + (size_t)n * 192, len = 0, off = 0;
  char* hdr = (char*)malloc(cap);
  len += (size_t)snprintf(hdr + len, cap - len, "{\"__metadata__\":{\"format\":\"pt\"}");
  for (int k = 0; k < n; ++k) {
    if (o[k].nd == 2)
      len += (size_t)snprintf(hdr + len, cap - len, ",\"%s\":{\"dtype\":\"%s\",\"shape\":[%lld,%lld],\"data_offsets\":[%zu,%zu]}",
                              o[k].name, o[k].dtype, o[k].shape[0], o[k].shape[1], off, off + o[k].nbytes);
    else
      len += (size_t)snprintf(hdr + len, cap - len, ",\"%s\":{\"dtype\":\"%s\",\"shape\":[%lld],\"data_offsets\":[%zu,%zu]}",
                              o[k].name, o[k].dtype, o[k].shape[0], off, off + o[k].nbytes);
    off += o[k].nbytes;
  }
  len += (size_t)snprintf(hdr + len, cap - len, "}");
  while (len % 8) hdr[len++] = ' ';
  int rc = -1;
  FILE* f = fopen(path, "wb");
  if (f) {
    const uint64_t hl = (uint64_t)len;
    int ok = fwrite(&hl, 8, 1, f) == 1 && fwrite(hdr, 1, len, f) == len;
    for (int k = 0; k < n && ok; ++k) ok = fwrite(o[k].data, 1, o[k].nbytes, f) == o[k].nbytes;
    rc = (fclose(f) == 0 && ok) ? 0 : -1;
  }
  free(hdr);
  free(bf);
  free(o);
  return rc;
}

/* Test helper: zero the bf16 scales of one family of linears ("pg", "pp", "o" or "down" in layers
 * [l0, l1), or the model's "plproj"), so that its output is exactly zero (isolates parts of the
 * model when comparing against the reference engine on a checkpoint written afterwards).  Returns 0,
 * or -1 for an unknown family, a bad range or a per-layer-embedding family in a model without
 * per-layer embeddings. */
int or_e2e_zero_scales_range(void* mp, const char* what, int l0, int l1) {
  Model* m = (Model*)mp;
  const int ple_part = !strcmp(what, "plproj") || !strcmp(what, "pg") || !strcmp(what, "pp");
  if ((ple_part && !m->ple) || l0 < 0 || l1 > m->NL || l0 > l1) return -1;
  if (!strcmp(what, "plproj")) {
    memset(m->plproj.s, 0, sizeof(uint16_t) * (size_t)m->plproj.N * (m->plproj.K / 32));
    return 0;
  }
  for (int l = l0; l < l1; ++l) {
    TLayer* t = &m->L[l];
    Lin* L = !strcmp(what, "pg") ? &t->pg : !strcmp(what, "pp") ? &t->pp : !strcmp(what, "o") ? &t->o
           : !strcmp(what, "down") ? &t->down : NULL;
    if (!L) return -1;
    memset(L->s, 0, sizeof(uint16_t) * (size_t)L->N * (L->K / 32));
  }
  return 0;
}
int or_e2e_zero_scales(void* mp, const char* what) { return or_e2e_zero_scales_range(mp, what, 0, ((Model*)mp)->NL); }
