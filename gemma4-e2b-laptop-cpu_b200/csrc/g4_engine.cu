// The speculative greedy-decode engine on one GPU: the synthetic E2B target (g4_model.cuh), its
// MTP drafter, prompt lookup, batched verification and greedy acceptance.  The control flow is the
// reference's run_req spec loop (gemma4_engine.cpp:1582-1663) in chain mode; the forward pass is
// its fwd lambda (:1256-1502) and the draft step its draft_step (:1534-1563), both at the
// synthetic dimensions.  Every kernel launch goes to the engine's stream.
#include "g4_api.h"
#include "g4_layers.cuh"
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <vector>

namespace g4 {

#define ECK(call)                                                                                  \
  do {                                                                                             \
    cudaError_t e_ = (call);                                                                       \
    if (e_ != cudaSuccess) return set_error(G4_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)
#define RCK(call)              \
  do {                         \
    int rc_ = (call);          \
    if (rc_ != G4_OK) return rc_; \
  } while (0)

struct Lin {  // one int4 W4G32 matrix in device layout
  uint8_t* w = nullptr;
  uint16_t* s = nullptr;
  int N = 0, K = 0;
};
struct TLayer {
  Lin qkv, o, gu, down;
  float *in_ln, *post_attn, *pre_ff, *post_ff, *qn, *kn;
  bool global;
};
struct DLayerW {
  Lin q, o, gu, down;
  float *in_ln, *post_attn, *pre_ff, *post_ff, *qn;
  bool global;
};

// Phase timer: CUDA events at op boundaries on the engine stream; the time between an event and the
// next one is charged to the category recorded with the first (the reference's DECODE_STAGE /
// STAGE_PROF breakdown, gemma4_engine.cpp:1672, 1691).
enum Phase { PH_EMBED_NORM = 0, PH_LINEAR, PH_ATTN, PH_HEAD, PH_DRAFT, PH_COPY, PH_N };
struct PhaseTimer {
  bool on = false;
  std::vector<cudaEvent_t> ev;
  std::vector<int> cat;
  size_t used = 0;
  double acc[PH_N] = {0, 0, 0, 0, 0, 0};
  long long launches[PH_N] = {0, 0, 0, 0, 0, 0};
  void mark(cudaStream_t st, int c) {
    if (!on) return;
    if (used == ev.size()) { cudaEvent_t e; cudaEventCreate(&e); ev.push_back(e); cat.push_back(0); }
    cudaEventRecord(ev[used], st);
    cat[used] = c;
    ++used;
  }
  void flush() {  // after a stream sync
    if (!on || used < 2) { used = 0; return; }
    for (size_t i = 0; i + 1 < used; ++i) {
      float ms = 0;
      cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
      acc[cat[i]] += ms;
      launches[cat[i]]++;
    }
    used = 0;
  }
};

}  // namespace g4

struct g4_engine {
  g4_engine_config cfg;
  g4::ModelDims d;
  cudaStream_t st = nullptr;
  std::vector<void*> allocs;
  // weights
  std::vector<g4::TLayer> L;
  std::vector<g4::DLayerW> DL;
  g4::Lin dpre, dpost, dcent;
  float *fnorm = nullptr, *dnorm = nullptr;
  uint16_t* E = nullptr;
  // head
  uint8_t *hdata = nullptr, *hunp = nullptr, *sW4 = nullptr;
  uint16_t* sS4 = nullptr;
  float* scoef = nullptr;
  long long* hexc_ptr = nullptr;
  uint16_t* hexc_col = nullptr;
  float* hexc_delta = nullptr;
  uint8_t cb8[8];
  // caches and tables
  uint16_t *Kc = nullptr, *Vc = nullptr;  // [NL][ctx][HD]
  float* rope[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};  // [type][cos|sin] [ctx][HD/2]
  // activations (M <= MMAX)
  int MMAX = 32;
  float *x, *a, *qkv, *att, *o, *gu, *act, *hbuf, *mlp_in, *qs;
  int8_t* xq;
  float* xsx;
  int32_t* xsum;
  int* ctl;   // device: [0] = P (last committed target position), [8, 8 + MMAX) = the rows' tokens
  int* toks;  // = ctl + 8
  int* G;
  int* hio = nullptr;  // pinned host mirror: ctl [8 + MMAX], then G [MMAX], then drafts [8]
  void* attn_ws = nullptr;
  int* attn_cnt = nullptr;  // per-(row, head) counters of the captured rounds' attention, 0 between calls
  bool pdl_ok = true;       // captures use programmatic dependent launch unless that failed once
  size_t attn_ws_bytes = 0;
  void* head_ws = nullptr;
  size_t head_ws_bytes = 0;
  int* head_ns = nullptr;
  // drafter activations
  float *dcomb, *dx, *da, *dq, *dopt, *dgu, *dact, *dh, *bcur, *dscore, *cscore, *hprev, *hnext;
  int *cand, *dtok;
  bool i8_active = false;
  g4_engine_stats stats{};
  g4::PhaseTimer prof;
  // CUDA graphs of a decode round: the verify pass for M = 1..4 rows and the chain of k drafts;
  // positions are read from ctl[0] on the device, so one capture serves every round
  cudaGraphExec_t gverify[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  cudaGraphExec_t gdraft = nullptr;
  int gk_verify[5] = {0, 0, 0, 0, 0}, gk_draft = 0;  // kernel nodes of each graph
  cudaEvent_t tev[4] = {nullptr, nullptr, nullptr, nullptr};  // draft start/end, verify start/end
  int fake_n = 0;
  // decode state between g4_engine_decode calls
  std::vector<int> seq;  // prompt + committed tokens (prompt-lookup history)
  int P = -1, conf = 0;
  bool stopped = false;
};

using namespace g4;

extern "C" int g4_engine_default_config(g4_engine_config* c) {
  if (!c) return set_error(G4_ERR_INVALID, "g4_engine_default_config: null pointer");
  std::memset(c, 0, sizeof *c);
  c->hidden = 2048; c->n_layers = 30; c->mlp = 8192; c->vocab = 262144; c->ctx_max = 8192;
  c->prefill_block = 32; c->k_draft = 3; c->ngram = 2; c->ngram_len = 3; c->prefill_int8 = 1; c->decode_int8 = 1;
  c->head_screen = 1; c->screen_lim = 30000; c->attn_chunks = 8; c->att_par = 192; c->drafter = 1; c->seed = 20261201ull;
  c->graphs = 1;
  return G4_OK;
}

static int ealloc(g4_engine* e, void** p, size_t bytes) {
  cudaError_t r = cudaMalloc(p, bytes < 256 ? 256 : bytes);
  if (r != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_engine: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(r));
  e->allocs.push_back(*p);
  return G4_OK;
}
template <class T>
static int ealloc_t(g4_engine* e, T** p, size_t count) { return ealloc(e, reinterpret_cast<void**>(p), count * sizeof(T)); }

static unsigned gridfor(long long n, int block = 256) { return (unsigned)std::min<long long>((n + block - 1) / block, 1 << 20); }

// Generate a stack of int4 matrices (ids, row counts) as one device-layout matrix of K columns.
static int gen_lin(g4_engine* e, Lin& lin, const std::vector<std::pair<uint64_t, int>>& parts, int K, uint8_t* tmp) {
  int N = 0;
  for (auto& p : parts) N += p.second;
  lin.N = N; lin.K = K;
  RCK(ealloc_t(e, &lin.w, (size_t)N * K / 2));
  RCK(ealloc_t(e, &lin.s, (size_t)N * K / 32));
  size_t roff = 0, soff = 0;
  for (auto& p : parts) {
    const long long nb = (long long)p.second * K / 2, ns = (long long)p.second * K / 32;
    k_gen_w4<<<gridfor(nb), 256, 0, e->st>>>(e->cfg.seed, p.first, nb, tmp + roff);
    k_gen_scales<<<gridfor(ns), 256, 0, e->st>>>(e->cfg.seed, p.first | T_SCALES, ns, lin.s + soff);
    roff += nb; soff += ns;
  }
  RCK(g4_w4_pack(tmp, N, K, lin.w, e->st));
  return check_launch("gen_lin");
}
static int gen_norm(g4_engine* e, float** p, uint64_t id, int n, float mul) {
  RCK(ealloc_t(e, p, n));
  k_gen_norm<<<gridfor(n), 256, 0, e->st>>>(e->cfg.seed, id, n, mul, *p);
  return check_launch("gen_norm");
}

extern "C" int g4_engine_create(const g4_engine_config* cfg, g4_engine** out) {
  if (!cfg || !out) return set_error(G4_ERR_INVALID, "g4_engine_create: null pointer");
  const g4_engine_config c = *cfg;
  G4_REQUIRE(c.hidden % 256 == 0 && c.hidden >= 256 && c.hidden <= 2048 && c.mlp % 256 == 0 && c.n_layers >= 1 && c.vocab % 128 == 0 &&
                 c.vocab <= (1 << 18) && (c.vocab & (c.vocab - 1)) == 0 && c.ctx_max >= 64 && c.ctx_max <= 32768 &&
                 c.prefill_block >= 1 && c.prefill_block <= 32 && c.k_draft >= 0 && c.k_draft <= 3 && c.attn_chunks >= 1 &&
                 c.attn_chunks <= 16,
             "g4_engine_create: unsupported configuration");
  RCK(g4_device_init());
  g4_engine* e = new g4_engine();
  e->cfg = c;
  ModelDims& d = e->d;
  d.H = c.hidden; d.NL = c.n_layers; d.I = c.mlp; d.V = c.vocab; d.DCENT = c.vocab / d.DPER;
  d.DTOP = std::min(32, d.DCENT);
  auto fail = [&](int rc) { g4_engine_destroy(e); return rc; };
  if (cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking) != cudaSuccess) return fail(set_error(G4_ERR_CUDA, "stream"));
  const int H = d.H, QD = d.NQ * d.HD, I = d.I;
  uint8_t* tmp = nullptr;
  const size_t tmp_bytes = (size_t)std::max({(size_t)(QD + 2 * d.HD) * H / 2, (size_t)2 * I * H / 2, (size_t)I * H / 2,
                                              (size_t)QD * H / 2, (size_t)d.DCENT * H / 2, (size_t)H * 2 * H / 2});
  if (ealloc_t(e, &tmp, tmp_bytes)) return fail(G4_ERR_CUDA);
  e->L.resize(d.NL);
  for (int l = 0; l < d.NL; ++l) {
    TLayer& t = e->L[l];
    t.global = d.global_layer(l);
    int rc = gen_lin(e, t.qkv, {{layer_id(l, T_Q), QD}, {layer_id(l, T_K), d.HD}, {layer_id(l, T_V), d.HD}}, H, tmp);
    if (!rc) rc = gen_lin(e, t.o, {{layer_id(l, T_O), H}}, QD, tmp);
    if (!rc) rc = gen_lin(e, t.gu, {{layer_id(l, T_GATE), I}, {layer_id(l, T_UP), I}}, H, tmp);
    if (!rc) rc = gen_lin(e, t.down, {{layer_id(l, T_DOWN), H}}, I, tmp);
    if (!rc) rc = gen_norm(e, &t.in_ln, layer_id(l, T_IN_LN), H, 1.f);
    if (!rc) rc = gen_norm(e, &t.post_attn, layer_id(l, T_POST_ATTN), H, 1.f);
    if (!rc) rc = gen_norm(e, &t.pre_ff, layer_id(l, T_PRE_FF), H, 1.f);
    if (!rc) rc = gen_norm(e, &t.post_ff, layer_id(l, T_POST_FF), H, 1.f);
    if (!rc) rc = gen_norm(e, &t.qn, layer_id(l, T_QN), d.HD, 0.0625f);
    if (!rc) rc = gen_norm(e, &t.kn, layer_id(l, T_KN), d.HD, 1.f);
    if (rc) return fail(rc);
  }
  if (gen_norm(e, &e->fnorm, T_FNORM, H, 1.f)) return fail(G4_ERR_CUDA);
  // embedding / tied head, packed exact head, screen
  const long long EV = (long long)d.V * H;
  if (ealloc_t(e, &e->E, (size_t)EV)) return fail(G4_ERR_CUDA);
  k_gen_embed<<<gridfor(EV), 256, 0, e->st>>>(c.seed, EV, e->E);
  {
    void* ws = nullptr;
    if (ealloc(e, &ws, std::max<size_t>(2048, 8 * (size_t)d.V))) return fail(G4_ERR_CUDA);
    int rc = g4_bf16p_codebook(e->E, EV, e->cb8, ws, std::max<size_t>(2048, 8 * (size_t)d.V), e->st);
    long long total = 0;
    if (!rc && ealloc_t(e, &e->hexc_ptr, (size_t)d.V + 1)) rc = G4_ERR_CUDA;
    if (!rc) rc = g4_bf16p_count(e->E, d.V, H, e->cb8, e->hexc_ptr, ws, 8 * (size_t)d.V, &total, e->st);
    if (!rc && ealloc_t(e, &e->hdata, (size_t)d.V * (H / 32) * 44)) rc = G4_ERR_CUDA;
    if (!rc && ealloc_t(e, &e->hexc_col, (size_t)std::max(1LL, total))) rc = G4_ERR_CUDA;
    if (!rc && ealloc_t(e, &e->hexc_delta, (size_t)std::max(1LL, total))) rc = G4_ERR_CUDA;
    if (!rc) rc = g4_bf16p_pack(e->E, d.V, H, e->cb8, e->hdata, e->hexc_ptr, e->hexc_col, e->hexc_delta, e->st);
    if (!rc && H % 64 == 0) {  // the unpacked copy that the head GEMV reads
      if (ealloc_t(e, &e->hunp, (size_t)d.V * (H / 32) * 64)) rc = G4_ERR_CUDA;
      if (!rc) rc = g4_bf16p_unpack(e->hdata, e->cb8, d.V, H, e->hunp, e->st);
    }
    if (!rc && ealloc_t(e, &e->sW4, (size_t)d.V * H / 2)) rc = G4_ERR_CUDA;
    if (!rc && ealloc_t(e, &e->sS4, (size_t)d.V * H / 32)) rc = G4_ERR_CUDA;
    if (!rc && ealloc_t(e, &e->scoef, (size_t)d.V)) rc = G4_ERR_CUDA;
    if (!rc) rc = g4_screen_build(e->E, d.V, H, e->sW4, e->sS4, e->scoef, e->st);
    if (rc) return fail(rc);
  }
  // drafter
  if (c.drafter) {
    int rc = gen_lin(e, e->dpre, {{T_DPRE, H}}, 2 * H, tmp);
    if (!rc) rc = gen_lin(e, e->dpost, {{T_DPOST, H}}, H, tmp);
    if (!rc) rc = gen_lin(e, e->dcent, {{T_DCENT, d.DCENT}}, H, tmp);
    if (!rc) rc = gen_norm(e, &e->dnorm, T_DNORM, H, 1.f);
    e->DL.resize(d.DL);
    for (int l = 0; l < d.DL && !rc; ++l) {
      DLayerW& t = e->DL[l];
      t.global = (l == d.DL - 1);
      rc = gen_lin(e, t.q, {{dlayer_id(l, T_Q), QD}}, H, tmp);
      if (!rc) rc = gen_lin(e, t.o, {{dlayer_id(l, T_O), H}}, QD, tmp);
      if (!rc) rc = gen_lin(e, t.gu, {{dlayer_id(l, T_GATE), I}, {dlayer_id(l, T_UP), I}}, H, tmp);
      if (!rc) rc = gen_lin(e, t.down, {{dlayer_id(l, T_DOWN), H}}, I, tmp);
      if (!rc) rc = gen_norm(e, &t.in_ln, dlayer_id(l, T_IN_LN), H, 1.f);
      if (!rc) rc = gen_norm(e, &t.post_attn, dlayer_id(l, T_POST_ATTN), H, 1.f);
      if (!rc) rc = gen_norm(e, &t.pre_ff, dlayer_id(l, T_PRE_FF), H, 1.f);
      if (!rc) rc = gen_norm(e, &t.post_ff, dlayer_id(l, T_POST_FF), H, 1.f);
      if (!rc) rc = gen_norm(e, &t.qn, dlayer_id(l, T_QN), d.HD, 0.0625f);
    }
    if (rc) return fail(rc);
  }
  // KV cache and RoPE tables (host, double -> float, as gemma4_engine.cpp:1246-1247)
  const size_t kvn = (size_t)d.NL * c.ctx_max * d.HD;
  if (ealloc_t(e, &e->Kc, kvn) || ealloc_t(e, &e->Vc, kvn)) return fail(G4_ERR_CUDA);
  cudaMemsetAsync(e->Kc, 0, kvn * 2, e->st);
  cudaMemsetAsync(e->Vc, 0, kvn * 2, e->st);
  {
    const int hh = d.HD / 2;
    std::vector<float> cs((size_t)c.ctx_max * hh), sn((size_t)c.ctx_max * hh);
    for (int ty = 0; ty < 2; ++ty) {
      const double theta = ty ? 1e6 : 1e4;
      for (int p = 0; p < c.ctx_max; ++p)
        for (int j = 0; j < hh; ++j) {
          const double inv = 1.0 / pow(theta, (2.0 * j) / d.HD);
          const double ang = p * inv;
          cs[(size_t)p * hh + j] = (float)cos(ang);
          sn[(size_t)p * hh + j] = (float)sin(ang);
        }
      if (ealloc_t(e, &e->rope[ty][0], cs.size()) || ealloc_t(e, &e->rope[ty][1], sn.size())) return fail(G4_ERR_CUDA);
      if (cudaMemcpy(e->rope[ty][0], cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
          cudaMemcpy(e->rope[ty][1], sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(set_error(G4_ERR_CUDA, "rope tables"));
    }
  }
  // activations
  const int MM = e->MMAX;
  int rc = ealloc_t(e, &e->x, (size_t)MM * H);
  if (!rc) rc = ealloc_t(e, &e->a, (size_t)MM * std::max(H, I));
  if (!rc) rc = ealloc_t(e, &e->qkv, (size_t)MM * (QD + 2 * d.HD));
  if (!rc) rc = ealloc_t(e, &e->att, (size_t)MM * QD);
  if (!rc) rc = ealloc_t(e, &e->qs, (size_t)4 * QD);
  if (!rc) rc = ealloc_t(e, &e->o, (size_t)MM * H);
  if (!rc) rc = ealloc_t(e, &e->gu, (size_t)MM * 2 * I);
  if (!rc) rc = ealloc_t(e, &e->act, (size_t)MM * I);
  if (!rc) rc = ealloc_t(e, &e->hbuf, (size_t)MM * H);
  if (!rc) rc = ealloc_t(e, &e->mlp_in, (size_t)MM * H);
  const size_t kmax = (size_t)std::max({2 * H, I, QD});  // widest linear input
  if (!rc) rc = ealloc_t(e, &e->xq, (size_t)MM * kmax);
  if (!rc) rc = ealloc_t(e, &e->xsx, (size_t)MM * kmax / 32);
  if (!rc) rc = ealloc_t(e, &e->xsum, (size_t)MM * kmax / 32);
  if (!rc) rc = ealloc_t(e, &e->ctl, (size_t)MM + 8);
  if (!rc) {
    e->toks = e->ctl + 8;
    if (cudaHostAlloc(reinterpret_cast<void**>(&e->hio), sizeof(int) * (2 * (size_t)MM + 16), cudaHostAllocDefault) != cudaSuccess)
      rc = set_error(G4_ERR_CUDA, "g4_engine_create: pinned host buffer");
  }
  for (int i = 0; i < 4 && !rc; ++i)
    if (cudaEventCreate(&e->tev[i]) != cudaSuccess) rc = set_error(G4_ERR_CUDA, "g4_engine_create: events");
  if (!rc) rc = ealloc_t(e, &e->G, (size_t)MM);
  e->attn_ws_bytes = g4_attn_splitkv_ws_bytes(4, d.NQ, d.HD, 0, c.ctx_max - 1, c.attn_chunks);
  if (!rc) rc = ealloc(e, &e->attn_ws, e->attn_ws_bytes);
  if (!rc) rc = ealloc_t(e, &e->attn_cnt, 64);
  if (!rc && cudaMemsetAsync(e->attn_cnt, 0, 64 * sizeof(int), e->st) != cudaSuccess)  // captured attention's counters
    rc = set_error(G4_ERR_CUDA, "g4_engine_create: counter reset");
  e->head_ws_bytes = g4_head_screen_ws_bytes(4, d.V, c.screen_lim);
  if (!rc) rc = ealloc(e, &e->head_ws, e->head_ws_bytes);
  if (!rc) rc = ealloc_t(e, &e->head_ns, 4);
  if (!rc) rc = ealloc_t(e, &e->dcomb, (size_t)2 * H);
  if (!rc) rc = ealloc_t(e, &e->dx, (size_t)H);
  if (!rc) rc = ealloc_t(e, &e->da, (size_t)std::max({H, I, QD}));
  if (!rc) rc = ealloc_t(e, &e->dq, (size_t)QD);
  if (!rc) rc = ealloc_t(e, &e->dopt, (size_t)QD);
  if (!rc) rc = ealloc_t(e, &e->dgu, (size_t)2 * I);
  if (!rc) rc = ealloc_t(e, &e->dact, (size_t)I);
  if (!rc) rc = ealloc_t(e, &e->dh, (size_t)H);
  if (!rc) rc = ealloc_t(e, &e->bcur, (size_t)H);
  if (!rc) rc = ealloc_t(e, &e->hprev, (size_t)H);
  if (!rc) rc = ealloc_t(e, &e->hnext, (size_t)H);
  if (!rc) rc = ealloc_t(e, &e->dscore, (size_t)d.DCENT);
  if (!rc) rc = ealloc_t(e, &e->cscore, (size_t)d.DTOP * d.DPER);
  if (!rc) rc = ealloc_t(e, &e->cand, (size_t)d.DTOP * d.DPER);
  if (!rc) rc = ealloc_t(e, &e->dtok, 4);
  if (rc) return fail(rc);
  if (cudaStreamSynchronize(e->st) != cudaSuccess) return fail(set_error(G4_ERR_CUDA, "g4_engine_create: %s", cudaGetErrorString(cudaGetLastError())));
  *out = e;
  return G4_OK;
}

extern "C" void g4_engine_destroy(g4_engine* e) {
  if (!e) return;
  if (e->st) cudaStreamSynchronize(e->st);
  for (auto& g : e->gverify)
    if (g) cudaGraphExecDestroy(g);
  if (e->gdraft) cudaGraphExecDestroy(e->gdraft);
  for (auto& ev : e->tev)
    if (ev) cudaEventDestroy(ev);
  if (e->hio) cudaFreeHost(e->hio);
  for (void* p : e->allocs) cudaFree(p);
  if (e->st) cudaStreamDestroy(e->st);
  delete e;
}

// int4 linear: W4A8 when int8 activations are active and M >= 2 (lin_multi :311), or always for the
// drafter (force_i8); otherwise the float W4G32 path.  prequant: the producer of X already wrote its
// quantisation to xq/xsx/xsum (fused row kernels, attention merge).
static bool i8_path(const g4_engine* e, int M, bool force_i8) { return (e->i8_active && M >= 2) || force_i8; }
static QuantOut quant_out(g4_engine* e, int M, bool force_i8) {
  return i8_path(e, M, force_i8) ? QuantOut{e->xq, e->xsx, e->xsum} : QuantOut{nullptr, nullptr, nullptr};
}
static int lin(g4_engine* e, const Lin& w, const float* X, int M, float* Y, bool force_i8 = false, bool prequant = false) {
  if (i8_path(e, M, force_i8)) {
    if (!prequant) RCK(g4_w4a8_quant(X, M, w.K, e->xq, e->xsx, e->xsum, e->st));
    int m0 = 0;
    while (m0 < M) {  // the GEMV serves up to 8 activation rows per launch; rows are independent
      const int mm = std::min(8, M - m0);
      RCK(g4_w4a8_gemm(w.w, w.s, e->xq + (size_t)m0 * w.K, e->xsx + (size_t)m0 * (w.K / 32),
                       e->xsum + (size_t)m0 * (w.K / 32), mm, w.N, w.K, Y + (size_t)m0 * w.N, w.N, e->st));
      m0 += mm;
    }
    return G4_OK;
  }
  int m0 = 0;
  while (m0 < M) {
    const int mm = std::min(8, M - m0);
    RCK(g4_w4g32_gemm(w.w, w.s, X + (size_t)m0 * w.K, nullptr, mm, w.N, w.K, Y + (size_t)m0 * w.N, w.N, e->st));
    m0 += mm;
  }
  return G4_OK;
}

// One target forward over M tokens at positions pos0.. (fwd, :1256-1502).  toks are device ints;
// when want, rows hf.. get the final-normed hidden in hbuf and the greedy next token in G.  With
// dyn the positions are ctl[0] + 1.. read on the device (pos0 unused; M <= 4 and the split-KV path,
// i.e. position + M > att_par, which the caller guarantees), so that the launches can be captured
// once and replayed at every position.  Per layer: norm(+quant) -> qkv -> q/k norms, RoPE, KV
// write -> attention(+quant) -> o -> residual + pre-MLP norm(+quant) -> gate/up -> GeGLU(+quant)
// -> down -> residual + the next layer's input norm(+quant) (the final norm after the last layer).
static int forward(g4_engine* e, int M, int pos0, bool want, int hf, bool dyn = false) {
  const ModelDims& d = e->d;
  const int H = d.H, QD = d.NQ * d.HD, ld = QD + 2 * d.HD;
  const float sqrtH = sqrtf((float)H);
  PhaseTimer& pf = e->prof;
  const QuantOut qo = quant_out(e, M, false);
  pf.mark(e->st, PH_EMBED_NORM);
  RCK(launch("k_embed", k_embed, dim3(M), dim3(256), 0, e->st, e->E, e->toks, H, sqrtH, e->x));
  RCK(launch("k_norm_q", k_norm_q, dim3(M), dim3(256), 0, e->st, e->x, e->L[0].in_ln, H, e->a, 0, qo));
  RCK(check_launch("k_norm_q"));
  for (int l = 0; l < d.NL; ++l) {
    const TLayer& t = e->L[l];
    const int ty = t.global ? 1 : 0;
    pf.mark(e->st, PH_LINEAR);
    RCK(lin(e, t.qkv, e->a, M, e->qkv, false, true));
    uint16_t* Kc = e->Kc + (size_t)l * e->cfg.ctx_max * d.HD;
    uint16_t* Vc = e->Vc + (size_t)l * e->cfg.ctx_max * d.HD;
    pf.mark(e->st, PH_EMBED_NORM);
    const bool split = dyn || (M <= 4 && pos0 + M > e->cfg.att_par);
    // split-KV reads the rotated queries from qs ([M][QD]); the per-row paths read them in place
    if (d.HD % 64 == 0 && d.HD <= 512 && d.NQ + 2 <= 16)  // warp per head
      RCK(launch("k_qkv_post_w", k_qkv_post_w, dim3(M), dim3(32 * (d.NQ + 2)), 0, e->st, e->qkv, ld, d.NQ, d.HD,
                 dyn ? 1 : pos0, dyn ? e->ctl : nullptr, t.qn, t.kn, e->rope[ty][0], e->rope[ty][1], Kc, Vc,
                 split ? e->qs : e->qkv, split ? QD : ld));
    else
      RCK(launch("k_qkv_post", k_qkv_post, dim3(dim3(M, d.NQ + 2)), dim3(256), 0, e->st, e->qkv, ld, d.NQ, d.HD, dyn ? 1 : pos0, dyn ? e->ctl : nullptr,
                                                       t.qn, t.kn, e->rope[ty][0], e->rope[ty][1], Kc, Vc,
                                                       split ? e->qs : e->qkv, split ? QD : ld));
    RCK(check_launch("k_qkv_post"));
    pf.mark(e->st, PH_ATTN);
    bool att_q = false;
    if (dyn) {
      const int max_len = t.global ? e->cfg.ctx_max : std::min(e->cfg.ctx_max, d.WINDOW + 4);
      RCK(attn_splitkv_dev(Kc, Vc, e->qs, M, d.NQ, d.HD, e->ctl, 1, 1, t.global ? 0 : d.WINDOW, max_len,
                           e->cfg.attn_chunks, e->att, e->attn_ws, e->attn_ws_bytes, e->st, qo, e->attn_cnt));
      att_q = true;
    } else if (split) {
      // split-KV (:1305-1327)
      int pos[4], lo[4], kmin = 1 << 30;
      for (int m = 0; m < M; ++m) {
        pos[m] = pos0 + m;
        lo[m] = t.global ? 0 : std::max(0, pos[m] - (d.WINDOW - 1));
        kmin = std::min(kmin, lo[m]);
      }
      RCK(g4_attn_splitkv(Kc, Vc, e->qs, pos, lo, M, d.NQ, d.HD, kmin, pos0 + M - 1, e->cfg.attn_chunks, e->att, e->attn_ws,
                          e->attn_ws_bytes, e->st));
    } else {
      const int variant = (M >= 4 && pos0 + M > 64) ? 0 : 1;  // attn_tile, else per-(row, head) (:1328-1355)
      const int len_max = (t.global ? pos0 + M : std::min(pos0 + M, d.WINDOW));
      k_attn_rows<<<dim3(M, d.NQ), 256, sizeof(float) * len_max, e->st>>>(Kc, Vc, e->qkv, ld, d.NQ, d.HD, pos0,
                                                                           t.global ? 0 : d.WINDOW, variant, e->att, QD);
      RCK(check_launch("k_attn_rows"));
    }
    pf.mark(e->st, PH_LINEAR);
    RCK(lin(e, t.o, e->att, M, e->o, false, att_q));
    pf.mark(e->st, PH_EMBED_NORM);
    RCK(launch("k_post_attn_q", k_post_attn_q, dim3(M), dim3(256), 0, e->st, e->o, e->x, t.post_attn, t.pre_ff, e->mlp_in, H, qo));
    pf.mark(e->st, PH_LINEAR);
    RCK(lin(e, t.gu, e->mlp_in, M, e->gu, false, true));
    pf.mark(e->st, PH_EMBED_NORM);
    RCK(launch("k_act_q", k_act_q, dim3((unsigned)((long long)M * d.I / 256)), dim3(256), 0, e->st, e->gu, d.I, M, e->act, qo));
    pf.mark(e->st, PH_LINEAR);
    RCK(lin(e, t.down, e->act, M, e->o, false, true));
    pf.mark(e->st, PH_EMBED_NORM);
    if (l + 1 < d.NL)  // residual (layer scalar 1) and the next layer's input norm
      RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(M), dim3(256), 0, e->st, e->o, e->x, t.post_ff, 1.0f, H, e->L[l + 1].in_ln, e->a, 0, qo));
    else  // residual and the final norm (rounded) of every row into hbuf
      RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(M), dim3(256), 0, e->st, e->o, e->x, t.post_ff, 1.0f, H, e->fnorm, e->hbuf, 1,
                                           QuantOut{nullptr, nullptr, nullptr}));
    RCK(check_launch("layer"));
  }
  pf.mark(e->st, PH_HEAD);
  if (!want) return G4_OK;
  // head in groups of 4 rows (:1500)
  for (int r0 = hf; r0 < M; r0 += 4) {
    const int mh = std::min(4, M - r0);
    if (e->cfg.head_screen) {
      RCK(head_screen_impl(e->sW4, e->sS4, e->scoef, e->hdata, e->hunp, e->cb8, e->hexc_ptr, e->hexc_col, e->hexc_delta,
                           d.V, H, e->hbuf + (size_t)r0 * H, mh, e->cfg.screen_lim, e->G + r0, e->head_ns, e->head_ws,
                           e->head_ws_bytes, e->st));
    } else {
      float* logits = static_cast<float*>(e->head_ws);
      if (e->hunp)
        RCK(g4_bf16p_unpacked_gemm(e->hunp, e->hexc_ptr, e->hexc_col, e->hexc_delta, d.V, H, e->hbuf + (size_t)r0 * H, mh,
                                   logits, d.V, e->st));
      else
        RCK(g4_bf16p_gemm(e->hdata, e->cb8, e->hexc_ptr, e->hexc_col, e->hexc_delta, d.V, H, e->hbuf + (size_t)r0 * H, mh,
                          logits, d.V, e->st));
      RCK(g4_head_argmax(logits, mh, d.V, d.V, e->G + r0, static_cast<char*>(e->head_ws) + sizeof(float) * (size_t)4 * d.V,
                         64, e->st));
    }
  }
  pf.mark(e->st, PH_COPY);
  return G4_OK;
}

// One draft step (draft_step, :1534-1563): token *dtok_in, hidden h (device), query position pos,
// last valid target position P; writes the drafted token to *dtok_out and the next hidden to bcur.
// With dyn, P is ctl[0] on the device and pos = P + 1 + j (pos and P unused).  Every drafter linear
// runs W4A8 at M = 1, its input quantised by the kernel that produces it.
static int draft_step(g4_engine* e, const int* dtok_in, const float* h, int pos, int P, int* dtok_out, bool dyn = false,
                      int j = 0) {
  const ModelDims& d = e->d;
  const int H = d.H;
  const QuantOut qo{e->xq, e->xsx, e->xsum};
  e->prof.mark(e->st, PH_DRAFT);
  RCK(launch("k_draft_in", k_draft_in, dim3(8), dim3(256), 0, e->st, e->E, dtok_in, h, H, sqrtf((float)H), e->dcomb));
  RCK(lin(e, e->dpre, e->dcomb, 1, e->dx, true));
  RCK(launch("k_round", k_round, dim3(gridfor(H)), dim3(256), 0, e->st, e->dx, H));
  RCK(launch("k_norm_q", k_norm_q, dim3(1), dim3(256), 0, e->st, e->dx, e->DL[0].in_ln, H, e->da, 0, qo));
  for (int l = 0; l < d.DL; ++l) {
    const DLayerW& t = e->DL[l];
    const int ty = t.global ? 1 : 0;
    // target layer whose KV the drafter reads: the last global layer, or the last sliding layer
    int tl = -1;
    for (int l2 = d.NL - 1; l2 >= 0; --l2)
      if (d.global_layer(l2) == t.global) { tl = l2; break; }
    if (tl < 0) return set_error(G4_ERR_UNSUPPORTED, "draft_step: the target has no %s layer", t.global ? "global" : "sliding");
    RCK(lin(e, t.q, e->da, 1, e->dq, true, true));
    RCK(launch("k_q_post", k_q_post, dim3(d.NQ), dim3(256), 0, e->st, e->dq, d.HD, dyn ? 1 + j : pos, dyn ? e->ctl : nullptr, t.qn, e->rope[ty][0],
                                      e->rope[ty][1]));
    const uint16_t* Kt = e->Kc + (size_t)tl * e->cfg.ctx_max * d.HD;
    const uint16_t* Vt = e->Vc + (size_t)tl * e->cfg.ctx_max * d.HD;
    bool att_q = false;
    if (dyn) {
      const int max_len = t.global ? e->cfg.ctx_max : std::min(e->cfg.ctx_max, d.WINDOW);
      RCK(attn_splitkv_dev(Kt, Vt, e->dq, 1, d.NQ, d.HD, e->ctl, 0, 1 + j, t.global ? 0 : d.WINDOW, max_len,
                           e->cfg.attn_chunks, e->dopt, e->attn_ws, e->attn_ws_bytes, e->st, qo, e->attn_cnt));
      att_q = true;
    } else {
      const int lo = t.global ? 0 : std::max(0, pos - (d.WINDOW - 1));
      const int pp = P;
      RCK(g4_attn_splitkv(Kt, Vt, e->dq, &pp, &lo, 1, d.NQ, d.HD, lo, P, e->cfg.attn_chunks, e->dopt, e->attn_ws,
                          e->attn_ws_bytes, e->st));
    }
    RCK(lin(e, t.o, e->dopt, 1, e->da, true, att_q));
    // o residual (no layer scalar), then the pre-MLP norm (rounded)
    RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(1), dim3(256), 0, e->st, e->da, e->dx, t.post_attn, 0.0f, H, t.pre_ff, e->da, 1, qo));
    RCK(lin(e, t.gu, e->da, 1, e->dgu, true, true));
    RCK(launch("k_act_q", k_act_q, dim3((unsigned)(d.I / 256)), dim3(256), 0, e->st, e->dgu, d.I, 1, e->dact, qo));
    RCK(lin(e, t.down, e->dact, 1, e->da, true, true));
    // MLP residual with the layer scalar 1, then the next layer's input norm or the final norm
    if (l + 1 < d.DL)
      RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(1), dim3(256), 0, e->st, e->da, e->dx, t.post_ff, 1.0f, H, e->DL[l + 1].in_ln, e->da, 0, qo));
    else
      RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(1), dim3(256), 0, e->st, e->da, e->dx, t.post_ff, 1.0f, H, e->dnorm, e->dh, 1, qo));
    RCK(check_launch("draft layer"));
  }
  RCK(lin(e, e->dpost, e->dh, 1, e->bcur, true, true));
  RCK(lin(e, e->dcent, e->dh, 1, e->dscore, true, true));
  RCK(launch("k_round", k_round, dim3(gridfor(H)), dim3(256), 0, e->st, e->bcur, H));
  const int nc = d.DTOP * d.DPER;
  RCK(launch("k_topk_cand", k_topk_cand, dim3((d.DCENT + 31) / 32), dim3(256), sizeof(float) * d.DCENT, e->st, e->dscore, d.DCENT, d.DTOP, d.DPER, d.V, e->cand));
  RCK(launch("k_cand_scores", k_cand_scores, dim3((nc * 16 + 255) / 256), dim3(256), 0, e->st, e->E, e->cand, nc, e->dh, H, e->cscore));
  RCK(launch("k_cand_best", k_cand_best, dim3(1), dim3(1024), 0, e->st, e->cscore, e->cand, nc, dtok_out));
  e->prof.mark(e->st, PH_COPY);
  return check_launch("draft_step");
}

extern "C" int g4_engine_forward(g4_engine* e, const int32_t* toks, int M, int pos0, int want, int hf, int int8,
                                 int32_t* G, float* hbuf) {
  G4_REQUIRE(e && toks && M >= 1 && M <= e->MMAX && pos0 >= 0 && pos0 + M <= e->cfg.ctx_max && hf >= 0 && hf < M,
             "g4_engine_forward: bad arguments");
  e->i8_active = int8 != 0;
  ECK(cudaMemcpyAsync(e->toks, toks, sizeof(int) * M, cudaMemcpyHostToDevice, e->st));
  RCK(forward(e, M, pos0, want != 0, hf));
  if (want && G) ECK(cudaMemcpyAsync(G + hf, e->G + hf, sizeof(int) * (M - hf), cudaMemcpyDeviceToHost, e->st));
  if (want && hbuf)
    ECK(cudaMemcpyAsync(hbuf + (size_t)hf * e->d.H, e->hbuf + (size_t)hf * e->d.H, sizeof(float) * (M - hf) * e->d.H,
                        cudaMemcpyDeviceToHost, e->st));
  ECK(cudaStreamSynchronize(e->st));
  return G4_OK;
}

extern "C" int g4_engine_draft(g4_engine* e, int32_t tok, const float* h, int pos, int P, int32_t* out_tok, float* h_next) {
  G4_REQUIRE(e && h && out_tok && e->cfg.drafter && pos < e->cfg.ctx_max && P >= 0, "g4_engine_draft: bad arguments");
  ECK(cudaMemcpyAsync(e->dtok, &tok, sizeof(int), cudaMemcpyHostToDevice, e->st));
  ECK(cudaMemcpyAsync(e->hbuf, h, sizeof(float) * e->d.H, cudaMemcpyHostToDevice, e->st));
  RCK(draft_step(e, e->dtok, e->hbuf, pos, P, e->dtok + 1));
  ECK(cudaMemcpyAsync(out_tok, e->dtok + 1, sizeof(int), cudaMemcpyDeviceToHost, e->st));
  if (h_next) ECK(cudaMemcpyAsync(h_next, e->bcur, sizeof(float) * e->d.H, cudaMemcpyDeviceToHost, e->st));
  ECK(cudaStreamSynchronize(e->st));
  return G4_OK;
}

static bool is_stop(int t) { return t == 106 || t == 1; }

extern "C" int g4_engine_fake_ctx(g4_engine* e, int n) {
  G4_REQUIRE(e && n >= 0 && n + 16 <= e->cfg.ctx_max, "g4_engine_fake_ctx: bad arguments (n=%d ctx_max=%d)", n,
             e ? e->cfg.ctx_max : 0);
  const int HD = e->d.HD;
  std::vector<uint16_t> kb((size_t)n * HD), vb((size_t)n * HD);
  uint32_t rs = 12345;
  auto rnd = [&]() {
    rs = rs * 1664525u + 1013904223u;
    const float f = ((int)(rs >> 9) % 2001 - 1000) / 700.0f;
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);  // round to nearest even (finite values)
    return (uint16_t)(u >> 16);
  };
  ECK(cudaStreamSynchronize(e->st));
  for (int l = 0; l < e->d.NL; ++l) {
    for (size_t i = 0; i < (size_t)n * HD; ++i) {
      kb[i] = rnd();
      vb[i] = rnd();
    }
    const size_t off = (size_t)l * e->cfg.ctx_max * HD;
    ECK(cudaMemcpy(e->Kc + off, kb.data(), kb.size() * 2, cudaMemcpyHostToDevice));
    ECK(cudaMemcpy(e->Vc + off, vb.data(), vb.size() * 2, cudaMemcpyHostToDevice));
  }
  e->fake_n = n;
  return G4_OK;
}

// run_req (:1582-1680), split in two: prefill in blocks (int8 per ENGINE_PREFILL_INT8, :1595), then
// resumable decode rounds (chain mode): prompt lookup or k MTP drafts -> one verify forward ->
// greedy acceptance.  The committed sequence stays on the host (it is the prompt-lookup history).
extern "C" int g4_engine_prefill(g4_engine* e, const int32_t* prompt, int n, int32_t* first_token) {
  G4_REQUIRE(e && prompt && n >= 1 && e->fake_n + n + 8 <= e->cfg.ctx_max,
             "g4_engine_prefill: bad arguments (n=%d fake context %d ctx_max=%d)", n, e ? e->fake_n : 0,
             e ? e->cfg.ctx_max : 0);
  const int H = e->d.H, FN = e->fake_n;
  auto t0 = std::chrono::steady_clock::now();
  e->i8_active = e->cfg.prefill_int8 != 0;
  int done = 0, last_M = 0;
  while (done < n) {
    const int M = std::min(e->cfg.prefill_block, n - done);
    const bool last = done + M == n;
    ECK(cudaMemcpyAsync(e->toks, prompt + done, sizeof(int) * M, cudaMemcpyHostToDevice, e->st));
    RCK(forward(e, M, FN + done, last, last ? M - 1 : 0));
    done += M;
    last_M = M;
  }
  int first = 0;
  ECK(cudaMemcpyAsync(&first, e->G + (last_M - 1), sizeof(int), cudaMemcpyDeviceToHost, e->st));
  ECK(cudaMemcpyAsync(e->hprev, e->hbuf + (size_t)(last_M - 1) * H, sizeof(float) * H, cudaMemcpyDeviceToDevice, e->st));
  ECK(cudaStreamSynchronize(e->st));
  e->prof.flush();
  e->seq.assign(prompt, prompt + n);
  e->seq.push_back(first);
  e->P = FN + n - 1;
  e->conf = first;
  e->stopped = is_stop(first);
  e->stats = g4_engine_stats{};
  e->stats.prefill_tokens = n;
  e->stats.prefill_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  if (first_token) *first_token = first;
  return G4_OK;
}

// Record the launches of body() on the engine stream into an executable graph, its kernels launched
// for programmatic dependent launch; if that capture fails, record it again with ordinary launches.
template <class F>
static int capture_once(g4_engine* e, cudaGraphExec_t* out, F body, bool pdl, int* kernels) {
  ECK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
  pdl_enabled() = pdl;
  const int rc = body();
  pdl_enabled() = false;
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(e->st, &g);
  if (rc != G4_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return set_error(G4_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
  size_t nn = 0;
  if (kernels && cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn > 0) {
    std::vector<cudaGraphNode_t> nodes(nn);
    *kernels = 0;
    if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
      for (size_t i = 0; i < nn; ++i) {
        cudaGraphNodeType ty;
        if (cudaGraphNodeGetType(nodes[i], &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++*kernels;
      }
  }
  const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return set_error(G4_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ie));
  return G4_OK;
}
template <class F>
static int capture(g4_engine* e, cudaGraphExec_t* out, F body, int* kernels) {
  if (e->cfg.graphs == 1 && e->pdl_ok) {
    if (capture_once(e, out, body, true, kernels) == G4_OK) return G4_OK;
    cudaGetLastError();
    e->pdl_ok = false;
  }
  return capture_once(e, out, body, false, kernels);
}

// The k MTP drafts of a round from ctl (tokens[0] = the confirmed token, ctl[0] = P) and hprev:
// draft j reads the drafter hidden of draft j-1 and writes its token to tokens[1 + j].
static int draft_chain(g4_engine* e, bool dyn) {
  const int H = e->d.H;
  ECK(cudaMemcpyAsync(e->dtok, e->toks, sizeof(int), cudaMemcpyDeviceToDevice, e->st));
  const float* hcur = e->hprev;
  for (int j = 0; j < e->cfg.k_draft; ++j) {
    RCK(draft_step(e, e->dtok + (j & 1), hcur, e->P + 1 + j, e->P, e->dtok + ((j + 1) & 1), dyn, j));
    ECK(cudaMemcpyAsync(e->toks + 1 + j, e->dtok + ((j + 1) & 1), sizeof(int), cudaMemcpyDeviceToDevice, e->st));
    ECK(cudaMemcpyAsync(e->hnext, e->bcur, sizeof(float) * H, cudaMemcpyDeviceToDevice, e->st));
    hcur = e->hnext;
  }
  return G4_OK;
}

extern "C" int g4_engine_decode(g4_engine* e, int max_rounds, int max_tokens, int32_t* out, int* n_out,
                                g4_engine_stats* stats) {
  G4_REQUIRE(e && n_out && max_rounds >= 0 && max_tokens >= 0 && !e->seq.empty(), "g4_engine_decode: call g4_engine_prefill first");
  const int H = e->d.H, MM = e->MMAX;
  auto t0 = std::chrono::steady_clock::now();
  cudaEvent_t ev0, ev1;
  ECK(cudaEventCreate(&ev0));
  ECK(cudaEventCreate(&ev1));
  ECK(cudaEventRecord(ev0, e->st));
  e->i8_active = e->cfg.decode_int8 && e->cfg.prefill_int8;  // (:1600)
  int* hctl = e->hio;                  // [0] = P, [8..] = tokens
  int* hG = e->hio + 8 + MM;           // verified tokens
  int* hdr = e->hio + 8 + 2 * MM;      // drafts read back
  int produced = 0, rounds = 0;
  int block[8];
  while (rounds < max_rounds && produced < max_tokens && !e->stopped) {
    if (e->P + 1 + 8 >= e->cfg.ctx_max) return set_error(G4_ERR_UNSUPPORTED, "g4_engine_decode: context full (%d)", e->cfg.ctx_max);
    block[0] = e->conf;
    int nd = 0;
    bool used_ng = false;
    const std::vector<int>& seq = e->seq;
    if (e->cfg.ngram > 0) {  // prompt lookup (:1624-1628)
      const int Ls = (int)seq.size(), NG = e->cfg.ngram;
      if (Ls > NG)
        for (int i = Ls - NG - 1; i >= 0; --i) {
          bool eq = true;
          for (int t = 0; t < NG; ++t)
            if (seq[i + t] != seq[Ls - NG + t]) { eq = false; break; }
          if (eq) {
            for (int j = 0; j < e->cfg.ngram_len && j < 7 && i + NG + j < Ls; ++j) block[1 + nd++] = seq[i + NG + j];
            break;
          }
        }
      if (nd > 0) { used_ng = true; e->stats.ngram_rounds++; }
    }
    const bool drafting = !used_ng && e->cfg.drafter && e->cfg.k_draft > 0;
    const int M = (drafting ? e->cfg.k_draft : nd) + 1;
    // replay captured graphs once the split-KV path applies to every row (positions > att_par)
    const bool use_g = e->cfg.graphs && !e->prof.on && M <= 4 && e->P + 1 > e->cfg.att_par;
    hctl[0] = e->P;
    for (int i = 0; i <= nd; ++i) hctl[8 + i] = block[i];
    const int nsend = 8 + (drafting ? 1 : M);
    ECK(cudaMemcpyAsync(e->ctl, hctl, sizeof(int) * nsend, cudaMemcpyHostToDevice, e->st));
    e->stats.h2d_bytes += sizeof(int) * nsend;
    if (drafting) {
      ECK(cudaEventRecord(e->tev[0], e->st));
      if (use_g) {
        if (!e->gdraft) RCK(capture(e, &e->gdraft, [&] { return draft_chain(e, true); }, &e->gk_draft));
        ECK(cudaGraphLaunch(e->gdraft, e->st));
        e->stats.kernel_launches += e->gk_draft;
      } else {
        const long long l0 = launch_count();
        RCK(draft_chain(e, false));
        e->stats.kernel_launches += launch_count() - l0;
      }
      ECK(cudaEventRecord(e->tev[1], e->st));
      e->stats.drafted += e->cfg.k_draft;
      e->stats.draft_steps += e->cfg.k_draft;
      nd = e->cfg.k_draft;
    }
    ECK(cudaEventRecord(e->tev[2], e->st));
    if (use_g) {
      if (!e->gverify[M]) RCK(capture(e, &e->gverify[M], [&] { return forward(e, M, 0, true, 0, true); }, &e->gk_verify[M]));
      ECK(cudaGraphLaunch(e->gverify[M], e->st));
      e->stats.kernel_launches += e->gk_verify[M];
    } else {
      const long long l0 = launch_count();
      RCK(forward(e, M, e->P + 1, true, 0));
      e->stats.kernel_launches += launch_count() - l0;
    }
    ECK(cudaEventRecord(e->tev[3], e->st));
    ECK(cudaMemcpyAsync(hG, e->G, sizeof(int) * M, cudaMemcpyDeviceToHost, e->st));
    e->stats.d2h_bytes += sizeof(int) * M;
    if (drafting) {
      ECK(cudaMemcpyAsync(hdr, e->toks + 1, sizeof(int) * nd, cudaMemcpyDeviceToHost, e->st));
      e->stats.d2h_bytes += sizeof(int) * nd;
    }
    ECK(cudaStreamSynchronize(e->st));
    e->prof.flush();
    if (drafting) {
      for (int j = 0; j < nd; ++j) block[1 + j] = hdr[j];
      float ms = 0;
      cudaEventElapsedTime(&ms, e->tev[0], e->tev[1]);
      e->stats.draft_gpu_ms += ms;
    }
    {
      float ms = 0;
      cudaEventElapsedTime(&ms, e->tev[2], e->tev[3]);
      e->stats.verify_gpu_ms += ms;
      e->stats.verify_passes++;
      e->stats.verify_rows += M;
    }
    e->stats.rounds++;
    ++rounds;
    int nacc = 0;
    while (nacc < nd && block[nacc + 1] == hG[nacc]) ++nacc;
    e->stats.accepted += nacc;
    for (int i = 0; i <= nacc; ++i) {
      e->seq.push_back(hG[i]);
      if (out && produced < max_tokens) out[produced] = hG[i];
      ++produced;
      if (is_stop(hG[i])) { e->stopped = true; break; }
    }
    e->conf = hG[nacc];
    ECK(cudaMemcpyAsync(e->hprev, e->hbuf + (size_t)nacc * H, sizeof(float) * H, cudaMemcpyDeviceToDevice, e->st));
    e->P += nacc + 1;
  }
  ECK(cudaEventRecord(ev1, e->st));
  ECK(cudaEventSynchronize(ev1));
  float gms = 0;
  cudaEventElapsedTime(&gms, ev0, ev1);
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  e->stats.decode_gpu_ms += gms;
  e->stats.decode_tokens += std::min(produced, max_tokens);
  e->stats.decode_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  *n_out = std::min(produced, max_tokens);
  if (stats) *stats = e->stats;
  return G4_OK;
}

extern "C" int g4_engine_generate(g4_engine* e, const int32_t* prompt, int n, int n_new, int32_t* out, int* n_out,
                                  g4_engine_stats* stats) {
  G4_REQUIRE(e && prompt && out && n_out && n >= 1 && n_new >= 1 && n + n_new + 8 <= e->cfg.ctx_max,
             "g4_engine_generate: bad arguments (n=%d n_new=%d ctx_max=%d)", n, n_new, e->cfg.ctx_max);
  int first = 0;
  RCK(g4_engine_prefill(e, prompt, n, &first));
  out[0] = first;
  int got = 0;
  if (n_new > 1 && !e->stopped) RCK(g4_engine_decode(e, 1 << 30, n_new - 1, out + 1, &got, nullptr));
  int total = 1 + got;
  for (int i = 0; i < total; ++i)
    if (is_stop(out[i])) { total = i + 1; break; }
  *n_out = total;
  if (stats) *stats = e->stats;
  return G4_OK;
}

// Phase times (ms) accumulated while profiling is on: [0] embed/norms/rope/residual, [1] linears,
// [2] attention, [3] head, [4] drafter, [5] copies between phases; enable != 0 turns it on and
// clears the totals, enable == 0 turns it off.  out may be NULL.
extern "C" int g4_engine_phase_times(g4_engine* e, int enable, double* out_ms, long long* out_marks) {
  G4_REQUIRE(e, "g4_engine_phase_times: null engine");
  if (out_ms) for (int i = 0; i < PH_N; ++i) out_ms[i] = e->prof.acc[i];
  if (out_marks) for (int i = 0; i < PH_N; ++i) out_marks[i] = e->prof.launches[i];
  if (enable >= 0) {
    e->prof.on = enable != 0;
    for (int i = 0; i < PH_N; ++i) { e->prof.acc[i] = 0; e->prof.launches[i] = 0; }
    e->prof.used = 0;
  }
  return G4_OK;
}
