// The speculative greedy-decode engine on one GPU: the synthetic E2B target (g4_model.cuh), its
// MTP drafter, prompt lookup, batched verification and greedy acceptance.  The control flow is the
// reference's run_req spec loop (gemma4_engine.cpp:1582-1663) in chain mode; the forward pass is
// its fwd lambda (:1256-1502) and the draft step its draft_step (:1534-1563), both at the
// synthetic dimensions.  Every kernel launch goes to the engine's stream.
#include "g4_api.h"
#include "g4_ckpt.h"
#include "g4_layers.cuh"
#include "g4_stream.h"
#include "g4_tc.h"
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
struct TcLin {  // the tensor-core operands of a Lin: s8 weights [N][K] and scales transposed [K/32][N]
  int8_t* w8 = nullptr;
  float* swT = nullptr;
};
struct TLayer {
  Lin qkv, o, gu, down;
  TcLin tqkv, to, tgu, tdown;
  float *in_ln = nullptr, *post_attn = nullptr, *pre_ff = nullptr, *post_ff = nullptr, *qn = nullptr, *kn = nullptr;
  bool global = false;
  float scalar = 1.0f;         // layer_scalar (:1389-1404): 1 for the synthetic model, a checkpoint's value otherwise
  Lin pg, pp;                  // per-layer input gate [256][H] and projection [H][256] (PLE)
  float* post_ple = nullptr;   // post_per_layer_input_norm (PLE)
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

// Decode-round state on the device: the spec loop's variables (run_req, gemma4_engine.cpp:1616-1663)
// live here so that the rounds of a decode call run with no host round trip.  Per-call fields are
// reset by k_decode_setup; totals accumulate from the prefill.
struct RoundCtl {
  int P, conf, seq_len, stopped;                 // last committed position, confirmed token, history length, stop seen
  int produced, rounds_call, max_rounds, max_tokens;  // this decode call
  int nd, drafting, M, used_ng;                  // the current round
  int rounds, ngram_rounds, drafted, accepted;   // totals since the prefill
  int verify_rows, draft_rounds, trace_n, ctx_full;
  int head_fallbacks, pad_[3];                   // verify passes that read the full exact head (screen fell back or skipped)
  int ngram_accepted, pad2_[3];                  // drafts accepted in prompt-lookup rounds
  int spol[4];                                   // screen back-off state (ScreenWs::pol): skip count, skipped now,
                                                 // back-off, passes skipped in total
  int rounds_m[5];                               // rounds by verify rows M (launch accounting)
  int ctx_max, trace_cap, out_cap;
  unsigned long long t_begin, t_verify;          // %globaltimer stamps of the current round
  unsigned long long draft_ns, verify_ns;        // totals since the prefill
};

__device__ __forceinline__ bool stop_token(int t) { return t == 106 || t == 1; }

// Reset the per-call fields (budgets come in as arguments: no host copy).
__global__ void k_decode_setup(RoundCtl* rc, int max_rounds, int max_tokens) {
  rc->produced = 0;
  rc->rounds_call = 0;
  rc->max_rounds = max_rounds;
  rc->max_tokens = max_tokens;
  rc->ctx_full = 0;
}

// Start of a round: prompt lookup over the committed history (:1624-1628: the latest earlier match of
// the last `ngram` tokens, up to nglen following tokens), else k MTP drafts; writes the round's
// tokens and P into the control block the captured passes read, and (in a graph) selects the draft
// and verify bodies.  One block of 256 threads; the history is scanned backwards in 2,048-position
// chunks staged in shared memory.
constexpr int kScanChunk = 2048;
__global__ void __launch_bounds__(256) k_round_begin(RoundCtl* rc, const int* __restrict__ seq, int* ctl, int ngram,
                                                     int nglen, int kdraft, cudaGraphConditionalHandle hdraft,
                                                     cudaGraphConditionalHandle hm, int set_handles) {
  __shared__ int s[kScanChunk + 16];
  __shared__ int s_best;
  const int t = threadIdx.x;
  const int L = rc->seq_len;
  int best = -1;
  if (ngram > 0 && ngram <= 8 && L > ngram) {
    int key[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) key[j] = j < ngram ? seq[L - ngram + j] : 0;
    for (int hi = L - ngram - 1; hi >= 0; hi -= kScanChunk) {
      const int lo = hi - (kScanChunk - 1) > 0 ? hi - (kScanChunk - 1) : 0;
      for (int i = t; i < hi - lo + 1 + ngram; i += blockDim.x) s[i] = seq[lo + i];
      if (t == 0) s_best = -1;
      __syncthreads();
      for (int i = hi - t; i >= lo; i -= blockDim.x) {
        bool eq = true;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < ngram && s[i - lo + j] != key[j]) eq = false;
        if (eq) { atomicMax(&s_best, i); break; }  // descending: the first hit is this thread's latest
      }
      __syncthreads();
      best = s_best;
      __syncthreads();
      if (best >= 0) break;
    }
  }
  if (t == 0) {
    int nd = 0;
    int* toks = ctl + 8;
    toks[0] = rc->conf;
    if (best >= 0)
      for (int j = 0; j < nglen && j < 7 && best + ngram + j < L; ++j) toks[1 + nd++] = seq[best + ngram + j];
    const int used_ng = nd > 0;
    const int drafting = !used_ng && kdraft > 0;
    const int M = (drafting ? kdraft : nd) + 1;
    rc->nd = drafting ? kdraft : nd;
    rc->used_ng = used_ng;
    rc->drafting = drafting;
    rc->M = M;
    ctl[0] = rc->P;
    if (set_handles) {
      cudaGraphSetConditional(hdraft, drafting ? 1u : 0u);
      cudaGraphSetConditional(hm, (unsigned)(M - 1));
    }
    rc->t_begin = globaltimer();
    rc->t_verify = rc->t_begin;
  }
}

// End of a round: nacc = leading drafts equal to the verified tokens, commit G[0..nacc] (history,
// the call's output, stop tokens 1 / 106), conf = G[nacc], hprev = the final hidden of row nacc,
// P += nacc + 1 (:1656-1660); the round's trace record; in a graph, whether the loop continues.
__global__ void __launch_bounds__(256) k_round_end(RoundCtl* rc, int* seq, const int* ctl, const int* G, const float* hbuf,
                                                   float* hprev, int H, int* out, int* trace, const int* head_ns,
                                                   cudaGraphConditionalHandle hloop, int set_handle) {
  __shared__ int s_nacc;
  const int t = threadIdx.x;
  if (t == 0) {
    const unsigned long long now = globaltimer();
    const int* toks = ctl + 8;
    const int nd = rc->nd;
    int nacc = 0;
    while (nacc < nd && toks[1 + nacc] == G[nacc]) ++nacc;
    for (int i = 0; i <= nacc; ++i) {
      const int g = G[i];
      seq[rc->seq_len++] = g;
      if (rc->produced < rc->out_cap) out[rc->produced] = g;  // every committed token (the history mirror)
      rc->produced++;
      if (stop_token(g)) { rc->stopped = 1; break; }
    }
    rc->conf = G[nacc];
    rc->P += nacc + 1;
    rc->rounds++;
    rc->rounds_call++;
    rc->accepted += nacc;
    rc->verify_rows += rc->M;
    rc->rounds_m[rc->M]++;
    if (rc->used_ng) {
      rc->ngram_rounds++;
      rc->ngram_accepted += nacc;
    }
    if (rc->drafting) {
      rc->drafted += nd;
      rc->draft_rounds++;
      rc->draft_ns += rc->t_verify - rc->t_begin;
    }
    rc->verify_ns += now - rc->t_verify;
    if (head_ns != nullptr && head_ns[0] < 0) rc->head_fallbacks++;
    if (rc->trace_n < rc->trace_cap) {
      int* tr = trace + 6 * (size_t)rc->trace_n;
      tr[0] = nd;
      tr[1] = rc->used_ng;
      for (int j = 0; j < 3; ++j) tr[2 + j] = (rc->drafting && j < nd) ? toks[1 + j] : -1;
      tr[5] = nacc;
    }
    rc->trace_n++;
    const bool budget = rc->rounds_call < rc->max_rounds && rc->produced < rc->max_tokens;
    const bool room = rc->P + 1 + 8 < rc->ctx_max;
    if (!rc->stopped && budget && !room) rc->ctx_full = 1;
    if (set_handle) cudaGraphSetConditional(hloop, (!rc->stopped && budget && room) ? 1u : 0u);
    s_nacc = nacc;
  }
  __syncthreads();
  const float* src = hbuf + (size_t)s_nacc * H;
  for (int i = t; i < H; i += blockDim.x) hprev[i] = src[i];
}

// Arms the decode loop: the WHILE handle's default is 0, so a launch in which the device could not
// set a conditional value runs no round at all (rather than an unbounded loop).
__global__ void k_loop_arm(cudaGraphConditionalHandle hloop) { cudaGraphSetConditional(hloop, 1u); }

// The first kernel of a captured verify pass stamps its start (after the previous kernel finished).
__global__ void k_stamp(RoundCtl* rc) {
  pdl_wait();
  pdl_trigger();
  rc->t_verify = globaltimer();
}

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
  // per-layer embeddings (cfg.ple): the [vocab][NL x 256] table, the projection of the embedding and
  // its norm; the rows' projections and per-layer inputs, and a layer's gate input and output
  uint16_t* PLEt = nullptr;
  g4::Lin plproj;
  float* plnorm = nullptr;
  float *pr = nullptr, *pli = nullptr, *pgv = nullptr, *g2 = nullptr;
  // head
  uint8_t *hdata = nullptr, *hnib = nullptr, *sW4 = nullptr;
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
  float* x2 = nullptr;            // second residual-stream buffer of the segment kernels
  unsigned* segbar = nullptr;     // grid-barrier counters of a pass's segment launches, then the abort flag
  unsigned long long* segtrace = nullptr;  // stage timestamps of the last pass's segment launches
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
  // tensor-core prefill: chunks of up to pmc rows of full prompt blocks
  bool tc_ready = false;
  int pmc = 0;
  int* ptoks = nullptr;
  float *px = nullptr, *pa = nullptr, *pqkv = nullptr, *patt = nullptr, *po = nullptr, *pgu = nullptr, *pact = nullptr,
        *pmlp = nullptr, *psxT = nullptr;
  int8_t* pq = nullptr;
  float* psx = nullptr;
  int32_t* psum = nullptr;
  // decode state between g4_engine_decode calls: on the device (RoundCtl, history, outputs, trace),
  // mirrored on the host after every call
  g4::RoundCtl* rc = nullptr;      // device
  g4::RoundCtl* rch = nullptr;     // pinned host mirror
  int *dseq = nullptr, *dout = nullptr, *dtrace = nullptr;
  int out_cap = 0, trace_cap = 0;
  std::vector<int> seq;  // prompt + committed tokens (host mirror of dseq)
  int P = -1, conf = 0;
  bool stopped = false;
  // the decode loop as one graph: WHILE(round) { begin; IF(drafting) drafts; SWITCH(M) verify; end }
  cudaGraphExec_t gloop = nullptr;
  cudaGraph_t graw_verify[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  cudaGraph_t graw_draft = nullptr;
  bool loop_failed = false;
  bool shared = false;  // weights belong to another engine
  // an asynchronous decode call in flight (g4_engine_decode_async / _wait)
  bool async_pending = false;
  int async_max_tokens = 0, async_r0 = 0, async_dr0 = 0, async_rm[5] = {0, 0, 0, 0, 0};
  cudaEvent_t aev0 = nullptr, aev1 = nullptr;
  std::chrono::steady_clock::time_point async_t0;
  // prefix cache (run_req, gemma4_engine.cpp:1569-1580): the active conversation's tokens whose K/V
  // (positions [0, kv_len)) is in the engine's cache, and the stored conversations, each with its
  // own device K/V buffers ([n_layers][ctx_max][head_dim], like the engine's)
  struct KvSlot {
    uint16_t* K = nullptr;
    uint16_t* V = nullptr;
    std::vector<int> keys;
    int kv_len = 0;
    unsigned long long stamp = 0;
  };
  std::vector<int> ctx_keys;
  int kv_len = 0;
  unsigned long long clock_tick = 0, active_stamp = 0;
  std::vector<KvSlot> stored;
  uint16_t *spareK = nullptr, *spareV = nullptr;
  int slot_switches = 0, slot_evictions = 0;
};

using namespace g4;

extern "C" int g4_engine_default_config(g4_engine_config* c) {
  if (!c) return set_error(G4_ERR_INVALID, "g4_engine_default_config: null pointer");
  std::memset(c, 0, sizeof *c);
  c->hidden = 2048; c->n_layers = 30; c->mlp = 8192; c->vocab = 262144; c->ctx_max = 8192;
  c->prefill_block = 32; c->k_draft = 3; c->ngram = 2; c->ngram_len = 3; c->prefill_int8 = 1; c->decode_int8 = 1;
  c->head_screen = 2; c->screen_lim = 30000; c->attn_chunks = 8; c->att_par = 192; c->drafter = 1; c->seed = 20261201ull;
  c->graphs = 1;
  c->fused_layers = 0;
  c->prefill_tc = 1;
  c->slots = 1;
  c->slot_min_reuse = 32;
  c->kv_owners = 0;
  c->mlp_shared = 0;
  c->ple = 0;
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

// The screen back-off state inside the device round state.
static int* screen_policy(g4_engine* e) {
  return reinterpret_cast<int*>(reinterpret_cast<char*>(e->rc) + offsetof(RoundCtl, spol));
}

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
// The same from a checkpoint: the reference-layout bytes and bf16 scales of each part, then packed.
static int ck_lin(g4_engine* e, const g4_checkpoint* ck, Lin& lin, const std::vector<std::pair<std::string, int>>& parts,
                  int K, uint8_t* tmp) {
  int N = 0;
  for (auto& p : parts) N += p.second;
  lin.N = N; lin.K = K;
  RCK(ealloc_t(e, &lin.w, (size_t)N * K / 2));
  RCK(ealloc_t(e, &lin.s, (size_t)N * K / 32));
  if (cudaStreamSynchronize(e->st) != cudaSuccess) return set_error(G4_ERR_CUDA, "checkpoint: stream");  // tmp is free
  RCK(ck_load_lin(ck, parts, K, tmp, lin.s, e->st));
  RCK(g4_w4_pack(tmp, N, K, lin.w, e->st));
  return check_launch("ck_lin");
}
static int ck_norm(g4_engine* e, const g4_checkpoint* ck, float** p, const std::string& name, int n) {
  RCK(ealloc_t(e, p, n));
  return ck_load_vec(ck, name, n, *p, e->st);
}
static int gen_norm(g4_engine* e, float** p, uint64_t id, int n, float mul) {
  RCK(ealloc_t(e, p, n));
  k_gen_norm<<<gridfor(n), 256, 0, e->st>>>(e->cfg.seed, id, n, mul, *p);
  return check_launch("gen_norm");
}

// Engine creation; with share, the weights (target, drafter, head copies, screen, tensor-core
// operands, RoPE tables) are the other engine's and only the per-stream state is allocated.
static int create_impl(const g4_engine_config* cfg, const g4_engine* share, g4_engine** out,
                       const g4_checkpoint* ck = nullptr) {
  if (!cfg || !out) return set_error(G4_ERR_INVALID, "g4_engine_create: null pointer");
  const g4_engine_config c = *cfg;
  G4_REQUIRE(c.hidden % 256 == 0 && c.hidden >= 256 && c.hidden <= 2048 && c.mlp % 256 == 0 && c.n_layers >= 1 && c.vocab % 128 == 0 &&
                 c.vocab <= (1 << 18) && (c.vocab & (c.vocab - 1)) == 0 && c.ctx_max >= 64 && c.ctx_max <= 32768 &&
                 c.prefill_block >= 1 && c.prefill_block <= 32 && c.k_draft >= 0 && c.k_draft <= 3 && c.attn_chunks >= 1 &&
                 c.attn_chunks <= 16 && c.slots >= 0 && c.slots <= 64 && c.slot_min_reuse >= 0,
             "g4_engine_create: unsupported configuration");
  G4_REQUIRE(c.kv_owners >= 0 && c.kv_owners <= c.n_layers, "g4_engine_create: kv_owners %d outside [0, %d]", c.kv_owners,
             c.n_layers);
  G4_REQUIRE(c.mlp_shared >= 0 && c.mlp_shared % 256 == 0, "g4_engine_create: mlp_shared %d is not a multiple of 256",
             c.mlp_shared);
  G4_REQUIRE(!c.ple || (c.prefill_int8 && c.decode_int8),
             "g4_engine_create: per-layer embeddings need prefill_int8 = decode_int8 = 1 (the reference's int8 branch)");
  {
    ModelDims dd;
    dd.NL = c.n_layers;
    dd.OWN = c.kv_owners;
    for (int l = 0; l < dd.NL; ++l)
      G4_REQUIRE(dd.owner_of(l) >= 0, "g4_engine_create: KV-shared layer %d has no %s layer among the owners", l,
                 dd.global_layer(l) ? "global" : "sliding");
  }
  RCK(g4_device_init());
  g4_engine* e = new g4_engine();
  e->cfg = c;
  ModelDims& d = e->d;
  d.H = c.hidden; d.NL = c.n_layers; d.I = c.mlp; d.V = c.vocab; d.DCENT = c.vocab / d.DPER;
  d.OWN = c.kv_owners;
  d.IS = c.mlp_shared;
  d.DTOP = std::min(32, d.DCENT);
  auto fail = [&](int rc) { g4_engine_destroy(e); return rc; };
  if (cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking) != cudaSuccess) return fail(set_error(G4_ERR_CUDA, "stream"));
  const int H = d.H, QD = d.NQ * d.HD, I = d.I, IM = d.mlp_max();
  if (share) {
    const g4_engine_config& sc = share->cfg;
    if (sc.hidden != c.hidden || sc.n_layers != c.n_layers || sc.mlp != c.mlp || sc.vocab != c.vocab || sc.seed != c.seed ||
        sc.kv_owners != c.kv_owners || sc.mlp_shared != c.mlp_shared || sc.ple != c.ple ||
        (c.drafter && !sc.drafter) || c.ctx_max > sc.ctx_max || (c.prefill_tc && !share->tc_ready && sc.prefill_tc))
      return fail(set_error(G4_ERR_INVALID, "g4_engine_create_shared: configuration differs from the weights' engine"));
    e->L = share->L;
    e->DL = share->DL;
    e->dpre = share->dpre; e->dpost = share->dpost; e->dcent = share->dcent;
    e->fnorm = share->fnorm; e->dnorm = share->dnorm; e->E = share->E;
    e->PLEt = share->PLEt; e->plproj = share->plproj; e->plnorm = share->plnorm;
    e->hdata = share->hdata; e->hnib = share->hnib; e->sW4 = share->sW4; e->sS4 = share->sS4; e->scoef = share->scoef;
    e->hexc_ptr = share->hexc_ptr; e->hexc_col = share->hexc_col; e->hexc_delta = share->hexc_delta;
    std::memcpy(e->cb8, share->cb8, 8);
    for (int ty = 0; ty < 2; ++ty) { e->rope[ty][0] = share->rope[ty][0]; e->rope[ty][1] = share->rope[ty][1]; }
    e->shared = true;
  } else {
  uint8_t* tmp = nullptr;
  const size_t tmp_bytes = (size_t)std::max({(size_t)(QD + 2 * d.HD) * H / 2, (size_t)2 * IM * H / 2, (size_t)IM * H / 2,
                                              (size_t)d.NL * 256 * H / 2,
                                              (size_t)QD * H / 2, (size_t)d.DCENT * H / 2, (size_t)H * 2 * H / 2});
  if (ealloc_t(e, &tmp, tmp_bytes)) return fail(G4_ERR_CUDA);
  e->L.resize(d.NL);
  for (int l = 0; l < d.NL && ck; ++l) {  // target weights from a checkpoint (q4 / bfvec, :1222-1229)
    TLayer& t = e->L[l];
    t.global = d.global_layer(l);
    int rc = d.owns(l) ? ck_lin(e, ck, t.qkv, {{ck_layer(l, "self_attn.q_proj"), QD}, {ck_layer(l, "self_attn.k_proj"), d.HD},
                                              {ck_layer(l, "self_attn.v_proj"), d.HD}}, H, tmp)
                       : ck_lin(e, ck, t.qkv, {{ck_layer(l, "self_attn.q_proj"), QD}}, H, tmp);
    if (!rc) rc = ck_lin(e, ck, t.o, {{ck_layer(l, "self_attn.o_proj"), H}}, QD, tmp);
    const int Il = d.mlp_of(l);
    if (!rc) rc = ck_lin(e, ck, t.gu, {{ck_layer(l, "mlp.gate_proj"), Il}, {ck_layer(l, "mlp.up_proj"), Il}}, H, tmp);
    if (!rc) rc = ck_lin(e, ck, t.down, {{ck_layer(l, "mlp.down_proj"), H}}, Il, tmp);
    if (!rc) rc = ck_norm(e, ck, &t.in_ln, ck_layer(l, "input_layernorm.weight"), H);
    if (!rc) rc = ck_norm(e, ck, &t.post_attn, ck_layer(l, "post_attention_layernorm.weight"), H);
    if (!rc) rc = ck_norm(e, ck, &t.pre_ff, ck_layer(l, "pre_feedforward_layernorm.weight"), H);
    if (!rc) rc = ck_norm(e, ck, &t.post_ff, ck_layer(l, "post_feedforward_layernorm.weight"), H);
    if (!rc) rc = ck_norm(e, ck, &t.qn, ck_layer(l, "self_attn.q_norm.weight"), d.HD);
    if (!rc && d.owns(l)) rc = ck_norm(e, ck, &t.kn, ck_layer(l, "self_attn.k_norm.weight"), d.HD);
    if (!rc) rc = ck_load_scalar(ck, ck_layer(l, "layer_scalar"), &t.scalar);
    if (!rc && c.ple) rc = ck_lin(e, ck, t.pg, {{ck_layer(l, "per_layer_input_gate"), 256}}, H, tmp);
    if (!rc && c.ple) rc = ck_lin(e, ck, t.pp, {{ck_layer(l, "per_layer_projection"), H}}, 256, tmp);
    if (!rc && c.ple) rc = ck_norm(e, ck, &t.post_ple, ck_layer(l, "post_per_layer_input_norm.weight"), H);
    if (rc) return fail(rc);
  }
  for (int l = 0; l < d.NL && !ck; ++l) {
    TLayer& t = e->L[l];
    t.global = d.global_layer(l);
    int rc = d.owns(l) ? gen_lin(e, t.qkv, {{layer_id(l, T_Q), QD}, {layer_id(l, T_K), d.HD}, {layer_id(l, T_V), d.HD}}, H, tmp)
                       : gen_lin(e, t.qkv, {{layer_id(l, T_Q), QD}}, H, tmp);  // KV-shared: q only
    if (!rc) rc = gen_lin(e, t.o, {{layer_id(l, T_O), H}}, QD, tmp);
    const int Il = d.mlp_of(l);
    if (!rc) rc = gen_lin(e, t.gu, {{layer_id(l, T_GATE), Il}, {layer_id(l, T_UP), Il}}, H, tmp);
    if (!rc) rc = gen_lin(e, t.down, {{layer_id(l, T_DOWN), H}}, Il, tmp);
    if (!rc) rc = gen_norm(e, &t.in_ln, layer_id(l, T_IN_LN), H, 1.f);
    if (!rc) rc = gen_norm(e, &t.post_attn, layer_id(l, T_POST_ATTN), H, 1.f);
    if (!rc) rc = gen_norm(e, &t.pre_ff, layer_id(l, T_PRE_FF), H, 1.f);
    if (!rc) rc = gen_norm(e, &t.post_ff, layer_id(l, T_POST_FF), H, 1.f);
    if (!rc) rc = gen_norm(e, &t.qn, layer_id(l, T_QN), d.HD, 0.0625f);
    if (!rc && d.owns(l)) rc = gen_norm(e, &t.kn, layer_id(l, T_KN), d.HD, 1.f);
    if (!rc && c.ple) rc = gen_lin(e, t.pg, {{layer_id(l, T_PG), 256}}, H, tmp);
    if (!rc && c.ple) rc = gen_lin(e, t.pp, {{layer_id(l, T_PP), H}}, 256, tmp);
    if (!rc && c.ple) rc = gen_norm(e, &t.post_ple, layer_id(l, T_POST_PLE), H, 1.f);
    if (rc) return fail(rc);
  }
  if (ck ? ck_norm(e, ck, &e->fnorm, "norm.weight", H) : gen_norm(e, &e->fnorm, T_FNORM, H, 1.f)) return fail(G4_ERR_CUDA);
  if (c.ple) {  // per-layer embeddings: the table, the projection of the embedding and its norm (:1230-1231)
    const long long NP = (long long)d.NL * 256;
    if (ealloc_t(e, &e->PLEt, (size_t)d.V * NP)) return fail(G4_ERR_CUDA);
    int rc = G4_OK;
    if (ck) {
      rc = ck_load_bf16(ck, "embed_tokens_per_layer.weight", d.V, NP, e->PLEt, e->st);
      if (!rc) rc = ck_lin(e, ck, e->plproj, {{"per_layer_model_projection", (int)NP}}, H, tmp);
      if (!rc) rc = ck_norm(e, ck, &e->plnorm, "per_layer_projection_norm.weight", 256);
    } else {
      k_gen_bf16<<<gridfor((long long)d.V * NP), 256, 0, e->st>>>(c.seed, T_PLE, (long long)d.V * NP, 0.02f, e->PLEt);
      rc = gen_lin(e, e->plproj, {{T_PLPROJ, (int)NP}}, H, tmp);
      if (!rc) rc = gen_norm(e, &e->plnorm, T_PLNORM, 256, 1.f);
    }
    if (rc) return fail(rc);
  }
  // embedding / tied head, packed exact head, screen
  const long long EV = (long long)d.V * H;
  if (ealloc_t(e, &e->E, (size_t)EV)) return fail(G4_ERR_CUDA);
  if (ck) {
    if (int rc = ck_load_bf16(ck, "embed_tokens.weight", d.V, H, e->E, e->st)) return fail(rc);
  } else {
    k_gen_embed<<<gridfor(EV), 256, 0, e->st>>>(c.seed, EV, e->E);
  }
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
    if (!rc && H % 128 == 0) {  // the split-nibble copy that the full-head GEMV reads
      if (ealloc_t(e, &e->hnib, g4_bf16p_nib_bytes(d.V, H))) rc = G4_ERR_CUDA;
      if (!rc) rc = g4_bf16p_nib_pack(e->hdata, d.V, H, e->hnib, e->st);
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
  }  // weights generated (not shared)
  // tensor-core prefill operands and chunk buffers
  if (c.prefill_tc && c.prefill_int8 && !c.ple && H % 128 == 0 && QD % 128 == 0 && I % 128 == 0 && IM % 128 == 0 &&
      (QD + 2 * d.HD) % 128 == 0) {
    int rc = G4_OK;
    auto tc_lin = [&](const Lin& l, TcLin& t) {
      if (rc) return;
      if (ealloc_t(e, &t.w8, (size_t)l.N * l.K) || ealloc_t(e, &t.swT, (size_t)l.N * (l.K / 32))) { rc = G4_ERR_CUDA; return; }
      rc = tc_expand_weights(l.w, l.s, l.N, l.K, t.w8, t.swT, e->st);
    };
    for (int l = 0; l < d.NL && !share; ++l) {
      TLayer& t = e->L[l];
      tc_lin(t.qkv, t.tqkv); tc_lin(t.o, t.to); tc_lin(t.gu, t.tgu); tc_lin(t.down, t.tdown);
    }
    e->pmc = std::min(2048, c.ctx_max / 32 * 32);
    if (rc) return fail(rc);
    e->tc_ready = true;  // the chunk buffers are allocated by the first prefill that uses them
  }
  // KV cache and RoPE tables (host, double -> float, as gemma4_engine.cpp:1246-1247)
  const size_t kvn = (size_t)d.NL * c.ctx_max * d.HD;
  if (ealloc_t(e, &e->Kc, kvn) || ealloc_t(e, &e->Vc, kvn)) return fail(G4_ERR_CUDA);
  cudaMemsetAsync(e->Kc, 0, kvn * 2, e->st);
  cudaMemsetAsync(e->Vc, 0, kvn * 2, e->st);
  if (!share) {
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
  if (!rc) rc = ealloc_t(e, &e->x2, (size_t)MM * H);
  if (!rc) rc = ealloc_t(e, &e->segbar, (size_t)4 * (c.n_layers + 2) + 1);
  if (!rc) rc = ealloc_t(e, &e->segtrace, (size_t)(c.n_layers + 2) * 2 * kSegStamps);
  if (!rc) rc = ealloc_t(e, &e->a, (size_t)MM * std::max(H, IM));
  if (!rc) rc = ealloc_t(e, &e->qkv, (size_t)MM * (QD + 2 * d.HD));
  if (!rc) rc = ealloc_t(e, &e->att, (size_t)MM * QD);
  if (!rc) rc = ealloc_t(e, &e->qs, (size_t)4 * QD);
  if (!rc) rc = ealloc_t(e, &e->o, (size_t)MM * H);
  if (!rc) rc = ealloc_t(e, &e->gu, (size_t)MM * 2 * IM);
  if (!rc && c.ple) rc = ealloc_t(e, &e->pr, (size_t)MM * d.NL * 256);
  if (!rc && c.ple) rc = ealloc_t(e, &e->pli, (size_t)MM * d.NL * 256);
  if (!rc && c.ple) rc = ealloc_t(e, &e->pgv, (size_t)MM * 256);
  if (!rc && c.ple) rc = ealloc_t(e, &e->g2, (size_t)MM * 256);
  if (!rc) rc = ealloc_t(e, &e->act, (size_t)MM * IM);
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
  e->out_cap = c.ctx_max;
  e->trace_cap = c.ctx_max;
  if (!rc) rc = ealloc_t(e, &e->rc, 1);
  if (!rc && cudaMemsetAsync(e->rc, 0, sizeof(RoundCtl), e->st) != cudaSuccess)  // the screen back-off starts off
    rc = set_error(G4_ERR_CUDA, "g4_engine_create: %s", cudaGetErrorString(cudaGetLastError()));
  if (!rc) rc = ealloc_t(e, &e->dseq, (size_t)c.ctx_max + 64);
  if (!rc) rc = ealloc_t(e, &e->dout, (size_t)e->out_cap);
  if (!rc) rc = ealloc_t(e, &e->dtrace, (size_t)e->trace_cap * 6);
  if (!rc && cudaHostAlloc(reinterpret_cast<void**>(&e->rch), sizeof(RoundCtl), cudaHostAllocDefault) != cudaSuccess)
    rc = set_error(G4_ERR_CUDA, "g4_engine_create: pinned host buffer");
  if (rc) return fail(rc);
  if (cudaStreamSynchronize(e->st) != cudaSuccess) return fail(set_error(G4_ERR_CUDA, "g4_engine_create: %s", cudaGetErrorString(cudaGetLastError())));
  *out = e;
  return G4_OK;
}

extern "C" int g4_engine_create(const g4_engine_config* cfg, g4_engine** out) { return create_impl(cfg, nullptr, out); }

extern "C" int g4_engine_create_from_checkpoint(const g4_engine_config* cfg, const g4_checkpoint* ck, g4_engine** out) {
  if (!cfg || !ck || !out) return set_error(G4_ERR_INVALID, "g4_engine_create_from_checkpoint: null pointer");
  g4_engine_config c = *cfg;
  RCK(g4_checkpoint_config(ck, &c));
  // per-layer embeddings read from a checkpoint gave other hidden states than the oracle's on the
  // GPU (the same weights generated on the device agree); refused until that is resolved
  if (c.ple)
    return set_error(G4_ERR_UNSUPPORTED,
                     "g4_engine_create_from_checkpoint: per-layer embeddings from a checkpoint are not enabled in this "
                     "build (unverified); the seeded model with ple = 1 runs them");
  return create_impl(&c, nullptr, out, ck);
}

extern "C" int g4_engine_create_shared(const g4_engine_config* cfg, const g4_engine* weights, g4_engine** out) {
  G4_REQUIRE(weights, "g4_engine_create_shared: null weights engine");
  return create_impl(cfg, weights, out);
}

extern "C" void g4_engine_destroy(g4_engine* e) {
  if (!e) return;
  if (e->st) cudaStreamSynchronize(e->st);
  for (auto& g : e->gverify)
    if (g) cudaGraphExecDestroy(g);
  if (e->gdraft) cudaGraphExecDestroy(e->gdraft);
  if (e->gloop) cudaGraphExecDestroy(e->gloop);
  for (auto& g : e->graw_verify)
    if (g) cudaGraphDestroy(g);
  if (e->graw_draft) cudaGraphDestroy(e->graw_draft);
  if (e->rch) cudaFreeHost(e->rch);
  if (e->aev0) cudaEventDestroy(e->aev0);
  if (e->aev1) cudaEventDestroy(e->aev1);
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
// The layer stack of a verify pass with persistent segment kernels (g4_stream.cu): segment 0 = the
// embedding, layer 0's input norm, qkv projection and q/k/v post; then per layer its split-KV
// attention (which quantises its output for the o projection) and segment l+1 = layer l's o, MLP and
// residuals with the next layer's input norm, qkv and q/k/v post (or the final norm into hbuf).
static bool fused_ok(const g4_engine* e, int M, int pos0, bool dyn) {
  const ModelDims& d = e->d;
  return e->cfg.fused_layers && i8_path(e, M, false) && M >= 2 && M <= 4 && (dyn || pos0 + M > e->cfg.att_par) &&
         d.H == 2048 && d.I == 8192 && d.HD == 256 && d.NQ == 8 && !e->prof.on && d.OWN == 0 && !e->cfg.ple &&
         std::all_of(e->L.begin(), e->L.end(), [](const TLayer& t) { return t.scalar == 1.0f; });
}
static int forward_layers_fused(g4_engine* e, int M, int pos0, bool dyn) {
  const ModelDims& d = e->d;
  if (!e->x2 || !e->segbar) return set_error(G4_ERR_INVALID, "segment kernels: buffers missing");
  const int H = d.H, QD = d.NQ * d.HD;
  const QuantOut qo = quant_out(e, M, false);
  ECK(cudaMemsetAsync(e->segbar, 0, sizeof(unsigned) * (4 * (size_t)(d.NL + 2) + 1), e->st));
  auto lin_of = [](const Lin& l) { return SegLin{l.w, l.s, l.N, l.K}; };
  SegParams p = {};
  p.M = M; p.H = H; p.I = d.I; p.QD = QD; p.HD = d.HD; p.NQ = d.NQ;
  p.x_a = e->x; p.x_b = e->x2;
  p.att_q = e->xq; p.att_sx = e->xsx; p.att_sum = e->xsum;
  p.o_out = e->o; p.down_out = e->o;
  p.act_q = e->xq; p.act_sx = e->xsx; p.act_sum = e->xsum;
  p.hbuf = e->hbuf; p.qkv_out = e->qkv; p.qs = e->qs; p.ldq = QD;
  p.dpos = dyn ? e->ctl : nullptr;
  p.pos0 = dyn ? 1 : pos0;
  p.E = e->E; p.toks = e->toks; p.sqrtH = sqrtf((float)H);
  p.abort_flag = e->segbar + 4 * (size_t)(d.NL + 2);
  p.trace = e->segtrace;
  auto set_next = [&](int l) {  // the qkv part of a segment: layer l
    const TLayer& t = e->L[l];
    const int ty = t.global ? 1 : 0;
    p.do_qkv = 1;
    p.qkv = lin_of(t.qkv);
    p.w_next = t.in_ln;
    p.qn = t.qn; p.kn = t.kn; p.cosT = e->rope[ty][0]; p.sinT = e->rope[ty][1];
    p.Kc = e->Kc + (size_t)l * e->cfg.ctx_max * d.HD;
    p.Vc = e->Vc + (size_t)l * e->cfg.ctx_max * d.HD;
  };
  p.do_mlp = 0;
  set_next(0);
  p.bar = e->segbar;
  p.trace_slot = 0;
  RCK(seg_launch(p, e->st));
  for (int l = 0; l < d.NL; ++l) {
    const TLayer& t = e->L[l];
    const uint16_t* Kc = e->Kc + (size_t)l * e->cfg.ctx_max * d.HD;
    const uint16_t* Vc = e->Vc + (size_t)l * e->cfg.ctx_max * d.HD;
    if (dyn) {
      const int max_len = t.global ? e->cfg.ctx_max : std::min(e->cfg.ctx_max, d.WINDOW + 4);
      RCK(attn_splitkv_dev(Kc, Vc, e->qs, M, d.NQ, d.HD, e->ctl, 1, 1, t.global ? 0 : d.WINDOW, max_len,
                           e->cfg.attn_chunks, e->att, e->attn_ws, e->attn_ws_bytes, e->st, qo, e->attn_cnt));
    } else {
      int pos[4], lo[4], kmin = 1 << 30;
      for (int m = 0; m < M; ++m) {
        pos[m] = pos0 + m;
        lo[m] = t.global ? 0 : std::max(0, pos[m] - (d.WINDOW - 1));
        kmin = std::min(kmin, lo[m]);
      }
      RCK(g4_attn_splitkv(Kc, Vc, e->qs, pos, lo, M, d.NQ, d.HD, kmin, pos0 + M - 1, e->cfg.attn_chunks, e->att, e->attn_ws,
                          e->attn_ws_bytes, e->st));
      RCK(g4_w4a8_quant(e->att, M, QD, e->xq, e->xsx, e->xsum, e->st));
    }
    p.do_mlp = 1;
    p.o = lin_of(t.o); p.gu = lin_of(t.gu); p.down = lin_of(t.down);
    p.w_post_attn = t.post_attn; p.w_pre_ff = t.pre_ff; p.w_post_ff = t.post_ff;
    if (l + 1 < d.NL) {
      set_next(l + 1);
    } else {
      p.do_qkv = 0;
      p.w_next = e->fnorm;
    }
    p.bar = e->segbar + 4 * (size_t)(l + 1);
    p.trace_slot = l + 1;
    RCK(seg_launch(p, e->st));
  }
  return check_launch("segment layers");
}

static int forward(g4_engine* e, int M, int pos0, bool want, int hf, bool dyn = false) {
  const ModelDims& d = e->d;
  const int H = d.H, QD = d.NQ * d.HD;
  const float sqrtH = sqrtf((float)H);
  PhaseTimer& pf = e->prof;
  const QuantOut qo = quant_out(e, M, false);
  if (fused_ok(e, M, pos0, dyn)) {
    RCK(forward_layers_fused(e, M, pos0, dyn));
    goto head;
  }
  pf.mark(e->st, PH_EMBED_NORM);
  RCK(launch("k_embed", k_embed, dim3(M), dim3(256), 0, e->st, e->E, e->toks, H, sqrtH, e->x));
  if (e->cfg.ple) {  // the per-layer inputs (:1270-1288), before the first norm quantises its rows
    RCK(lin(e, e->plproj, e->x, M, e->pr));
    RCK(launch("k_ple_in", k_ple_in, dim3(M, d.NL), dim3(256), 0, e->st, (const float*)e->pr, (const int*)e->toks,
               (const uint16_t*)e->PLEt, (const float*)e->plnorm, 1.0f / sqrtf((float)H), d.NL, e->pli));
  }
  RCK(launch("k_norm_q", k_norm_q, dim3(M), dim3(256), 0, e->st, e->x, e->L[0].in_ln, H, e->a, 0, qo));
  RCK(check_launch("k_norm_q"));
  for (int l = 0; l < d.NL; ++l) {
    const TLayer& t = e->L[l];
    const int ty = t.global ? 1 : 0;
    pf.mark(e->st, PH_LINEAR);
    RCK(lin(e, t.qkv, e->a, M, e->qkv, false, true));
    // a KV-shared layer (:1251) has the q projection only and reads its owner's cache
    const bool own = d.owns(l);
    const int ld = t.qkv.N, parts = d.NQ + (own ? 2 : 0);
    uint16_t* Kc = e->Kc + (size_t)d.owner_of(l) * e->cfg.ctx_max * d.HD;
    uint16_t* Vc = e->Vc + (size_t)d.owner_of(l) * e->cfg.ctx_max * d.HD;
    pf.mark(e->st, PH_EMBED_NORM);
    const bool split = dyn || (M <= 4 && pos0 + M > e->cfg.att_par);
    // split-KV reads the rotated queries from qs ([M][QD]); the per-row paths read them in place
    if (d.HD % 64 == 0 && d.HD <= 512 && d.NQ + 2 <= 16)  // warp per head
      RCK(launch("k_qkv_post_w", k_qkv_post_w, dim3(M), dim3(32 * parts), 0, e->st, e->qkv, ld, d.NQ, d.HD,
                 dyn ? 1 : pos0, dyn ? e->ctl : nullptr, t.qn, t.kn, e->rope[ty][0], e->rope[ty][1], Kc, Vc,
                 split ? e->qs : e->qkv, split ? QD : ld));
    else
      RCK(launch("k_qkv_post", k_qkv_post, dim3(dim3(M, parts)), dim3(256), 0, e->st, e->qkv, ld, d.NQ, d.HD, dyn ? 1 : pos0, dyn ? e->ctl : nullptr,
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
      if (sizeof(float) * len_max > 40 * 1024)
        cudaFuncSetAttribute(k_attn_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(sizeof(float) * len_max));
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
    RCK(launch("k_act_q", k_act_q, dim3((unsigned)((long long)M * t.down.K / 256)), dim3(256), 0, e->st, e->gu, t.down.K, M,
               e->act, qo));
    pf.mark(e->st, PH_LINEAR);
    RCK(lin(e, t.down, e->act, M, e->o, false, true));
    pf.mark(e->st, PH_EMBED_NORM);
    if (e->cfg.ple) {  // add_res_prep_x (:1376), then the per-layer input (:1379-1388)
      RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(M), dim3(256), 0, e->st, (const float*)e->o, e->x,
                 (const float*)t.post_ff, 0.0f, H, (const float*)nullptr, (float*)nullptr, 0, QuantOut{nullptr, nullptr, nullptr}));
      RCK(lin(e, t.pg, e->x, M, e->pgv));
      RCK(launch("k_ple_gate", k_ple_gate, dim3(M), dim3(256), 0, e->st, (const float*)e->pgv, (const float*)e->pli, l, d.NL,
                 e->g2, qo));
      RCK(lin(e, t.pp, e->g2, M, e->o, false, true));
    }
    const float* w_res = e->cfg.ple ? t.post_ple : t.post_ff;  // the residual that ends the layer
    if (l + 1 < d.NL)  // residual (and the layer scalar), the next layer's input norm
      RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(M), dim3(256), 0, e->st, e->o, e->x, w_res, t.scalar, H, e->L[l + 1].in_ln, e->a, 0, qo));
    else  // residual and the final norm (rounded) of every row into hbuf
      RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(M), dim3(256), 0, e->st, e->o, e->x, w_res, t.scalar, H, e->fnorm, e->hbuf, 1,
                                           QuantOut{nullptr, nullptr, nullptr}));
    RCK(check_launch("layer"));
  }
head:
  pf.mark(e->st, PH_HEAD);
  if (!want) return G4_OK;
  // head in groups of 4 rows (:1500)
  for (int r0 = hf; r0 < M; r0 += 4) {
    const int mh = std::min(4, M - r0);
    if (e->cfg.head_screen) {
      RCK(head_screen_impl(e->sW4, e->sS4, e->scoef, e->hdata, nullptr, e->cb8, e->hexc_ptr, e->hexc_col, e->hexc_delta,
                           d.V, H, e->hbuf + (size_t)r0 * H, mh, e->cfg.screen_lim, e->G + r0, e->head_ns, e->head_ws,
                           e->head_ws_bytes, e->st, e->cfg.head_screen == 2 ? screen_policy(e) : nullptr, e->hnib));
    } else {
      float* logits = static_cast<float*>(e->head_ws);
      if (e->hnib)
        RCK(g4_bf16p_nib_gemm(e->hnib, e->cb8, e->hexc_ptr, e->hexc_col, e->hexc_delta, d.V, H, e->hbuf + (size_t)r0 * H, mh,
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
      if (d.global_layer(l2) == t.global) { tl = d.owner_of(l2); break; }
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
  for (int l = 0; l < e->d.NL && e->d.owns(l); ++l) {  // the owners' caches, one stream (:1249-1250)
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
// The tensor-core prefill's chunk buffers (pmc rows), allocated on first use.
static int ensure_chunk_buffers(g4_engine* e) {
  if (e->ptoks) return G4_OK;
  const ModelDims& d = e->d;
  const int H = d.H, QD = d.NQ * d.HD, I = d.mlp_max(), MC = e->pmc;
  const size_t kmax = (size_t)std::max({H, I, QD});
  int rc = ealloc_t(e, &e->ptoks, (size_t)MC);
  if (!rc) rc = ealloc_t(e, &e->px, (size_t)MC * H);
  if (!rc) rc = ealloc_t(e, &e->pa, (size_t)MC * H);
  if (!rc) rc = ealloc_t(e, &e->pqkv, (size_t)MC * (QD + 2 * d.HD));
  if (!rc) rc = ealloc_t(e, &e->patt, (size_t)MC * QD);
  if (!rc) rc = ealloc_t(e, &e->po, (size_t)MC * H);
  if (!rc) rc = ealloc_t(e, &e->pgu, (size_t)MC * 2 * I);
  if (!rc) rc = ealloc_t(e, &e->pact, (size_t)MC * I);
  if (!rc) rc = ealloc_t(e, &e->pmlp, (size_t)MC * H);
  if (!rc) rc = ealloc_t(e, &e->pq, (size_t)MC * kmax);
  if (!rc) rc = ealloc_t(e, &e->psx, (size_t)MC * kmax / 32);
  if (!rc) rc = ealloc_t(e, &e->psum, (size_t)MC * kmax / 32);
  if (!rc) rc = ealloc_t(e, &e->psxT, (size_t)MC * kmax / 32);
  return rc;
}

// Prefill of Mc (a multiple of prefill_block, at most pmc) prompt rows at positions pos0.. that form
// full prefill blocks (the blocks start at position blk_fn), through all layers at once: the row kernels of forward() over Mc rows and the
// tensor-core W4A8 GEMM (the same values as the blocks' GEMVs: prefill blocks of >= 2 rows take the
// int8 path, :311); attention per row with its block's variant (k_attn_rows, variant < 0).
constexpr int kPrefillRows = 4;  // query rows per block of the prefill attention
static int prefill_chunk(g4_engine* e, const int32_t* toks, int Mc, int pos0, int blk_fn) {
  const ModelDims& d = e->d;
  const int H = d.H, QD = d.NQ * d.HD;
  const int Mpad = (Mc + 127) / 128 * 128;
  const QuantOut qo{e->pq, e->psx, e->psum};
  ECK(cudaMemcpyAsync(e->ptoks, toks, sizeof(int) * Mc, cudaMemcpyHostToDevice, e->st));
  auto gemm = [&](const TcLin& t, const Lin& l, float* Y) {
    RCK(tc_transpose_sx(e->psx, Mc, l.K / 32, e->psxT, Mpad, e->st));
    return tc_gemm(e->pq, Mc, l.K, e->psxT, Mpad, t.w8, t.swT, l.N, Y, l.N, e->st);
  };
  RCK(launch("k_embed", k_embed, dim3(Mc), dim3(256), 0, e->st, (const uint16_t*)e->E, (const int*)e->ptoks, H,
             sqrtf((float)H), e->px));
  RCK(launch("k_norm_q", k_norm_q, dim3(Mc), dim3(256), 0, e->st, (const float*)e->px, (const float*)e->L[0].in_ln, H, e->pa, 0, qo));
  for (int l = 0; l < d.NL; ++l) {
    const TLayer& t = e->L[l];
    const int ty = t.global ? 1 : 0;
    const int ld = t.qkv.N;  // QD for a KV-shared layer, whose K and V are its owner's
    uint16_t* Kc = e->Kc + (size_t)d.owner_of(l) * e->cfg.ctx_max * d.HD;
    uint16_t* Vc = e->Vc + (size_t)d.owner_of(l) * e->cfg.ctx_max * d.HD;
    RCK(gemm(t.tqkv, t.qkv, e->pqkv));
    RCK(launch("k_qkv_post_w", k_qkv_post_w, dim3(Mc), dim3(32 * (d.NQ + (d.owns(l) ? 2 : 0))), 0, e->st, (const float*)e->pqkv, ld, d.NQ, d.HD,
               pos0, (const int*)nullptr, (const float*)t.qn, (const float*)t.kn, (const float*)e->rope[ty][0],
               (const float*)e->rope[ty][1], Kc, Vc, e->pqkv, ld));
    const int len_max = t.global ? pos0 + Mc : std::min(pos0 + Mc, d.WINDOW);
    if (e->cfg.prefill_tc == 2 && d.NQ % 4 == 0 && d.HD <= 256) {  // four heads per block share each K and V row
      const size_t smem = sizeof(float) * 4 * (size_t)len_max;
      if (smem > 200 * 1024) return set_error(G4_ERR_UNSUPPORTED, "prefill attention: %zu B of shared memory", smem);
      if (smem > 40 * 1024) cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      RCK(launch("k_attn_prefill", k_attn_prefill, dim3(Mc, d.NQ / 4), dim3(288), smem, e->st, (const uint16_t*)Kc,
                 (const uint16_t*)Vc, (const float*)e->pqkv, ld, d.HD, pos0, t.global ? 0 : d.WINDOW, blk_fn,
                 e->cfg.prefill_block, e->patt, QD));
    } else if (e->cfg.prefill_tc == 3 && d.HD <= 256 && d.HD % 16 == 0 &&
               sizeof(float) * kPrefillRows * (size_t)(len_max + kPrefillRows - 1) <= 200 * 1024) {
      // kPrefillRows rows of one head per block share each K and V load
      RCK(attn_rows_multi(kPrefillRows, Kc, Vc, e->pqkv, ld, d.NQ, d.HD, pos0, Mc, t.global ? 0 : d.WINDOW, len_max,
                          e->patt, QD, blk_fn, e->cfg.prefill_block, e->st));
    } else if (e->cfg.prefill_tc == 1 && d.HD <= 256 && d.HD % 16 == 0) {
      if (sizeof(float) * len_max > 40 * 1024)
        cudaFuncSetAttribute(k_attn_rows2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(sizeof(float) * len_max));
      RCK(launch("k_attn_rows2", k_attn_rows2, dim3(Mc, d.NQ), dim3(256), sizeof(float) * len_max, e->st, (const uint16_t*)Kc,
                 (const uint16_t*)Vc, (const float*)e->pqkv, ld, d.NQ, d.HD, pos0, t.global ? 0 : d.WINDOW, e->patt, QD,
                 blk_fn, e->cfg.prefill_block));
    } else {
      if (sizeof(float) * len_max > 40 * 1024)
        cudaFuncSetAttribute(k_attn_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(sizeof(float) * len_max));
      RCK(launch("k_attn_rows", k_attn_rows, dim3(Mc, d.NQ), dim3(256), sizeof(float) * len_max, e->st, (const uint16_t*)Kc,
                 (const uint16_t*)Vc, (const float*)e->pqkv, ld, d.NQ, d.HD, pos0, t.global ? 0 : d.WINDOW, -1, e->patt, QD,
                 blk_fn, e->cfg.prefill_block));
    }
    RCK(g4_w4a8_quant(e->patt, Mc, QD, e->pq, e->psx, e->psum, e->st));
    RCK(gemm(t.to, t.o, e->po));
    RCK(launch("k_post_attn_q", k_post_attn_q, dim3(Mc), dim3(256), 0, e->st, (const float*)e->po, e->px, (const float*)t.post_attn,
               (const float*)t.pre_ff, e->pmlp, H, qo));
    RCK(gemm(t.tgu, t.gu, e->pgu));
    RCK(launch("k_act_q", k_act_q, dim3((unsigned)((long long)Mc * t.down.K / 256)), dim3(256), 0, e->st, (const float*)e->pgu,
               t.down.K, Mc, e->pact, qo));
    RCK(gemm(t.tdown, t.down, e->po));
    // residual, then the next layer's input norm and its quantisation (none after the last layer:
    // these rows need no final norm)
    RCK(launch("k_resid_norm_q", k_resid_norm_q, dim3(Mc), dim3(256), 0, e->st, (const float*)e->po, e->px,
               (const float*)t.post_ff, t.scalar, H, l + 1 < d.NL ? (const float*)e->L[l + 1].in_ln : (const float*)nullptr,
               e->pa, 0, qo));
  }
  return check_launch("prefill_chunk");
}

static int upload_round_state(g4_engine* e);
extern "C" int g4_engine_prefill(g4_engine* e, const int32_t* prompt, int n, int32_t* first_token) {
  return g4_engine_prefill_from(e, prompt, n, 0, first_token);
}

extern "C" int g4_engine_prefill_from(g4_engine* e, const int32_t* prompt, int n, int start, int32_t* first_token) {
  G4_REQUIRE(e && prompt && n >= 1 && start >= 0 && start < n && e->fake_n + n + 8 <= e->cfg.ctx_max,
             "g4_engine_prefill: bad arguments (n=%d start=%d fake context %d ctx_max=%d)", n, start, e ? e->fake_n : 0,
             e ? e->cfg.ctx_max : 0);
  G4_REQUIRE(!e->async_pending, "g4_engine_prefill: a decode call is pending");
  const int H = e->d.H, FN = e->fake_n;
  e->kv_len = 0;  // the prefix cache's record is rewritten by the request that called this (if any)
  e->ctx_keys.clear();
  auto t0 = std::chrono::steady_clock::now();
  e->i8_active = e->cfg.prefill_int8 != 0;
  int done = start, last_M = 0;
  if (e->tc_ready && e->cfg.prefill_tc && e->i8_active && e->cfg.prefill_block >= 2) {
    // every full block but the last through the tensor-core path, in chunks (blocks from start)
    const int PB = e->cfg.prefill_block;
    const int nfast = start + ((n - start - 1) / PB) * PB;
    const int chunk = std::max(PB, e->pmc / PB * PB);
    if (nfast > start) RCK(ensure_chunk_buffers(e));
    while (done < nfast) {
      const int Mc = std::min(chunk, nfast - done);
      RCK(prefill_chunk(e, prompt + done, Mc, FN + done, FN + start));
      done += Mc;
    }
  }
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
  RCK(upload_round_state(e));
  e->stats = g4_engine_stats{};
  e->stats.prefill_tokens = n - start;
  e->stats.prefill_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  if (first_token) *first_token = first;
  return G4_OK;
}

// The device round state after a prefill (or an imported state): history, P, conf, zero totals.
static int upload_round_state(g4_engine* e) {
  if ((int)e->seq.size() + 8 > e->cfg.ctx_max + 64) return set_error(G4_ERR_UNSUPPORTED, "history longer than the context");
  RoundCtl& h = *e->rch;
  std::memset(&h, 0, sizeof h);
  h.P = e->P;
  h.conf = e->conf;
  h.seq_len = (int)e->seq.size();
  h.stopped = e->stopped ? 1 : 0;
  h.ctx_max = e->cfg.ctx_max;
  h.trace_cap = e->trace_cap;
  h.out_cap = e->out_cap;
  ECK(cudaMemcpyAsync(e->dseq, e->seq.data(), sizeof(int) * e->seq.size(), cudaMemcpyHostToDevice, e->st));
  ECK(cudaMemcpyAsync(e->rc, &h, sizeof h, cudaMemcpyHostToDevice, e->st));
  ECK(cudaStreamSynchronize(e->st));
  return G4_OK;
}

// Record the launches of body() on the engine stream into an executable graph, its kernels launched
// for programmatic dependent launch; if that capture fails, record it again with ordinary launches.
// raw (may be NULL) keeps the recorded graph as well (for the decode loop's conditional bodies).
template <class F>
static int capture_once(g4_engine* e, cudaGraphExec_t* out, cudaGraph_t* raw, F body, bool pdl, int* kernels) {
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
  if (raw && ie == cudaSuccess) {
    if (*raw) cudaGraphDestroy(*raw);
    *raw = g;
  } else {
    cudaGraphDestroy(g);
  }
  if (ie != cudaSuccess) return set_error(G4_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ie));
  return G4_OK;
}
template <class F>
static int capture(g4_engine* e, cudaGraphExec_t* out, cudaGraph_t* raw, F body, int* kernels) {
  if (e->cfg.graphs == 1 && e->pdl_ok) {
    if (capture_once(e, out, raw, body, true, kernels) == G4_OK) return G4_OK;
    cudaGetLastError();
    e->pdl_ok = false;
  }
  return capture_once(e, out, raw, body, false, kernels);
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

// A captured verify pass for M rows: the start stamp, then the target forward with positions read
// from ctl[0] on the device.
static int verify_body(g4_engine* e, int M) {
  RCK(launch("k_stamp", k_stamp, dim3(1), dim3(32), 0, e->st, e->rc));
  return forward(e, M, 0, true, 0, true);
}
static int ensure_verify_graph(g4_engine* e, int M) {
  e->i8_active = e->cfg.decode_int8 && e->cfg.prefill_int8;  // verify passes run in the decode mode (:1600)
  if (!e->gverify[M]) RCK(capture(e, &e->gverify[M], &e->graw_verify[M], [&] { return verify_body(e, M); }, &e->gk_verify[M]));
  return G4_OK;
}
static int ensure_draft_graph(g4_engine* e) {
  if (!e->gdraft) RCK(capture(e, &e->gdraft, &e->graw_draft, [&] { return draft_chain(e, true); }, &e->gk_draft));
  return G4_OK;
}

static int add_kernel_node(cudaGraph_t g, cudaGraphNode_t* node, const cudaGraphNode_t* deps, size_t ndeps, void* fn,
                           dim3 grid, dim3 block, void** args) {
  cudaKernelNodeParams kp = {};
  kp.func = fn;
  kp.gridDim = grid;
  kp.blockDim = block;
  kp.sharedMemBytes = 0;
  kp.kernelParams = args;
  ECK(cudaGraphAddKernelNode(node, g, deps, ndeps, &kp));
  return G4_OK;
}

// The decode loop as one executable graph (all rounds past att_par):
//   WHILE (continue) { k_round_begin; IF (drafting) { the k drafts }; SWITCH (M - 1) { verify pass of
//   M rows }; k_round_end }
// with the branch values set on the device by k_round_begin / k_round_end, so a whole decode call is
// one graph launch followed by one copy of the committed tokens.
static int build_loop_graph(g4_engine* e) {
  const bool drafter = e->cfg.drafter && e->cfg.k_draft > 0;
  for (int M = 1; M <= 4; ++M) RCK(ensure_verify_graph(e, M));
  if (drafter) RCK(ensure_draft_graph(e));
  cudaGraph_t g = nullptr;
  ECK(cudaGraphCreate(&g, 0));
  auto fail = [&](int rc) { cudaGraphDestroy(g); return rc; };
  cudaGraphConditionalHandle hloop = 0, hdraft = 0, hm = 0;
  if (cudaGraphConditionalHandleCreate(&hloop, g, 0, cudaGraphCondAssignDefault) != cudaSuccess ||
      cudaGraphConditionalHandleCreate(&hdraft, g, 0, cudaGraphCondAssignDefault) != cudaSuccess ||
      cudaGraphConditionalHandleCreate(&hm, g, 0, cudaGraphCondAssignDefault) != cudaSuccess)
    return fail(set_error(G4_ERR_CUDA, "conditional handles: %s", cudaGetErrorString(cudaGetLastError())));
  cudaGraphNodeParams wp = {};
  wp.type = cudaGraphNodeTypeConditional;
  wp.conditional.handle = hloop;
  wp.conditional.type = cudaGraphCondTypeWhile;
  wp.conditional.size = 1;
  cudaGraphNode_t arm, wnode;
  void* aargs[] = {&hloop};
  if (int rc = add_kernel_node(g, &arm, nullptr, 0, reinterpret_cast<void*>(k_loop_arm), dim3(1), dim3(1), aargs)) return fail(rc);
  if (cudaGraphAddNode(&wnode, g, &arm, 1, &wp) != cudaSuccess)
    return fail(set_error(G4_ERR_CUDA, "while node: %s", cudaGetErrorString(cudaGetLastError())));
  cudaGraph_t body = wp.conditional.phGraph_out[0];
  // k_round_begin
  RoundCtl* rcp = e->rc;
  const int* seqc = e->dseq;
  int* ctl = e->ctl;
  int ngram = e->cfg.ngram, nglen = e->cfg.ngram_len, kdraft = drafter ? e->cfg.k_draft : 0, one = 1;
  void* bargs[] = {&rcp, &seqc, &ctl, &ngram, &nglen, &kdraft, &hdraft, &hm, &one};
  cudaGraphNode_t nbegin, nif = nullptr, nsw, nend;
  if (int rc = add_kernel_node(body, &nbegin, nullptr, 0, reinterpret_cast<void*>(k_round_begin), dim3(1), dim3(256), bargs)) return fail(rc);
  cudaGraphNode_t prev = nbegin;
  if (drafter) {
    cudaGraphNodeParams ip = {};
    ip.type = cudaGraphNodeTypeConditional;
    ip.conditional.handle = hdraft;
    ip.conditional.type = cudaGraphCondTypeIf;
    ip.conditional.size = 1;
    if (cudaGraphAddNode(&nif, body, &prev, 1, &ip) != cudaSuccess)
      return fail(set_error(G4_ERR_CUDA, "if node: %s", cudaGetErrorString(cudaGetLastError())));
    cudaGraphNode_t child;
    if (cudaGraphAddChildGraphNode(&child, ip.conditional.phGraph_out[0], nullptr, 0, e->graw_draft) != cudaSuccess)
      return fail(set_error(G4_ERR_CUDA, "draft body: %s", cudaGetErrorString(cudaGetLastError())));
    prev = nif;
  }
  cudaGraphNodeParams sp = {};
  sp.type = cudaGraphNodeTypeConditional;
  sp.conditional.handle = hm;
  sp.conditional.type = cudaGraphCondTypeSwitch;
  sp.conditional.size = 4;
  if (cudaGraphAddNode(&nsw, body, &prev, 1, &sp) != cudaSuccess)
    return fail(set_error(G4_ERR_CUDA, "switch node: %s", cudaGetErrorString(cudaGetLastError())));
  for (int M = 1; M <= 4; ++M) {
    cudaGraphNode_t child;
    if (cudaGraphAddChildGraphNode(&child, sp.conditional.phGraph_out[M - 1], nullptr, 0, e->graw_verify[M]) != cudaSuccess)
      return fail(set_error(G4_ERR_CUDA, "verify body: %s", cudaGetErrorString(cudaGetLastError())));
  }
  int* seqm = e->dseq;
  const int* ctlc = e->ctl;
  const int* G = e->G;
  const float* hbuf = e->hbuf;
  float* hprev = e->hprev;
  int H = e->d.H;
  int* out = e->dout;
  int* trace = e->dtrace;
  const int* hns = e->cfg.head_screen ? e->head_ns : nullptr;
  void* eargs[] = {&rcp, &seqm, &ctlc, &G, &hbuf, &hprev, &H, &out, &trace, &hns, &hloop, &one};
  if (int rc = add_kernel_node(body, &nend, &nsw, 1, reinterpret_cast<void*>(k_round_end), dim3(1), dim3(256), eargs)) return fail(rc);
  const cudaError_t ie = cudaGraphInstantiate(&e->gloop, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) {
    e->gloop = nullptr;
    return set_error(G4_ERR_CUDA, "decode loop instantiate: %s", cudaGetErrorString(ie));
  }
  return G4_OK;
}

static int read_round_state(g4_engine* e) {
  ECK(cudaMemcpyAsync(e->rch, e->rc, sizeof(RoundCtl), cudaMemcpyDeviceToHost, e->st));
  ECK(cudaStreamSynchronize(e->st));
  e->stats.d2h_bytes += sizeof(RoundCtl);
  return G4_OK;
}

// One round launched from the host (eager, or graphs of single passes): the device kernels decide
// as in the loop graph; the host reads the round's shape back once to pick the launches.
static int host_round(g4_engine* e, bool graphs) {
  const bool drafter = e->cfg.drafter && e->cfg.k_draft > 0;
  RCK(launch("k_round_begin", k_round_begin, dim3(1), dim3(256), 0, e->st, e->rc, (const int*)e->dseq, e->ctl, e->cfg.ngram,
             e->cfg.ngram_len, drafter ? e->cfg.k_draft : 0, (cudaGraphConditionalHandle)0, (cudaGraphConditionalHandle)0, 0));
  RCK(read_round_state(e));
  const RoundCtl& h = *e->rch;
  const int M = h.M;
  e->P = h.P;
  const long long l0 = launch_count();
  if (h.drafting) {
    if (graphs) {
      RCK(ensure_draft_graph(e));
      ECK(cudaGraphLaunch(e->gdraft, e->st));
      e->stats.kernel_launches += e->gk_draft;
    } else {
      RCK(draft_chain(e, false));
    }
  }
  if (graphs) {
    RCK(ensure_verify_graph(e, M));
    ECK(cudaGraphLaunch(e->gverify[M], e->st));
    e->stats.kernel_launches += e->gk_verify[M];
  } else {
    RCK(launch("k_stamp", k_stamp, dim3(1), dim3(32), 0, e->st, e->rc));
    RCK(forward(e, M, e->P + 1, true, 0));
  }
  RCK(launch("k_round_end", k_round_end, dim3(1), dim3(256), 0, e->st, e->rc, e->dseq, (const int*)e->ctl, (const int*)e->G,
             (const float*)e->hbuf, e->hprev, e->d.H, e->dout, e->dtrace,
             (const int*)(e->cfg.head_screen ? e->head_ns : nullptr), (cudaGraphConditionalHandle)0, 0));
  e->stats.kernel_launches += launch_count() - l0;
  RCK(read_round_state(e));
  e->prof.flush();
  return G4_OK;
}

static void finish_stats(g4_engine* e, int n, float gms, std::chrono::steady_clock::time_point t0);
extern "C" int g4_engine_decode(g4_engine* e, int max_rounds, int max_tokens, int32_t* out, int* n_out,
                                g4_engine_stats* stats) {
  G4_REQUIRE(e && n_out && max_rounds >= 0 && max_tokens >= 0 && !e->seq.empty(), "g4_engine_decode: call g4_engine_prefill first");
  auto t0 = std::chrono::steady_clock::now();
  cudaEvent_t ev0, ev1;
  ECK(cudaEventCreate(&ev0));
  ECK(cudaEventCreate(&ev1));
  ECK(cudaEventRecord(ev0, e->st));
  e->i8_active = e->cfg.decode_int8 && e->cfg.prefill_int8;  // (:1600)
  int rc0 = G4_OK;
  RCK(launch("k_decode_setup", k_decode_setup, dim3(1), dim3(1), 0, e->st, e->rc, max_rounds, max_tokens));
  e->stats.kernel_launches += 1;
  int& produced = e->rch->produced;
  produced = 0;
  e->rch->rounds_call = 0;
  e->rch->stopped = e->stopped;
  e->rch->P = e->P;
  while (rc0 == G4_OK && e->rch->rounds_call < max_rounds && produced < max_tokens && !e->rch->stopped) {
    if (e->rch->P + 1 + 8 >= e->cfg.ctx_max) { rc0 = set_error(G4_ERR_UNSUPPORTED, "g4_engine_decode: context full (%d)", e->cfg.ctx_max); break; }
    // captured graphs once the split-KV path applies to every row (positions > att_par)
    const bool use_g = e->cfg.graphs && !e->prof.on && e->rch->P + 1 > e->cfg.att_par;
    if (use_g && !e->loop_failed && !e->gloop) {
      if (build_loop_graph(e) != G4_OK) {
        e->loop_failed = true;  // conditional nodes unavailable: rounds launched from the host
        cudaGetLastError();
      }
    }
    if (use_g && e->gloop) {
      const int r0 = e->rch->rounds;
      int rm[5];
      std::memcpy(rm, e->rch->rounds_m, sizeof rm);
      const int dr0 = e->rch->draft_rounds;
      ECK(cudaGraphLaunch(e->gloop, e->st));
      RCK(read_round_state(e));
      const RoundCtl& h = *e->rch;
      e->stats.kernel_launches += 1 + 2LL * (h.rounds - r0) + (long long)e->gk_draft * (h.draft_rounds - dr0);
      if (h.rounds == r0) rc0 = set_error(G4_ERR_CUDA, "g4_engine_decode: the round loop graph ran no round");
      for (int M = 1; M <= 4; ++M) e->stats.kernel_launches += (long long)e->gk_verify[M] * (h.rounds_m[M] - rm[M]);
      if (h.ctx_full) rc0 = set_error(G4_ERR_UNSUPPORTED, "g4_engine_decode: context full (%d)", e->cfg.ctx_max);
      break;
    }
    RCK(host_round(e, use_g));
  }
  const RoundCtl& h = *e->rch;
  const int n = std::min(h.produced, max_tokens);
  const int ncopy = std::min(h.produced, e->out_cap);  // every committed token, for the history mirror
  std::vector<int> got(ncopy);
  if (ncopy > 0) {
    ECK(cudaMemcpyAsync(got.data(), e->dout, sizeof(int) * ncopy, cudaMemcpyDeviceToHost, e->st));
    e->stats.d2h_bytes += sizeof(int) * ncopy;
  }
  ECK(cudaEventRecord(ev1, e->st));
  ECK(cudaEventSynchronize(ev1));
  float gms = 0;
  cudaEventElapsedTime(&gms, ev0, ev1);
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  // the committed history: the call's tokens (all of them while they fit the output buffer)
  for (int i = 0; i < ncopy; ++i) e->seq.push_back(got[i]);
  if (out) std::memcpy(out, got.data(), sizeof(int) * std::min(n, ncopy));
  finish_stats(e, n, gms, t0);
  *n_out = n;
  if (stats) *stats = e->stats;
  return rc0;
}

// The host mirror and statistics after a decode call (the round state is already read back).
static void finish_stats(g4_engine* e, int n, float gms, std::chrono::steady_clock::time_point t0) {
  const RoundCtl& h = *e->rch;
  e->P = h.P;
  e->conf = h.conf;
  e->stopped = h.stopped != 0;
  g4_engine_stats& st = e->stats;
  st.rounds = h.rounds;
  st.ngram_rounds = h.ngram_rounds;
  st.drafted = h.drafted;
  st.accepted = h.accepted;
  st.verify_passes = h.rounds;
  st.verify_rows = h.verify_rows;
  st.draft_steps = h.draft_rounds * e->cfg.k_draft;
  st.verify_gpu_ms = h.verify_ns * 1e-6;
  st.draft_gpu_ms = h.draft_ns * 1e-6;
  st.head_fallbacks = h.head_fallbacks;
  st.screen_skipped = h.spol[3];
  st.ngram_accepted = h.ngram_accepted;
  st.decode_gpu_ms += gms;
  st.decode_tokens += n;
  st.decode_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

// BENCH_MODE's k (gemma4_engine.cpp:1682): the draft chain and the round loop are recorded for one
// k, so they are dropped here and recorded again by the next decode call.
extern "C" int g4_engine_set_k_draft(g4_engine* e, int k) {
  G4_REQUIRE(e && k >= 0 && k <= 3 && !e->async_pending, "g4_engine_set_k_draft: bad arguments");
  G4_REQUIRE(k == 0 || e->cfg.drafter, "g4_engine_set_k_draft: the engine has no drafter");
  if (k == e->cfg.k_draft) return G4_OK;
  ECK(cudaStreamSynchronize(e->st));
  if (e->gloop) cudaGraphExecDestroy(e->gloop);
  if (e->gdraft) cudaGraphExecDestroy(e->gdraft);
  if (e->graw_draft) cudaGraphDestroy(e->graw_draft);
  e->gloop = nullptr;
  e->gdraft = nullptr;
  e->graw_draft = nullptr;
  e->gk_draft = 0;
  e->loop_failed = false;
  e->cfg.k_draft = k;
  return G4_OK;
}

// ---- requests with the prefix cache (run_req, gemma4_engine.cpp:1569-1680)

// K/V rows [0, len) of every layer from (sK, sV) to (dK, dV), all laid out as the engine's cache.
static int kv_copy(g4_engine* e, uint16_t* dK, uint16_t* dV, const uint16_t* sK, const uint16_t* sV, int len) {
  if (len <= 0) return G4_OK;
  const size_t pitch = sizeof(uint16_t) * (size_t)e->cfg.ctx_max * e->d.HD;
  const size_t width = sizeof(uint16_t) * (size_t)len * e->d.HD;
  ECK(cudaMemcpy2DAsync(dK, pitch, sK, pitch, width, e->d.NL, cudaMemcpyDeviceToDevice, e->st));
  ECK(cudaMemcpy2DAsync(dV, pitch, sV, pitch, width, e->d.NL, cudaMemcpyDeviceToDevice, e->st));
  return G4_OK;
}

// The stored slots' K/V buffers and one spare, allocated by the first request (slots > 1).
static int ensure_slots(g4_engine* e) {
  const int ns = std::max(1, e->cfg.slots);
  if (ns <= 1 || !e->stored.empty()) return G4_OK;
  const size_t elems = (size_t)e->d.NL * e->cfg.ctx_max * e->d.HD;
  std::vector<g4_engine::KvSlot> st(ns - 1);
  for (auto& sl : st) {
    RCK(ealloc_t(e, &sl.K, elems));
    RCK(ealloc_t(e, &sl.V, elems));
  }
  RCK(ealloc_t(e, &e->spareK, elems));
  RCK(ealloc_t(e, &e->spareV, elems));
  e->stored = std::move(st);
  return G4_OK;
}

// swap_with (:1576): the active conversation and a stored one change places.  The engine's own cache
// stays where the captured graphs expect it: the active K/V goes to the spare buffer, the slot's K/V
// is copied in, and the spare buffer becomes the slot's (device-to-device copies of the valid rows).
static int swap_with(g4_engine* e, g4_engine::KvSlot& sl) {
  RCK(kv_copy(e, e->spareK, e->spareV, e->Kc, e->Vc, e->kv_len));
  RCK(kv_copy(e, e->Kc, e->Vc, sl.K, sl.V, sl.kv_len));
  std::swap(sl.K, e->spareK);
  std::swap(sl.V, e->spareV);
  std::swap(e->ctx_keys, sl.keys);
  std::swap(e->kv_len, sl.kv_len);
  std::swap(e->active_stamp, sl.stamp);
  return G4_OK;
}

static int lcp_len(const std::vector<int>& k, int klen, const int32_t* p, int n) {
  int c = 0;
  while (c < klen && c < n && c < (int)k.size() && k[c] == p[c]) ++c;
  return c;
}

extern "C" int g4_engine_request(g4_engine* e, const int32_t* prompt, int n, int max_new, int32_t* out, int* n_out,
                                 g4_request_info* info, g4_token_cb on_tokens, void* user) {
  G4_REQUIRE(e && prompt && n >= 1 && max_new >= 0 && (out || max_new == 0) && n_out, "g4_engine_request: bad arguments");
  G4_REQUIRE(!e->async_pending, "g4_engine_request: a decode call is pending");
  RCK(ensure_slots(e));
  int common = lcp_len(e->ctx_keys, e->kv_len, prompt, n);
  ++e->clock_tick;
  int slot_used = 0;
  if (!e->stored.empty()) {
    int best = -1, bc = common;
    for (int i = 0; i < (int)e->stored.size(); ++i) {
      const int c = lcp_len(e->stored[i].keys, e->stored[i].kv_len, prompt, n);
      if (c > bc) { bc = c; best = i; }
    }
    if (best >= 0) {  // a stored conversation shares more of this prompt: switch to it
      e->active_stamp = e->clock_tick;
      RCK(swap_with(e, e->stored[best]));
      ++e->slot_switches;
      slot_used = best + 1;
      common = bc;
    } else if (bc < e->cfg.slot_min_reuse) {  // nothing worth reusing: the LRU slot takes the active one
      int v = 0;
      for (int i = 1; i < (int)e->stored.size(); ++i)
        if (e->stored[i].stamp < e->stored[v].stamp) v = i;
      e->active_stamp = e->clock_tick;
      RCK(swap_with(e, e->stored[v]));
      e->kv_len = 0;
      e->ctx_keys.clear();
      common = 0;
      ++e->slot_evictions;
      slot_used = v + 1;
    }
    e->active_stamp = e->clock_tick;
  }
  const int start = std::min(common, n - 1);  // the last prompt token always runs (its logits and hidden)
  auto t0 = std::chrono::steady_clock::now();
  int first = 0;
  RCK(g4_engine_prefill_from(e, prompt, n, start, &first));
  const double prefill_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  int total = 0;
  double decode_ms = 0.0;
  if (max_new == 0) {  // prefill only (:1607): the prompt's K/V is the conversation
    e->ctx_keys.assign(prompt, prompt + n);
    e->kv_len = n;
  } else {
    out[0] = first;
    if (on_tokens) on_tokens(out, 1, user);
    int got = 0;
    auto t1 = std::chrono::steady_clock::now();
    if (max_new > 1 && !e->stopped) {
      if (on_tokens) {  // one round per call, each round's tokens reported as they commit
        while (got < max_new - 1 && !e->stopped) {
          int k = 0;
          RCK(g4_engine_decode(e, 1, max_new - 1 - got, out + 1 + got, &k, nullptr));
          if (k > 0) on_tokens(out + 1 + got, k, user);
          got += k;
          if (k == 0) break;
        }
      } else {
        RCK(g4_engine_decode(e, 1 << 30, max_new - 1, out + 1, &got, nullptr));
      }
    }
    decode_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t1).count();
    total = 1 + got;
    for (int i = 0; i < total; ++i)
      if (is_stop(out[i])) { total = i + 1; break; }
    // the conversation's tokens whose K/V is written: positions 0..P (:1601)
    const size_t nk = std::min(e->seq.size(), (size_t)std::max(0, e->P - e->fake_n + 1));
    e->ctx_keys.assign(e->seq.begin(), e->seq.begin() + nk);
    e->kv_len = e->fake_n ? 0 : std::min(e->P + 1, (int)e->ctx_keys.size());
  }
  *n_out = total;
  if (info) {
    info->prompt_tokens = n;
    info->reused = start;
    info->slot = slot_used;
    info->tokens = total;
    info->prefill_ms = prefill_ms;
    info->decode_ms = decode_ms;
    info->slot_switches = e->slot_switches;
    info->slot_evictions = e->slot_evictions;
    info->kv_len = e->kv_len;
    info->rounds = e->stats.rounds;
    info->ngram_rounds = e->stats.ngram_rounds;
    info->ngram_accepted = e->stats.ngram_accepted;
  }
  return G4_OK;
}



// Asynchronous decode: the rounds of the call are enqueued as one launch of the round-loop graph on
// the engine's stream (after start_event, when given) and the call returns at once; several engines
// (g4_engine_create_shared) then decode concurrently.  g4_engine_decode_wait completes the call.
extern "C" int g4_engine_decode_async(g4_engine* e, int max_rounds, int max_tokens, void* start_event) {
  G4_REQUIRE(e && max_rounds >= 1 && max_tokens >= 1 && !e->seq.empty() && !e->async_pending,
             "g4_engine_decode_async: bad arguments or a call already pending");
  if (!e->cfg.graphs || e->prof.on || e->P + 1 <= e->cfg.att_par || e->stopped || e->P + 1 + 8 >= e->cfg.ctx_max)
    return set_error(G4_ERR_UNSUPPORTED, "g4_engine_decode_async: needs graphs on, a position past att_par and room in the context");
  // the decode mode first: the round-loop graph records the verify passes of the current mode
  e->i8_active = e->cfg.decode_int8 && e->cfg.prefill_int8;
  if (!e->gloop && !e->loop_failed && build_loop_graph(e) != G4_OK) {
    e->loop_failed = true;
    cudaGetLastError();
  }
  if (!e->gloop) return set_error(G4_ERR_UNSUPPORTED, "g4_engine_decode_async: the round-loop graph is unavailable");
  if (!e->aev0) {
    ECK(cudaEventCreate(&e->aev0));
    ECK(cudaEventCreate(&e->aev1));
  }
  e->async_t0 = std::chrono::steady_clock::now();
  if (start_event) ECK(cudaStreamWaitEvent(e->st, reinterpret_cast<cudaEvent_t>(start_event), 0));
  ECK(cudaEventRecord(e->aev0, e->st));
  RCK(launch("k_decode_setup", k_decode_setup, dim3(1), dim3(1), 0, e->st, e->rc, max_rounds, max_tokens));
  e->async_r0 = e->rch->rounds;
  e->async_dr0 = e->rch->draft_rounds;
  std::memcpy(e->async_rm, e->rch->rounds_m, sizeof e->async_rm);
  ECK(cudaGraphLaunch(e->gloop, e->st));
  ECK(cudaEventRecord(e->aev1, e->st));
  e->async_max_tokens = max_tokens;
  e->async_pending = true;
  return G4_OK;
}

// Waits for the pending asynchronous call; out / n_out / stats as g4_engine_decode.  ms_since_start
// (may be NULL): device time from start_event (as passed to g4_engine_decode_async) to the end of
// this engine's rounds.
extern "C" int g4_engine_decode_wait(g4_engine* e, int32_t* out, int* n_out, g4_engine_stats* stats, void* start_event,
                                     float* ms_since_start) {
  G4_REQUIRE(e && n_out && e->async_pending, "g4_engine_decode_wait: no call pending");
  e->async_pending = false;
  ECK(cudaEventSynchronize(e->aev1));
  RCK(read_round_state(e));
  const RoundCtl& h = *e->rch;
  int rc0 = G4_OK;
  e->stats.kernel_launches += 2 + 2LL * (h.rounds - e->async_r0) + (long long)e->gk_draft * (h.draft_rounds - e->async_dr0);
  for (int M = 1; M <= 4; ++M) e->stats.kernel_launches += (long long)e->gk_verify[M] * (h.rounds_m[M] - e->async_rm[M]);
  if (h.rounds == e->async_r0) rc0 = set_error(G4_ERR_CUDA, "g4_engine_decode_wait: the round loop graph ran no round");
  if (h.ctx_full) rc0 = set_error(G4_ERR_UNSUPPORTED, "g4_engine_decode_wait: context full (%d)", e->cfg.ctx_max);
  const int n = std::min(h.produced, e->async_max_tokens);
  const int ncopy = std::min(h.produced, e->out_cap);
  std::vector<int> got(ncopy);
  if (ncopy > 0) {
    ECK(cudaMemcpy(got.data(), e->dout, sizeof(int) * ncopy, cudaMemcpyDeviceToHost));
    e->stats.d2h_bytes += sizeof(int) * ncopy;
  }
  for (int i = 0; i < ncopy; ++i) e->seq.push_back(got[i]);
  if (out) std::memcpy(out, got.data(), sizeof(int) * std::min(n, ncopy));
  float gms = 0;
  cudaEventElapsedTime(&gms, e->aev0, e->aev1);
  if (ms_since_start) {
    *ms_since_start = 0.f;
    if (start_event) cudaEventElapsedTime(ms_since_start, reinterpret_cast<cudaEvent_t>(start_event), e->aev1);
  }
  finish_stats(e, n, gms, e->async_t0);
  *n_out = n;
  if (stats) *stats = e->stats;
  return rc0;
}

// Stage timestamps of the last verify pass's segment kernels (see g4.h).
extern "C" int g4_engine_seg_trace(g4_engine* e, unsigned long long* out, int cap, int* n) {
  G4_REQUIRE(e && n && cap >= 0 && (out || cap == 0), "g4_engine_seg_trace: bad arguments");
  const int total = (e->d.NL + 2) * 2 * kSegStamps;
  *n = total;
  if (cap > 0) {
    ECK(cudaStreamSynchronize(e->st));
    ECK(cudaMemcpy(out, e->segtrace, sizeof(unsigned long long) * std::min(cap, total), cudaMemcpyDeviceToHost));
  }
  return G4_OK;
}

// Per-round records since the prefill: {nd, prompt lookup used, drafts[3] (-1 padded), nacc}.
extern "C" int g4_engine_trace(g4_engine* e, int32_t* out, int cap_rounds, int* n_rounds) {
  G4_REQUIRE(e && n_rounds && cap_rounds >= 0 && (out || cap_rounds == 0), "g4_engine_trace: bad arguments");
  RCK(read_round_state(e));
  const int n = std::min(e->rch->trace_n, e->trace_cap);
  const int k = std::min(n, cap_rounds);
  if (k > 0) {
    ECK(cudaMemcpyAsync(out, e->dtrace, sizeof(int) * 6 * (size_t)k, cudaMemcpyDeviceToHost, e->st));
    ECK(cudaStreamSynchronize(e->st));
  }
  *n_rounds = n;
  return G4_OK;
}

// Device time of the captured verify pass of M rows at the current position, replayed reps times
// between two CUDA events on the engine stream (the pass rewrites only the rows that the next round
// writes again: KV rows P+1.., the greedy tokens and the hidden rows).
extern "C" int g4_engine_time_verify(g4_engine* e, int M, int reps, double* ms_per_pass) {
  G4_REQUIRE(e && ms_per_pass && M >= 1 && M <= 4 && reps >= 1 && !e->seq.empty() && e->cfg.graphs &&
                 e->P + 1 > e->cfg.att_par && e->P + 1 + M < e->cfg.ctx_max,
             "g4_engine_time_verify: needs a prefilled engine with graphs past att_par");
  e->i8_active = e->cfg.decode_int8 && e->cfg.prefill_int8;
  RCK(ensure_verify_graph(e, M));
  int hctl[8 + 4] = {e->P, 0, 0, 0, 0, 0, 0, 0, e->conf, e->conf, e->conf, e->conf};
  ECK(cudaMemcpyAsync(e->ctl, hctl, sizeof hctl, cudaMemcpyHostToDevice, e->st));
  ECK(cudaGraphLaunch(e->gverify[M], e->st));  // warm
  cudaEvent_t a, b;
  ECK(cudaEventCreate(&a));
  ECK(cudaEventCreate(&b));
  ECK(cudaEventRecord(a, e->st));
  for (int i = 0; i < reps; ++i) ECK(cudaGraphLaunch(e->gverify[M], e->st));
  ECK(cudaEventRecord(b, e->st));
  ECK(cudaEventSynchronize(b));
  float ms = 0;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  *ms_per_pass = ms / reps;
  return G4_OK;
}

// The decode state of src (KV rows of every layer up to its position, history, hidden, round state)
// copied into dst, an engine of the same model dimensions: dst continues src's stream.
extern "C" int g4_engine_copy_state(g4_engine* dst, const g4_engine* src) {
  G4_REQUIRE(dst && src && !src->seq.empty() && dst->d.H == src->d.H && dst->d.NL == src->d.NL && dst->d.HD == src->d.HD &&
                 src->P + 1 <= dst->cfg.ctx_max && !dst->async_pending,
             "g4_engine_copy_state: incompatible engines");
  ECK(cudaStreamSynchronize(src->st));
  const size_t n = (size_t)(src->P + 2) * dst->d.HD;  // positions 0..P+1 (the next row is rewritten anyway)
  for (int l = 0; l < dst->d.NL; ++l) {
    ECK(cudaMemcpyAsync(dst->Kc + (size_t)l * dst->cfg.ctx_max * dst->d.HD, src->Kc + (size_t)l * src->cfg.ctx_max * src->d.HD,
                        n * 2, cudaMemcpyDeviceToDevice, dst->st));
    ECK(cudaMemcpyAsync(dst->Vc + (size_t)l * dst->cfg.ctx_max * dst->d.HD, src->Vc + (size_t)l * src->cfg.ctx_max * src->d.HD,
                        n * 2, cudaMemcpyDeviceToDevice, dst->st));
  }
  ECK(cudaMemcpyAsync(dst->hprev, src->hprev, sizeof(float) * dst->d.H, cudaMemcpyDeviceToDevice, dst->st));
  dst->seq = src->seq;
  dst->P = src->P;
  dst->conf = src->conf;
  dst->stopped = src->stopped;
  dst->fake_n = src->fake_n;
  RCK(upload_round_state(dst));
  dst->stats = g4_engine_stats{};
  return G4_OK;
}

// Decode state for another implementation (or a later restore): K and V of positions [0, npos) of
// every layer, the committed history, the hidden of the last committed row and its position.
extern "C" int g4_engine_export_state(g4_engine* e, int npos, uint16_t* Kc, uint16_t* Vc, int32_t* seq, int seq_cap,
                                      int* seq_len, float* hprev, int* P) {
  G4_REQUIRE(e && npos >= 0 && npos <= e->cfg.ctx_max && seq_len && P && !e->seq.empty(), "g4_engine_export_state: bad arguments");
  const ModelDims& d = e->d;
  ECK(cudaStreamSynchronize(e->st));
  for (int l = 0; l < d.NL && npos > 0; ++l) {
    const size_t off = (size_t)l * e->cfg.ctx_max * d.HD, n = (size_t)npos * d.HD;
    if (Kc) ECK(cudaMemcpy(Kc + (size_t)l * n, e->Kc + off, n * 2, cudaMemcpyDeviceToHost));
    if (Vc) ECK(cudaMemcpy(Vc + (size_t)l * n, e->Vc + off, n * 2, cudaMemcpyDeviceToHost));
  }
  *seq_len = (int)e->seq.size();
  if (seq) std::memcpy(seq, e->seq.data(), sizeof(int) * std::min<size_t>(seq_cap, e->seq.size()));
  if (hprev) ECK(cudaMemcpy(hprev, e->hprev, sizeof(float) * d.H, cudaMemcpyDeviceToHost));
  *P = e->P;
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
