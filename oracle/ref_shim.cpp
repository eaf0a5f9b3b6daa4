// TEST INFRASTRUCTURE ONLY: a C-ABI shim over the reference engine's own kernels, compiled
// from the reference sources where they lie (oracle/Makefile passes -I <reference>/engine) into
// oracle/_ref/libg4ref.so.  Nothing of the reference is copied here: the engine translation unit
// is included with `main` renamed, the same trick the reference's own bench/attn_bench.cpp:2-4
// uses, and every function below only marshals arguments into the reference's structures.
// Used to pin the plain-C oracle (tests/golden) and as the timed CPU baseline in bench.py.
#define main engine_main
#include "gemma4_engine.cpp"
#undef main

#include <sched.h>

extern "C" {

// Start the reference's persistent pool on CPUs 0..T-1 (gemma4_engine.cpp:73-134).  The calling
// thread is restored to its previous affinity afterwards so the host process is not confined.
int ref_pool_start(int T) {
  static bool started = false;
  if (started) return POOL.T;
  cpu_set_t old; sched_getaffinity(0, sizeof(old), &old);
  std::vector<int> cpus; for (int i = 0; i < T; ++i) cpus.push_back(i);
  POOL.start(cpus);
  sched_setaffinity(0, sizeof(old), &old);
  atexit([] { POOL.shutdown(); });
  started = true;
  return POOL.T;
}

// W4G32 float path through the engine's own dispatch: XP::prep (:180-194) + lin_multi (:310-317)
// -> lin_task (:243-255) -> w4::gemm_rows_tile<MT> (w4g32_avx2.h:65-96).
void ref_w4g32_gemm(const uint8_t* W, const uint16_t* S, const float* X, int M, int N, int K, float* Y) {
  static XP xp;
  Q4 q; q.w = W; q.s = S; q.N = N; q.K = K; q.p8 = nullptr;
  G_I8_ACTIVE = false;
  xp.prep(X, K, M);
  lin1(xp, q, Y);
}

// w4a8::quant (w4a8_avx2.h:30-42).
void ref_w4a8_quant(const float* X, int M, int K, int8_t* q, float* sx, int32_t* sum) {
  w4a8::XQ xq; w4a8::quant(X, M, K, xq);
  std::memcpy(q, xq.q.data(), (size_t)M * K);
  std::memcpy(sx, xq.sx.data(), sizeof(float) * (size_t)M * (K / 32));
  std::memcpy(sum, xq.sum.data(), sizeof(int32_t) * (size_t)M * (K / 32));
}

// W4A8 path: repack_tiles (w4a8_avx2.h:20-27) then, for M>=2, the engine's lin_multi int8 branch
// (:311-312 -> i8_task :304-309 -> w4a8::tile<MT>); for M=1 tile<1> directly over all tiles.
void ref_w4a8_gemm(const uint8_t* W, const uint16_t* S, const float* X, int M, int N, int K, float* Y) {
  static XP xp; static w4a8::Packed pk;
  w4a8::repack_alloc(N, K, pk); w4a8::repack_tiles(W, S, N, K, pk, 0, N / 8);
  Q4 q; q.w = W; q.s = S; q.N = N; q.K = K; q.p8 = &pk;
  if (M >= 2) {
    G_I8_ACTIVE = true;
    xp.prep(X, K, M);
    lin1(xp, q, Y);
    G_I8_ACTIVE = false;
  } else {
    w4a8::XQ xq; w4a8::quant(X, M, K, xq);
    for (int t = 0; t < N / 8; ++t) w4a8::tile<1>(pk, t, xq, 0, Y);
  }
}

// bf16p::pack (bf16_exp3_head.h:26-49).  Returns the exception count; the outputs are copied
// only when it fits the caller's capacity.
int64_t ref_bf16p_pack(const uint16_t* E, int N, int K, const uint8_t* cb8, uint8_t* data,
                       int64_t* exc_ptr, uint16_t* exc_col, float* exc_delta, int64_t cap) {
  bf16p::Packed P; bf16p::pack(E, N, K, cb8, P);
  const int64_t ne = (int64_t)P.exc_col.size();
  std::memcpy(data, P.data.data(), P.data.size());
  std::memcpy(exc_ptr, P.exc_ptr.data(), sizeof(int64_t) * (N + 1));
  if (ne <= cap) {
    std::memcpy(exc_col, P.exc_col.data(), sizeof(uint16_t) * ne);
    std::memcpy(exc_delta, P.exc_delta.data(), sizeof(float) * ne);
  }
  return ne;
}

// Exact head logits through the engine's head_task (:574-579 -> bf16p::rows_tile<MT>).
void ref_bf16p_gemm(const uint16_t* E, int N, int K, const uint8_t* cb8, const float* X, int M, float* Y) {
  static bf16p::Packed P; bf16p::pack(E, N, K, cb8, P);
  HeadArg ha; ha.P = &P; ha.h = X; ha.logit = Y; ha.M = M;
  POOL.run(head_task, &ha);
}

// Split-KV attention: attn_task (:743-877) over the pool's T threads, then attn_merge (:1019-1059).
void ref_attn_splitkv(const uint16_t* Kc, const uint16_t* Vc, int hd, int nh, int M, const float* q,
                      const int* pos, const int* lo, int kmin, int kmax, float* out) {
  AttnArg aa; aa.Kc = Kc; aa.Vc = Vc; aa.hd = hd; aa.nh = nh; aa.M = M; aa.kmin = kmin; aa.kmax = kmax;
  float* outp[4];
  for (int m = 0; m < M; ++m) {
    aa.q[m] = q + (size_t)m * nh * hd; aa.pos[m] = pos[m]; aa.lo[m] = lo[m];
    aa.skip_lo[m] = 1; aa.skip_hi[m] = 0; outp[m] = out + (size_t)m * nh * hd;
  }
  G_I8_ACTIVE = false;
  POOL.run(attn_task, &aa);
  attn_merge(aa, POOL.active_count(), outp, nullptr);
}

// The tiled prefill attention of a block of M rows at positions pos0.. (fwd's TILED branch,
// :1328-1336): attn_tile (:1061-1083) over tiles of QB rows x 8 heads on the pool's threads.  q rows
// (already normed and rotated) qstride apart, att rows 8*hd apart, bf16-rounded.
struct TileArg {
  const uint16_t *Kc, *Vc;
  int hd, sliding, qstride, pos0, M, ntiles;
  const float* q;
  float* att;
};
static void tile_task(void* p, int tid, int T) {
  const TileArg* a = static_cast<const TileArg*>(p);
  for (int t = tid; t < a->ntiles; t += T) attn_tile(a->Kc, a->Vc, a->hd, a->sliding != 0, a->q, a->qstride, a->pos0, a->M, a->att, t, tid);
}
void ref_attn_tile_run(const uint16_t* Kc, const uint16_t* Vc, int hd, int sliding, const float* q, int qstride, int pos0,
                       int M, float* att) {
  TileArg a{Kc, Vc, hd, sliding, qstride, pos0, M, (M + QB - 1) / QB, q, att};
  POOL.run(tile_task, &a);
}

// The reference screen_task (:460-538) at its hard-coded K=1536, N=262144, then eval_row's
// threshold filter (:1453-1467).  Writes the per-row L, the filtered survivors in list order and
// their count (or -1 when a per-thread list overflowed).
void ref_screen_1536(const uint8_t* W4, const uint16_t* S4, const float* coef, const float* H, int M,
                     const float* pre_thr, float* L_out, int* cnt_out, int* surv_out, int lim) {
  static ScrArg SA; static XP XH; static float hn[4];
  SCR.w.assign(W4, W4 + (size_t)262144 * 768);
  SCR.s.assign(S4, S4 + (size_t)262144 * 48);
  SCR.coef.assign(coef, coef + 262144);
  SCR.on = true;
  XH.prep(H, 1536, M);
  for (int m = 0; m < M; ++m) hn[m] = (float)sqrt(ss_avx2(H + (size_t)m * 1536, 1536));
  for (int m = 0; m < M; ++m) {
    SA.pre_thr[m] = pre_thr[m];
    SA.shared_best[m].store(pre_thr[m], std::memory_order_relaxed);
    SA.overflow[m].store(false, std::memory_order_relaxed);
  }
  SA.S = &SCR; SA.x = &XH; SA.hn = hn; SA.M = M; SA.nxt.store(0, std::memory_order_relaxed);
  POOL.run(screen_task, &SA);
  const int actT = POOL.active_count();
  auto cap = [](float s) { return r16(30.0f * tanhf(s / 30.0f)); };
  for (int m = 0; m < M; ++m) {
    float L = -1e30f; for (int t = 0; t < actT; ++t) L = std::max(L, SA.tmax[t][m]);
    L_out[m] = L;
    if (SA.overflow[m].load()) { cnt_out[m] = -1; continue; }
    float Lr = r16(L), cmL = cap(Lr), lo = Lr - 64.0f, hi = Lr;
    for (int it = 0; it < 40; ++it) { float mid = 0.5f * (lo + hi); if (cap(r16(mid)) == cmL) hi = mid; else lo = mid; }
    const float thr = hi - 0.25f;
    int tot = 0;
    for (int t = 0; t < actT; ++t)
      for (int k = 0; k < SA.t_cnt[t][m]; ++k)
        if (SA.t_u[t][m][k] >= thr) { if (tot < lim) surv_out[(size_t)m * lim + tot] = SA.t_idx[t][m][k]; ++tot; }
    cnt_out[m] = tot > lim ? -1 : tot;
  }
}

// One int4 matrix (reference layout) prepared for the engine's dispatch: its Q4 descriptor and the
// load-time W4A8 repack (w4a8::repack_tiles, as q4() does under ENGINE_DECODE_INT8, :175).
struct RefLin { Q4 q; w4a8::Packed pk; };
void* ref_lin_prepare(const uint8_t* W, const uint16_t* S, int N, int K) {
  RefLin* r = new RefLin;
  r->q.w = W; r->q.s = S; r->q.N = N; r->q.K = K;
  w4a8::repack_alloc(N, K, r->pk);
  w4a8::repack_tiles(W, S, N, K, r->pk, 0, N / 8);
  r->q.p8 = &r->pk;
  return r;
}
// Y = X W^T through the engine's lin1 (:310-317): W4A8 (i8_task) when i8 and M >= 2, else the float
// W4G32 path (lin_task); with i8 at M = 1 (the synthetic drafter's int8 linears) i8_task over the
// pool with one activation row.
void ref_lin_run(void* h, const float* X, int M, float* Y, int i8) {
  static XP xp;
  RefLin* r = static_cast<RefLin*>(h);
  xp.prep(X, r->q.K, M);
  if (i8 && M == 1) {
    w4a8::quant(X, 1, r->q.K, xp.xq);
    xp.qdone = true;
    I8Arg a; a.x = &xp; a.nj = 1; a.cum[0] = 0; a.q[0] = &r->q; a.y[0] = Y; a.cum[1] = r->q.N / 8;
    POOL.run(i8_task, &a);
    return;
  }
  G_I8_ACTIVE = i8 != 0;
  lin1(xp, r->q, Y);
  G_I8_ACTIVE = false;
}
// The packed exact head (bf16p::pack) and its logits for M <= 4 rows through head_task (:574-579).
void* ref_head_prepare(const uint16_t* E, int N, int K, const uint8_t* cb8) {
  bf16p::Packed* P = new bf16p::Packed;
  bf16p::pack(E, N, K, cb8, *P);
  return P;
}
void ref_head_run(void* h, const float* X, int M, float* Y) {
  HeadArg ha; ha.P = static_cast<bf16p::Packed*>(h); ha.h = X; ha.logit = Y; ha.M = M;
  POOL.run(head_task, &ha);
}

// gelu8 / exp8 on n values (gemma4_engine.cpp:43-60), 8 at a time (n a multiple of 8).
void ref_gelu8(const float* x, int n, float* y) { for (int i = 0; i < n; i += 8) _mm256_storeu_ps(y + i, gelu8(_mm256_loadu_ps(x + i))); }
void ref_exp8(const float* x, int n, float* y) { for (int i = 0; i < n; i += 8) _mm256_storeu_ps(y + i, exp8(_mm256_loadu_ps(x + i))); }

}  // extern "C"
