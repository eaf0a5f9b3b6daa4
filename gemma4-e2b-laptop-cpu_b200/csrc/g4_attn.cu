// Split-KV decode attention for up to 4 query rows and 8 query heads sharing one KV head.
//
// The reference splits the key range [kmin, kmax] into T contiguous chunks, one per pool thread
// (attn_task, gemma4_engine.cpp:743-877), and merges the partial softmaxes exactly
// (attn_merge :1019-1059).  The fp32 results depend on that split, so the GPU keeps it: the
// chunk boundaries are kmin + t*len/T, and within a chunk every sum runs in key order.  The work
// is spread over the GPU differently:
//   k_attn_scores  all (key, row, head) scores at once; each score is one half-warp, lane c
//                  running the reference's AVX partial sum c (elements c, c+16, ...), then the
//                  two 8-lane halves added and the 8-lane tree of hsum (:786-797);
//   k_attn_stats   per (chunk, row, head): the chunk max, the exp8 weights and their sum in key
//                  order;
//   k_attn_accum   per (chunk, row, head, dim): O = fma(w, v, O) over the chunk's keys in order;
//   k_attn_merge   per (row, head, dim): the rescale and normalisation of attn_merge, output
//                  rounded to bf16.
// There is no softmax scale: the reference folds it into q (q_norm), as does the caller here.
#include "g4_api.h"
#include "g4_async.cuh"
#include "g4_common.cuh"
#include <cstdlib>

namespace g4 {

struct AttnDesc {
  int M, nh, hd, kmin, kmax, T;
  int pos[4], lo[4];
  // Positions read on the device (a captured decode step whose position changes between replays):
  // when dynP is set, row m's last key is *dynP + base_add + m and its first key is
  // max(0, *dynP + q_add + m - (window - 1)) (0 for window == 0); kmin/kmax follow from them.
  const int* dynP;
  int base_add, q_add, window;
  QuantOut qo;  // when qo.q is set, the merge also quantises each row of out for a W4A8 linear
};

__device__ __forceinline__ AttnDesc resolve(const AttnDesc& d0) {
  AttnDesc d = d0;
  if (d.dynP != nullptr) {
    const int P = *d.dynP;
    d.kmin = 1 << 30;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      if (m < d.M) {
        d.pos[m] = P + d.base_add + m;
        d.lo[m] = d.window ? max(0, P + d.q_add + m - (d.window - 1)) : 0;
        d.kmin = min(d.kmin, d.lo[m]);
      } else {
        d.pos[m] = -1;
        d.lo[m] = 0;
      }
    }
    d.kmax = P + d.base_add + d.M - 1;
  }
  return d;
}

// Row m's first and last key, selected without indexing the descriptor's arrays (a runtime index
// would move the descriptor to local memory).
__device__ __forceinline__ int sel4(const int (&a)[4], int m) {
  int r = a[0];
  r = m == 1 ? a[1] : r;
  r = m == 2 ? a[2] : r;
  r = m == 3 ? a[3] : r;
  return r;
}
__device__ __forceinline__ int dlo(const AttnDesc& d, int m) { return sel4(d.lo, m); }
__device__ __forceinline__ int dpos(const AttnDesc& d, int m) { return sel4(d.pos, m); }
__device__ __forceinline__ bool allowed(const AttnDesc& d, int m, int p) { return p >= dlo(d, m) && p <= dpos(d, m); }
__device__ __forceinline__ int chunk_lo(const AttnDesc& d, int t) {
  const int len = d.kmax - d.kmin + 1;
  return d.kmin + (int)((long long)t * len / d.T);
}

// Workspace layout (floats): S [M*nh][len] scores then weights (one contiguous run of keys per
// (row, head)), AM [T][M*nh], AL [T][M*nh], AO [T][M*nh][hd].
struct AttnWs {
  float *S, *AM, *AL, *AO;
};
__host__ __device__ inline size_t attn_ws_floats(int M, int nh, int hd, int len, int T) {
  return (size_t)len * M * nh + 2 * (size_t)T * M * nh + (size_t)T * M * nh * hd;
}
__device__ __forceinline__ AttnWs attn_ws(float* base, const AttnDesc& d) {
  const int len = d.kmax - d.kmin + 1;
  AttnWs w;
  w.S = base;
  w.AM = w.S + (size_t)len * d.M * d.nh;
  w.AL = w.AM + (size_t)d.T * d.M * d.nh;
  w.AO = w.AL + (size_t)d.T * d.M * d.nh;
  return w;
}

// ---- scores.  A block takes kScoreKeys consecutive keys, copies their K rows into shared memory
// (one bulk copy) and transposes them so that the elements c, c+16, ... of partial c sit together
// (lane slots of kLaneStr bytes, an odd multiple of 16, so a half-warp's 16-byte loads are
// conflict-free); each (row, head) pair gets one half-warp: lane c runs the reference's AVX
// partial sum c (elements c, c+16, ... in order; q for the pair stays in registers), then the two
// 8-lane halves are added and reduced with the 8-lane tree of hsum (:786-797).
constexpr int kScoreKeys = 32;
template <int STEPS>
struct ScoreTile {
  static constexpr int kLaneStr = ((STEPS * 2 / 16) | 1) * 16;  // bytes per lane slot
  static constexpr int kKeyStr = 16 * kLaneStr;                   // bytes per transposed key
};
__host__ __device__ inline size_t attn_scores_smem(int hd) {
  const int steps = hd / 16, lane_str = ((steps * 2 / 16) | 1) * 16;
  return 128 + (size_t)kScoreKeys * hd * 2 + (size_t)kScoreKeys * 16 * lane_str;
}
template <int STEPS>  // hd / 16
__global__ void __launch_bounds__(512) k_attn_scores(const uint16_t* __restrict__ Kc, const float* __restrict__ q,
                                                     AttnDesc d0, float* __restrict__ ws) {
  constexpr int HD = STEPS * 16, LS = ScoreTile<STEPS>::kLaneStr, KS = ScoreTile<STEPS>::kKeyStr;
  extern __shared__ __align__(128) uint8_t sm_raw[];
  const AttnDesc d = resolve(d0);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm_raw);
  const uint4* kraw = reinterpret_cast<const uint4*>(sm_raw + 128);
  uint8_t* ktt = sm_raw + 128 + (size_t)kScoreKeys * HD * 2;
  const AttnWs w = attn_ws(ws, d);
  const int len = d.kmax - d.kmin + 1;
  const int p0 = d.kmin + blockIdx.x * kScoreKeys;
  if (p0 > d.kmax) {  // grid sized for the longest key range (positions read on the device)
    pdl_wait();
    pdl_trigger();
    return;
  }
  const int nk = min(kScoreKeys, d.kmax + 1 - p0);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // keys before the first query row's position were written by earlier passes: requested before
  // the wait on the previous kernel (the KV write of the current rows), the current rows after it
  const int nold = min(nk, max(0, d.pos[0] - p0));
  if (threadIdx.x == 0) {
    mbar_expect_tx(bar, (uint32_t)nk * HD * 2);
    if (nold > 0) bulk_g2s(sm_raw + 128, Kc + (size_t)p0 * HD, (uint32_t)nold * HD * 2, bar);
  }
  pdl_wait();
  pdl_trigger();
  if (nk > nold && threadIdx.x == 0)
    bulk_g2s(sm_raw + 128 + (size_t)nold * HD * 2, Kc + (size_t)(p0 + nold) * HD, (uint32_t)(nk - nold) * HD * 2, bar);
  const int hw = threadIdx.x >> 4, c = threadIdx.x & 15;
  const bool live_mh = hw < d.M * d.nh;
  const int m = live_mh ? hw / d.nh : 0, h = live_mh ? hw % d.nh : 0;
  float qr[STEPS];
  const float* qh = q + ((size_t)m * d.nh + h) * HD;
#pragma unroll
  for (int i = 0; i < STEPS; ++i) qr[i] = qh[c + 16 * i];
  if (!cta_wait(bar, 0)) return;
  // transpose: element e = c + 16 i of a key goes to lane slot c, position i
  for (int e8 = threadIdx.x; e8 < nk * (HD / 8); e8 += blockDim.x) {
    const int key = e8 / (HD / 8), e0 = (e8 % (HD / 8)) * 8;
    const uint4 v = kraw[e8];
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    uint16_t* kd = reinterpret_cast<uint16_t*>(ktt + (size_t)key * KS);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + j;
      kd[((e & 15) * LS >> 1) + (e >> 4)] = (uint16_t)(wv[j >> 1] >> (16 * (j & 1)));
    }
  }
  __syncthreads();
  float* srow = w.S + (size_t)hw * len + (p0 - d.kmin);
  auto score = [&](int k) {  // lane c's partial for key k
    const uint4* kp = reinterpret_cast<const uint4*>(ktt + (size_t)k * KS + c * LS);
    float acc = 0.f;
#pragma unroll
    for (int v4 = 0; v4 < STEPS / 8; ++v4) {
      const uint4 t4 = kp[v4];
      const uint32_t wv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t u = wv[j >> 1];
        acc = fmaf(qr[8 * v4 + j], __uint_as_float((j & 1) ? (u & 0xFFFF0000u) : (u << 16)), acc);
      }
    }
    return acc;
  };
  int k = 0;
  for (; k + 4 <= nk; k += 4) {  // four keys at a time: independent chains for latency hiding
    float acc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[u] = score(k + u);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float sc = hsum8_octet(__fadd_rn(acc[u], __shfl_xor_sync(FULL, acc[u], 8)));
      if (c == 0 && live_mh && allowed(d, m, p0 + k + u)) srow[k + u] = sc;
    }
  }
  for (; k < nk; ++k) {
    const float acc = score(k);
    const float sc = hsum8_octet(__fadd_rn(acc, __shfl_xor_sync(FULL, acc, 8)));
    if (c == 0 && live_mh && allowed(d, m, p0 + k)) srow[k] = sc;
  }
}

// ---- chunk statistics: block = (chunk t, 8 (row, head) pairs), one warp per pair.  The warp holds the
// chunk's allowed scores in registers (key c0 + 32*j + lane in slot j); max is order-free; the
// weights exp8(s - max) are elementwise and overwrite the scores; their sum runs in key order
// (each slot's 32 keys are handed over by shuffles).  Longer chunks run in segments of
// 32*kStatSlots keys.
constexpr int kStatSlots = 32;
__global__ void __launch_bounds__(256) k_attn_stats(AttnDesc d0, float* __restrict__ ws) {
  pdl_wait();
  pdl_trigger();
  const AttnDesc d = resolve(d0);
  const AttnWs w = attn_ws(ws, d);
  const int mh = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31, t = blockIdx.x;
  if (mh >= d.M * d.nh) return;
  const int m = mh / d.nh, len = d.kmax - d.kmin + 1;
  const int c0 = max(chunk_lo(d, t), dlo(d, m)), c1 = min(chunk_lo(d, t + 1), dpos(d, m) + 1);  // allowed keys of the chunk
  float* srow = w.S + (size_t)mh * len - d.kmin;
  constexpr int SEG = 32 * kStatSlots;
  const bool one = c1 - c0 <= SEG;  // the whole chunk fits the registers: load it once
  float v[kStatSlots];
  float mx = -1e30f;
  for (int sb = c0; sb < c1; sb += SEG) {
#pragma unroll
    for (int j = 0; j < kStatSlots; ++j) {
      const int p = sb + 32 * j + lane;
      v[j] = p < c1 ? srow[p] : -1e30f;
      mx = fmaxf(mx, v[j]);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  float l8 = 0.f;
  for (int sb = c0; sb < c1; sb += SEG) {
    if (!one) {
#pragma unroll
      for (int j = 0; j < kStatSlots; ++j) {
        const int p = sb + 32 * j + lane;
        v[j] = p < c1 ? srow[p] : -1e30f;
      }
    }
#pragma unroll
    for (int j = 0; j < kStatSlots; ++j) {
      const int pb = sb + 32 * j;
      if (pb >= c1) break;  // warp-uniform
      const int p = pb + lane;
      float wt = 0.f;
      if (p < c1) {
        wt = exp8(__fsub_rn(v[j], mx));
        srow[p] = wt;
      }
      const int nb = min(32, c1 - pb);
      if (nb == 32) {
        float x[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) x[k] = __shfl_sync(FULL, wt, k);
#pragma unroll
        for (int k = 0; k < 32; ++k) l8 = __fadd_rn(l8, x[k]);  // every lane adds in key order
      } else {
        for (int k = 0; k < nb; ++k) l8 = __fadd_rn(l8, __shfl_sync(FULL, wt, k));
      }
    }
  }
  if (lane == 0) {
    const size_t ix = (size_t)t * d.M * d.nh + mh;
    w.AM[ix] = mx;
    w.AL[ix] = (dlo(d, m) > dpos(d, m)) ? 0.0f : l8;
  }
}

// cp.async (Ampere-style asynchronous copy) of 4 / 16 bytes global -> shared, grouped.
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// ---- O accumulation: block = (chunk t, 16-dim slice, group of 8 (row, head) pairs).  Thread =
// (pair g of the group, dim pair dp): one packed f32x2 fma chain over the chunk's allowed keys in
// order.  V slices and weights of kAccKeys keys at a time are staged in shared memory with
// asynchronous copies, double-buffered so that the next tile loads while this one is consumed.
constexpr int kAccKeys = 128;
__global__ void __launch_bounds__(64) k_attn_accum(const uint16_t* __restrict__ Vc, AttnDesc d0, float* __restrict__ ws) {
  pdl_wait();
  pdl_trigger();
  const AttnDesc d = resolve(d0);
  __shared__ __align__(16) uint32_t vs[2][kAccKeys][8];    // 16 bf16 dims per key
  __shared__ __align__(16) float wsm[2][8][kAccKeys + 1];  // weights [pair][key], padded against bank conflicts
  const AttnWs w = attn_ws(ws, d);
  const int t = blockIdx.x, i0 = blockIdx.y * 16, mhb = blockIdx.z * 8;
  const int nmh = d.M * d.nh, len = d.kmax - d.kmin + 1;
  const int g = threadIdx.x >> 3, dp = threadIdx.x & 7;
  const int ng = min(8, nmh - mhb);  // live pairs in this group
  const bool live = g < ng;
  const int mh = mhb + (live ? g : 0), m = mh / d.nh;
  const int c0 = chunk_lo(d, t), c1 = chunk_lo(d, t + 1);
  const int a = max(c0, dlo(d, m)), b = min(c1 - 1, dpos(d, m));
  auto stage = [&](int buf, int pb) {
    const int nk = min(kAccKeys, c1 - pb);
    for (int e = threadIdx.x; e < nk * 2; e += 64)  // V: 2 x 16 B per key
      cp_async16(&vs[buf][e >> 1][(e & 1) * 4], Vc + (size_t)(pb + (e >> 1)) * d.hd + i0 + (e & 1) * 8);
    for (int r = 0; r < ng; ++r) {
      const float* src = w.S + (size_t)(mhb + r) * len + (pb - d.kmin);
      for (int k = threadIdx.x; k < nk; k += 64) cp_async4(&wsm[buf][r][k], src + k);
    }
  };
  float2 o = make_float2(0.f, 0.f);
  stage(0, c0);
  cp_async_commit();
  for (int pb = c0, it = 0; pb < c1; pb += kAccKeys, ++it) {
    if (pb + kAccKeys < c1) stage((it + 1) & 1, pb + kAccKeys);
    cp_async_commit();  // possibly empty group: keeps the wait count uniform
    cp_async_wait_1();
    __syncthreads();
    const int buf = it & 1;
    if (live) {
      const int nk = min(kAccKeys, c1 - pb);
      const int ka = max(a, pb) - pb, kb = min(b, pb + nk - 1) - pb;
#pragma unroll 4
      for (int k = ka; k <= kb; ++k) {
        const uint32_t vv = vs[buf][k][dp];
        const float wt = wsm[buf][g][k];
        o = __ffma2_rn(make_float2(wt, wt), make_float2(__uint_as_float(vv << 16), __uint_as_float(vv & 0xFFFF0000u)), o);
      }
    }
    __syncthreads();
  }
  if (live) {
    float* ao = w.AO + ((size_t)t * nmh + mh) * d.hd + i0 + 2 * dp;
    ao[0] = o.x;
    ao[1] = o.y;
  }
}

// ---- merge: block per (row, head), thread per dim.  M0 = max of the chunk maxima with L > 0;
// sc_t = expf(M_t - M0) (correctly rounded here); l = sum L_t*sc_t in double in chunk order (each
// product exact); out = r16((sum_t fma(O_t, sc_t)) * (float)(1/l)).  The per-chunk factors are
// computed once per block.
__global__ void __launch_bounds__(512) k_attn_merge(AttnDesc d0, const float* __restrict__ ws, float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sc[64], al[64];
  __shared__ float inv_l, s_m0;
  const AttnDesc d = resolve(d0);
  const AttnWs w = attn_ws(const_cast<float*>(ws), d);
  const int mh = blockIdx.x, i = threadIdx.x, nmh = d.M * d.nh;
  // chunk factors: maxima and sums loaded in parallel, M0 and l (in chunk order) by thread 0
  if (i < d.T) {
    const size_t ix = (size_t)i * nmh + mh;
    al[i] = w.AL[ix];
    sc[i] = al[i] > 0 ? w.AM[ix] : -1e30f;
  }
  __syncthreads();
  if (i == 0) {
    float M0 = -1e30f;
    for (int t = 0; t < d.T; ++t) M0 = fmaxf(M0, sc[t]);
    s_m0 = M0;
  }
  __syncthreads();
  if (i < d.T) sc[i] = al[i] > 0 ? exp_cr(__fsub_rn(sc[i], s_m0)) : 0.f;
  __syncthreads();
  if (i == 0) {
    double l = 0;
    for (int t = 0; t < d.T; ++t)
      if (al[t] > 0) l = fma((double)al[t], (double)sc[t], l);
    inv_l = (float)(1.0 / l);
  }
  __syncthreads();
  if (i >= d.hd) return;
  float acc = 0.f;
  if (d.T <= 16) {  // every chunk's O loaded at once, then the chain in chunk order
    float aov[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) aov[t] = t < d.T ? w.AO[((size_t)t * nmh + mh) * d.hd + i] : 0.f;
#pragma unroll
    for (int t = 0; t < 16; ++t)
      if (t < d.T && al[t] > 0) acc = fmaf(aov[t], sc[t], acc);
  } else {
    for (int t = 0; t < d.T; ++t) {
      if (!(al[t] > 0)) continue;
      acc = fmaf(w.AO[((size_t)t * nmh + mh) * d.hd + i], sc[t], acc);
    }
  }
  const float v = r16(__fmul_rn(acc, inv_l));
  out[(size_t)mh * d.hd + i] = v;
  if (d.qo.q) {  // blockDim == hd, a multiple of 32: warp w holds group w of this head's dims
    int8_t qv;
    float sx;
    int32_t tot;
    quant_group32(v, qv, sx, tot);
    const size_t flat = (size_t)mh * d.hd + i;
    d.qo.q[flat] = qv;
    if ((threadIdx.x & 31) == 0) {
      d.qo.sx[flat >> 5] = sx;
      d.qo.sum[flat >> 5] = tot;
    }
  }
}

// ---- chunk kernel for long chunks (global layers): statistics, accumulation and merge in one
// launch after k_attn_scores.  Block = (chunk t, 32-dim slice, group of 8 (row, head) pairs),
// 256 threads.  The chunk's V slice (64 bytes of each key) is requested by cp.async before the
// wait on the previous kernel (the cache rows were written two launches earlier, by the KV write,
// which had completed before the scores kernel started).  Warp p loads pair p's allowed scores of
// the chunk into shared memory, takes their max and turns them into exp8 weights in place (as
// k_attn_stats).  Then, concurrently, warps 0-3 run the weight sums of pairs w and w+4 in key
// order (32 weights at a time handed to every lane by shuffles), and warps 4-7 (thread = pair x
// dim pair) run the O chains over the chunk's keys in order, with the weights and V of the next 8
// keys loaded while the current 8 are accumulated (as k_attn_accum).  The last of the T blocks of
// a (slice, group) merges the chunks for its 32 dims (as k_attn_merge) and quantises them when
// asked.  Same values as the four-kernel path.
constexpr int kChunkMaxKeys = 1536;
constexpr int kChunkWs = kChunkMaxKeys + 4;  // a multiple of 4 whose rows start in distinct banks
__host__ __device__ inline size_t attn_chunk_smem() {
  return sizeof(float) * 8 * kChunkWs + (size_t)kChunkMaxKeys * 64;
}
__device__ __forceinline__ void cp_async16_g(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__global__ void __launch_bounds__(256) k_attn_chunk(const uint16_t* __restrict__ Vc, AttnDesc d0, float* __restrict__ ws,
                                                    int* __restrict__ counters, float* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t csm[];
  float* wsm = reinterpret_cast<float*>(csm);                                  // [8][kChunkWs]
  uint32_t* vsl = reinterpret_cast<uint32_t*>(csm + sizeof(float) * 8 * kChunkWs);  // [key - cl][16]
  __shared__ float smx[8], sl8[8];
  __shared__ int s_last;
  const AttnDesc d = resolve(d0);  // positions come from the host-written control word
  const int t = blockIdx.x, y = blockIdx.y, grp = blockIdx.z, i0 = y * 32;
  const int nmh = d.M * d.nh, len = d.kmax - d.kmin + 1, G8 = (nmh + 7) / 8;
  const int mhb = grp * 8, ng = min(8, nmh - mhb);
  const int cl = chunk_lo(d, t), ch = chunk_lo(d, t + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < (ch - cl) * 4; e += 256)  // 4 x 16 B per key (32 bf16 dims)
    cp_async16_g(vsl + (size_t)e * 4, Vc + (size_t)(cl + (e >> 2)) * d.hd + i0 + (e & 3) * 8);
  asm volatile("cp.async.commit_group;" ::: "memory");
  pdl_wait();  // the scores come from the previous kernel
  pdl_trigger();
  const AttnWs w = attn_ws(ws, d);
  constexpr int WS = kChunkWs;  // weights of pair p at wsm[p * WS + (k - cl)]
  // scores of pair `warp` -> shared memory, max, weights
  if (warp < ng) {
    const int mh = mhb + warp, m = mh / d.nh;
    const int a = max(cl, dlo(d, m)), b = min(ch - 1, dpos(d, m));
    const float* srow = w.S + (size_t)mh * len - d.kmin;
    float* wp = wsm + warp * WS - cl;
    float mx = -1e30f;
    constexpr int kPer = kChunkMaxKeys / 32;
    float v[kPer];  // every score load in flight at once
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int k = a + lane + 32 * j;
      v[j] = k <= b ? __ldcg(srow + k) : -1e30f;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) mx = fmaxf(mx, v[j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    const int jn = b >= a ? (b - a + 32) / 32 : 0;  // slots holding keys (warp-uniform)
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (j >= jn) break;
      const int k = a + lane + 32 * j;
      if (k <= b) wp[k] = exp8(__fsub_rn(v[j], mx));
    }
    if (lane == 0) smx[warp] = mx;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    // in-order weight sums, one lane per pair, four weights per 16-byte load
    if (lane < ng) {
      const int mh = mhb + lane, m = mh / d.nh;
      const float* wr = wsm + lane * WS;
      int k = max(cl, dlo(d, m)) - cl;
      const int ke = min(ch - 1, dpos(d, m)) - cl;  // inclusive
      float l8 = 0.f;
      for (; k <= ke && (k & 3); ++k) l8 = __fadd_rn(l8, wr[k]);
      if (k + 3 <= ke) {
        float4 cur = *reinterpret_cast<const float4*>(wr + k);
        for (; k + 7 <= ke; k += 4) {
          const float4 nxt = *reinterpret_cast<const float4*>(wr + k + 4);
          l8 = __fadd_rn(l8, cur.x);
          l8 = __fadd_rn(l8, cur.y);
          l8 = __fadd_rn(l8, cur.z);
          l8 = __fadd_rn(l8, cur.w);
          cur = nxt;
        }
        l8 = __fadd_rn(l8, cur.x);
        l8 = __fadd_rn(l8, cur.y);
        l8 = __fadd_rn(l8, cur.z);
        l8 = __fadd_rn(l8, cur.w);
        k += 4;
      }
      for (; k <= ke; ++k) l8 = __fadd_rn(l8, wr[k]);
      sl8[lane] = (dlo(d, m) > dpos(d, m)) ? 0.0f : l8;
    }
  } else if (warp >= 4) {
    // O chains: thread = (pair p, dim pair dp) over this block's 32 dims; 8 keys per step, their
    // weights in two 16-byte loads
    const int at = threadIdx.x - 128, p = at >> 4, dp = at & 15;
    const bool live = p < ng;
    const int mh = mhb + (live ? p : 0), m = mh / d.nh;
    int k = max(cl, dlo(d, m)) - cl;
    const int ke = live ? min(ch - 1, dpos(d, m)) - cl : k - 1;  // inclusive
    const float* wr = wsm + (live ? p : 0) * WS;
    const uint32_t* vr = vsl + dp;
    float2 o = make_float2(0.f, 0.f);
    auto step = [&](float wt, uint32_t vv) {
      o = __ffma2_rn(make_float2(wt, wt), make_float2(__uint_as_float(vv << 16), __uint_as_float(vv & 0xFFFF0000u)), o);
    };
    for (; k <= ke && (k & 3); ++k) step(wr[k], vr[(size_t)k * 16]);
#pragma unroll 2
    for (; k + 7 <= ke; k += 8) {
      const float4 w0 = *reinterpret_cast<const float4*>(wr + k), w1 = *reinterpret_cast<const float4*>(wr + k + 4);
      uint32_t vv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) vv[u] = vr[(size_t)(k + u) * 16];
      step(w0.x, vv[0]); step(w0.y, vv[1]); step(w0.z, vv[2]); step(w0.w, vv[3]);
      step(w1.x, vv[4]); step(w1.y, vv[5]); step(w1.z, vv[6]); step(w1.w, vv[7]);
    }
    for (; k <= ke; ++k) step(wr[k], vr[(size_t)k * 16]);
    if (live) {
      float* ao = w.AO + ((size_t)t * nmh + mh) * d.hd + i0 + 2 * dp;
      ao[0] = o.x;
      ao[1] = o.y;
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < ng) {  // every slice writes the same statistics
    w.AM[(size_t)t * nmh + mhb + threadIdx.x] = smx[threadIdx.x];
    w.AL[(size_t)t * nmh + mhb + threadIdx.x] = sl8[threadIdx.x];
  }
  __threadfence();
  __syncthreads();
  int* cnt = counters + (size_t)y * G8 + grp;
  if (threadIdx.x == 0) s_last = atomicAdd(cnt, 1) == d.T - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (warp < ng) {
    // merge (k_attn_merge) for pair `warp`, dim i0 + lane
    const int mh = mhb + warp;
    constexpr int kT = 16;  // every load first (T <= 16), then the factors, then l and O in chunk order
    float alv[kT], amv[kT], aov[kT];
#pragma unroll
    for (int tt = 0; tt < kT; ++tt) {
      const size_t jx = (size_t)tt * nmh + mh;
      const bool in = tt < d.T;
      alv[tt] = in ? __ldcg(&w.AL[jx]) : 0.f;
      amv[tt] = in ? __ldcg(&w.AM[jx]) : 0.f;
      aov[tt] = in ? __ldcg(&w.AO[jx * d.hd + i0 + lane]) : 0.f;
    }
    float M0 = -1e30f;
#pragma unroll
    for (int tt = 0; tt < kT; ++tt)
      if (alv[tt] > 0) M0 = fmaxf(M0, amv[tt]);
    double l = 0;
    float acc = 0.f;
#pragma unroll
    for (int tt = 0; tt < kT; ++tt) {
      if (!(alv[tt] > 0)) continue;
      const float sc = exp_cr(__fsub_rn(amv[tt], M0));
      l = fma((double)alv[tt], (double)sc, l);
      acc = fmaf(aov[tt], sc, acc);
    }
    const float inv = (float)(1.0 / l);
    const float v = r16(__fmul_rn(acc, inv));
    const size_t flat = (size_t)mh * d.hd + i0 + lane;
    out[flat] = v;
    if (d.qo.q) {
      int8_t qv;
      float sxv;
      int32_t tot;
      quant_group32(v, qv, sxv, tot);
      d.qo.q[flat] = qv;
      if (lane == 0) {
        d.qo.sx[flat >> 5] = sxv;
        d.qo.sum[flat >> 5] = tot;
      }
    }
  }
  if (threadIdx.x == 0) *cnt = 0;  // ready for the next launch
}

// ---- one-kernel split-KV for short chunks (sliding-window layers): block = (chunk t, (row, head)
// pair).  The chunk's K and V rows arrive in shared memory by two bulk copies (its rows are
// contiguous in the cache; one copy per row costs microseconds of issue time); the block
// then computes the chunk's scores (half-warp per key, as k_attn_scores), the chunk max, the exp8
// weights and their in-order sum (as k_attn_stats), and O for every dim over the chunk's keys in
// order (as k_attn_accum); the last of the T blocks of a pair to finish (a counter per pair, zeroed
// before the launch) merges the chunks (as k_attn_merge) and quantises the row when asked.  Same
// values as the four-kernel path.
constexpr int kAttnShortKeys = 96;  // longest chunk served by k_attn_short
__host__ __device__ inline size_t attn_short_smem(int hd) {
  return 128 + 2 * (size_t)kAttnShortKeys * hd * 2 + sizeof(float) * kAttnShortKeys;
}

template <int STEPS>
__global__ void __launch_bounds__(256) k_attn_short(const uint16_t* __restrict__ Kc, const uint16_t* __restrict__ Vc,
                                                    const float* __restrict__ q, AttnDesc d0, float* __restrict__ ws,
                                                    int* __restrict__ counters, float* __restrict__ out) {
  extern __shared__ __align__(128) uint8_t sm_raw[];
  __shared__ float red_f[8];
  __shared__ float msc[64], red_f_am[32];
  __shared__ float s_l8, s_inv;
  __shared__ int s_last;
  const AttnDesc d = resolve(d0);
  const AttnWs w = attn_ws(ws, d);
  const int t = blockIdx.x, mh = blockIdx.y, nmh = d.M * d.nh;
  const int m = mh / d.nh, h = mh % d.nh;
  const int c0 = max(chunk_lo(d, t), dlo(d, m)), c1 = min(chunk_lo(d, t + 1), dpos(d, m) + 1);
  const int n = max(0, c1 - c0);
  const int rs = d.hd * 2;  // shared-memory row stride (bytes)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm_raw);
  uint8_t* ks = sm_raw + 128;
  uint8_t* vs = ks + (size_t)kAttnShortKeys * rs;
  float* sc = reinterpret_cast<float*>(vs + (size_t)kAttnShortKeys * rs);
  const int hw = threadIdx.x >> 4, c = threadIdx.x & 15, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // The chunk's rows are contiguous: one copy for K, one for V.  Keys before the first query row's
  // position were written by earlier passes, so their rows are requested before the wait on the
  // previous kernel (the KV write of the current rows); the current rows follow after it.
  const int nold = min(n, max(0, d.pos[0] - c0));
  const uint32_t rb = (uint32_t)d.hd * 2;
  if (n > 0 && threadIdx.x == 0) {
    mbar_expect_tx(bar, 2u * rb * (uint32_t)n);
    if (nold > 0) {
      bulk_g2s(ks, Kc + (size_t)c0 * d.hd, rb * (uint32_t)nold, bar);
      bulk_g2s(vs, Vc + (size_t)c0 * d.hd, rb * (uint32_t)nold, bar);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (n > nold && threadIdx.x == 0) {
    bulk_g2s(ks + (size_t)nold * rs, Kc + (size_t)(c0 + nold) * d.hd, rb * (uint32_t)(n - nold), bar);
    bulk_g2s(vs + (size_t)nold * rs, Vc + (size_t)(c0 + nold) * d.hd, rb * (uint32_t)(n - nold), bar);
  }
  float qr[STEPS];
  {
    const float* qh = q + ((size_t)m * d.nh + h) * d.hd;
#pragma unroll
    for (int i = 0; i < STEPS; ++i) qr[i] = qh[c + 16 * i];
  }
  if (n > 0 && !cta_wait(bar, 0)) return;
  // scores, two keys per half-warp iteration (independent chains)
  const int nk32 = (n + 31) / 32 * 32;  // both half-warps of a warp run the same iterations
  for (int k = hw; k < nk32; k += 32) {
    const uint16_t* kr0 = reinterpret_cast<const uint16_t*>(ks + (size_t)min(k, n - 1) * rs);
    const uint16_t* kr1 = reinterpret_cast<const uint16_t*>(ks + (size_t)min(k + 16, n - 1) * rs);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < STEPS; ++i) {
      a0 = fmaf(qr[i], bf2f(kr0[c + 16 * i]), a0);
      a1 = fmaf(qr[i], bf2f(kr1[c + 16 * i]), a1);
    }
    const float s0 = hsum8_octet(__fadd_rn(a0, __shfl_xor_sync(FULL, a0, 8)));
    const float s1 = hsum8_octet(__fadd_rn(a1, __shfl_xor_sync(FULL, a1, 8)));
    if (c == 0 && k < n) sc[k] = s0;
    if (c == 0 && k + 16 < n) sc[k + 16] = s1;
  }
  __syncthreads();
  // chunk max (order-free), then the weights
  float mx = -1e30f;
  for (int k = threadIdx.x; k < n; k += blockDim.x) mx = fmaxf(mx, sc[k]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if (lane == 0) red_f[wid] = mx;
  __syncthreads();
  mx = red_f[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, red_f[i]);
  for (int k = threadIdx.x; k < n; k += blockDim.x) sc[k] = exp8(__fsub_rn(sc[k], mx));
  __syncthreads();
  // in-order sum of the weights (warp 0)
  if (wid == 0) {
    float l8 = 0.f;
    for (int kb = 0; kb < n; kb += 32) {
      const float wt = kb + lane < n ? sc[kb + lane] : 0.f;
      const int nb = min(32, n - kb);
      if (nb == 32) {
        float x[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) x[k] = __shfl_sync(FULL, wt, k);
#pragma unroll
        for (int k = 0; k < 32; ++k) l8 = __fadd_rn(l8, x[k]);
      } else {
        for (int k = 0; k < nb; ++k) l8 = __fadd_rn(l8, __shfl_sync(FULL, wt, k));
      }
    }
    if (lane == 0) s_l8 = l8;
  }
  // O over the chunk's keys in order, thread per dim
  const size_t ix = (size_t)t * nmh + mh;
  for (int i = threadIdx.x; i < d.hd; i += blockDim.x) {
    float o = 0.f;
    const uint8_t* vp = vs + (size_t)i * 2;
#pragma unroll 8
    for (int k = 0; k < n; ++k) o = fmaf(sc[k], bf2f(*reinterpret_cast<const uint16_t*>(vp + (size_t)k * rs)), o);
    w.AO[ix * d.hd + i] = o;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    w.AM[ix] = mx;
    w.AL[ix] = (dlo(d, m) > dpos(d, m)) ? 0.0f : s_l8;
  }
  __threadfence();  // every thread's partial results are visible device-wide before the count
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&counters[mh], 1) == d.T - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // merge (k_attn_merge) by the last block of the pair: every load first (the chunks' O values
  // of this thread's dim, the chunk maxima and sums), then the factors in parallel, l in order
  float aov[8];
  if ((int)threadIdx.x < d.hd)
#pragma unroll
    for (int tt = 0; tt < 8; ++tt)
      if (tt < d.T) aov[tt] = __ldcg(&w.AO[((size_t)tt * nmh + mh) * d.hd + threadIdx.x]);
  if (threadIdx.x < d.T) {
    const size_t jx = (size_t)threadIdx.x * nmh + mh;
    msc[32 + threadIdx.x] = __ldcg(&w.AL[jx]);
    red_f_am[threadIdx.x] = __ldcg(&w.AM[jx]);
  }
  __syncthreads();
  if (threadIdx.x < d.T) {
    float M0 = -1e30f;
    for (int tt = 0; tt < d.T; ++tt)
      if (msc[32 + tt] > 0) M0 = fmaxf(M0, red_f_am[tt]);
    msc[threadIdx.x] = msc[32 + threadIdx.x] > 0 ? exp_cr(__fsub_rn(red_f_am[threadIdx.x], M0)) : 0.f;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double l = 0;
    for (int tt = 0; tt < d.T; ++tt)
      if (msc[32 + tt] > 0) l = fma((double)msc[32 + tt], (double)msc[tt], l);
    s_inv = (float)(1.0 / l);
    counters[mh] = 0;  // ready for the next launch
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d.hd; i += blockDim.x) {
    float acc = 0.f;
    if (i == (int)threadIdx.x && d.T <= 8) {
#pragma unroll
      for (int tt = 0; tt < 8; ++tt)
        if (tt < d.T && msc[32 + tt] > 0) acc = fmaf(aov[tt], msc[tt], acc);
    } else {
      for (int tt = 0; tt < d.T; ++tt)
        if (msc[32 + tt] > 0) acc = fmaf(__ldcg(&w.AO[((size_t)tt * nmh + mh) * d.hd + i]), msc[tt], acc);
    }
    const float v = r16(__fmul_rn(acc, s_inv));
    out[(size_t)mh * d.hd + i] = v;
    if (d.qo.q) {
      int8_t qv;
      float sxv;
      int32_t tot;
      quant_group32(v, qv, sxv, tot);
      const size_t flat = (size_t)mh * d.hd + i;
      d.qo.q[flat] = qv;
      if (lane == 0) {
        d.qo.sx[flat >> 5] = sxv;
        d.qo.sum[flat >> 5] = tot;
      }
    }
  }
}

}  // namespace g4

G4_STATUS_READER(attn)

using namespace g4;

static int fill_desc(AttnDesc& d, const uint16_t* Kc, const uint16_t* Vc, int M, int nh, int hd, const int* pos,
                     const int* lo, int kmin, int kmax, int T) {
  G4_REQUIRE(aligned(Kc, 16) && aligned(Vc, 16), "attention: K and V caches must be 16-byte aligned");
  G4_REQUIRE(M >= 1 && M <= 4 && nh >= 1 && nh <= 8 && hd >= 16 && hd <= 512 && hd % 32 == 0 && T >= 1 && T <= 64,
             "attention: unsupported shape M=%d nh=%d hd=%d T=%d", M, nh, hd, T);
  G4_REQUIRE(pos && lo && kmin >= 0 && kmax >= kmin, "attention: bad key range [%d, %d]", kmin, kmax);
  d.M = M; d.nh = nh; d.hd = hd; d.kmin = kmin; d.kmax = kmax; d.T = T;
  d.dynP = nullptr; d.base_add = d.q_add = d.window = 0;
  d.qo = QuantOut{nullptr, nullptr, nullptr};
  for (int m = 0; m < 4; ++m) { d.pos[m] = m < M ? pos[m] : -1; d.lo[m] = m < M ? lo[m] : 0; }
  for (int m = 0; m < M; ++m)
    G4_REQUIRE(lo[m] >= kmin && pos[m] <= kmax, "attention: row %d range [%d, %d] outside [%d, %d]", m, lo[m], pos[m],
               kmin, kmax);
  return G4_OK;
}

static size_t attn_counter_offset(int M, int nh, int hd, int len, int T);
static int attn_counter_count(int M, int nh, int hd) {
  const int a = M * nh, b = (hd / 32) * ((M * nh + 7) / 8);
  return a > b ? a : b;
}

// Scores, then either the chunk kernel (chunks of at most kChunkMaxKeys keys) or statistics,
// accumulation and merge as three kernels.  zeroed_counters as for launch_attn_short; NULL = the
// workspace's, reset first.  four = true forces the three-kernel tail (the allocation-free entry
// point, whose fixed scratch has no counters).
static int launch_attn(const uint16_t* Kc, const uint16_t* Vc, const float* q, const AttnDesc& d, float* w, float* out,
                       cudaStream_t st, int max_len = 0, int* zeroed_counters = nullptr, bool four = false) {
  const int len = max_len > 0 ? max_len : d.kmax - d.kmin + 1, nmh = d.M * d.nh;
  const size_t ssm = attn_scores_smem(d.hd);
  int rc = G4_OK;
  const dim3 sgrid((len + kScoreKeys - 1) / kScoreKeys), sblk(nmh * 16);
  if (d.hd == 256) rc = launch("k_attn_scores", k_attn_scores<16>, sgrid, sblk, ssm, st, Kc, q, d, w);
  else if (d.hd == 512) {
    cudaFuncSetAttribute(k_attn_scores<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm);
    rc = launch("k_attn_scores", k_attn_scores<32>, sgrid, sblk, ssm, st, Kc, q, d, w);
  }
  else if (d.hd == 128) rc = launch("k_attn_scores", k_attn_scores<8>, sgrid, sblk, ssm, st, Kc, q, d, w);
  else return set_error(G4_ERR_UNSUPPORTED, "attention: hd=%d (supported: 128, 256, 512)", d.hd);
  if (rc) return rc;
  static const bool chunk_on = [] {  // G4_ATTN_CHUNK=0/1 overrides the default (experiments)
    const char* e = getenv("G4_ATTN_CHUNK");
    return e ? e[0] == '1' : true;
  }();
  if (chunk_on && !four && d.T <= 16 && (len + d.T - 1) / d.T + 1 <= kChunkMaxKeys && d.hd % 32 == 0) {
    int* counters = zeroed_counters;
    if (counters == nullptr) {
      counters = reinterpret_cast<int*>(reinterpret_cast<char*>(w) + attn_counter_offset(d.M, d.nh, d.hd, len, d.T));
      cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int) * (size_t)attn_counter_count(d.M, d.nh, d.hd), st);
      if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "attention: counter reset: %s", cudaGetErrorString(e));
    }
    const size_t csm = attn_chunk_smem();
    cudaFuncSetAttribute(k_attn_chunk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csm);
    return launch("k_attn_chunk", k_attn_chunk, dim3(d.T, d.hd / 32, (nmh + 7) / 8), dim3(256), csm, st, Vc, d, w,
                  counters, out);
  }
  if (int rc_ = launch("k_attn_stats", k_attn_stats, dim3(d.T, (nmh + 7) / 8), dim3(256), 0, st, d, w)) return rc_;
  if (int rc_ = launch("k_attn_accum", k_attn_accum, dim3(d.T, d.hd / 16, (nmh + 7) / 8), dim3(64), 0, st, Vc, d, w))
    return rc_;
  if (int rc_ = launch("k_attn_merge", k_attn_merge, dim3(nmh), dim3(d.hd > 64 ? d.hd : 64), 0, st, d, w, out)) return rc_;
  return check_launch("k_attn_merge");
}

// Workspace of g4_attn_splitkv: the partial results (attn_ws_floats), then the int counters of the
// one-kernel and chunk paths (one per (row, head) pair, or per (32-dim slice, group of 8 pairs)).
static size_t attn_counter_offset(int M, int nh, int hd, int len, int T) {
  return (sizeof(float) * attn_ws_floats(M, nh, hd, len, T) + 15) / 16 * 16;
}
extern "C" size_t g4_attn_splitkv_ws_bytes(int M, int nh, int hd, int kmin, int kmax, int T) {
  return attn_counter_offset(M, nh, hd, kmax - kmin + 1, T) + sizeof(int) * (size_t)attn_counter_count(M, nh, hd);
}

// One-kernel path (k_attn_short) when every chunk has at most kAttnShortKeys keys; max_len bounds
// the key range (the device may pick a shorter one) and sizes the workspace.
// zeroed_counters: caller-owned per-pair counters known to be 0 (the merging block of every pair
// leaves its counter at 0 again); NULL = use the workspace's and reset them first.
static int launch_attn_short(const uint16_t* Kc, const uint16_t* Vc, const float* q, const AttnDesc& d, void* ws,
                             float* out, cudaStream_t st, int max_len, int* zeroed_counters = nullptr) {
  const int nmh = d.M * d.nh;
  const size_t smem = attn_short_smem(d.hd);
  int* counters = zeroed_counters;
  if (counters == nullptr) {
    counters = reinterpret_cast<int*>(static_cast<char*>(ws) + attn_counter_offset(d.M, d.nh, d.hd, max_len, d.T));
    cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int) * (size_t)nmh, st);
    if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "attention: counter reset: %s", cudaGetErrorString(e));
  }
  float* w = static_cast<float*>(ws);
  const dim3 grid(d.T, nmh);
  if (d.hd == 256) {
    cudaFuncSetAttribute(k_attn_short<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (int rc = launch("k_attn_short", k_attn_short<16>, grid, dim3(256), smem, st, Kc, Vc, q, d, w, counters, out))
      return rc;
  } else if (d.hd == 128) {
    cudaFuncSetAttribute(k_attn_short<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (int rc = launch("k_attn_short", k_attn_short<8>, grid, dim3(256), smem, st, Kc, Vc, q, d, w, counters, out))
      return rc;
  } else {
    return set_error(G4_ERR_UNSUPPORTED, "attention: hd=%d", d.hd);
  }
  return check_launch("k_attn_short");
}
static bool short_fits(int max_len, int T, int hd) {
  // chunk_lo(t+1) - chunk_lo(t) <= ceil(len / T); T <= 64 for the merge factors
  return (max_len + T - 1) / T <= kAttnShortKeys && T <= 32 && (hd == 256 || hd == 128);
}

extern "C" int g4_attn_splitkv(const uint16_t* Kc, const uint16_t* Vc, const float* q, const int* pos, const int* lo,
                               int M, int nh, int hd, int kmin, int kmax, int T, float* out, void* ws, size_t ws_bytes,
                               void* stream) {
  G4_REQUIRE(Kc && Vc && q && out && ws, "g4_attn_splitkv: null pointer");
  AttnDesc d;
  if (int rc = fill_desc(d, Kc, Vc, M, nh, hd, pos, lo, kmin, kmax, T)) return rc;
  const size_t need = g4_attn_splitkv_ws_bytes(M, nh, hd, kmin, kmax, T);
  if (ws_bytes < need) return set_error(G4_ERR_NOMEM, "g4_attn_splitkv: workspace %zu < %zu bytes", ws_bytes, need);
  G4_REQUIRE(aligned(ws, 16), "g4_attn_splitkv: workspace must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const int len = kmax - kmin + 1;
  if (short_fits(len, T, hd)) return launch_attn_short(Kc, Vc, q, d, ws, out, st, len);
  return launch_attn(Kc, Vc, q, d, static_cast<float*>(ws), out, st);
}

// Engine-internal form for captured decode steps: the key ranges come from the position *dP on the
// device (see AttnDesc::dynP); max_len bounds kmax - kmin + 1 over every position the capture will
// see and sizes the score grid (blocks past kmax return at once).  ws must hold max_len keys.
int g4::attn_splitkv_dev(const uint16_t* Kc, const uint16_t* Vc, const float* q, int M, int nh, int hd, const int* dP,
                         int base_add, int q_add, int window, int max_len, int T, float* out, void* ws, size_t ws_bytes,
                         cudaStream_t st, QuantOut qo, int* zeroed_counters) {
  G4_REQUIRE(Kc && Vc && q && out && ws && dP && max_len >= 1, "attn_splitkv_dev: bad arguments");
  int pos[4] = {0, 0, 0, 0}, lo[4] = {0, 0, 0, 0};
  for (int m = 0; m < M && m < 4; ++m) pos[m] = m;
  AttnDesc d;
  if (int rc = fill_desc(d, Kc, Vc, M, nh, hd, pos, lo, 0, M - 1, T)) return rc;
  d.dynP = dP; d.base_add = base_add; d.q_add = q_add; d.window = window;
  d.qo = qo;
  const size_t need = g4_attn_splitkv_ws_bytes(M, nh, hd, 0, max_len - 1, T);
  if (ws_bytes < need) return set_error(G4_ERR_NOMEM, "attn_splitkv_dev: workspace %zu < %zu bytes", ws_bytes, need);
  if (short_fits(max_len, T, hd)) return launch_attn_short(Kc, Vc, q, d, ws, out, st, max_len, zeroed_counters);
  return launch_attn(Kc, Vc, q, d, static_cast<float*>(ws), out, st, max_len, zeroed_counters);
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant of g4_attn_splitkv.
//
// Some callers cannot hand this library a workspace: code embedded in a host that owns every
// byte of device memory through its own arena and forbids foreign allocations, or a decode loop
// on a latency-critical thread where a cudaMalloc/cudaFree could stall on a device-wide
// synchronisation.  This entry point takes only inputs and outputs; its scratch is the fixed
// array below, a file-scope device global of kAttnNoAllocFloats floats (1,312,768 bytes) that every
// GPU which loads libg4.so holds until the process exits.  It serves M <= 4 rows, nh <= 8 heads,
// hd <= 256, T <= 8 chunks and up to 8,192 keys (kmax - kmin + 1); larger calls are rejected.
//
// In host code the name g_attn_scratch only stands for the array; the device address comes from
// cudaGetSymbolAddress, looked up again by every call made outside stream capture (so an address
// from before a cudaDeviceReset, after which the module is loaded anew, is never reused) and taken
// from the last such lookup on that device by calls made while the stream is being captured; make
// one call on the device before capturing.  All calls on a device share the array
// and it keeps the previous call's contents; every word a call reads is written earlier in the
// same call, so nothing needs clearing, but two calls whose kernels overlap on the GPU (two
// streams, or two host threads) race on it and must be serialised by the caller.
constexpr size_t kAttnNoAllocFloats = (size_t)8192 * 4 * 8 + 2 * (size_t)8 * 4 * 8 + (size_t)8 * 4 * 8 * 256;
static __device__ __align__(256) float g_attn_scratch[kAttnNoAllocFloats];

#include <mutex>
static std::mutex g_attn_scratch_mu;
static float* g_attn_scratch_dev[128];

static int attn_scratch_for_current_device(cudaStream_t st, float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_attn_splitkv_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return set_error(G4_ERR_UNSUPPORTED, "g4_attn_splitkv_noalloc: device %d", dev);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(st, &cs);
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_attn_splitkv_noalloc: cudaStreamIsCapturing: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_attn_scratch_mu);
  if (cs == cudaStreamCaptureStatusNone || g_attn_scratch_dev[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(G4_ERR_CUDA, "g4_attn_splitkv_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_attn_scratch_dev[dev] = static_cast<float*>(p);
  }
  *out = g_attn_scratch_dev[dev];
  return G4_OK;
}

extern "C" int g4_attn_splitkv_noalloc(const uint16_t* Kc, const uint16_t* Vc, const float* q, const int* pos,
                                       const int* lo, int M, int nh, int hd, int kmin, int kmax, int T, float* out,
                                       void* stream) {
  G4_REQUIRE(Kc && Vc && q && out, "g4_attn_splitkv_noalloc: null pointer");
  AttnDesc d;
  if (int rc = fill_desc(d, Kc, Vc, M, nh, hd, pos, lo, kmin, kmax, T)) return rc;
  const int len = kmax - kmin + 1;
  if (hd > 256 || T > 8 || len > 8192 || attn_ws_floats(M, nh, hd, len, T) > kAttnNoAllocFloats)
    return set_error(G4_ERR_UNSUPPORTED,
                     "g4_attn_splitkv_noalloc: M=%d nh=%d hd=%d T=%d keys=%d exceed the fixed scratch "
                     "(hd <= 256, T <= 8, keys <= 8192); use g4_attn_splitkv with a workspace",
                     M, nh, hd, T, len);
  cudaStream_t st = as_stream(stream);
  float* w = nullptr;
  if (int rc = attn_scratch_for_current_device(st, &w)) return rc;
  return launch_attn(Kc, Vc, q, d, w, out, st, 0, nullptr, /*four=*/true);
}
