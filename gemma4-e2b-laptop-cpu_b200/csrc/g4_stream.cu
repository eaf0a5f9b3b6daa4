// The verify pass's layer stack as persistent "segment" kernels (sm_100a).
//
// One launch covers everything of a decoder layer between two attentions: the o projection of
// layer l, the post-attention residual and pre-MLP norm, the fused gate/up projection with GeGLU
// and the down projection's int8 quantisation, the down projection, the post-MLP residual and the
// next layer's input norm, the qkv projection of layer l+1, and its q/k/v norms, RoPE and KV write
// (the reference's fwd, gemma4_engine.cpp:1262-1404, from :1358 of one layer to :1323 of the next).
// The first launch of a pass starts at the embedding (:1264), the last ends at the final norm
// (:1402).  Split-KV attention stays a separate kernel (g4_attn.cu) between the launches.
//
// Grid: one CTA per SM (persistent), 8 consumer warps + 1 producer warp.  The producer streams the
// CTA's share of the segment's weight rows -- fixed tiles of 16 rows (K = 2048) or 4 rows
// (K = 8192), 16 KB of int4 weights + 2 KB of bf16 scales each -- through a ring of shared-memory
// slots with 1D bulk copies (the TMA engine), in consumption order and independent of the
// activation dependencies, after first asking L2 to prefetch all of them; so HBM keeps streaming
// while the consumers wait at a stage boundary.  Stages are separated by grid barriers (an atomic
// arrival counter per barrier, bounded polling).  Activations that cross CTAs go through global
// memory (L2) and are read with ld.global.cg; each CTA recomputes the row norms it needs (M <= 4
// rows of 2048) instead of waiting for another stage.
//
// Arithmetic is exactly that of the per-kernel path: the W4A8 group dots are integer-exact
// (8 dp4a per activation row) and each (weight row, activation row) runs the fp32 chain
// row = fma(float(a32), sw*sx, row) over its groups in order (w4a8_avx2.h:57-58); norms take the
// sum of squares in double over the reference's 16 ordered partials; quantisation is
// w4a8::quant's (w4a8_avx2.h:30-42).  Only the int8 path (M = 2..4 rows) runs here.
#include "g4_api.h"
#include "g4_async.cuh"
#include "g4_common.cuh"
#include "g4_stream.h"
#include <algorithm>

namespace g4 {

constexpr int kSegConsumers = 256;
constexpr int kSegThreads = kSegConsumers + 32;
constexpr int kSegRowPad = 16;                                   // bytes after each weight row in a slot
constexpr int kSegScaleOff = 16 * (1024 + kSegRowPad);          // 16 rows of K = 2048 (4 rows of 8192 fit too)
constexpr int kSegSlot = kSegScaleOff + 2048;                   // 18,688 bytes
constexpr int kSegNS = 5;                                       // ring slots
constexpr int kSegKmax = 8192;

// Tile geometry of one matrix: rows per tile R (16 for K = 2048, 4 for K = 8192), tiles grouped in
// units that stay on one CTA (4 for the gate/up pair: gate rows 32u..32u+31 and the same up rows).
struct SegMatDev {
  const uint8_t* w;
  const uint16_t* s;
  int N, K, R, ntiles, tpu, off;
};

struct SegShared {
  uint64_t full[kSegNS], empty[kSegNS];
  double part[8][4][16];
  uint32_t keys[8][4][8];
  double chain[4][16];
  float r[4];
  int flag;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Number of units of matrix mat that CTA c owns, and the k-th of them.
__device__ __forceinline__ int seg_units(const SegMatDev& mt, int c, int G) {
  const int nunits = mt.ntiles / mt.tpu;
  const int first = ((c - mt.off) % G + G) % G;
  return first < nunits ? (nunits - 1 - first) / G + 1 : 0;
}
__device__ __forceinline__ int seg_unit(const SegMatDev& mt, int c, int G, int k) {
  return ((c - mt.off) % G + G) % G + k * G;
}
// First weight row of tile j (0 <= j < tpu) of unit u.
__device__ __forceinline__ int seg_tile_row(const SegMatDev& mt, int u, int j, int half_rows) {
  if (mt.tpu == 4) return (j < 2 ? 0 : half_rows) + 32 * u + 16 * (j & 1);  // gate / up halves
  return (u * mt.tpu + j) * mt.R;
}

// ------------------------------------------------------------------------------- grid barrier
// Monotonic arrival counter per barrier (zeroed before the launch); gives up after the wait limit
// and raises the abort flag so that every CTA leaves at its next barrier.  local_ok: this thread's
// status so far; the result is the same for every consumer thread of every CTA that returns true.
__device__ bool grid_barrier(unsigned* ctr, unsigned* abort_flag, unsigned G, bool local_ok, SegShared& sh) {
  if (!local_ok) sh.flag = 1;
  consumer_sync();
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    bool ok = sh.flag == 0;
    if (ok) {
      __threadfence();
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    }
    const unsigned long long t0 = globaltimer();
    while (ok) {
      unsigned v, ab;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= G) break;
      asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(ab) : "l"(abort_flag) : "memory");
      if (ab != 0u || globaltimer() - t0 > kWaitLimitNs) { ok = false; break; }
    }
    if (!ok) {
      sh.flag = 1;
      atomicOr(&g_dev_status, kStatusTimeout);
      atomicExch(abort_flag, 1u);
    }
    ok_s = ok ? 1 : 0;
  }
  consumer_sync();
  return ok_s != 0;
}

// ---------------------------------------------------------------------------- row prologues
// The norm prologues work on M <= 4 rows of H = 2048 floats in shared memory; thread t (< 256) owns
// float4 blocks t and t + 256 of every row.  Each helper is compiled once (not inlined) and loops
// over the rows, so that the code a launch runs once stays small: a launch runs on every SM once,
// and each new line of code is an instruction-cache miss.
constexpr int kH = 2048;

__device__ __forceinline__ float4 r16x4(float4 a) { return make_float4(r16(a.x), r16(a.y), r16(a.z), r16(a.w)); }
// (a * r) * w per element
__device__ __forceinline__ float4 scale4(float4 a, float r, float4 w) {
  return make_float4(__fmul_rn(__fmul_rn(a.x, r), w.x), __fmul_rn(__fmul_rn(a.y, r), w.y),
                     __fmul_rn(__fmul_rn(a.z, r), w.z), __fmul_rn(__fmul_rn(a.w, r), w.w));
}
// r16(x + r16((o * r) * w)) per element
__device__ __forceinline__ float4 resid4(float4 x, float4 o, float r, float4 w) {
  const float4 u = r16x4(scale4(o, r, w));
  return r16x4(make_float4(__fadd_rn(x.x, u.x), __fadd_rn(x.y, u.y), __fadd_rn(x.z, u.z), __fadd_rn(x.w, u.w)));
}

// rows [M][kH] from global memory (written earlier in this pass: read through L2), optionally
// rounded to bf16, into shared memory; all 2M loads are in flight before the first store.
__device__ __noinline__ void seg_load_rows(float* dst, const float* src, int M, int round) {
  const int t = threadIdx.x;
  float4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < 2 * M) v[i] = ldcg4(src + (size_t)(i >> 1) * kH + 4 * (t + 256 * (i & 1)));
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < 2 * M) reinterpret_cast<float4*>(dst + (size_t)(i >> 1) * kH)[t + 256 * (i & 1)] = round ? r16x4(v[i]) : v[i];
}

// rows [M][kH] from shared memory to global memory
__device__ __noinline__ void seg_store_rows(float* dst, const float* src, int M) {
  const int t = threadIdx.x;
  for (int i = 0; i < 2 * M; ++i)
    reinterpret_cast<float4*>(dst + (size_t)(i >> 1) * kH)[t + 256 * (i & 1)] =
        reinterpret_cast<const float4*>(src + (size_t)(i >> 1) * kH)[t + 256 * (i & 1)];
}

// x = r16(E[tok] * sqrt(H)) for the M tokens (:1264)
__device__ __noinline__ void seg_embed(float* dst, const uint16_t* E, const int* toks, int M, float sqrtH) {
  const int t = threadIdx.x;
  uint2 b[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < 2 * M) {
      const uint16_t* er = E + (size_t)__ldcg(toks + (i >> 1)) * kH;
      b[i] = __ldg(reinterpret_cast<const uint2*>(er) + t + 256 * (i & 1));
    }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < 2 * M)
      reinterpret_cast<float4*>(dst + (size_t)(i >> 1) * kH)[t + 256 * (i & 1)] =
          make_float4(r16(__fmul_rn(bf2f(b[i].x & 0xFFFFu), sqrtH)), r16(__fmul_rn(bf2f(b[i].x >> 16), sqrtH)),
                      r16(__fmul_rn(bf2f(b[i].y & 0xFFFFu), sqrtH)), r16(__fmul_rn(bf2f(b[i].y >> 16), sqrtH)));
}

// Exponent keys for the exactness test (see seg_rms): bytes (kmax, 255 - kmin) of the nonzero
// elements' biased exponents; a value that is not bf16-valued or not finite fails the test.
__device__ __forceinline__ uint32_t seg_ekeys(float x) {
  const uint32_t b = __float_as_uint(x) & 0x7FFFFFFFu;
  const uint32_t e = max(b >> 23, 1u);
  const uint32_t key = ((b & 0xFFFFu) != 0u || e == 255u) ? ((255u << 8) | 254u) : ((e << 8) | (255u - e));
  return b == 0u ? 0u : key;
}

// RMS scales sh.r[m] of the M rows in shared memory, in the reference's order (ss_avx2,
// :326-343): per row the sum of squares in double over 16 partials (element j to partial j % 16,
// each in element order), combined ((p_b + p_4+b) + (p_8+b + p_12+b)), then (t0 + t2) + (t1 + t3);
// r = 1 / sqrtf((float)(ss / n) + 1e-6).  A partial whose elements are bf16-valued with nonzero
// exponents spanning at most 15 is an exact sum in double in any order (every square is a multiple
// of 2^(2 e_min - 268) and 128 of them stay below 2^53 such units), so it is summed as a tree;
// any other partial runs the sequential chain.
__device__ __noinline__ void seg_rms(const float* rows, int M, SegShared& sh) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
#pragma unroll 1
  for (int m = 0; m < M; ++m) {
    const float4 v0 = reinterpret_cast<const float4*>(rows + (size_t)m * kH)[t];
    const float4 v1 = reinterpret_cast<const float4*>(rows + (size_t)m * kH)[t + 256];
    const float c[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    double d[4];
    uint32_t k01 = 0u, k23 = 0u;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const double a = c[e], b = c[4 + e];
      d[e] = fma(b, b, a * a);  // element order within the thread: block t, then block t + 256
    }
    k01 = __vmaxu4(seg_ekeys(c[0]) | (seg_ekeys(c[1]) << 16), seg_ekeys(c[4]) | (seg_ekeys(c[5]) << 16));
    k23 = __vmaxu4(seg_ekeys(c[2]) | (seg_ekeys(c[3]) << 16), seg_ekeys(c[6]) | (seg_ekeys(c[7]) << 16));
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
#pragma unroll
      for (int e = 0; e < 4; ++e) d[e] += __shfl_xor_sync(FULL, d[e], o);
      k01 = __vmaxu4(k01, __shfl_xor_sync(FULL, k01, o));
      k23 = __vmaxu4(k23, __shfl_xor_sync(FULL, k23, o));
    }
    if (lane < 4) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sh.part[w][m][4 * lane + e] = d[e];
      sh.keys[w][m][2 * lane] = k01;
      sh.keys[w][m][2 * lane + 1] = k23;
    }
  }
  consumer_sync();
  if (t < 16 * M) {
    const int m = t >> 4, p = t & 15;
    double s = 0.0;
    uint32_t kw = 0u;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) {
      s += sh.part[ww][m][p];
      kw = __vmaxu4(kw, sh.keys[ww][m][p >> 1]);
    }
    const uint32_t kk = (kw >> (16 * (p & 1))) & 0xFFFFu;
    const int kmax = (int)(kk >> 8), kmin = 255 - (int)(kk & 0xFFu);
    if (kmax - kmin > 15) {  // the chain in element order, 8 loads in flight ahead of it
      s = 0.0;
      const float* xr = rows + (size_t)m * kH;
#pragma unroll 1
      for (int i = p; i < kH; i += 128) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = xr[i + 16 * u];
#pragma unroll
        for (int u = 0; u < 8; ++u) { const double x = v[u]; s = fma(x, x, s); }
      }
    }
    sh.chain[m][p] = s;
  }
  consumer_sync();
  if (t < M) {
    double tb[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) tb[b] = (sh.chain[t][b] + sh.chain[t][4 + b]) + (sh.chain[t][8 + b] + sh.chain[t][12 + b]);
    const double ss = (tb[0] + tb[2]) + (tb[1] + tb[3]);
    sh.r[t] = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(ss * (1.0 / (double)kH)), 1e-6f)));  // kH a power of two
  }
  consumer_sync();
}

// x = r16(x + r16((o * r_m) * w)) for the M rows in shared memory (r from seg_rms of o)
__device__ __noinline__ void seg_resid(float* x, const float* o, float4 w0, float4 w1, int M, const SegShared& sh) {
  const int t = threadIdx.x;
#pragma unroll 1
  for (int m = 0; m < M; ++m) {
    const float r = sh.r[m];
    float4* xm = reinterpret_cast<float4*>(x + (size_t)m * kH);
    const float4* om = reinterpret_cast<const float4*>(o + (size_t)m * kH);
    xm[t] = resid4(xm[t], om[t], r, w0);
    xm[t + 256] = resid4(xm[t + 256], om[t + 256], r, w1);
  }
}

// w4a8::quant of the float4 block f of row m into shared memory: a 32-group is the 8 consecutive
// threads holding its blocks (all 32 lanes call it together).
__device__ __forceinline__ void quant4_smem(float4 y, int f, int m, int8_t* q, int qstride, float* sx, int32_t* sm) {
  float amax = fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w)));
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, o));
  const float s = __fdiv_rn(amax, 127.0f);
  const float inv = s > 0.f ? __frcp_rn(s) : 0.0f;  // = __fdiv_rn(1.0f, s): both correctly rounded
  const float c[4] = {y.x, y.y, y.z, y.w};
  int32_t tot = 0;
  uint32_t packed = 0u;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float v = __fmul_rn(c[e], inv);
    const int32_t rr = (v > -2147483648.f && v < 2147483648.f) ? __float2int_rn(v) : INT32_MIN;
    tot += rr;
    const int32_t r16v = rr < -32768 ? -32768 : (rr > 32767 ? 32767 : rr);
    const int32_t qq = r16v < -128 ? -128 : (r16v > 127 ? 127 : r16v);
    packed |= ((uint32_t)qq & 0xFFu) << (8 * e);
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) tot += __shfl_xor_sync(FULL, tot, o);
  *reinterpret_cast<uint32_t*>(q + (size_t)m * qstride + 4 * f) = packed;
  if ((threadIdx.x & 7) == 0) {
    sx[m * 256 + (f >> 3)] = s;
    sm[m * 256 + (f >> 3)] = tot;
  }
}

// y = (x * r_m) * w (rounded to bf16 when round) for the M rows: to out (global, when not NULL) or
// quantised into the stage's int8 activations q / sx / sm (stride kH + 16).
__device__ __noinline__ void seg_scale(const float* x, float4 w0, float4 w1, int M, int round, const SegShared& sh, int8_t* q,
                                       float* sx, int32_t* sm, float* out) {
  const int t = threadIdx.x;
#pragma unroll 1
  for (int m = 0; m < M; ++m) {
    const float r = sh.r[m];
    const float4* xm = reinterpret_cast<const float4*>(x + (size_t)m * kH);
    float4 y0 = scale4(xm[t], r, w0), y1 = scale4(xm[t + 256], r, w1);
    if (round) { y0 = r16x4(y0); y1 = r16x4(y1); }
    if (out) {
      reinterpret_cast<float4*>(out + (size_t)m * kH)[t] = y0;
      reinterpret_cast<float4*>(out + (size_t)m * kH)[t + 256] = y1;
    } else {
      quant4_smem(y0, t, m, q, kH + 16, sx, sm);
      quant4_smem(y1, t + 256, m, q, kH + 16, sx, sm);
    }
  }
}

// ------------------------------------------------------------------------------------ kernel
struct SegSmem {
  uint8_t* slots;   // kSegNS x kSegSlot
  int8_t* q;        // [M][K + 16] int8 activations
  float* sx;        // [M][256]
  int32_t* sm;      // [M][256]
  int* ac;          // phase-1 integer dots of a round (kSegAcBytes)
  float* ra;        // [M][2048] prologue rows A and B (alias ac: used only between GEMV stages)
  float* rb;
  uint16_t* scl;    // the round's tile scales (kSegSclBytes)
  float* gub;       // [8 tiles][4][16] gate/up outputs of a round
};

// Load the int8 activations [M][K] (+ scales, sums) of a stage from global memory (written earlier
// in this pass by other CTAs or kernels) into shared memory.
template <int M>
__device__ void load_act(const int8_t* q, const float* sx, const int32_t* sm, int K, const SegSmem& S) {
  const int G = K >> 5;
  const int n16 = K >> 4;
  for (int i = threadIdx.x; i < M * n16; i += kSegConsumers) {
    const int m = i / n16, c = i % n16;
    const int4 v = __ldcg(reinterpret_cast<const int4*>(q + (size_t)m * K) + c);
    *reinterpret_cast<int4*>(S.q + (size_t)m * (K + 16) + 16 * c) = v;
  }
  for (int i = threadIdx.x; i < M * G; i += kSegConsumers) {
    const int m = i / G, g = i % G;
    S.sx[m * 256 + g] = __ldcg(sx + (size_t)m * G + g);
    S.sm[m * 256 + g] = __ldcg(sm + (size_t)m * G + g);
  }
}

// A GEMV stage over this CTA's tiles of one matrix, in rounds of up to kSegRoundTiles(M) tiles:
//   phase 1 (all 256 threads): as each tile lands, thread (group g, row subset) computes the exact
//     integer dots a32 = sum t*xq - 8*sum of its rows for all M activation rows into ac, and the
//     tile's bf16 scales are copied out; the ring slot is then freed;
//   phase 2: one thread per (tile, row, activation row) runs the fp32 chain
//     row = fma(float(a32), sw*sx, row) over the groups in order.
// Output rows go to Y (or, for the gate/up pair, to the GeGLU of the round's units, whose int8
// quantisation is written to aq / asx / asum).
constexpr int kSegAcBytes = 68 * 1024;   // 4 or 8 tiles x 16 x 4 or 2 rows x 68 ints
constexpr int kSegSclBytes = 18 * 1024;  // 8 tiles x 16 rows x 72 bf16
template <int M>
__device__ __forceinline__ int seg_round_tiles() { return M == 2 ? 8 : 4; }

template <int M>
__device__ __noinline__ bool gemv_stage(const SegMatDev mt, int ring, float* Y, int ldy, int half_rows, const SegSmem S,
                                        SegShared& sh, bool geglu, int8_t* aq, float* asx, int32_t* asum) {
  const int G = gridDim.x, c = blockIdx.x, t = threadIdx.x;
  constexpr int MT = M == 3 ? 4 : M;
  const int R = mt.R, K = mt.K, NG = K >> 5;
  const int acs = NG + 4;                 // ac row stride (ints): 16-byte pad, bank-spread rows
  const int scs = NG + 8;                 // scale row stride (bf16)
  const int RS = kSegConsumers / NG;      // row subsets in phase 1 (4 for K = 2048, 1 for 8192)
  const int ntr = seg_round_tiles<M>();
  const int nunits = seg_units(mt, c, G);
  const int ntl = nunits * mt.tpu;
  // phase-1 role: group g, rows rsub, rsub + RS, ...; its activations stay in registers all stage
  const int g = t % NG, rsub = t / NG;
  int4 qa[M], qb[M];
  int bias[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    qa[m] = *reinterpret_cast<const int4*>(S.q + (size_t)m * (K + 16) + (size_t)g * 32);
    qb[m] = *reinterpret_cast<const int4*>(S.q + (size_t)m * (K + 16) + (size_t)g * 32 + 16);
    bias[m] = -8 * S.sm[m * 256 + g];
  }
  bool ok = true;
  for (int base = 0; base < ntl; base += ntr) {
    const int nt = min(ntr, ntl - base);
    for (int ti = 0; ti < nt; ++ti) {
      const int i = base + ti;
      const int slot = (ring + i) % kSegNS;
      if (!mbar_wait(&sh.full[slot], (uint32_t)(((ring + i) / kSegNS) & 1))) ok = false;
      const uint8_t* sb = S.slots + (size_t)slot * kSegSlot;
      if (ok) {
        for (int r = rsub; r < R; r += RS) {
          const uint4 wv = *reinterpret_cast<const uint4*>(sb + (size_t)r * ((K >> 1) + kSegRowPad) + (size_t)g * 16);
          const uint32_t lo0 = wv.x & 0x0F0F0F0Fu, lo1 = wv.y & 0x0F0F0F0Fu, lo2 = wv.z & 0x0F0F0F0Fu, lo3 = wv.w & 0x0F0F0F0Fu;
          const uint32_t hi0 = (wv.x >> 4) & 0x0F0F0F0Fu, hi1 = (wv.y >> 4) & 0x0F0F0F0Fu, hi2 = (wv.z >> 4) & 0x0F0F0F0Fu,
                         hi3 = (wv.w >> 4) & 0x0F0F0F0Fu;
          int* acr = S.ac + ((size_t)(ti * R + r) * MT) * acs + g;
#pragma unroll
          for (int m = 0; m < M; ++m) {
            int a0 = bias[m], a1 = 0;  // the integer dot is exact in any order
            a0 = __dp4a((int)lo0, qa[m].x, a0);
            a1 = __dp4a((int)lo1, qa[m].y, a1);
            a0 = __dp4a((int)lo2, qa[m].z, a0);
            a1 = __dp4a((int)lo3, qa[m].w, a1);
            a0 = __dp4a((int)hi0, qb[m].x, a0);
            a1 = __dp4a((int)hi1, qb[m].y, a1);
            a0 = __dp4a((int)hi2, qb[m].z, a0);
            a1 = __dp4a((int)hi3, qb[m].w, a1);
            acr[(size_t)m * acs] = a0 + a1;
          }
        }
        // the tile's scales, to a bank-spread copy
        const int cpr = NG >> 3;  // 16-byte chunks per scale row
        if (t < R * cpr) {
          const int rr = t / cpr, ch = t % cpr;
          *reinterpret_cast<uint4*>(S.scl + (size_t)(ti * R + rr) * scs + ch * 8) =
              *reinterpret_cast<const uint4*>(sb + kSegScaleOff + (size_t)rr * NG * 2 + ch * 16);
        }
      }
      consumer_sync();  // every thread is done with the slot
      if (t == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sh.empty[slot])) : "memory");
    }
    // phase 2: chain (tile ti, activation row m, row r), r fastest
    const int per_tile = R * M;
    if (ok && t < nt * per_tile) {
      const int ti = t / per_tile, rem = t % per_tile, r = rem % R, m = rem / R;
      const int* acr = S.ac + ((size_t)(ti * R + r) * MT + m) * acs;
      const uint16_t* scr = S.scl + (size_t)(ti * R + r) * scs;
      const float* sxm = S.sx + m * 256;
      float row = 0.f;
#pragma unroll 2
      for (int g8 = 0; g8 < NG; g8 += 8) {
        const int4 a_lo = *reinterpret_cast<const int4*>(acr + g8), a_hi = *reinterpret_cast<const int4*>(acr + g8 + 4);
        const uint4 s8 = *reinterpret_cast<const uint4*>(scr + g8);
        const float4 x_lo = *reinterpret_cast<const float4*>(sxm + g8), x_hi = *reinterpret_cast<const float4*>(sxm + g8 + 4);
        const int av[8] = {a_lo.x, a_lo.y, a_lo.z, a_lo.w, a_hi.x, a_hi.y, a_hi.z, a_hi.w};
        const uint32_t sw[4] = {s8.x, s8.y, s8.z, s8.w};
        const float xv[8] = {x_lo.x, x_lo.y, x_lo.z, x_lo.w, x_hi.x, x_hi.y, x_hi.z, x_hi.w};
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint32_t b = (u & 1) ? (sw[u >> 1] >> 16) : (sw[u >> 1] & 0xFFFFu);
          row = fmaf((float)av[u], __fmul_rn(bf2f(b), xv[u]), row);
        }
      }
      const int u = seg_unit(mt, c, G, (base + ti) / mt.tpu), tj = (base + ti) % mt.tpu;
      const int n0 = seg_tile_row(mt, u, tj, half_rows);
      if (geglu) S.gub[((size_t)ti * 4 + m) * 16 + r] = row;
      else Y[(size_t)m * ldy + n0 + r] = row;
    }
    consumer_sync();
    if (geglu && ok) {
      // GeGLU of the round's units (tiles 4k..4k+3: gate rows 0-15, 16-31, up rows 0-15, 16-31 of
      // one unit): act = r16(r16(gelu(r16 g)) * r16 u), then the 32-group quantisation
      const int w = t >> 5, lane = t & 31;
      const int units = nt / 4;
      for (int pi = w; pi < units * M; pi += 8) {
        const int ur = pi / M, mm = pi % M;
        const int u = seg_unit(mt, c, G, (base + 4 * ur) / 4);
        const float gv = r16(S.gub[((size_t)(4 * ur + (lane >> 4)) * 4 + mm) * 16 + (lane & 15)]);
        const float uv = r16(S.gub[((size_t)(4 * ur + 2 + (lane >> 4)) * 4 + mm) * 16 + (lane & 15)]);
        const float v = r16(__fmul_rn(r16(gelu(gv)), uv));
        int8_t qv;
        float sxv;
        int32_t tot;
        quant_group32(v, qv, sxv, tot);
        const int I = half_rows;
        aq[(size_t)mm * I + 32 * u + lane] = qv;
        if (lane == 0) {
          asx[(size_t)mm * (I >> 5) + u] = sxv;
          asum[(size_t)mm * (I >> 5) + u] = tot;
        }
      }
      consumer_sync();
    }
  }
  return ok;
}

// Producer warp (lane 0): L2 prefetch of every tile of this CTA, then the ring of bulk copies.
__device__ void seg_producer(const SegMatDev* mats, int nmats, const int* half_rows, SegSmem S, SegShared& sh,
                             unsigned* abort_flag) {
  if ((threadIdx.x & 31) != 0) return;
  const int G = gridDim.x, c = blockIdx.x;
  for (int s = 0; s < nmats; ++s) {
    const SegMatDev& mt = mats[s];
    const int nu = seg_units(mt, c, G);
    for (int k = 0; k < nu; ++k) {
      const int u = seg_unit(mt, c, G, k);
      for (int tj = 0; tj < mt.tpu; ++tj) {
        const int n0 = seg_tile_row(mt, u, tj, half_rows[s]);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(mt.w + (size_t)n0 * (mt.K >> 1)),
                     "r"((uint32_t)(mt.R * (mt.K >> 1))) : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(mt.s + (size_t)n0 * (mt.K >> 5)),
                     "r"((uint32_t)(mt.R * (mt.K >> 5) * 2)) : "memory");
      }
    }
  }
  int ring = 0;
  for (int s = 0; s < nmats; ++s) {
    const SegMatDev& mt = mats[s];
    const int nu = seg_units(mt, c, G);
    const uint32_t rowb = (uint32_t)(mt.K >> 1), sb = (uint32_t)(mt.R * (mt.K >> 5) * 2);
    for (int k = 0; k < nu; ++k) {
      const int u = seg_unit(mt, c, G, k);
      for (int tj = 0; tj < mt.tpu; ++tj, ++ring) {
        const int slot = ring % kSegNS;
        if (ring >= kSegNS) {  // wait until the consumers freed the slot's previous tile
          const uint32_t par = (uint32_t)(((ring / kSegNS) - 1) & 1);
          if (!mbar_wait(&sh.empty[slot], par)) {
            atomicOr(&g_dev_status, kStatusTimeout);
            atomicExch(abort_flag, 1u);
            return;
          }
        }
        const int n0 = seg_tile_row(mt, u, tj, half_rows[s]);
        uint8_t* dst = S.slots + (size_t)slot * kSegSlot;
        mbar_expect_tx(&sh.full[slot], (uint32_t)mt.R * rowb + sb);
        for (int r = 0; r < mt.R; ++r)
          bulk_g2s(dst + (size_t)r * (rowb + kSegRowPad), mt.w + (size_t)(n0 + r) * rowb, rowb, &sh.full[slot]);
        bulk_g2s(dst + kSegScaleOff, mt.s + (size_t)n0 * (mt.K >> 5), sb, &sh.full[slot]);
      }
    }
  }
  // no copy may still be landing when the CTA exits: wait (bounded) for the last fill of every slot
  for (int k = ring - 1; k >= 0 && k >= ring - kSegNS; --k)
    if (!mbar_wait(&sh.full[k % kSegNS], (uint32_t)((k / kSegNS) & 1))) atomicOr(&g_dev_status, kStatusInflight);
}

template <int M>
__global__ void __launch_bounds__(kSegThreads, 1) k_seg(const __grid_constant__ SegParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ SegShared sh;
  SegSmem S;
  S.slots = smem;
  S.q = reinterpret_cast<int8_t*>(smem + (size_t)kSegNS * kSegSlot);
  S.sx = reinterpret_cast<float*>(S.q + (size_t)M * (kSegKmax + 16));
  S.sm = reinterpret_cast<int32_t*>(S.sx + M * 256);
  S.ac = reinterpret_cast<int*>(S.sm + M * 256);
  S.ra = reinterpret_cast<float*>(S.ac);
  S.rb = S.ra + (size_t)M * kH;
  S.scl = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(S.ac) + kSegAcBytes);
  S.gub = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(S.scl) + kSegSclBytes);
  const int t = threadIdx.x;
  if (t == 0) {
    for (int i = 0; i < kSegNS; ++i) { mbar_init(&sh.full[i], 1); mbar_init(&sh.empty[i], 1); }
    fence_mbar_init();
    sh.flag = 0;
  }
  __syncthreads();
  // the matrices of this launch, in stage order (the producer streams their tiles in this order)
  SegMatDev mats[4];
  int half[4] = {0, 0, 0, 0};
  int nm = 0, i_o = -1, i_gu = -1, i_dn = -1, i_qkv = -1;
  if (p.do_mlp) {
    i_o = nm;  mats[nm++] = SegMatDev{p.o.w, p.o.s, p.o.N, p.o.K, 16, p.o.N / 16, 1, 0};
    i_gu = nm; half[nm] = p.I; mats[nm++] = SegMatDev{p.gu.w, p.gu.s, p.gu.N, p.gu.K, 16, p.gu.N / 16, 4, 37};
    i_dn = nm; mats[nm++] = SegMatDev{p.down.w, p.down.s, p.down.N, p.down.K, 4, p.down.N / 4, 1, 74};
  }
  if (p.do_qkv) { i_qkv = nm; mats[nm++] = SegMatDev{p.qkv.w, p.qkv.s, p.qkv.N, p.qkv.K, 16, p.qkv.N / 16, 1, 111}; }
  const bool tracer = p.trace != nullptr && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1);
  unsigned long long* trc = tracer ? p.trace + ((size_t)p.trace_slot * 2 + (blockIdx.x ? 1 : 0)) * kSegStamps : nullptr;
  auto stamp = [&](int k) {
    if (trc && (threadIdx.x == 0 || threadIdx.x == kSegConsumers)) trc[k] = globaltimer();
  };
  if (t >= kSegConsumers) {  // producer warp: weights are read-only, no wait on earlier kernels
    stamp(20);
    seg_producer(mats, nm, half, S, sh, p.abort_flag);
    stamp(22);
    return;
  }
  stamp(0);
  // the norm weights of this launch (read-only) in registers before the wait on the previous kernel
  float4 w_pa[2], w_pf[2], w_pff[2], w_nx[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    w_pa[k] = p.do_mlp ? __ldg(reinterpret_cast<const float4*>(p.w_post_attn) + t + 256 * k) : z;
    w_pf[k] = p.do_mlp ? __ldg(reinterpret_cast<const float4*>(p.w_pre_ff) + t + 256 * k) : z;
    w_pff[k] = p.do_mlp ? __ldg(reinterpret_cast<const float4*>(p.w_post_ff) + t + 256 * k) : z;
    w_nx[k] = __ldg(reinterpret_cast<const float4*>(p.w_next) + t + 256 * k);
  }
  pdl_wait();
  stamp(1);
  const unsigned G = gridDim.x;
  int ring = 0;
  bool ok = true;
  int bar = 0;
  auto tiles = [&](int i) { return seg_units(mats[i], blockIdx.x, G) * mats[i].tpu; };

  if (p.do_mlp) {
    // ---- S1: o projection of the attention output (quantised by the attention kernel)
    load_act<M>(p.att_q, p.att_sx, p.att_sum, p.o.K, S);
    consumer_sync();
    stamp(2);
    ok = gemv_stage<M>(mats[i_o], ring, p.o_out, p.H, 0, S, sh, false, nullptr, nullptr, nullptr) && ok;
    ring += tiles(i_o);
    stamp(3);
    ok = grid_barrier(p.bar + bar++, p.abort_flag, G, ok, sh);
    stamp(4);
    // ---- S2: o = r16(o); x = r16(x + r16((o*r)*w_post)); mlp_in = r16((x*r')*w_pre), quantised;
    //          then gate/up with GeGLU and the down projection's quantisation
    if (ok) {
      seg_load_rows(S.ra, p.o_out, M, 1);
      seg_load_rows(S.rb, p.x_a, M, 0);
      consumer_sync();
      seg_rms(S.ra, M, sh);
      stamp(5);
      seg_resid(S.rb, S.ra, w_pa[0], w_pa[1], M, sh);
      consumer_sync();
      if (blockIdx.x == 0) seg_store_rows(p.x_b, S.rb, M);
      seg_rms(S.rb, M, sh);
      seg_scale(S.rb, w_pf[0], w_pf[1], M, 1, sh, S.q, S.sx, S.sm, nullptr);
      consumer_sync();
      stamp(6);
      ok = gemv_stage<M>(mats[i_gu], ring, nullptr, 0, p.I, S, sh, true, p.act_q, p.act_sx, p.act_sum) && ok;
      stamp(7);
    }
    ring += tiles(i_gu);
    ok = grid_barrier(p.bar + bar++, p.abort_flag, G, ok, sh);
    stamp(8);
    // ---- S3: down projection
    if (ok) {
      load_act<M>(p.act_q, p.act_sx, p.act_sum, p.down.K, S);
      consumer_sync();
      stamp(9);
      ok = gemv_stage<M>(mats[i_dn], ring, p.down_out, p.H, 0, S, sh, false, nullptr, nullptr, nullptr) && ok;
      stamp(10);
    }
    ring += tiles(i_dn);
    ok = grid_barrier(p.bar + bar++, p.abort_flag, G, ok, sh);
    stamp(11);
    // ---- S4: o = r16(down); x = r16(x + r16((o*r)*w_post_ff)) (layer scalar 1); then the next
    //          layer's input norm (x*r')*w_in, quantised, or the final norm (rounded) into hbuf
    if (ok) {
      seg_load_rows(S.ra, p.down_out, M, 1);
      seg_load_rows(S.rb, p.x_b, M, 0);
      consumer_sync();
      stamp(16);
      seg_rms(S.ra, M, sh);
      stamp(17);
      seg_resid(S.rb, S.ra, w_pff[0], w_pff[1], M, sh);
      consumer_sync();
      if (blockIdx.x == 0) seg_store_rows(p.x_a, S.rb, M);
      stamp(18);
      seg_rms(S.rb, M, sh);
      stamp(19);
      if (!p.do_qkv) {  // final norm, rounded (:1402)
        if (blockIdx.x == 0) seg_scale(S.rb, w_nx[0], w_nx[1], M, 1, sh, nullptr, nullptr, nullptr, p.hbuf);
      } else {
        seg_scale(S.rb, w_nx[0], w_nx[1], M, 0, sh, S.q, S.sx, S.sm, nullptr);
      }
      consumer_sync();
    }
  } else if (p.do_qkv) {
    // ---- first launch of a pass: x = r16(E[tok] * sqrt(H)) (:1264), a = (x*r)*w_in, quantised
    seg_embed(S.rb, p.E, p.toks, M, p.sqrtH);
    consumer_sync();
    if (blockIdx.x == 0) seg_store_rows(p.x_a, S.rb, M);
    seg_rms(S.rb, M, sh);
    seg_scale(S.rb, w_nx[0], w_nx[1], M, 0, sh, S.q, S.sx, S.sm, nullptr);
    consumer_sync();
  }
  if (p.do_qkv) {
    // ---- qkv projection of the next layer
    stamp(12);
    if (ok) ok = gemv_stage<M>(mats[i_qkv], ring, p.qkv_out, p.qkv.N, 0, S, sh, false, nullptr, nullptr, nullptr) && ok;
    stamp(13);
    ok = grid_barrier(p.bar + bar++, p.abort_flag, G, ok, sh);
    stamp(14);
    // ---- S5: q/k/v norms, RoPE and the KV write (:1290-1303), warp per (row, part)
    if (ok) {
      const int HD = p.HD, hh = HD >> 1, per = HD >> 6, nparts = p.NQ + 2;
      const int lane = t & 31, gw = blockIdx.x * 8 + (t >> 5);
      if (gw < M * nparts) {
        const int m = gw / nparts, part = gw % nparts;
        const int pos = (p.dpos ? __ldcg(p.dpos) : 0) + p.pos0 + m;
        const float* w = part < p.NQ ? p.qn : (part == p.NQ ? p.kn : nullptr);
        const float* src = p.qkv_out + (size_t)m * p.qkv.N + (size_t)part * HD;
        float xl[4], xh[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = lane + 32 * k;
          xl[k] = k < per ? __ldcg(src + j) : 0.f;
          xh[k] = k < per ? __ldcg(src + j + hh) : 0.f;
        }
        double s = 0.0;  // lanes 0..15: partial `lane` (elements lane, lane + 16, ... in order; HD = 256)
        if (lane < 16) {
          float v[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] = __ldcg(src + lane + 16 * k);
#pragma unroll
          for (int k = 0; k < 16; ++k) { const double d = v[k]; s = fma(d, d, s); }
        }
        double u = s + __shfl_down_sync(FULL, s, 4);
        double tt = u + __shfl_down_sync(FULL, u, 8);
        double v2 = tt + __shfl_down_sync(FULL, tt, 2);
        double ss = v2 + __shfl_down_sync(FULL, v2, 1);
        ss = __shfl_sync(FULL, ss, 0);
        const double mean = (HD & (HD - 1)) == 0 ? ss * (1.0 / (double)HD) : ss / (double)HD;
        const float r = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)mean, 1e-6f)));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (k >= per) break;
          const int j = lane + 32 * k;
          const float a = w ? r16(__fmul_rn(__fmul_rn(xl[k], r), w[j])) : r16(__fmul_rn(xl[k], r));
          const float b = w ? r16(__fmul_rn(__fmul_rn(xh[k], r), w[j + hh])) : r16(__fmul_rn(xh[k], r));
          if (part == p.NQ + 1) {
            p.Vc[(size_t)pos * HD + j] = (uint16_t)f2bf(a);
            p.Vc[(size_t)pos * HD + j + hh] = (uint16_t)f2bf(b);
            continue;
          }
          const float cs = p.cosT[(size_t)pos * hh + j], sn = p.sinT[(size_t)pos * hh + j];
          const float ra = fmaf(a, cs, -__fmul_rn(b, sn));  // rope_avx2 (:394-402)
          const float rb = fmaf(b, cs, __fmul_rn(a, sn));
          if (part == p.NQ) {
            p.Kc[(size_t)pos * HD + j] = (uint16_t)f2bf(ra);
            p.Kc[(size_t)pos * HD + j + hh] = (uint16_t)f2bf(rb);
          } else {
            float* dst = p.qs + (size_t)m * p.ldq + (size_t)part * HD;
            dst[j] = ra;
            dst[j + hh] = rb;
          }
        }
      }
    }
  }
  stamp(15);
  (void)ok;
}

}  // namespace g4

G4_STATUS_READER(stream)

using namespace g4;

namespace g4 {
size_t seg_smem_bytes(int M) {
  return (size_t)kSegNS * kSegSlot + (size_t)M * (kSegKmax + 16) + (size_t)M * 256 * 8 + kSegAcBytes + kSegSclBytes +
         (size_t)8 * 4 * 16 * 4;
}

int seg_check(const SegParams& p) {
  const bool shapes = p.H == 2048 && p.HD == 256 && p.NQ == 8 && p.QD == 2048 && (!p.do_mlp || (p.o.N == p.H && p.o.K == p.QD &&
                      p.gu.N == 2 * p.I && p.gu.K == p.H && p.down.N == p.H && p.down.K == p.I && p.I == 8192)) &&
                      (!p.do_qkv || (p.qkv.N == p.QD + 2 * p.HD && p.qkv.K == p.H));
  if (!shapes || p.M < 2 || p.M > 4) return set_error(G4_ERR_UNSUPPORTED, "segment kernel: unsupported shape");
  return G4_OK;
}

// Launch with one CTA per SM (the shared memory allows no second one): the grid barriers need every
// CTA resident at once, which holds because the grid is no larger than the SM count and the only
// other kernels in flight are the one before it in the stream, which does not wait for this one,
// and the one after it, which (programmatic launch) starts only once every CTA here has issued
// launch_dependents, i.e. is resident.  Every barrier wait is bounded in any case.  Programmatic
// dependent launch lets the producer's weight stream start under the previous kernel when the
// engine records a pass.
int seg_launch(const SegParams& p, cudaStream_t st) {
  if (int rc = seg_check(p)) return rc;
  static int nsm = 0;
  if (nsm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || nsm <= 0) nsm = 148;
  }
  const size_t smem = seg_smem_bytes(p.M);
  auto go = [&](auto kern) -> int {
    if (inflight_fault().load(std::memory_order_relaxed))
      return set_error(G4_ERR_TIMEOUT, "k_seg: refused: a kernel ended with copies in flight (device status bit 1)");
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kSegThreads, smem) != cudaSuccess || occ < 1)
      return set_error(G4_ERR_UNSUPPORTED, "segment kernel: %zu B of shared memory do not fit an SM", smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nsm);
    cfg.blockDim = dim3(kSegThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    if (occ * nsm < nsm) return set_error(G4_ERR_UNSUPPORTED, "segment kernel: grid does not fit");
    // attribute sets tried in order: programmatic (when recording a pass), ordinary, cooperative
    cudaError_t e = cudaErrorUnknown;
    for (int variant = pdl_enabled() ? 0 : 1; variant < 3; ++variant) {
      cudaLaunchAttribute at[2];
      int na = 0;
      if (variant == 2) {
        at[na].id = cudaLaunchAttributeCooperative;
        at[na].val.cooperative = 1;
        ++na;
      }
      if (variant == 0) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
      }
      cfg.attrs = at;
      cfg.numAttrs = na;
      e = cudaLaunchKernelEx(&cfg, kern, p);
      if (e == cudaSuccess) break;
      cudaGetLastError();
    }
    if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "k_seg: %s", cudaGetErrorString(e));
    ++launch_count();
    return G4_OK;
  };
  switch (p.M) {
    case 2: return go(k_seg<2>);
    case 3: return go(k_seg<3>);
    default: return go(k_seg<4>);
  }
}
}  // namespace g4
