// W4G32 and W4A8 linears for decode and draft verification (M <= 8 activation rows).
//
// Both GEMVs stream the int4 weights once from HBM in the device layout made by g4_w4_pack
// (per 32-group, byte b holds element b in its low nibble and element 16+b in its high
// nibble).  That one layout serves both kernels:
//   * float path: lane j of a row needs elements 2j, 16+2j, 2j+1, 17+2j of every group, which
//     are the four nibbles of the little-endian u16 at byte 2j, in exactly the order in which
//     the reference's lane j multiplies them (w4g32_avx2.h:74-91);
//   * int8 path: the low nibbles of word k are elements 4k..4k+3 and the high nibbles elements
//     16+4k..16+4k+3, so each masked word pairs with a natural-order word of int8 activations
//     in one dp4a.
#include "g4_api.h"
#include "g4_common.cuh"
#include "g4_async.cuh"
#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <mutex>

namespace g4 {

// ---------------------------------------------------------------------------------- relayout
// Reference layout byte b = element 2b | element 2b+1 << 4  ->  device layout byte b =
// element b | element 16+b << 4.  One thread per 32-group.
__global__ void k_w4_pack(const uint8_t* __restrict__ W, long long groups, uint8_t* __restrict__ Wp) {
  pdl_wait();
  pdl_trigger();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= groups) return;
  const uint4 v = reinterpret_cast<const uint4*>(W)[i];
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
  uint32_t t[32];
#pragma unroll
  for (int b = 0; b < 16; ++b) {
    const uint32_t byte = (in[b >> 2] >> (8 * (b & 3))) & 0xFFu;
    t[2 * b] = byte & 15u;
    t[2 * b + 1] = byte >> 4;
  }
  uint32_t out[4] = {0, 0, 0, 0};
#pragma unroll
  for (int b = 0; b < 16; ++b) out[b >> 2] |= (t[b] | (t[16 + b] << 4)) << (8 * (b & 3));
  reinterpret_cast<uint4*>(Wp)[i] = make_uint4(out[0], out[1], out[2], out[3]);
}

// ---------------------------------------------------------------------------- group sums
// gsum[m][g] = ((x0 + x1) + x2) + ... + x31 starting from 0 (w4g32_avx2.h:22; XP::prep
// gemma4_engine.cpp:191).  One thread per (m, g).
__global__ void k_gsum(const float* __restrict__ X, int MG, int G, float* __restrict__ gs) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= MG) return;
  const float* x = X + (size_t)(i / G) * G * 32 + (size_t)(i % G) * 32;
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 32; ++k) s = __fadd_rn(s, x[k]);
  gs[i] = s;
}

// ------------------------------------------------------------------------- W4G32 float GEMV
// Each CTA owns ROWS = 8*R weight rows.  Thread 0 streams the rows into shared memory with 1D
// bulk copies (the TMA engine), CH groups per chunk, NB chunk buffers in a ring; every row is
// padded by 16 bytes so the octets' reads fall in different banks.  One octet (8 lanes) works on
// R rows, lane j owning the reference's AVX lane j: per group
//   a = t(2j)x(2j); a = fma(t(16+2j), x(16+2j), a); a = fma(t(2j+1), ...); a = fma(t(17+2j), ...)
//   row = fma(a, scale, row); off = fma(scale, gsum, off)   (the reference build fuses this one)
// and finally y = hsum8(row) - 8*off.  With R = 2 the two rows' chains run as packed f32x2
// operations (each half an IEEE fp32 op, so the results are the same bits).
struct GemvGeom {
  int G, CH, nchunk, NB, rowb;
};
__host__ __device__ inline GemvGeom gemv_geom(int K, int CH, int NB) {
  GemvGeom g;
  g.G = K >> 5;
  g.CH = CH;
  g.nchunk = g.G / CH;
  g.NB = NB < g.nchunk ? NB : g.nchunk;
  g.rowb = CH * 16 + 16;
  return g;
}

// 4 int4 values (nibbles of v, low first) -> exact floats via the 2^23 bias.
__device__ __forceinline__ void nib4_to_f(uint32_t v, float& t0, float& t1, float& t2, float& t3) {
  const uint32_t lo = v & 0x0F0Fu, hi = (v >> 4) & 0x0F0Fu;
  const float2 a = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650)),
                                          __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650))),
                              make_float2(-8388608.0f, -8388608.0f));
  const float2 b = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7651)),
                                          __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7651))),
                              make_float2(-8388608.0f, -8388608.0f));
  t0 = a.x; t1 = a.y; t2 = b.x; t3 = b.y;
}

template <int M, int R, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
k_w4g32(const uint8_t* __restrict__ Wp, const uint16_t* __restrict__ S, const float* __restrict__ X,
        const float* __restrict__ gsum_in, int N, int K, float* __restrict__ Y, int ldy, int CH, int NBmax) {
  constexpr int T = WARPS * 32;
  constexpr int ROWS = WARPS * 4 * R;
  const GemvGeom geo = gemv_geom(K, CH, NBmax);
  const int G = geo.G;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint8_t* wbuf = smem + 128;
  uint16_t* sc = reinterpret_cast<uint16_t*>(wbuf + (size_t)geo.NB * ROWS * geo.rowb);
  float* gs = reinterpret_cast<float*>(sc + (size_t)ROWS * G);
  const int n0 = blockIdx.x * ROWS;
  const int nvalid = min(ROWS, N - n0);

  if (threadIdx.x == 0) {
    for (int b = 0; b < geo.NB; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int c) {
    const int b = c % geo.NB;
    const uint32_t wbytes = (uint32_t)geo.CH * 16;
    mbar_expect_tx(&bars[b], nvalid * wbytes + (c == 0 ? (uint32_t)nvalid * G * 2 : 0u));
    for (int r = 0; r < nvalid; ++r)
      bulk_g2s(wbuf + ((size_t)b * ROWS + r) * geo.rowb, Wp + (size_t)(n0 + r) * (K >> 1) + (size_t)c * wbytes, wbytes,
               &bars[b]);
    if (c == 0) bulk_g2s(sc, S + (size_t)n0 * G, (uint32_t)nvalid * G * 2, &bars[b]);
  };
  if (threadIdx.x == 0)
    for (int c = 0; c < geo.NB; ++c) issue(c);

  pdl_wait();  // the weights above are read-only; activations come from the previous kernel
  pdl_trigger();

  // group sums (given, or ((x0 + x1) + ...) + x31 from 0, w4g32_avx2.h:22) while the copies fly
  if (gsum_in != nullptr) {
    for (int i = threadIdx.x; i < M * G; i += T) gs[i] = gsum_in[i];
  } else {
    for (int i = threadIdx.x; i < M * G; i += T) {
      const float4* x4 = reinterpret_cast<const float4*>(X + (size_t)(i / G) * K + (size_t)(i % G) * 32);
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 v = __ldg(x4 + k);
        s = __fadd_rn(s, v.x); s = __fadd_rn(s, v.y); s = __fadd_rn(s, v.z); s = __fadd_rn(s, v.w);
      }
      gs[i] = s;
    }
  }
  __syncthreads();

  const int oct = threadIdx.x >> 3, j = threadIdx.x & 7;
  float2 row[M], off[M];  // .x = row oct*R, .y = row oct*R+1 (unused when R == 1)
#pragma unroll
  for (int m = 0; m < M; ++m) { row[m] = make_float2(0.f, 0.f); off[m] = make_float2(0.f, 0.f); }
  const int r0 = oct * R;

  for (int c = 0; c < geo.nchunk; ++c) {
    const int b = c % geo.NB;
    if (!cta_wait(&bars[b], (uint32_t)(c / geo.NB) & 1u)) return;
    const uint8_t* wb = wbuf + (size_t)b * ROWS * geo.rowb;
    for (int gl = 0; gl < geo.CH; gl += 8) {
      const int gbase = c * geo.CH + gl;
      uint4 s4[R];
#pragma unroll
      for (int i = 0; i < R; ++i) s4[i] = *reinterpret_cast<const uint4*>(sc + (size_t)(r0 + i) * G + gbase);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int g = gbase + u;
        float t[R][4], scl[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const uint32_t v = *reinterpret_cast<const uint16_t*>(wb + (size_t)(r0 + i) * geo.rowb + (gl + u) * 16 + 2 * j);
          nib4_to_f(v, t[i][0], t[i][1], t[i][2], t[i][3]);
          const uint32_t sw = (u < 2 ? s4[i].x : u < 4 ? s4[i].y : u < 6 ? s4[i].z : s4[i].w);
          scl[i] = bf2f((u & 1) ? (sw >> 16) : (sw & 0xFFFFu));
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float* xg = X + (size_t)m * K + (size_t)g * 32;
          const float2 xa = __ldg(reinterpret_cast<const float2*>(xg + 2 * j));
          const float2 xb = __ldg(reinterpret_cast<const float2*>(xg + 16 + 2 * j));
          const float gsv = gs[m * G + g];
          if constexpr (R == 2) {
            float2 a = __fmul2_rn(make_float2(t[0][0], t[1][0]), make_float2(xa.x, xa.x));
            a = __ffma2_rn(make_float2(t[0][1], t[1][1]), make_float2(xb.x, xb.x), a);
            a = __ffma2_rn(make_float2(t[0][2], t[1][2]), make_float2(xa.y, xa.y), a);
            a = __ffma2_rn(make_float2(t[0][3], t[1][3]), make_float2(xb.y, xb.y), a);
            const float2 s2 = make_float2(scl[0], scl[1]);
            row[m] = __ffma2_rn(a, s2, row[m]);
            off[m] = __ffma2_rn(s2, make_float2(gsv, gsv), off[m]);
          } else {
            float a = __fmul_rn(t[0][0], xa.x);
            a = fmaf(t[0][1], xb.x, a);
            a = fmaf(t[0][2], xa.y, a);
            a = fmaf(t[0][3], xb.y, a);
            row[m].x = fmaf(a, scl[0], row[m].x);
            off[m].x = fmaf(scl[0], gsv, off[m].x);
          }
        }
      }
    }
    if (c + geo.NB < geo.nchunk) {
      __syncthreads();
      if (threadIdx.x == 0) { fence_proxy_async_smem(); issue(c + geo.NB); }
    }
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const float h0 = hsum8_octet(row[m].x);
    if (j == 0 && r0 < nvalid) Y[(size_t)m * ldy + n0 + r0] = __fsub_rn(h0, __fmul_rn(8.f, off[m].x));
    if constexpr (R == 2) {
      const float h1 = hsum8_octet(row[m].y);
      if (j == 0 && r0 + 1 < nvalid) Y[(size_t)m * ldy + n0 + r0 + 1] = __fsub_rn(h1, __fmul_rn(8.f, off[m].y));
    }
  }
}

// W4G32 float GEMV, row-per-thread variant for tall matrices (the head screen: 262,144 rows).
// One thread runs the eight lane chains of its row, so each 16-byte group of weights is decoded
// once for all M activation rows.  The thread reads its row's weights and scales straight from
// global memory through L1 (16-byte loads; a row's 128-byte lines serve 8 consecutive loads of its
// thread), so occupancy is set by registers; a persistent grid takes 256-row tiles in turn.  The
// activations sit in shared memory as [k][4] (one 16-byte broadcast load per element), the group
// sums as [g][4].  Values are those of k_w4g32: per lane j and group, a = t(2j)x(2j);
// a = fma(t(16+2j), x(16+2j), a); a = fma(t(2j+1), ...); a = fma(t(17+2j), ...);
// row_j = fma(a, s, row_j); off = fma(s, gsum, off); y = hsum8(row) - 8 off.
constexpr int kWrThreads = 256;
__host__ __device__ inline size_t w4g32_rows_smem(int K) { return (size_t)K * 16 + (size_t)(K / 32) * 16; }

template <int M>
__global__ void __launch_bounds__(kWrThreads) k_w4g32_rows(const uint8_t* __restrict__ Wp, const uint16_t* __restrict__ S,
                                                            const float* __restrict__ X, int N, int K,
                                                            float* __restrict__ Y, int ldy) {
  extern __shared__ __align__(16) float4 xs[];  // [K], then group sums [G]
  pdl_wait();
  pdl_trigger();
  const int G = K >> 5;
  float4* gs = xs + K;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    float v[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) v[m] = m < M ? X[(size_t)m * K + i] : 0.f;
    xs[i] = make_float4(v[0], v[1], v[2], v[3]);
  }
  for (int g = threadIdx.x; g < G; g += blockDim.x) {  // ((x0 + x1) + ...) + x31 from 0 (w4g32_avx2.h:22)
    float v[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      float sm = 0.f;
      if (m < M)
        for (int k = 0; k < 32; ++k) sm = __fadd_rn(sm, X[(size_t)m * K + g * 32 + k]);
      v[m] = sm;
    }
    gs[g] = make_float4(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n - (int)threadIdx.x < N; n += gridDim.x * blockDim.x) {
    if (n >= N) continue;
    const uint4* wrow = reinterpret_cast<const uint4*>(Wp + (size_t)n * (K >> 1));
    const uint4* srow = reinterpret_cast<const uint4*>(S + (size_t)n * G);
    float2 row[8][2], off[2];
#pragma unroll
    for (int j = 0; j < 8; ++j) row[j][0] = row[j][1] = make_float2(0.f, 0.f);
    off[0] = off[1] = make_float2(0.f, 0.f);
#pragma unroll 1
    for (int g8 = 0; g8 < G; g8 += 8) {
      const uint4 s8 = __ldg(srow + (g8 >> 3));
      const uint32_t s8w[4] = {s8.x, s8.y, s8.z, s8.w};
      uint4 wq[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) wq[u] = __ldg(wrow + g8 + u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int g = g8 + u;
        const uint32_t w4[4] = {wq[u].x, wq[u].y, wq[u].z, wq[u].w};
        const float scl = bf2f((u & 1) ? (s8w[u >> 1] >> 16) : (s8w[u >> 1] & 0xFFFFu));
        const float2 sc2 = make_float2(scl, scl);
        const float4* xg = xs + g * 32;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t v = (w4[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;  // bytes 2j, 2j+1
          float t0, t1, t2, t3;
          nib4_to_f(v, t0, t1, t2, t3);
          const float4 x0 = xg[2 * j], x1 = xg[16 + 2 * j], x2 = xg[2 * j + 1], x3 = xg[17 + 2 * j];
          float2 a0 = __fmul2_rn(make_float2(t0, t0), make_float2(x0.x, x0.y));
          float2 a1 = __fmul2_rn(make_float2(t0, t0), make_float2(x0.z, x0.w));
          a0 = __ffma2_rn(make_float2(t1, t1), make_float2(x1.x, x1.y), a0);
          a1 = __ffma2_rn(make_float2(t1, t1), make_float2(x1.z, x1.w), a1);
          a0 = __ffma2_rn(make_float2(t2, t2), make_float2(x2.x, x2.y), a0);
          a1 = __ffma2_rn(make_float2(t2, t2), make_float2(x2.z, x2.w), a1);
          a0 = __ffma2_rn(make_float2(t3, t3), make_float2(x3.x, x3.y), a0);
          a1 = __ffma2_rn(make_float2(t3, t3), make_float2(x3.z, x3.w), a1);
          row[j][0] = __ffma2_rn(a0, sc2, row[j][0]);
          row[j][1] = __ffma2_rn(a1, sc2, row[j][1]);
        }
        const float4 gv = gs[g];
        off[0] = __ffma2_rn(sc2, make_float2(gv.x, gv.y), off[0]);
        off[1] = __ffma2_rn(sc2, make_float2(gv.z, gv.w), off[1]);
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int p = m >> 1;
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (m & 1) ? row[j][p].y : row[j][p].x;
      const float h = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[4]), __fadd_rn(v[1], v[5])),
                                __fadd_rn(__fadd_rn(v[2], v[6]), __fadd_rn(v[3], v[7])));
      const float o = (m & 1) ? off[p].y : off[p].x;
      Y[(size_t)m * ldy + n] = __fsub_rn(h, __fmul_rn(8.f, o));
    }
  }
}

// W4G32 float GEMV fed by the TMA (the head screen's tall matrix), same values as k_w4g32_rows.
// Two threads share a row: thread half h runs lane chains 4h..4h+3 over every group in order, and
// the two halves meet in the final hsum8 through one shuffle.  A persistent CTA of 256 threads
// takes 128-row blocks (2048 blocks for the 262,144-row screen balance over 2 CTAs per SM to
// within 1%); per pipeline item two 2D tensor-map loads bring 8 groups of all 128 rows into one of
// kTwNS stages: the weights as a [128][128 B] box under the 128-byte swizzle (chunk u of row r
// lands at chunk u ^ (r & 7), so a 16-thread phase of 8-byte loads hits 8 distinct bank quads) and
// the bf16 scales as a [128][16 B] box.  Rows past N read as zeros and are not stored.  The
// activations sit in shared memory as element pairs [k/2][NP] float4 {x_m(2q), x_m+1(2q),
// x_m(2q+1), x_m+1(2q+1)}, which serve a lane's elements 2j, 2j+1 and 16+2j, 17+2j in two loads.
constexpr int kTwRows = 128, kTwThreads = 256, kTwNS = 4;
constexpr int kTwStage = kTwRows * 128 + kTwRows * 16;  // 18 KB, a multiple of the swizzle span
// With two activation-row pairs (M > 2) a float4 of padding follows every 4 element pairs, so that
// the two threads of a row (elements 8h.., 16+8h..) read bank-disjoint 16-byte slots.
__host__ __device__ constexpr int w4g32_xpad(int NP, int q) { return NP == 2 ? (q >> 2) : 0; }
__host__ __device__ inline size_t w4g32_tma_smem(int M, int K) {
  const int NP = (M + 1) / 2;
  return 1024 + (size_t)kTwNS * kTwStage + ((size_t)(K / 2) * NP + w4g32_xpad(NP, K / 2)) * 16 + (size_t)(K / 32) * NP * 8;
}

template <int M>
__global__ void __launch_bounds__(kTwThreads, 2)
k_w4g32_rows_tma(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ts,
                 const float* __restrict__ X, int N, int K, float* __restrict__ Y, int ldy, const int* __restrict__ skip) {
  constexpr int NP = (M + 1) / 2;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kTwNS];
  uint8_t* stages = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // 1024-byte aligned
  float4* xs = reinterpret_cast<float4*>(stages + (size_t)kTwNS * kTwStage);       // [K/2][NP]
  float2* gs = reinterpret_cast<float2*>(xs + (size_t)(K / 2) * NP + w4g32_xpad(NP, K / 2));  // [G][NP]
  pdl_wait();
  pdl_trigger();
  if (skip != nullptr && *skip != 0) return;  // before any copy is issued
  const int G = K >> 5, nch = G >> 3;
  const int nblk = (N + kTwRows - 1) / kTwRows;
  const int myblk = nblk > (int)blockIdx.x ? (nblk - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int nitems = myblk * nch;
  const int t = threadIdx.x, rl = t >> 1, half = t & 1;
  if (t == 0) {
    for (int b = 0; b < kTwNS; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i, int st) {  // thread 0
    const int blk = blockIdx.x + (i / nch) * gridDim.x, c = i % nch;
    uint8_t* sb = stages + (size_t)st * kTwStage;
    mbar_expect_tx(&bars[st], (uint32_t)kTwStage);
    tma_load_2d(sb, &tw, c * 128, blk * kTwRows, &bars[st]);
    tma_load_2d(sb + kTwRows * 128, &ts, c * 8, blk * kTwRows, &bars[st]);
  };
  if (t == 0)
    for (int b = 0; b < kTwNS && b < nitems; ++b) issue(b, b);
  for (int q = t; q < K / 2; q += kTwThreads) {
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int m0 = 2 * p, m1 = 2 * p + 1;
      const float a0 = X[(size_t)m0 * K + 2 * q], b0 = X[(size_t)m0 * K + 2 * q + 1];
      const float a1 = m1 < M ? X[(size_t)m1 * K + 2 * q] : 0.f, b1 = m1 < M ? X[(size_t)m1 * K + 2 * q + 1] : 0.f;
      xs[(size_t)q * NP + p + w4g32_xpad(NP, q)] = make_float4(a0, a1, b0, b1);
    }
  }
  for (int g = t; g < G; g += kTwThreads) {  // ((x0 + x1) + ...) + x31 from 0 (w4g32_avx2.h:22)
    float v[2 * NP];
#pragma unroll
    for (int m = 0; m < 2 * NP; ++m) {
      float sm = 0.f;
      if (m < M)
        for (int k = 0; k < 32; ++k) sm = __fadd_rn(sm, X[(size_t)m * K + g * 32 + k]);
      v[m] = sm;
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) gs[(size_t)g * NP + p] = make_float2(v[2 * p], v[2 * p + 1]);
  }
  __syncthreads();
  float2 row[4][NP], off[NP];
  for (int i = 0; i < nitems; ++i) {
    const int st = i % kTwNS;
    const int blk = blockIdx.x + (i / nch) * gridDim.x, c = i % nch;
    const int n = blk * kTwRows + rl;
    if (!cta_wait(&bars[st], (uint32_t)(i / kTwNS) & 1u)) return;
    if (c == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int p = 0; p < NP; ++p) row[j][p] = make_float2(0.f, 0.f);
#pragma unroll
      for (int p = 0; p < NP; ++p) off[p] = make_float2(0.f, 0.f);
    }
    const uint8_t* sb = stages + (size_t)st * kTwStage;
    uint2 wq[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      wq[u] = *reinterpret_cast<const uint2*>(sb + rl * 128 + ((u ^ (rl & 7)) << 4) + half * 8);
    const uint4 s8 = *reinterpret_cast<const uint4*>(sb + kTwRows * 128 + rl * 16);
    __syncthreads();  // every thread has its words in registers: the stage can be refilled
    if (t == 0 && i + kTwNS < nitems) {
      fence_proxy_async_smem();
      issue(i + kTwNS, st);
    }
    const uint32_t s8w[4] = {s8.x, s8.y, s8.z, s8.w};
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int g = c * 8 + u;
      const float scl = bf2f((u & 1) ? (s8w[u >> 1] >> 16) : (s8w[u >> 1] & 0xFFFFu));
      const float2 sc2 = make_float2(scl, scl);
      const float4* xg = xs + (size_t)g * 16 * NP + w4g32_xpad(NP, g * 16);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = 4 * half + jj;  // lane chain: bytes 2j, 2j+1 of the group
        const uint32_t v = ((jj < 2 ? wq[u].x : wq[u].y) >> (16 * (jj & 1))) & 0xFFFFu;
        float t0, t1, t2, t3;
        nib4_to_f(v, t0, t1, t2, t3);
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const float4 A = xg[j * NP + p + w4g32_xpad(NP, j)], B = xg[(8 + j) * NP + p + w4g32_xpad(NP, 8 + j)];
          float2 a = __fmul2_rn(make_float2(t0, t0), make_float2(A.x, A.y));
          a = __ffma2_rn(make_float2(t1, t1), make_float2(B.x, B.y), a);
          a = __ffma2_rn(make_float2(t2, t2), make_float2(A.z, A.w), a);
          a = __ffma2_rn(make_float2(t3, t3), make_float2(B.z, B.w), a);
          row[jj][p] = __ffma2_rn(a, sc2, row[jj][p]);
        }
      }
#pragma unroll
      for (int p = 0; p < NP; ++p) off[p] = __ffma2_rn(sc2, gs[(size_t)g * NP + p], off[p]);
    }
    if (c == nch - 1) {
      // lanes 4..7 of the row come from the other half; fadd is commutative, so both halves get
      // ((v0 + v4) + (v1 + v5)) + ((v2 + v6) + (v3 + v7)) bit for bit
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        float2 w[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          w[jj].x = __shfl_xor_sync(0xffffffffu, row[jj][p].x, 1);
          w[jj].y = __shfl_xor_sync(0xffffffffu, row[jj][p].y, 1);
        }
        const float hx = __fadd_rn(__fadd_rn(__fadd_rn(row[0][p].x, w[0].x), __fadd_rn(row[1][p].x, w[1].x)),
                                   __fadd_rn(__fadd_rn(row[2][p].x, w[2].x), __fadd_rn(row[3][p].x, w[3].x)));
        const float hy = __fadd_rn(__fadd_rn(__fadd_rn(row[0][p].y, w[0].y), __fadd_rn(row[1][p].y, w[1].y)),
                                   __fadd_rn(__fadd_rn(row[2][p].y, w[2].y), __fadd_rn(row[3][p].y, w[3].y)));
        if (n < N) {
          if (half == 0) Y[(size_t)(2 * p) * ldy + n] = __fsub_rn(hx, __fmul_rn(8.f, off[p].x));
          else if (2 * p + 1 < M) Y[(size_t)(2 * p + 1) * ldy + n] = __fsub_rn(hy, __fmul_rn(8.f, off[p].y));
        }
      }
    }
  }
}

// ------------------------------------------------------------------------ W4A8 quantisation
// One warp per (row, 32-group), lane i owning element i: amax, sx = amax/127, inv = sx>0 ? 1/sx
// : 0, r = RNE(x*inv) (x86 cvtps_epi32 semantics: out of range or NaN -> INT32_MIN), sum of the
// unsaturated r, q = r saturated to int16 then int8 (w4a8_avx2.h:30-42).
__global__ void k_w4a8_quant(const float* __restrict__ X, int MG, int G, int8_t* __restrict__ q,
                             float* __restrict__ sx, int32_t* __restrict__ sum) {
  pdl_wait();
  pdl_trigger();
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= MG) return;
  const size_t base = (size_t)wid * 32;  // [m][K] with K = 32G: group wid starts at 32*wid
  int8_t qv;
  float s;
  int32_t tot;
  quant_group32(X[base + lane], qv, s, tot);
  q[base + lane] = qv;
  if (lane == 0) { sx[wid] = s; sum[wid] = tot; }
  (void)G;
}

// ------------------------------------------------------------------------------ W4A8 GEMV
// Each CTA owns 8 weight rows streamed into shared memory as in k_w4g32.  Per chunk, phase 1
// has each thread take one group for all 8 rows (its int8 activations, scale and sum are loaded
// once and reused across the rows): the integer-exact group dot a32 = sum t*xq - 8*sum (eight
// dp4a per activation row) and the scale sw*sx go to shared memory.  Phase 2 runs the fp32
// chain row = fma(float(a32), sw*sx, row) over the groups in order (w4a8_avx2.h:57-58).
constexpr int kW4A8Rows = 8;

template <int M, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
k_w4a8(const uint8_t* __restrict__ Wp, const uint16_t* __restrict__ S, const int8_t* __restrict__ q,
       const float* __restrict__ sx, const int32_t* __restrict__ sum, int N, int K, float* __restrict__ Y, int ldy,
       int CH, int NBmax) {
  constexpr int T = WARPS * 32;
  constexpr int ROWS = kW4A8Rows;
  const GemvGeom geo = gemv_geom(K, CH, NBmax);
  const int G = geo.G;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint8_t* wbuf = smem + 128;
  uint16_t* sc = reinterpret_cast<uint16_t*>(wbuf + (size_t)geo.NB * ROWS * geo.rowb);
  float2* ac = reinterpret_cast<float2*>(sc + (size_t)ROWS * G);  // [ROWS*M][CH+1]
  const int n0 = blockIdx.x * ROWS;
  const int nvalid = min(ROWS, N - n0);
  const int acs = geo.CH + 1;

  if (threadIdx.x == 0) {
    for (int b = 0; b < geo.NB; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int c) {
    const int b = c % geo.NB;
    const uint32_t wbytes = (uint32_t)geo.CH * 16;
    mbar_expect_tx(&bars[b], nvalid * wbytes + (c == 0 ? (uint32_t)nvalid * G * 2 : 0u));
    for (int r = 0; r < nvalid; ++r)
      bulk_g2s(wbuf + ((size_t)b * ROWS + r) * geo.rowb, Wp + (size_t)(n0 + r) * (K >> 1) + (size_t)c * wbytes, wbytes,
               &bars[b]);
    if (c == 0) bulk_g2s(sc, S + (size_t)n0 * G, (uint32_t)nvalid * G * 2, &bars[b]);
  };
  if (threadIdx.x == 0)
    for (int c = 0; c < geo.NB; ++c) issue(c);

  pdl_wait();  // the weights above are read-only; activations come from the previous kernel
  pdl_trigger();

  // chain slots: thread t owns (row, activation row) pairs t, t+T, ... of the ROWS*M chains
  constexpr int CPT = (ROWS * M + T - 1) / T;
  float row[CPT];
#pragma unroll
  for (int k = 0; k < CPT; ++k) row[k] = 0.f;
  for (int c = 0; c < geo.nchunk; ++c) {
    const int b = c % geo.NB;
    if (!cta_wait(&bars[b], (uint32_t)(c / geo.NB) & 1u)) return;
    const uint8_t* wb = wbuf + (size_t)b * ROWS * geo.rowb;
    for (int gl = threadIdx.x; gl < geo.CH; gl += T) {
      const int g = c * geo.CH + gl;
      int4 qa[M], qb[M];
      int bias[M];
      float sxm[M];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const int4* qp = reinterpret_cast<const int4*>(q + (size_t)m * K + (size_t)g * 32);
        qa[m] = __ldg(qp);
        qb[m] = __ldg(qp + 1);
        bias[m] = -8 * __ldg(sum + (size_t)m * G + g);
        sxm[m] = __ldg(sx + (size_t)m * G + g);
      }
#pragma unroll 2
      for (int r = 0; r < ROWS; ++r) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wb + (size_t)r * geo.rowb + gl * 16);
        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) { lo[k] = w4[k] & 0x0F0F0F0Fu; hi[k] = (w4[k] >> 4) & 0x0F0F0F0Fu; }
        const float sw = bf2f(sc[(size_t)r * G + g]);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          int acc = bias[m];
          acc = __dp4a((int)lo[0], qa[m].x, acc);
          acc = __dp4a((int)lo[1], qa[m].y, acc);
          acc = __dp4a((int)lo[2], qa[m].z, acc);
          acc = __dp4a((int)lo[3], qa[m].w, acc);
          acc = __dp4a((int)hi[0], qb[m].x, acc);
          acc = __dp4a((int)hi[1], qb[m].y, acc);
          acc = __dp4a((int)hi[2], qb[m].z, acc);
          acc = __dp4a((int)hi[3], qb[m].w, acc);
          ac[(size_t)(r * M + m) * acs + gl] = make_float2((float)acc, __fmul_rn(sw, sxm[m]));
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
      const int ci = threadIdx.x + k * T;  // = r*M + m
      if (ci < ROWS * M) {
        const float2* a = ac + (size_t)ci * acs;
#pragma unroll 8
        for (int gl = 0; gl < geo.CH; ++gl) {
          const float2 v = a[gl];
          row[k] = fmaf(v.x, v.y, row[k]);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && c + geo.NB < geo.nchunk) { fence_proxy_async_smem(); issue(c + geo.NB); }
  }
#pragma unroll
  for (int k = 0; k < CPT; ++k) {
    const int ci = threadIdx.x + k * T, cr = ci / M, cm = ci % M;
    if (ci < ROWS * M && cr < nvalid) Y[(size_t)cm * ldy + n0 + cr] = row[k];
  }
}

// W4A8 GEMV, whole-block variant: a CTA requests all of its ROWS weight rows (every chunk, one
// mbarrier per chunk) and their scales at once, so that the whole matrix is in flight across the
// grid; phase 1 turns each chunk into (a32, sw*sx) pairs as it lands, kept for every group of the
// row in shared memory; phase 2 runs the ROWS*M fp32 chains over all groups in order.  The values
// are those of k_w4a8 (same integer dot, same product, same chain order).
template <int M, int ROWS, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
k_w4a8_all(const uint8_t* __restrict__ Wp, const uint16_t* __restrict__ S, const int8_t* __restrict__ q,
           const float* __restrict__ sx, const int32_t* __restrict__ sum, int N, int K, float* __restrict__ Y, int ldy,
           int CH) {
  constexpr int T = WARPS * 32;
  const int G = K >> 5, nchunk = G / CH;
  const int wrs = K >> 1;  // the CTA's rows sit as in memory (phase 1 reads one row at a time)
  const int acs = G + 1;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint8_t* wbuf = smem + 128;
  uint16_t* sc = reinterpret_cast<uint16_t*>(wbuf + (size_t)ROWS * wrs);
  float2* ac = reinterpret_cast<float2*>(sc + (size_t)ROWS * G);  // [ROWS*M][G+1]
  const int n0 = blockIdx.x * ROWS;
  const int nvalid = min(ROWS, N - n0);

  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    fence_mbar_init();
    // the CTA's rows and their scales are contiguous in memory: two bulk copies (one per row
    // costs issue time)
    const uint32_t wbytes = (uint32_t)nvalid * (uint32_t)(K >> 1), sbytes = (uint32_t)nvalid * G * 2;
    mbar_expect_tx(&bars[0], wbytes + sbytes);
    bulk_g2s(wbuf, Wp + (size_t)n0 * (K >> 1), wbytes, &bars[0]);
    bulk_g2s(sc, S + (size_t)n0 * G, sbytes, &bars[0]);
  }
  __syncthreads();  // the barrier is initialised before anyone polls it
  pdl_wait();  // the weights above are read-only; activations come from the previous kernel
  pdl_trigger();
  // phase 1: item (group gl of a chunk, row subset rs); with T > CH the rows of a group are split
  // over T / CH threads.  Each thread's activations for its first item are loaded before the
  // wait, so their latency overlaps the weights' arrival.
  const int RS = T > CH ? min(T / CH, ROWS) : 1;
  int4 qa[M], qb[M];
  int bias[M];
  float sxm[M];
  auto load_act = [&](int g) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int4* qp = reinterpret_cast<const int4*>(q + (size_t)m * K + (size_t)g * 32);
      qa[m] = __ldg(qp);
      qb[m] = __ldg(qp + 1);
      bias[m] = -8 * __ldg(sum + (size_t)m * G + g);
      sxm[m] = __ldg(sx + (size_t)m * G + g);
    }
  };
  if ((int)threadIdx.x < CH * RS) load_act(threadIdx.x % CH);
  for (int c = 0; c < nchunk; ++c) {
    if (c == 0 && !cta_wait(&bars[0], 0)) return;
    for (int idx = threadIdx.x; idx < CH * RS; idx += T) {
      const int gl = idx % CH, rs = idx / CH;
      const int g = c * CH + gl;
      if (c > 0 || idx >= T) load_act(g);
#pragma unroll 2
      for (int r = rs; r < ROWS; r += RS) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wbuf + (size_t)r * wrs + (size_t)g * 16);
        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) { lo[k] = w4[k] & 0x0F0F0F0Fu; hi[k] = (w4[k] >> 4) & 0x0F0F0F0Fu; }
        const float sw = bf2f(sc[(size_t)r * G + g]);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          int acc = bias[m];
          acc = __dp4a((int)lo[0], qa[m].x, acc);
          acc = __dp4a((int)lo[1], qa[m].y, acc);
          acc = __dp4a((int)lo[2], qa[m].z, acc);
          acc = __dp4a((int)lo[3], qa[m].w, acc);
          acc = __dp4a((int)hi[0], qb[m].x, acc);
          acc = __dp4a((int)hi[1], qb[m].y, acc);
          acc = __dp4a((int)hi[2], qb[m].z, acc);
          acc = __dp4a((int)hi[3], qb[m].w, acc);
          ac[(size_t)(r * M + m) * acs + g] = make_float2((float)acc, __fmul_rn(sw, sxm[m]));
        }
      }
    }
  }
  __syncthreads();
  const int ci = threadIdx.x;  // chain (row, activation row) = (ci / M, ci % M); T >= ROWS*M
  if (ci < ROWS * M) {
    const int cr = ci / M, cm = ci % M;
    const float2* a = ac + (size_t)ci * acs;
    float row = 0.f;
#pragma unroll 8
    for (int g = 0; g < G; ++g) {
      const float2 v = a[g];
      row = fmaf(v.x, v.y, row);
    }
    if (cr < nvalid) Y[(size_t)cm * ldy + n0 + cr] = row;
  }
}

// W4A8 GEMV, persistent ring variant: a grid of at most a few CTAs per SM, each taking blocks of
// ROWS weight rows in turn.  The activations (int8 rows, scales, sums) are staged in shared memory
// once per CTA; each block's rows and scales arrive by bulk copies into one of NS stages, issued
// NS blocks ahead, so the weight stream never waits for the arithmetic.  Per block, phase 1 gives
// every (group, row subset) to a thread (integer dots for all M activation rows) and phase 2 runs
// the ROWS*M fp32 chains in group order: the values of k_w4a8.
template <int M, int ROWS, int WARPS, int NS>
__global__ void __launch_bounds__(WARPS * 32)
k_w4a8_ring(const uint8_t* __restrict__ Wp, const uint16_t* __restrict__ S, const int8_t* __restrict__ q,
            const float* __restrict__ sx, const int32_t* __restrict__ sum, int N, int K, float* __restrict__ Y, int ldy) {
  constexpr int T = WARPS * 32;
  const int G = K >> 5;
  const int wrs = (K >> 1) + 16;
  const size_t wbytes = (size_t)ROWS * wrs, sbytes = ((size_t)ROWS * G * 2 + 15) / 16 * 16;
  const size_t stage_bytes = wbytes + sbytes;
  const int acs = G + 1;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint8_t* stages = smem + 128;
  int8_t* qs = reinterpret_cast<int8_t*>(stages + NS * stage_bytes);           // [M][K]
  float* sxs = reinterpret_cast<float*>(qs + (size_t)M * K);                     // [M][G]
  int32_t* sums = reinterpret_cast<int32_t*>(sxs + (size_t)M * G);               // [M][G]
  float2* ac = reinterpret_cast<float2*>(sums + (size_t)M * G);                  // [ROWS*M][G+1]
  const int nblk = (N + ROWS - 1) / ROWS;

  if (threadIdx.x == 0) {
    for (int b = 0; b < NS; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int blk, int st) {  // warp 0
    const int lane = threadIdx.x & 31;
    const int n0 = blk * ROWS, nvalid = min(ROWS, N - n0);
    uint8_t* wb = stages + (size_t)st * stage_bytes;
    if (lane == 0) mbar_expect_tx(&bars[st], (uint32_t)nvalid * (uint32_t)(K >> 1) + (uint32_t)nvalid * G * 2);
    __syncwarp();
    for (int r = lane; r < nvalid; r += 32)
      bulk_g2s(wb + (size_t)r * wrs, Wp + (size_t)(n0 + r) * (K >> 1), (uint32_t)(K >> 1), &bars[st]);
    if (lane == 0) bulk_g2s(wb + wbytes, S + (size_t)n0 * G, (uint32_t)nvalid * G * 2, &bars[st]);
  };
  if (threadIdx.x < 32)
    for (int b = 0; b < NS; ++b)
      if ((int)(blockIdx.x + b * gridDim.x) < nblk) issue(blockIdx.x + b * gridDim.x, b);
  pdl_wait();  // the weights above are read-only; activations come from the previous kernel
  pdl_trigger();
  // activations into shared memory (16-byte pieces; K % 256 == 0)
  for (int i = threadIdx.x; i < M * K / 16; i += T) reinterpret_cast<int4*>(qs)[i] = __ldg(reinterpret_cast<const int4*>(q) + i);
  for (int i = threadIdx.x; i < M * G; i += T) { sxs[i] = __ldg(sx + i); sums[i] = __ldg(sum + i); }
  __syncthreads();
  constexpr int RS_MAX = T;  // row subsets when T > G
  const int RS = T > G ? min(T / G, ROWS) : 1;
  (void)RS_MAX;
  int it = 0;
  for (int blk = blockIdx.x; blk < nblk; blk += gridDim.x, ++it) {
    const int st = it % NS;
    if (!cta_wait(&bars[st], (uint32_t)(it / NS) & 1u)) return;
    const uint8_t* wb = stages + (size_t)st * stage_bytes;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(wb + wbytes);
    const int n0 = blk * ROWS, nvalid = min(ROWS, N - n0);
    for (int idx = threadIdx.x; idx < G * RS; idx += T) {
      const int g = idx % G, rs = idx / G;
      int4 qa[M], qb[M];
      int bias[M];
      float sxm[M];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const int4* qp = reinterpret_cast<const int4*>(qs + (size_t)m * K + (size_t)g * 32);
        qa[m] = qp[0];
        qb[m] = qp[1];
        bias[m] = -8 * sums[m * G + g];
        sxm[m] = sxs[m * G + g];
      }
      for (int r = rs; r < ROWS; r += RS) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wb + (size_t)r * wrs + (size_t)g * 16);
        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) { lo[k] = w4[k] & 0x0F0F0F0Fu; hi[k] = (w4[k] >> 4) & 0x0F0F0F0Fu; }
        const float sw = bf2f(sc[(size_t)r * G + g]);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          int acc = bias[m];
          acc = __dp4a((int)lo[0], qa[m].x, acc);
          acc = __dp4a((int)lo[1], qa[m].y, acc);
          acc = __dp4a((int)lo[2], qa[m].z, acc);
          acc = __dp4a((int)lo[3], qa[m].w, acc);
          acc = __dp4a((int)hi[0], qb[m].x, acc);
          acc = __dp4a((int)hi[1], qb[m].y, acc);
          acc = __dp4a((int)hi[2], qb[m].z, acc);
          acc = __dp4a((int)hi[3], qb[m].w, acc);
          ac[(size_t)(r * M + m) * acs + g] = make_float2((float)acc, __fmul_rn(sw, sxm[m]));
        }
      }
    }
    __syncthreads();
    const int ci = threadIdx.x;
    if (ci < ROWS * M) {
      const int cr = ci / M, cm = ci % M;
      const float2* a = ac + (size_t)ci * acs;
      float row = 0.f;
#pragma unroll 8
      for (int g = 0; g < G; ++g) {
        const float2 v = a[g];
        row = fmaf(v.x, v.y, row);
      }
      if (cr < nvalid) Y[(size_t)cm * ldy + n0 + cr] = row;
    }
    __syncthreads();  // stage st and ac are free again
    if (threadIdx.x < 32 && blk + NS * (int)gridDim.x < nblk) {
      fence_proxy_async_smem();
      issue(blk + NS * gridDim.x, st);
    }
  }
}

}  // namespace g4

G4_STATUS_READER(linear)

using namespace g4;

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

extern "C" int g4_w4_pack(const uint8_t* W, int N, int K, uint8_t* Wp, void* stream) {
  G4_REQUIRE(W && Wp && N > 0 && K > 0 && K % 32 == 0, "g4_w4_pack: bad arguments N=%d K=%d", N, K);
  G4_REQUIRE(aligned(W, 16) && aligned(Wp, 16), "g4_w4_pack: W and Wp must be 16-byte aligned");
  const long long groups = (long long)N * (K / 32);
  k_w4_pack<<<(unsigned)((groups + 255) / 256), 256, 0, as_stream(stream)>>>(W, groups, Wp);
  return check_launch("k_w4_pack");
}

extern "C" int g4_w4g32_gsum(const float* X, int M, int K, float* gsum, void* stream) {
  G4_REQUIRE(X && gsum && M > 0 && K > 0 && K % 32 == 0, "g4_w4g32_gsum: bad arguments M=%d K=%d", M, K);
  const int MG = M * (K / 32);
  k_gsum<<<(MG + 255) / 256, 256, 0, as_stream(stream)>>>(X, MG, K / 32, gsum);
  return check_launch("k_gsum");
}

// Launch geometry: CH groups per chunk (64, or the largest of 32/16/8 dividing G), up to NB
// chunk buffers in flight.  Rows per CTA: 16 (R = 2 packed rows per octet) when that still gives
// at least two CTAs per SM, else 8.  G4_GEMV_CFG="R,WARPS,CH,NB" overrides this (tuning knob).
static int pick_ch(int G) { return G % 64 == 0 ? 64 : G % 32 == 0 ? 32 : G % 16 == 0 ? 16 : 8; }

struct GemvCfg { int R, WARPS, CH, NB; };
static GemvCfg gemv_cfg(int N, int G) {
  GemvCfg c{2, 2, pick_ch(G), 3};
  if ((N + 15) / 16 < 296) c.R = 1;
  if (const char* e = getenv("G4_GEMV_CFG")) sscanf(e, "%d,%d,%d,%d", &c.R, &c.WARPS, &c.CH, &c.NB);
  return c;
}
static size_t w4g32_smem(int M, int rows, const GemvGeom& g) {
  return 128 + (size_t)g.NB * rows * g.rowb + (size_t)rows * g.G * 2 + (size_t)M * g.G * 4;
}

template <int M, int R, int WARPS>
static int launch_w4g32_t(const uint8_t* Wp, const uint16_t* S, const float* X, const float* gsum, int N, int K,
                          float* Y, int ldy, int CH, int NB, cudaStream_t st) {
  constexpr int ROWS = WARPS * 4 * R;
  const GemvGeom g = gemv_geom(K, CH, NB);
  const size_t smem = w4g32_smem(M, ROWS, g);
  if (smem > 227 * 1024) return set_error(G4_ERR_UNSUPPORTED, "g4_w4g32_gemm: %zu B of shared memory", smem);
  if (smem > 40 * 1024) cudaFuncSetAttribute(k_w4g32<M, R, WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (int rc_ = launch("k_w4g32", k_w4g32<M, R, WARPS>, dim3((N + ROWS - 1) / ROWS), dim3(WARPS * 32), smem, st, Wp, S, X, gsum, N, K, Y, ldy, CH, NB)) return rc_;
  return check_launch("k_w4g32");
}

// Tensor maps of a packed W4G32 matrix for k_w4g32_rows_tma: the weights as bytes [N][K/2] in
// [128][128 B] boxes under the 128-byte swizzle, the bf16 scales as [N][K/32] in [128][8] boxes.
// Cached per (weights, scales, N, K).
static bool w4g32_tmaps(const uint8_t* Wp, const uint16_t* S, int N, int K, CUtensorMap* tw, CUtensorMap* ts) {
  static std::mutex mu;
  struct Entry { const void* w; const void* s; int N, K; CUtensorMap mw, ms; };
  static Entry cache[8];
  static int used = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].w == Wp && cache[i].s == S && cache[i].N == N && cache[i].K == K) {
      *tw = cache[i].mw;
      *ts = cache[i].ms;
      return true;
    }
  const uint64_t G = (uint64_t)K / 32;
  CUtensorMap mw, ms;
  if (!encode_tmap_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wp, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2, 128,
                      kTwRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT16, S, G, (uint64_t)N, G * 2, 8, kTwRows,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
    return false;
  if (used < 8) cache[used++] = Entry{Wp, S, N, K, mw, ms};
  *tw = mw;
  *ts = ms;
  return true;
}

template <int M>
static int launch_w4g32(const uint8_t* Wp, const uint16_t* S, const float* X, const float* gsum, int N, int K,
                        float* Y, int ldy, cudaStream_t st) {
  const GemvCfg c = gemv_cfg(N, K / 32);
  if (c.R == 2 && c.WARPS == 2) return launch_w4g32_t<M, 2, 2>(Wp, S, X, gsum, N, K, Y, ldy, c.CH, c.NB, st);
  if (c.R == 2 && c.WARPS == 4) return launch_w4g32_t<M, 2, 4>(Wp, S, X, gsum, N, K, Y, ldy, c.CH, c.NB, st);
  if (c.R == 1 && c.WARPS == 4) return launch_w4g32_t<M, 1, 4>(Wp, S, X, gsum, N, K, Y, ldy, c.CH, c.NB, st);
  return launch_w4g32_t<M, 1, 2>(Wp, S, X, gsum, N, K, Y, ldy, c.CH, c.NB, st);
}

static int w4g32_gemm_impl(const uint8_t* Wp, const uint16_t* S, const float* X, const float* gsum, int M, int N,
                           int K, float* Y, int ldy, void* stream, const int* skip) {
  G4_REQUIRE(Wp && S && X && Y, "g4_w4g32_gemm: null pointer");
  G4_REQUIRE(M >= 1 && M <= 8 && N > 0 && K > 0 && K % 256 == 0 && ldy >= N,
             "g4_w4g32_gemm: unsupported shape M=%d N=%d K=%d ldy=%d (K must be a multiple of 256)", M, N, K, ldy);
  G4_REQUIRE(aligned(Wp, 16) && aligned(S, 16) && aligned(X, 16) && (gsum == nullptr || aligned(gsum, 4)),
             "g4_w4g32_gemm: Wp, S and X must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  // tall matrices (the head screen): the TMA-fed variant, else the row-per-thread one
  const char* rv = getenv("G4_W4G32_ROWS");  // "0" / "direct" select other variants (experiments)
  CUtensorMap tw, ts;
  const size_t tsmem = w4g32_tma_smem(M, K);
  if (M <= 4 && gsum == nullptr && N >= 16384 && !rv && tsmem <= 113 * 1024 && w4g32_tmaps(Wp, S, N, K, &tw, &ts)) {
    auto go = [&](auto kern) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsmem);
      cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);  // 2 CTAs per SM
      int occ = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kTwThreads, tsmem) != cudaSuccess || occ < 1) occ = 1;
      const int grid = std::min((N + kTwRows - 1) / kTwRows, sm_count() * occ);
      if (int rc_ = launch("k_w4g32_rows_tma", kern, dim3(grid), dim3(kTwThreads), tsmem, st, tw, ts, X, N, K, Y, ldy, skip))
        return rc_;
      return check_launch("k_w4g32_rows_tma");
    };
    switch (M) {
      case 1: return go(k_w4g32_rows_tma<1>);
      case 2: return go(k_w4g32_rows_tma<2>);
      case 3: return go(k_w4g32_rows_tma<3>);
      default: return go(k_w4g32_rows_tma<4>);
    }
  }
  if (M <= 4 && gsum == nullptr && N >= 16384 && w4g32_rows_smem(K) <= 100 * 1024 && !(rv && rv[0] == '0')) {
    const size_t smem = w4g32_rows_smem(K);
    auto go = [&](auto kern) {
      if (smem > 40 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      int occ = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kWrThreads, smem) != cudaSuccess || occ < 1) occ = 1;
      const int grid = std::min((N + kWrThreads - 1) / kWrThreads, sm_count() * occ);
      if (int rc_ = launch("k_w4g32_rows", kern, dim3(grid), dim3(kWrThreads), smem, st, Wp, S, X, N, K, Y, ldy)) return rc_;
      return check_launch("k_w4g32_rows");
    };
    switch (M) {
      case 1: return go(k_w4g32_rows<1>);
      case 2: return go(k_w4g32_rows<2>);
      case 3: return go(k_w4g32_rows<3>);
      default: return go(k_w4g32_rows<4>);
    }
  }
  switch (M) {
    case 1: return launch_w4g32<1>(Wp, S, X, gsum, N, K, Y, ldy, st);
    case 2: return launch_w4g32<2>(Wp, S, X, gsum, N, K, Y, ldy, st);
    case 3: return launch_w4g32<3>(Wp, S, X, gsum, N, K, Y, ldy, st);
    case 4: return launch_w4g32<4>(Wp, S, X, gsum, N, K, Y, ldy, st);
    case 5: return launch_w4g32<5>(Wp, S, X, gsum, N, K, Y, ldy, st);
    case 6: return launch_w4g32<6>(Wp, S, X, gsum, N, K, Y, ldy, st);
    case 7: return launch_w4g32<7>(Wp, S, X, gsum, N, K, Y, ldy, st);
    default: return launch_w4g32<8>(Wp, S, X, gsum, N, K, Y, ldy, st);
  }
}

extern "C" int g4_w4g32_gemm(const uint8_t* Wp, const uint16_t* S, const float* X, const float* gsum, int M, int N,
                             int K, float* Y, int ldy, void* stream) {
  return w4g32_gemm_impl(Wp, S, X, gsum, M, N, K, Y, ldy, stream, nullptr);
}

int g4::w4g32_gemm_gated(const uint8_t* Wp, const uint16_t* S, const float* X, int M, int N, int K, float* Y, int ldy,
                         const int* skip, cudaStream_t st) {
  return w4g32_gemm_impl(Wp, S, X, nullptr, M, N, K, Y, ldy, st, skip);
}

extern "C" int g4_w4a8_quant(const float* X, int M, int K, int8_t* q, float* sx, int32_t* sum, void* stream) {
  G4_REQUIRE(X && q && sx && sum && M > 0 && K > 0 && K % 32 == 0, "g4_w4a8_quant: bad arguments M=%d K=%d", M, K);
  const int MG = M * (K / 32);
  const int threads = 256, per_block = threads / 32;
  if (int rc_ = launch("k_w4a8_quant", k_w4a8_quant, dim3((MG + per_block - 1) / per_block), dim3(threads), 0, as_stream(stream), X, MG, K / 32, q, sx, sum)) return rc_;
  return check_launch("k_w4a8_quant");
}

static size_t w4a8_smem(int M, const GemvGeom& g) {
  return 128 + (size_t)g.NB * kW4A8Rows * g.rowb + (size_t)kW4A8Rows * g.G * 2 + (size_t)kW4A8Rows * M * (g.CH + 1) * 8;
}

template <int M, int WARPS>
static int launch_w4a8_t(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx, const int32_t* sum,
                         int N, int K, float* Y, int ldy, int CH, int NB, cudaStream_t st) {
  const GemvGeom g = gemv_geom(K, CH, NB);
  const size_t smem = w4a8_smem(M, g);
  if (smem > 227 * 1024) return set_error(G4_ERR_UNSUPPORTED, "g4_w4a8_gemm: %zu B of shared memory", smem);
  if (smem > 40 * 1024) cudaFuncSetAttribute(k_w4a8<M, WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (int rc_ = launch("k_w4a8", k_w4a8<M, WARPS>, dim3((N + kW4A8Rows - 1) / kW4A8Rows), dim3(WARPS * 32), smem, st, Wp, S, q, sx, sum, N, K, Y, ldy, CH, NB)) return rc_;
  return check_launch("k_w4a8");
}

static size_t w4a8_all_smem(int M, int rows, int K) {
  const int G = K / 32;
  return 128 + (size_t)rows * (K / 2) + (size_t)rows * G * 2 + (size_t)rows * M * (G + 1) * 8;
}

template <int M, int ROWS, int WARPS>
static int launch_w4a8_all_t(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx, const int32_t* sum,
                             int N, int K, float* Y, int ldy, int CH, cudaStream_t st) {
  const size_t smem = w4a8_all_smem(M, ROWS, K);
  if (smem > 40 * 1024) cudaFuncSetAttribute(k_w4a8_all<M, ROWS, WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (int rc_ = launch("k_w4a8_all", k_w4a8_all<M, ROWS, WARPS>, dim3((N + ROWS - 1) / ROWS), dim3(WARPS * 32), smem, st, Wp, S, q, sx, sum, N, K, Y, ldy, CH)) return rc_;
  return check_launch("k_w4a8_all");
}

static size_t w4a8_ring_smem(int M, int rows, int K, int ns) {
  const int G = K / 32;
  const size_t stage = (size_t)rows * (K / 2 + 16) + ((size_t)rows * G * 2 + 15) / 16 * 16;
  return 128 + ns * stage + (size_t)M * K + (size_t)M * G * 8 + (size_t)rows * M * (G + 1) * 8;
}

template <int M, int ROWS, int WARPS, int NS>
static int launch_w4a8_ring_t(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx, const int32_t* sum,
                              int N, int K, float* Y, int ldy, int per_sm, cudaStream_t st) {
  const size_t smem = w4a8_ring_smem(M, ROWS, K, NS);
  auto kern = k_w4a8_ring<M, ROWS, WARPS, NS>;
  if (smem > 40 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, WARPS * 32, smem) != cudaSuccess || occ < 1) occ = 1;
  const int nblk = (N + ROWS - 1) / ROWS;
  const int grid = std::min(nblk, sm_count() * std::min(occ, per_sm));
  if (int rc_ = launch("k_w4a8_ring", kern, dim3(grid), dim3(WARPS * 32), smem, st, Wp, S, q, sx, sum, N, K, Y, ldy))
    return rc_;
  return check_launch("k_w4a8_ring");
}

// G4_W4A8_RING="rows,warps,stages,per_sm" selects the ring variant (rows 4/8/16, warps 2/4, stages
// 2/3/4) for experiments; unset, the whole-block variant runs.
template <int M>
static int launch_w4a8_ring(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx, const int32_t* sum,
                            int N, int K, float* Y, int ldy, cudaStream_t st, bool* done) {
  int R = 0, W = 4, NS = 3, per_sm = 4;  // off unless G4_W4A8_RING asks for it
  if (const char* e = getenv("G4_W4A8_RING")) sscanf(e, "%d,%d,%d,%d", &R, &W, &NS, &per_sm);
  *done = false;
  if (R <= 0) return G4_OK;
  if (R != 4 && R != 8 && R != 16) R = 8;
  if (W != 2 && W != 4) W = 4;
  if (NS < 2 || NS > 4) NS = 3;
  if (W * 32 < R * M) return G4_OK;
  if (w4a8_ring_smem(M, R, K, NS) > 220 * 1024) return G4_OK;
  *done = true;
#define G4_RING(RR, WW, SS) \
  if (R == RR && W == WW && NS == SS) return launch_w4a8_ring_t<M, RR, WW, SS>(Wp, S, q, sx, sum, N, K, Y, ldy, per_sm, st);
  G4_RING(4, 2, 2) G4_RING(4, 2, 3) G4_RING(4, 2, 4) G4_RING(4, 4, 2) G4_RING(4, 4, 3) G4_RING(4, 4, 4)
  G4_RING(8, 2, 2) G4_RING(8, 2, 3) G4_RING(8, 2, 4) G4_RING(8, 4, 2) G4_RING(8, 4, 3) G4_RING(8, 4, 4)
  G4_RING(16, 2, 2) G4_RING(16, 2, 3) G4_RING(16, 2, 4) G4_RING(16, 4, 2) G4_RING(16, 4, 3) G4_RING(16, 4, 4)
#undef G4_RING
  *done = false;
  return G4_OK;
}

template <int M>
static int launch_w4a8(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx, const int32_t* sum,
                       int N, int K, float* Y, int ldy, cudaStream_t st) {
  {
    bool done = false;
    const int rc = launch_w4a8_ring<M>(Wp, S, q, sx, sum, N, K, Y, ldy, st, &done);
    if (done || rc) return rc;
  }
  // whole-block variant (all rows of a CTA in flight at once) when its shared memory fits;
  // G4_W4A8_ALL="rows,warps" (rows 8/16, warps 2/4/8) overrides the choice for experiments
  int AR = (N >= 8192 && M <= 4) ? 16 : 8, AW = 4;
  if (const char* e = getenv("G4_W4A8_ALL")) sscanf(e, "%d,%d", &AR, &AW);
  if (AR != 16) AR = AR > 0 ? 8 : 0;
  if (AW != 2 && AW != 8) AW = 4;
  while (AW < 8 && AW * 32 < AR * M) AW *= 2;
  const int G = K / 32, ACH = pick_ch(G);
  if (AR > 0 && AW * 32 >= AR * M && G / ACH <= 16 && w4a8_all_smem(M, AR, K) <= 200 * 1024) {
#define G4_ALL(RR, WW) \
    if (AR == RR && AW == WW) return launch_w4a8_all_t<M, RR, WW>(Wp, S, q, sx, sum, N, K, Y, ldy, ACH, st);
    G4_ALL(8, 2) G4_ALL(8, 4) G4_ALL(8, 8) G4_ALL(16, 2) G4_ALL(16, 4) G4_ALL(16, 8)
#undef G4_ALL
  }
  int WARPS = 2, CH = pick_ch(K / 32), NB = 3;
  if (const char* e = getenv("G4_W4A8_CFG")) sscanf(e, "%d,%d,%d", &WARPS, &CH, &NB);
  if (WARPS == 1) return launch_w4a8_t<M, 1>(Wp, S, q, sx, sum, N, K, Y, ldy, CH, NB, st);
  if (WARPS == 4) return launch_w4a8_t<M, 4>(Wp, S, q, sx, sum, N, K, Y, ldy, CH, NB, st);
  return launch_w4a8_t<M, 2>(Wp, S, q, sx, sum, N, K, Y, ldy, CH, NB, st);
}

extern "C" int g4_w4a8_gemm(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx,
                            const int32_t* sum, int M, int N, int K, float* Y, int ldy, void* stream) {
  G4_REQUIRE(Wp && S && q && sx && sum && Y, "g4_w4a8_gemm: null pointer");
  G4_REQUIRE(M >= 1 && M <= 8 && N > 0 && K > 0 && K % 256 == 0 && ldy >= N,
             "g4_w4a8_gemm: unsupported shape M=%d N=%d K=%d ldy=%d (K must be a multiple of 256)", M, N, K, ldy);
  G4_REQUIRE(aligned(Wp, 16) && aligned(S, 16) && aligned(q, 16), "g4_w4a8_gemm: Wp, S and q must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  switch (M) {
    case 1: return launch_w4a8<1>(Wp, S, q, sx, sum, N, K, Y, ldy, st);
    case 2: return launch_w4a8<2>(Wp, S, q, sx, sum, N, K, Y, ldy, st);
    case 3: return launch_w4a8<3>(Wp, S, q, sx, sum, N, K, Y, ldy, st);
    case 4: return launch_w4a8<4>(Wp, S, q, sx, sum, N, K, Y, ldy, st);
    case 5: return launch_w4a8<5>(Wp, S, q, sx, sum, N, K, Y, ldy, st);
    case 6: return launch_w4a8<6>(Wp, S, q, sx, sum, N, K, Y, ldy, st);
    case 7: return launch_w4a8<7>(Wp, S, q, sx, sum, N, K, Y, ldy, st);
    default: return launch_w4a8<8>(Wp, S, q, sx, sum, N, K, Y, ldy, st);
  }
}
