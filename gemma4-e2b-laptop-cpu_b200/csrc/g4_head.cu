// Output head: the bf16-exp3 packed exact head (engine/bf16_exp3_head.h), the certified int4
// head screen (gemma4_engine.cpp:1235-1244, 454-538, 1409-1497) and the greedy pick with the
// softcap tie rule, all on the device.
//
// Logits stay exact: each packed row is decoded to its bf16 weights and dotted with h in the
// reference's fp32 order (lane j: weights j, 16+j, 8+j, 24+j of every group; hsum8; then the CSR
// exception patches y = y + delta*x, not fused, as the reference compiles under Zen 3 tuning).
// The screen finds the same survivor set as the reference's eval_row: lower/upper bounds s -+ c|h|
// (fused), L = max lower, survivors = {n : upper >= calc_thr(L)}.  Survivors are collected in any
// order: the pick (max of the rescored bf16 logits, then the lowest index whose capped value
// equals the max's) does not depend on it.  More than `lim` survivors means the full head runs,
// as the reference's fallback does.  The softcap r16(30*tanh(s/30)) is only ever applied to bf16
// values, so it is a 65,536-entry table built on the host with the same libm (g4_device_init).
#include "g4_api.h"
#include "g4_async.cuh"
#include "g4_common.cuh"
#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

namespace g4 {

__device__ float g_cap_table[65536];  // cap(bf16 value with these bits), as float

__device__ __forceinline__ float cap_bf(float v) { return g_cap_table[__float_as_uint(v) >> 16]; }  // v bf16-valued

// calc_thr (gemma4_engine.cpp:1455-1459): lowest z (40-step bisection on [r16(L)-64, r16(L)])
// whose capped bf16 value equals cap(r16(L)), minus 0.25.
__device__ float calc_thr(float L) {
  const float Lr = r16(L), cmL = cap_bf(Lr);
  float lo = __fsub_rn(Lr, 64.0f), hi = Lr;
  for (int it = 0; it < 40; ++it) {
    const float mid = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    if (cap_bf(r16(mid)) == cmL) hi = mid; else lo = mid;
  }
  return __fsub_rn(hi, 0.25f);
}

// float <-> order-preserving int for atomicMax
__device__ __forceinline__ int f2ord(float f) { const int i = __float_as_int(f); return i >= 0 ? i : i ^ 0x7FFFFFFF; }
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF); }

// ------------------------------------------------------------------------------- packing
// exponent histogram for the codebook (gemma4_engine.cpp:1232)
__global__ void k_exp_hist(const uint16_t* __restrict__ E, long long count, unsigned long long* __restrict__ hist) {
  __shared__ unsigned int h[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0;
  __syncthreads();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (long long)gridDim.x * blockDim.x)
    atomicAdd(&h[(E[i] >> 7) & 0xFF], 1u);
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[i], (unsigned long long)h[i]);
}

struct Codebook { uint8_t e[8]; };

// index of exponent e in the codebook; not found -> nearest (first on ties), exc = 1 (bf16_exp3_head.h:33-40)
__device__ __forceinline__ int cb_index(const Codebook& cb, int e, int& exc) {
  for (int i = 0; i < 8; ++i) if (cb.e[i] == e) { exc = 0; return i; }
  int best = 0, bd = 1 << 30;
  for (int i = 0; i < 8; ++i) { const int dd = abs((int)cb.e[i] - e); if (dd < bd) { bd = dd; best = i; } }
  exc = 1;
  return best;
}

// exceptions per row -> cnt[n] (block per row)
__global__ void k_bf16p_count(const uint16_t* __restrict__ E, int K, Codebook cb, long long* __restrict__ cnt) {
  const int n = blockIdx.x;
  int c = 0;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    int exc;
    cb_index(cb, (E[(size_t)n * K + k] >> 7) & 0xFF, exc);
    c += exc;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(FULL, c, o);
  __shared__ int ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < (int)(blockDim.x + 31) / 32; ++w) t += ws[w];
    cnt[n] = t;
  }
}

// exclusive scan of cnt[0..N) into ptr[0..N] (ptr[0] = 0); one block of 1024 threads, chunked.
__global__ void __launch_bounds__(1024) k_scan_rows(const long long* __restrict__ cnt, int N, long long* __restrict__ ptr) {
  __shared__ long long part[1024];
  const int per = (N + 1023) / 1024;
  const int a = threadIdx.x * per, b = min(N, a + per);
  long long s = 0;
  for (int i = a; i < b; ++i) s += cnt[i];
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    long long run = 0;
    for (int i = 0; i < 1024; ++i) { const long long v = part[i]; part[i] = run; run += v; }
  }
  __syncthreads();
  long long run = part[threadIdx.x];
  if (threadIdx.x == 0) ptr[0] = 0;
  for (int i = a; i < b; ++i) { run += cnt[i]; ptr[i + 1] = run; }
}

// fill the 44-byte groups and the exceptions of one row (block per row, thread per group);
// exceptions in (group, element) order at exc_ptr[n] + (exceptions of earlier groups) + rank.
__global__ void k_bf16p_fill(const uint16_t* __restrict__ E, int K, Codebook cb, uint8_t* __restrict__ data,
                             const long long* __restrict__ exc_ptr, uint16_t* __restrict__ exc_col,
                             float* __restrict__ exc_delta) {
  extern __shared__ int gcount[];  // [G] then scanned
  const int n = blockIdx.x, G = K >> 5;
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    int c = 0;
    for (int j = 0; j < 32; ++j) {
      int exc;
      cb_index(cb, (E[(size_t)n * K + g * 32 + j] >> 7) & 0xFF, exc);
      c += exc;
    }
    gcount[g] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int g = 0; g < G; ++g) { const int v = gcount[g]; gcount[g] = run; run += v; }
  }
  __syncthreads();
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    uint32_t sm[8] = {0, 0, 0, 0, 0, 0, 0, 0}, pl[3] = {0, 0, 0};
    long long e_out = exc_ptr[n] + gcount[g];
    for (int j = 0; j < 32; ++j) {
      const uint32_t w = E[(size_t)n * K + g * 32 + j];
      const uint32_t sign = w >> 15, e = (w >> 7) & 0xFF, m = w & 0x7F;
      int exc;
      const int idx = cb_index(cb, (int)e, exc);
      if (exc) {
        const uint32_t dec = (sign << 15) | ((uint32_t)cb.e[idx] << 7) | m;
        exc_col[e_out] = (uint16_t)(g * 32 + j);
        exc_delta[e_out] = __fsub_rn(bf2f(w), bf2f(dec));
        ++e_out;
      }
      sm[j >> 2] |= ((sign << 7) | m) << (8 * (j & 3));
      for (int k = 0; k < 3; ++k) pl[k] |= (uint32_t)((idx >> k) & 1) << j;
    }
    uint32_t* d = reinterpret_cast<uint32_t*>(data + ((size_t)n * G + g) * 44);
    for (int k = 0; k < 8; ++k) d[k] = sm[k];
    for (int k = 0; k < 3; ++k) d[8 + k] = pl[k];
  }
}

// ------------------------------------------------------------------------- exact head dot
struct HeadPacked {
  const uint8_t* data;
  const uint8_t* unp;  // the same head in the unpacked layout (g4_bf16p_unpack), or NULL
  const uint8_t* nib;  // the same head in the split-nibble layout (g4_bf16p_nib_pack), or NULL
  const long long* exc_ptr;
  const uint16_t* exc_col;
  const float* exc_delta;
  uint32_t cb_lo, cb_hi;  // codebook bytes 0-3 and 4-7
  int N, K;
};

// weight e (0..31) of a packed group held as sign/mant bytes and 3 planes
__device__ __forceinline__ float bf16p_w(const uint8_t* g, uint32_t p0, uint32_t p1, uint32_t p2, int e,
                                         uint32_t cb_lo, uint32_t cb_hi) {
  const uint32_t idx = ((p0 >> e) & 1u) | (((p1 >> e) & 1u) << 1) | (((p2 >> e) & 1u) << 2);
  const uint32_t ex = __byte_perm(cb_lo, cb_hi, idx) & 0xFFu;
  const uint32_t sm = g[e];
  return __uint_as_float((((sm & 0x80u) << 8) | (ex << 7) | (sm & 0x7Fu)) << 16);
}

// Row dot for one octet lane: returns the lane's partial sum over all groups (rows_tile order).
__device__ __forceinline__ float bf16p_lane_dot(const uint8_t* __restrict__ row, int G, const float* __restrict__ x,
                                                int j, uint32_t cb_lo, uint32_t cb_hi) {
  float acc = 0.f;
#pragma unroll 2
  for (int g = 0; g < G; ++g) {
    const uint8_t* gp = row + (size_t)g * 44;
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(gp + 32);
    const uint32_t p0 = pw[0], p1 = pw[1], p2 = pw[2];
    const float* xg = x + g * 32;
    acc = fmaf(bf16p_w(gp, p0, p1, p2, j, cb_lo, cb_hi), xg[j], acc);
    acc = fmaf(bf16p_w(gp, p0, p1, p2, 16 + j, cb_lo, cb_hi), xg[16 + j], acc);
    acc = fmaf(bf16p_w(gp, p0, p1, p2, 8 + j, cb_lo, cb_hi), xg[8 + j], acc);
    acc = fmaf(bf16p_w(gp, p0, p1, p2, 24 + j, cb_lo, cb_hi), xg[24 + j], acc);
  }
  return acc;
}

// exception patches of row n against x, in CSR order, unfused (bf16_exp3_head.h:103)
__device__ __forceinline__ float bf16p_patch(const HeadPacked& P, int n, const float* __restrict__ x, float y) {
  for (long long e = P.exc_ptr[n]; e < P.exc_ptr[n + 1]; ++e) y = __fadd_rn(y, __fmul_rn(P.exc_delta[e], x[P.exc_col[e]]));
  return y;
}

// Y[m*ldy + n] = raw logit (before r16).  Octet per row; 256 threads = 32 rows.  If `gate` is
// non-null the kernel does nothing unless *gate != 0 (device-side fallback decision).
template <int M>
__global__ void __launch_bounds__(256) k_bf16p_gemv(HeadPacked P, const float* __restrict__ X, float* __restrict__ Y,
                                                    int ldy, const int* __restrict__ gate) {
  pdl_wait();
  pdl_trigger();
  if (gate != nullptr && *gate == 0) return;
  const int j = threadIdx.x & 7;
  const int n_raw = blockIdx.x * 32 + (threadIdx.x >> 3);
  const bool live = n_raw < P.N;
  const int n = live ? n_raw : P.N - 1;
  const int G = P.K >> 5;
  const uint8_t* row = P.data + (size_t)n * G * 44;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const float* x = X + (size_t)m * P.K;
    const float acc = bf16p_lane_dot(row, G, x, j, P.cb_lo, P.cb_hi);
    const float y = hsum8_octet(acc);
    if (live && j == 0) Y[(size_t)m * ldy + n] = bf16p_patch(P, n, x, y);
  }
}

// Staged variant for K % 256 == 0 and K <= 2048 (the head widths of this model): a persistent
// grid, one CTA per SM, takes blocks of 32 rows in turn.  Each block's 32 packed rows arrive in
// shared memory by one bulk copy per row (issued by the lanes of warp 0), double-buffered against
// the previous block's arithmetic; rows sit 16 bytes further apart than in memory so that the four
// octets of a warp (four rows) read different banks.  The activations sit in shared memory as
// (row m, row m+1) pairs so
// that each decoded weight feeds two rows per packed f32x2 FMA.  Every octet lane runs exactly
// the chains of bf16p_lane_dot (per row m: elements j, 16+j, 8+j, 24+j of each group in group
// order), so the logits are those of k_bf16p_gemv.
constexpr int kHeadBlkRows = 32;
__host__ __device__ inline int head_row_stride(int K) { return (K / 32) * 44 + 16; }
__host__ __device__ inline size_t head_stage_bytes(int K) { return (size_t)kHeadBlkRows * head_row_stride(K); }
__host__ __device__ inline size_t head_smem_bytes(int M, int K) {
  return 128 + (size_t)((M + 1) / 2) * K * 8 + 2 * head_stage_bytes(K);
}

template <int M>
__global__ void __launch_bounds__(256) k_bf16p_gemv_staged(HeadPacked P, const float* __restrict__ X,
                                                           float* __restrict__ Y, int ldy,
                                                           const int* __restrict__ gate) {
  pdl_wait();
  pdl_trigger();
  constexpr int NP = (M + 1) / 2;
  if (gate != nullptr && *gate == 0) return;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  const int K = P.K, G = K >> 5;
  float2* xs = reinterpret_cast<float2*>(smem + 128);  // [NP][K]
  uint8_t* stage = smem + 128 + (size_t)NP * K * 8;
  const size_t sbytes = head_stage_bytes(K);
  const int nblk = (P.N + kHeadBlkRows - 1) / kHeadBlkRows;
  const int rowb = G * 44, rs = head_row_stride(K);
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int blk, int s) {  // warp 0, all lanes
    const int lane = threadIdx.x & 31;
    const int r0 = blk * kHeadBlkRows, nr = min(kHeadBlkRows, P.N - r0);
    if (lane == 0) mbar_expect_tx(&bars[s], (uint32_t)nr * rowb);
    __syncwarp();
    if (lane < nr)
      bulk_g2s(stage + s * sbytes + (size_t)lane * rs, P.data + (size_t)(r0 + lane) * rowb, (uint32_t)rowb, &bars[s]);
  };
  if (threadIdx.x < 32) {
    if ((int)blockIdx.x < nblk) issue(blockIdx.x, 0);
    if ((int)(blockIdx.x + gridDim.x) < nblk) issue(blockIdx.x + gridDim.x, 1);
  }
  for (int i = threadIdx.x; i < NP * K; i += blockDim.x) {
    const int p = i / K, k = i % K;
    const float a = X[(size_t)(2 * p) * K + k];
    const float b = (2 * p + 1 < M) ? X[(size_t)(2 * p + 1) * K + k] : 0.f;
    xs[i] = make_float2(a, b);
  }
  __syncthreads();
  const int j = threadIdx.x & 7, rl = threadIdx.x >> 3;  // octet lane, row in block
  const uint32_t cb_lo = P.cb_lo, cb_hi = P.cb_hi;
  int it = 0;
  for (int blk = blockIdx.x; blk < nblk; blk += gridDim.x, ++it) {
    const int s = it & 1;
    if (!cta_wait(&bars[s], (uint32_t)(it >> 1) & 1u)) return;
    const int n = blk * kHeadBlkRows + rl;
    const bool live = n < P.N;
    const uint8_t* row = stage + s * sbytes + (size_t)(live ? rl : 0) * rs;
    float2 acc[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) acc[p] = make_float2(0.f, 0.f);
#pragma unroll 2
    for (int g = 0; g < G; ++g) {
      const uint8_t* gp = row + g * 44;
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(gp + 32);
      // exponent codes of elements j, 8+j, 16+j, 24+j sit at bits j, j+8, j+16, j+24 of the planes
      const uint32_t c = ((pw[0] >> j) & 0x01010101u) | (((pw[1] >> j) & 0x01010101u) << 1) |
                         (((pw[2] >> j) & 0x01010101u) << 2);
      const uint32_t sel = (c & 7u) | ((c >> 4) & 0x70u) | ((c >> 8) & 0x700u) | ((c >> 12) & 0x7000u);
      const uint32_t ex4 = __byte_perm(cb_lo, cb_hi, sel);  // exponent of element j + 8i in byte i
      float w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t sm = gp[j + 8 * i];
        const uint32_t ex = (ex4 >> (8 * i)) & 0xFFu;
        w[i] = __uint_as_float((((sm & 0x80u) << 8) | (ex << 7) | (sm & 0x7Fu)) << 16);
      }
      const float2* xg = xs + g * 32 + j;
      // chain order of bf16p_lane_dot: elements j, 16+j, 8+j, 24+j
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const float2* xp = xg + (size_t)p * K;
        acc[p] = __ffma2_rn(make_float2(w[0], w[0]), xp[0], acc[p]);
        acc[p] = __ffma2_rn(make_float2(w[2], w[2]), xp[16], acc[p]);
        acc[p] = __ffma2_rn(make_float2(w[1], w[1]), xp[8], acc[p]);
        acc[p] = __ffma2_rn(make_float2(w[3], w[3]), xp[24], acc[p]);
      }
    }
    float y[M];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      y[2 * p] = hsum8_octet(acc[p].x);
      if (2 * p + 1 < M) y[2 * p + 1] = hsum8_octet(acc[p].y);
    }
    if (live && j == 0) {
      for (long long e = P.exc_ptr[n]; e < P.exc_ptr[n + 1]; ++e) {  // CSR order, unfused (bf16_exp3_head.h:103)
        const float dl = P.exc_delta[e];
        const int col = P.exc_col[e];
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float2 xv = xs[(size_t)(m >> 1) * K + col];
          y[m] = __fadd_rn(y[m], __fmul_rn(dl, (m & 1) ? xv.y : xv.x));
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) Y[(size_t)m * ldy + n] = y[m];
    }
    __syncthreads();  // every octet is done with this stage
    if (threadIdx.x < 32 && blk + 2 * (int)gridDim.x < nblk) {
      fence_proxy_async_smem();  // this stage's reads happen before the next bulk copies rewrite it
      issue(blk + 2 * gridDim.x, s);
    }
  }
}

// Row-per-thread variant: one thread runs all eight octet-lane chains of its row (the lanes of the
// reference's 8-wide vectors), so each group's exponent codes are decoded once for every
// activation row.  The thread reads its row straight from global memory, four groups (176 bytes)
// at a time as 11 aligned 16-byte loads through L1 (the 32 rows of a warp share no cache lines,
// each 128-byte line serves 8 consecutive loads of its thread), so occupancy is set by registers,
// not shared memory.  A persistent grid takes 256-row tiles in turn; the activations sit in shared
// memory as [k][pair] float2 (one 16-byte broadcast load per element for four rows).  Four weights
// at a time are decoded with byte permutes: the exponent codes of 4 consecutive elements are spread
// to bytes by one multiply per bit plane and turned into a permute selector over the 8-entry
// codebook; the sign/mantissa word and the 4 exponents give the bf16 high and low bytes, which 2
// permutes interleave into 2 x 2 floats.  Lane j's chain order (elements j, 16+j, 8+j, 24+j) is
// kept by visiting the element octets 0, 2, 1, 3 of each group.  Values are those of
// k_bf16p_gemv.
constexpr int kBrThreads = 256;
__host__ __device__ inline size_t head_rows_smem(int M, int K) { return (size_t)K * ((M + 1) / 2) * 8; }

template <int M>
__global__ void __launch_bounds__(kBrThreads) k_bf16p_rows(HeadPacked P, const float* __restrict__ X,
                                                           float* __restrict__ Y, int ldy, const int* __restrict__ gate) {
  constexpr int NP = (M + 1) / 2;
  pdl_wait();
  pdl_trigger();
  if (gate != nullptr && *gate == 0) return;
  extern __shared__ __align__(16) float2 xs[];  // [K][NP]
  const int K = P.K, G = K >> 5, rowb = G * 44;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    float v[2 * NP];
#pragma unroll
    for (int m = 0; m < 2 * NP; ++m) v[m] = m < M ? X[(size_t)m * K + i] : 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) xs[(size_t)i * NP + p] = make_float2(v[2 * p], v[2 * p + 1]);
  }
  __syncthreads();
  const uint32_t cb_lo = P.cb_lo, cb_hi = P.cb_hi;
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n - (int)threadIdx.x < P.N; n += gridDim.x * blockDim.x) {
    if (n >= P.N) continue;
    const uint4* rowp = reinterpret_cast<const uint4*>(P.data + (size_t)n * rowb);
    float2 acc[8][NP];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int p = 0; p < NP; ++p) acc[j][p] = make_float2(0.f, 0.f);
#pragma unroll 1
    for (int u = 0; u < G / 4; ++u) {
      uint32_t wv[44];
#pragma unroll
      for (int k = 0; k < 11; ++k) {
        const uint4 t4 = __ldg(rowp + u * 11 + k);
        wv[4 * k] = t4.x; wv[4 * k + 1] = t4.y; wv[4 * k + 2] = t4.z; wv[4 * k + 3] = t4.w;
      }
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        const int g = u * 4 + gg;
        const uint32_t* gw = wv + gg * 11;
        const uint32_t p0 = gw[8], p1 = gw[9], p2 = gw[10];
        const float2* xg = xs + (size_t)g * 32 * NP;
#pragma unroll
        for (int oi = 0; oi < 4; ++oi) {
          const int o8 = (oi == 1) ? 2 : (oi == 2 ? 1 : oi);  // element octets in chain order 0, 2, 1, 3
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int sh = 8 * o8 + 4 * h;  // elements sh .. sh+3 = lanes 4h .. 4h+3
            const uint32_t s0 = (((p0 >> sh) & 0xFu) * 0x00204081u) & 0x01010101u;
            const uint32_t s1 = (((p1 >> sh) & 0xFu) * 0x00204081u) & 0x01010101u;
            const uint32_t s2 = (((p2 >> sh) & 0xFu) * 0x00204081u) & 0x01010101u;
            const uint32_t cc = s0 | (s1 << 1) | (s2 << 2);  // code of element sh + k in byte k
            const uint32_t sel = __byte_perm(cc | (cc >> 4), 0u, 0x0020u);
            const uint32_t ex4 = __byte_perm(cb_lo, cb_hi, sel);
            const uint32_t smw = gw[sh >> 2];
            const uint32_t hb4 = (smw & 0x80808080u) | ((ex4 >> 1) & 0x7F7F7F7Fu);
            const uint32_t lb4 = ((ex4 << 7) & 0x80808080u) | (smw & 0x7F7F7F7Fu);
            const uint32_t t01 = __byte_perm(lb4, hb4, 0x5140u), t23 = __byte_perm(lb4, hb4, 0x7362u);
            const float wk[4] = {__uint_as_float(t01 << 16), __uint_as_float(t01 & 0xFFFF0000u),
                                 __uint_as_float(t23 << 16), __uint_as_float(t23 & 0xFFFF0000u)};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int e = sh + k, j = 4 * h + k;
#pragma unroll
              for (int p = 0; p < NP; ++p) acc[j][p] = __ffma2_rn(make_float2(wk[k], wk[k]), xg[e * NP + p], acc[j][p]);
            }
          }
        }
      }
    }
    float y[2 * NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      // hsum8: ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7))
      y[2 * p] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][p].x, acc[4][p].x), __fadd_rn(acc[1][p].x, acc[5][p].x)),
                           __fadd_rn(__fadd_rn(acc[2][p].x, acc[6][p].x), __fadd_rn(acc[3][p].x, acc[7][p].x)));
      y[2 * p + 1] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][p].y, acc[4][p].y), __fadd_rn(acc[1][p].y, acc[5][p].y)),
                               __fadd_rn(__fadd_rn(acc[2][p].y, acc[6][p].y), __fadd_rn(acc[3][p].y, acc[7][p].y)));
    }
    for (long long e = P.exc_ptr[n]; e < P.exc_ptr[n + 1]; ++e) {  // CSR order, unfused (bf16_exp3_head.h:103)
      const float dl = P.exc_delta[e];
      const int col = P.exc_col[e];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const float2 xv = xs[(size_t)col * NP + p];
        y[2 * p] = __fadd_rn(y[2 * p], __fmul_rn(dl, xv.x));
        y[2 * p + 1] = __fadd_rn(y[2 * p + 1], __fmul_rn(dl, xv.y));
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) Y[(size_t)m * ldy + n] = y[m];
  }
}

// Variant fed by the TMA, two threads per row: thread half h runs lane chains 4h..4h+3 (elements
// 4h..4h+3 of each octet) over every group in order, and the halves meet in the final hsum8
// through one shuffle.  A persistent CTA of 256 threads takes 128-row blocks (2 CTAs per SM; the
// 2048 blocks of the 262,144-row head balance to within 1%); per pipeline item one 2D tensor-map
// load brings 4 groups (176 bytes) of all 128 rows into one of kBtNS shared-memory stages as a dense
// [128][176] box (176 = 11 x 16 bytes, an odd multiple of 16, so 16-byte loads of 8 consecutive
// rows hit 8 different bank quads; rows past N read as zeros).  The arithmetic is that of
// k_bf16p_rows; the exception patches of activation row m run on half m & 1.
constexpr int kBtRows = 128, kBtThreads = 256, kBtNS = 3, kBtBox = 176;
__host__ __device__ inline size_t head_tma_smem(int M, int K) {
  return 128 + (size_t)kBtNS * kBtRows * kBtBox + (size_t)K * ((M + 1) / 2) * 8;
}

template <int M>
__global__ void __launch_bounds__(kBtThreads, 2) k_bf16p_rows_tma(const __grid_constant__ CUtensorMap tmap, HeadPacked P,
                                                                  const float* __restrict__ X, float* __restrict__ Y, int ldy,
                                                                  const int* __restrict__ gate) {
  constexpr int NP = (M + 1) / 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint8_t* stages = smem + 128;
  float2* xs = reinterpret_cast<float2*>(stages + (size_t)kBtNS * kBtRows * kBtBox);  // [K][NP]
  pdl_wait();
  pdl_trigger();
  if (gate != nullptr && *gate == 0) return;
  const int K = P.K, G = K >> 5, nch = G / 4;
  const int nblk = (P.N + kBtRows - 1) / kBtRows;
  const int myblk = nblk > (int)blockIdx.x ? (nblk - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int nitems = myblk * nch;
  const int t = threadIdx.x, rl = t >> 1, half = t & 1;
  if (t == 0) {
    for (int b = 0; b < kBtNS; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i, int st) {  // thread 0
    const int blk = blockIdx.x + (i / nch) * gridDim.x, c = i % nch;
    mbar_expect_tx(&bars[st], (uint32_t)(kBtRows * kBtBox));
    tma_load_2d(stages + (size_t)st * kBtRows * kBtBox, &tmap, c * kBtBox, blk * kBtRows, &bars[st]);
  };
  if (t == 0)
    for (int b = 0; b < kBtNS && b < nitems; ++b) issue(b, b);
  for (int i = t; i < K; i += kBtThreads) {
    float v[2 * NP];
#pragma unroll
    for (int m = 0; m < 2 * NP; ++m) v[m] = m < M ? X[(size_t)m * K + i] : 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) xs[(size_t)i * NP + p] = make_float2(v[2 * p], v[2 * p + 1]);
  }
  __syncthreads();
  const uint32_t cb_lo = P.cb_lo, cb_hi = P.cb_hi;
  const int hsh = 4 * half;
  float2 acc[4][NP];
  for (int i = 0; i < nitems; ++i) {
    const int st = i % kBtNS;
    const int blk = blockIdx.x + (i / nch) * gridDim.x, c = i % nch;
    const int n = blk * kBtRows + rl;
    if (!cta_wait(&bars[st], (uint32_t)(i / kBtNS) & 1u)) return;
    if (c == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int p = 0; p < NP; ++p) acc[j][p] = make_float2(0.f, 0.f);
    }
    const uint4* rowp = reinterpret_cast<const uint4*>(stages + ((size_t)st * kBtRows + rl) * kBtBox);
    uint32_t wv[44];
#pragma unroll
    for (int k = 0; k < 11; ++k) {
      const uint4 t4 = rowp[k];
      wv[4 * k] = t4.x; wv[4 * k + 1] = t4.y; wv[4 * k + 2] = t4.z; wv[4 * k + 3] = t4.w;
    }
    __syncthreads();  // every row has its words in registers: the stage can be refilled
    if (t == 0 && i + kBtNS < nitems) {
      fence_proxy_async_smem();
      issue(i + kBtNS, st);
    }
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) {
      const int g = c * 4 + gg;
      const uint32_t* gw = wv + gg * 11;
      const uint32_t p0 = gw[8], p1 = gw[9], p2 = gw[10];
      const float2* xg = xs + ((size_t)g * 32 + hsh) * NP;
#pragma unroll
      for (int oi = 0; oi < 4; ++oi) {
        const int o8 = (oi == 1) ? 2 : (oi == 2 ? 1 : oi);  // element octets in chain order 0, 2, 1, 3
        const int sh = 8 * o8 + hsh;
        const uint32_t s0 = (((p0 >> sh) & 0xFu) * 0x00204081u) & 0x01010101u;
        const uint32_t s1 = (((p1 >> sh) & 0xFu) * 0x00204081u) & 0x01010101u;
        const uint32_t s2 = (((p2 >> sh) & 0xFu) * 0x00204081u) & 0x01010101u;
        const uint32_t cc = s0 | (s1 << 1) | (s2 << 2);
        const uint32_t sel = __byte_perm(cc | (cc >> 4), 0u, 0x0020u);
        const uint32_t ex4 = __byte_perm(cb_lo, cb_hi, sel);
        const uint32_t smw = half ? gw[2 * o8 + 1] : gw[2 * o8];
        const uint32_t hb4 = (smw & 0x80808080u) | ((ex4 >> 1) & 0x7F7F7F7Fu);
        const uint32_t lb4 = ((ex4 << 7) & 0x80808080u) | (smw & 0x7F7F7F7Fu);
        const uint32_t t01 = __byte_perm(lb4, hb4, 0x5140u), t23 = __byte_perm(lb4, hb4, 0x7362u);
        const float wk[4] = {__uint_as_float(t01 << 16), __uint_as_float(t01 & 0xFFFF0000u),
                             __uint_as_float(t23 << 16), __uint_as_float(t23 & 0xFFFF0000u)};
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int p = 0; p < NP; ++p)
            acc[k][p] = __ffma2_rn(make_float2(wk[k], wk[k]), xg[(8 * o8 + k) * NP + p], acc[k][p]);
      }
    }
    if (c == nch - 1) {
      // lanes 4..7 come from the other half; fadd is commutative, so both halves hold
      // ((v0 + v4) + (v1 + v5)) + ((v2 + v6) + (v3 + v7)) bit for bit
      float y[2 * NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        float2 w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          w[k].x = __shfl_xor_sync(0xffffffffu, acc[k][p].x, 1);
          w[k].y = __shfl_xor_sync(0xffffffffu, acc[k][p].y, 1);
        }
        y[2 * p] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][p].x, w[0].x), __fadd_rn(acc[1][p].x, w[1].x)),
                             __fadd_rn(__fadd_rn(acc[2][p].x, w[2].x), __fadd_rn(acc[3][p].x, w[3].x)));
        y[2 * p + 1] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][p].y, w[0].y), __fadd_rn(acc[1][p].y, w[1].y)),
                                 __fadd_rn(__fadd_rn(acc[2][p].y, w[2].y), __fadd_rn(acc[3][p].y, w[3].y)));
      }
      if (n < P.N) {
        float yo[NP];  // this half's activation rows 2p + half
#pragma unroll
        for (int p = 0; p < NP; ++p) yo[p] = half ? y[2 * p + 1] : y[2 * p];
        for (long long e = P.exc_ptr[n]; e < P.exc_ptr[n + 1]; ++e) {  // CSR order, unfused (bf16_exp3_head.h:103)
          const float dl = P.exc_delta[e];
          const int col = P.exc_col[e];
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            const float2 xv = xs[(size_t)col * NP + p];
            yo[p] = __fadd_rn(yo[p], __fmul_rn(dl, half ? xv.y : xv.x));
          }
        }
#pragma unroll
        for (int p = 0; p < NP; ++p)
          if (2 * p + half < M) Y[(size_t)(2 * p + half) * ldy + n] = yo[p];
      }
    }
  }
}

// ------------------------------------------------------------------------------ greedy pick
// Slots per row m: [0] ordered-int max of r16 logits, [1] winner index.
__global__ void k_pick_init(int* __restrict__ slots, int M) {
  pdl_wait();
  pdl_trigger();
  const int m = threadIdx.x;
  if (m < M) { slots[2 * m] = f2ord(-1e30f); slots[2 * m + 1] = 0x7FFFFFFF; }
}
__global__ void k_pick_max(const float* __restrict__ Y, int N, int ldy, int* __restrict__ slots, const int* __restrict__ gate) {
  pdl_wait();
  pdl_trigger();
  if (gate != nullptr && *gate == 0) return;
  const int m = blockIdx.y;
  float mx = -1e30f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x) mx = fmaxf(mx, r16(Y[(size_t)m * ldy + i]));
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if ((threadIdx.x & 31) == 0) atomicMax(&slots[2 * m], f2ord(mx));
}
// lowest index with v >= mx - 2 and cap(v) == cap(mx) (gemma4_engine.cpp:1496)
__global__ void k_pick_idx(const float* __restrict__ Y, int N, int ldy, int* __restrict__ slots, const int* __restrict__ gate) {
  pdl_wait();
  pdl_trigger();
  if (gate != nullptr && *gate == 0) return;
  const int m = blockIdx.y;
  const float mx = ord2f(slots[2 * m]);
  const float cm = cap_bf(mx), lim = __fsub_rn(mx, 2.0f);
  int best = 0x7FFFFFFF;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x) {
    const float v = r16(Y[(size_t)m * ldy + i]);
    if (v >= lim && cap_bf(v) == cm) { best = i; break; }  // grid-stride: later i only larger
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) best = min(best, __shfl_xor_sync(FULL, best, o));
  if ((threadIdx.x & 31) == 0 && best != 0x7FFFFFFF) atomicMin(&slots[2 * m + 1], best);
}
__global__ void k_pick_out(const int* __restrict__ slots, int M, int* __restrict__ out, const int* __restrict__ gate) {
  pdl_wait();
  pdl_trigger();
  if (gate != nullptr && *gate == 0) return;
  const int m = threadIdx.x;
  if (m < M) out[m] = slots[2 * m + 1] == 0x7FFFFFFF ? -1 : slots[2 * m + 1];
}

// ---------------------------------------------------------------------------- screen build
// Block per row, thread per group for the int4 copy (device nibble layout: byte b = q[b] |
// q[16+b] << 4); then one thread sums e^2 and w^2 in double in the reference's (group, element)
// order and writes coef = fma(1e-4, sqrt(w2), sqrt(e2)) (gemma4_engine.cpp:1236-1243).
__global__ void k_screen_build(const uint16_t* __restrict__ E, int K, uint8_t* __restrict__ W4, uint16_t* __restrict__ S4,
                               float* __restrict__ coef) {
  extern __shared__ float scl[];  // [G] scale per group
  const int n = blockIdx.x, G = K >> 5;
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    float amax = 0.f, w[32];
    for (int i = 0; i < 32; ++i) { w[i] = bf2f(E[(size_t)n * K + g * 32 + i]); amax = fmaxf(amax, fabsf(w[i])); }
    const uint32_t sb = f2bf(__fdiv_rn(amax, 7.0f));
    const float sc = bf2f(sb);
    S4[(size_t)n * G + g] = (uint16_t)sb;
    scl[g] = sc;
    uint32_t qv[32];
    for (int i = 0; i < 32; ++i) {
      int v = sc > 0.f ? __float2int_rn(__fdiv_rn(w[i], sc)) : 0;
      v = max(-8, min(7, v));
      qv[i] = (uint32_t)(v + 8);
    }
    uint32_t out[4] = {0, 0, 0, 0};
    for (int b = 0; b < 16; ++b) out[b >> 2] |= (qv[b] | (qv[16 + b] << 4)) << (8 * (b & 3));
    reinterpret_cast<uint4*>(W4 + (size_t)n * (K >> 1))[g] = make_uint4(out[0], out[1], out[2], out[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double e2 = 0, w2 = 0;
    for (int g = 0; g < G; ++g) {
      const float sc = scl[g];
      for (int i = 0; i < 32; ++i) {
        const float w = bf2f(E[(size_t)n * K + g * 32 + i]);
        int v = sc > 0.f ? __float2int_rn(__fdiv_rn(w, sc)) : 0;
        v = max(-8, min(7, v));
        const double d = fma(-(double)v, (double)sc, (double)w);  // exact either way: v*sc is exact
        e2 = fma(d, d, e2);
        w2 = fma((double)w, (double)w, w2);
      }
    }
    coef[n] = (float)fma(1e-4, sqrt(w2), sqrt(e2));
  }
}

// ------------------------------------------------------------------------------------ screen
struct ScreenWs {
  float* s;      // [M][N] screen dots, later the fallback logits
  float* hn;     // [M]
  int* Lord;     // [M] ordered-int L
  float* thr;    // [M]
  int* cnt;      // [M] survivors
  int* fb;       // [1] fallback flag
  int* surv;     // [M][lim]
  float* fval;   // [M][lim]
  int* slots;    // [2M] pick slots
  // Screen back-off (nullable, caller-owned int[4]): {passes still to skip, this pass skipped,
  // current back-off, passes skipped in total}.  While the count is positive a pass skips the
  // screen and runs the full exact head at once (the winners are the same: the screen only
  // certifies a shortcut to the exact argmax).  A screen that falls back doubles the back-off
  // (1, 2, 4, .. kScreenBackoffMax passes); a screen that does not resets it.
  int* pol;
};
constexpr int kScreenBackoffMax = 64;
__device__ __forceinline__ bool screen_skipped(const ScreenWs& w) { return w.pol != nullptr && w.pol[1] != 0; }
static size_t screen_ws_layout(int M, int N, int lim, ScreenWs* w, char* base) {
  size_t off = 0;
  auto take = [&](size_t bytes) { char* p = base ? base + off : nullptr; off += (bytes + 255) & ~(size_t)255; return p; };
  char* s = take(sizeof(float) * (size_t)M * N);
  char* hn = take(sizeof(float) * M);
  char* L = take(sizeof(int) * M);
  char* thr = take(sizeof(float) * M);
  char* cnt = take(sizeof(int) * M);
  char* fb = take(sizeof(int));
  char* surv = take(sizeof(int) * (size_t)M * lim);
  char* fval = take(sizeof(float) * (size_t)M * lim);
  char* slots = take(sizeof(int) * 2 * M);
  if (w) {
    w->s = (float*)s; w->hn = (float*)hn; w->Lord = (int*)L; w->thr = (float*)thr; w->cnt = (int*)cnt; w->fb = (int*)fb;
    w->surv = (int*)surv; w->fval = (float*)fval; w->slots = (int*)slots;
    w->pol = nullptr;
  }
  return off;
}

// |h| per row in double, in the order of ss_avx2 (gemma4_engine.cpp:326-343); one warp per row.
__global__ void k_screen_init(const float* __restrict__ H, int K, int M, ScreenWs w) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x, lane = threadIdx.x;
  if (w.pol != nullptr) {  // back-off: this pass goes straight to the exact head
    const bool skip = w.pol[0] > 0;
    if (m == 0 && lane == 0) {
      w.pol[1] = skip ? 1 : 0;
      if (skip) *w.fb = 1;
    }
    if (skip) return;
  }
  double s = 0;
  if (lane < 16) {
    for (int i = 0; i < K; i += 16) { const double d = H[(size_t)m * K + i + lane]; s = fma(d, d, s); }
  }
  // lane l = 4a + b holds s[a][b]; t_b = (s0_b + s1_b) + (s2_b + s3_b); total = (t0 + t2) + (t1 + t3)
  double v[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) v[l] = __shfl_sync(FULL, s, l);
  if (lane == 0) {
    double t[4];
    for (int b = 0; b < 4; ++b) t[b] = (v[b] + v[4 + b]) + (v[8 + b] + v[12 + b]);
    w.hn[m] = (float)sqrt((t[0] + t[2]) + (t[1] + t[3]));
    w.Lord[m] = f2ord(-1e30f);
    w.cnt[m] = 0;
    if (m == 0) *w.fb = 0;
  }
}
// L = max over rows of fma(-c, hn, s) (screen_task :484, vmx)
__global__ void k_screen_L(const float* __restrict__ coef, int N, ScreenWs w) {
  pdl_wait();
  pdl_trigger();
  if (screen_skipped(w)) return;
  const int m = blockIdx.y;
  const float hn = w.hn[m];
  float mx = -1e30f;
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x)
    mx = fmaxf(mx, fmaf(-coef[n], hn, w.s[(size_t)m * N + n]));
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if ((threadIdx.x & 31) == 0) atomicMax(&w.Lord[m], f2ord(mx));
}
__global__ void k_screen_thr(int M, ScreenWs w) {
  pdl_wait();
  pdl_trigger();
  if (screen_skipped(w)) return;
  const int m = threadIdx.x;
  if (m < M) w.thr[m] = calc_thr(ord2f(w.Lord[m]));
}
// survivors: upper = fma(c, hn, s) >= thr (eval_row :1461); more than lim -> fallback flag.
// Warp-uniform iteration with one atomic per warp; the order of the list is irrelevant.
__global__ void k_screen_collect(const float* __restrict__ coef, int N, int lim, ScreenWs w) {
  pdl_wait();
  pdl_trigger();
  if (screen_skipped(w)) return;
  const int m = blockIdx.y, lane = threadIdx.x & 31;
  const float hn = w.hn[m], thr = w.thr[m];
  const int wstride = gridDim.x * blockDim.x;
  for (int base = (blockIdx.x * blockDim.x + threadIdx.x) & ~31; base < N; base += wstride) {
    const int n = base + lane;
    const bool pass = n < N && fmaf(coef[n], hn, w.s[(size_t)m * N + n]) >= thr;
    const unsigned mask = __ballot_sync(FULL, pass);
    if (mask == 0u) continue;
    int k0 = 0;
    if (lane == 0) k0 = atomicAdd(&w.cnt[m], __popc(mask));
    k0 = __shfl_sync(FULL, k0, 0);
    if (pass) {
      const int k = k0 + __popc(mask & ((1u << lane) - 1u));
      if (k < lim) w.surv[(size_t)m * lim + k] = n;
      else *w.fb = 1;
    }
  }
}
// rescore survivors with the exact head (octet per survivor, resc_task :540-571): fval = r16(y)
__global__ void __launch_bounds__(256) k_screen_rescore(HeadPacked P, const float* __restrict__ H, int lim, ScreenWs w) {
  pdl_wait();
  pdl_trigger();
  if (*w.fb) return;
  const int m = blockIdx.y;
  const int count = min(w.cnt[m], lim);
  const int j = threadIdx.x & 7;
  const int k_raw = blockIdx.x * 32 + (threadIdx.x >> 3);
  if (blockIdx.x * 32 >= count) return;  // whole block past the survivors (uniform)
  const bool live = k_raw < count;
  const int k = live ? k_raw : 0;
  const int n = w.surv[(size_t)m * lim + k];
  const int G = P.K >> 5;
  const float* x = H + (size_t)m * P.K;
  const float acc = bf16p_lane_dot(P.data + (size_t)n * G * 44, G, x, j, P.cb_lo, P.cb_hi);
  const float y = hsum8_octet(acc);
  if (live && j == 0) w.fval[(size_t)m * lim + k] = r16(bf16p_patch(P, n, x, y));
}
// pick among survivors: max value, then lowest index with the tie rule (eval_row :1469-1471 with
// ties to the lowest index).  One block per row.
__global__ void k_screen_pick(int lim, ScreenWs w, int* __restrict__ out, int* __restrict__ nsurv) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const int count = min(w.cnt[m], lim);
  if (threadIdx.x == 0) nsurv[m] = *w.fb ? -1 : count;
  if (*w.fb) return;
  __shared__ float smx[32];
  __shared__ int sidx[32];
  float mx = -1e30f;
  for (int k = threadIdx.x; k < count; k += blockDim.x) mx = fmaxf(mx, w.fval[(size_t)m * lim + k]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if ((threadIdx.x & 31) == 0) smx[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = -1e30f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, smx[i]);
  const float cm = cap_bf(mx), lo = __fsub_rn(mx, 2.0f);
  int best = 0x7FFFFFFF;
  for (int k = threadIdx.x; k < count; k += blockDim.x) {
    const float v = w.fval[(size_t)m * lim + k];
    if (v >= lo && cap_bf(v) == cm) best = min(best, w.surv[(size_t)m * lim + k]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) best = min(best, __shfl_xor_sync(FULL, best, o));
  if ((threadIdx.x & 31) == 0) sidx[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) best = min(best, sidx[i]);
    out[m] = best == 0x7FFFFFFF ? -1 : best;
  }
}
// fallback pick writes the winners (only when the flag is set)
__global__ void k_screen_fb_out(const int* __restrict__ slots, int M, const ScreenWs w, int* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int m = threadIdx.x;
  const bool fb = *w.fb != 0;
  if (fb && m < M) out[m] = slots[2 * m + 1] == 0x7FFFFFFF ? -1 : slots[2 * m + 1];
  if (w.pol != nullptr && m == 0) {  // back-off for the next passes
    if (w.pol[1] != 0) {
      w.pol[0] -= 1;
      w.pol[3] += 1;
    } else if (fb) {
      const int r = w.pol[2] > 0 ? min(2 * w.pol[2], kScreenBackoffMax) : 1;
      w.pol[2] = r;
      w.pol[0] = r;
    } else {
      w.pol[2] = 0;
    }
  }
}

// ---- vocab-parallel screen: one shard of the head's rows per GPU.  The single-GPU screen is
// split at its two global reductions, the bound L (a max over all rows) and the pick (the max
// candidate value, then the lowest index whose capped value equals the cap of that max); the
// caller reduces between the phases (all-reduce max / min across the shards).
__global__ void k_shard_L_out(const ScreenWs w, int M, float* __restrict__ L) {
  pdl_wait();
  pdl_trigger();
  const int m = threadIdx.x;
  if (m < M) L[m] = ord2f(w.Lord[m]);
}
__global__ void k_shard_set_L(const float* __restrict__ L, int M, ScreenWs w) {
  pdl_wait();
  pdl_trigger();
  const int m = threadIdx.x;
  if (m < M) w.Lord[m] = f2ord(L[m]);
}
// the shard's largest candidate value per row: the rescored survivors, or (fallback) the r16
// logits of every row, whose max k_pick_max left in slots
__global__ void k_shard_vmax(int lim, const ScreenWs w, const int* __restrict__ slots, float* __restrict__ vmax,
                             int* __restrict__ nsurv) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const int count = min(w.cnt[m], lim);
  __shared__ float smx[32];
  float mx = -1e30f;
  if (!*w.fb)
    for (int k = threadIdx.x; k < count; k += blockDim.x) mx = fmaxf(mx, w.fval[(size_t)m * lim + k]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if ((threadIdx.x & 31) == 0) smx[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, smx[i]);
    vmax[m] = *w.fb ? ord2f(slots[2 * m]) : mx;
    nsurv[m] = *w.fb ? -1 : count;
  }
}
// lowest shard index whose candidate v satisfies v >= gmax - 2 and cap(v) == cap(gmax), as a global
// index (row0 + local), or INT_MAX; survivors, or every row on the fallback
__global__ void k_shard_pick(const float* __restrict__ gmax, int lim, const ScreenWs w, int N, int row0,
                             int* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const float mx = gmax[m];
  const float cm = cap_bf(mx), lo = __fsub_rn(mx, 2.0f);
  __shared__ int sidx[32];
  int best = 0x7FFFFFFF;
  if (*w.fb) {
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
      const float v = r16(w.s[(size_t)m * N + i]);
      if (v >= lo && cap_bf(v) == cm) { best = i; break; }  // strided: later i only larger
    }
  } else {
    const int count = min(w.cnt[m], lim);
    for (int k = threadIdx.x; k < count; k += blockDim.x) {
      const float v = w.fval[(size_t)m * lim + k];
      if (v >= lo && cap_bf(v) == cm) best = min(best, w.surv[(size_t)m * lim + k]);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) best = min(best, __shfl_xor_sync(FULL, best, o));
  if ((threadIdx.x & 31) == 0) sidx[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) best = min(best, sidx[i]);
    out[m] = best == 0x7FFFFFFF ? 0x7FFFFFFF : row0 + best;
  }
}

}  // namespace g4

G4_STATUS_READER(head)

using namespace g4;

// ---------------------------------------------------------------------------- device init
static std::mutex g_init_mu;
static bool g_init_done[128];

static bool device_ready() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return false;
  std::lock_guard<std::mutex> lk(g_init_mu);
  return g_init_done[dev];
}

extern "C" int g4_device_init(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_device_init: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return set_error(G4_ERR_UNSUPPORTED, "g4_device_init: device %d", dev);
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (g_init_done[dev]) return G4_OK;
  // softcap of every bf16 value: r16(30 * tanhf(s / 30)) with the host libm (gemma4_engine.cpp:1410)
  std::vector<float> tab(65536);
  for (uint32_t b = 0; b < 65536; ++b) {
    uint32_t u = b << 16;
    float s;
    std::memcpy(&s, &u, 4);
    float c = 30.0f * tanhf(s / 30.0f);
    uint32_t cu;
    std::memcpy(&cu, &c, 4);
    if ((cu & 0x7fffffffu) > 0x7f800000u) cu = ((cu >> 16) | 0x40u) << 16;
    else cu = ((cu + 0x7fffu + ((cu >> 16) & 1u)) >> 16) << 16;
    std::memcpy(&tab[b], &cu, 4);
  }
  e = cudaMemcpyToSymbol(g_cap_table, tab.data(), sizeof(float) * 65536);
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_device_init: %s", cudaGetErrorString(e));
  g_init_done[dev] = true;
  return G4_OK;
}

#define G4_NEED_INIT(fn) \
  G4_REQUIRE(device_ready(), fn ": call g4_device_init() on this device first")

// ------------------------------------------------------------------------------ packing ABI
extern "C" int g4_bf16p_codebook(const uint16_t* E, long long count, uint8_t* cb8, void* ws, size_t ws_bytes,
                                 void* stream) {
  G4_REQUIRE(E && cb8 && ws && count > 0, "g4_bf16p_codebook: bad arguments");
  if (ws_bytes < 256 * sizeof(unsigned long long)) return set_error(G4_ERR_NOMEM, "g4_bf16p_codebook: workspace < 2048 B");
  cudaStream_t st = as_stream(stream);
  unsigned long long* hist = static_cast<unsigned long long*>(ws);
  cudaMemsetAsync(hist, 0, 256 * sizeof(unsigned long long), st);
  k_exp_hist<<<1184, 256, 0, st>>>(E, count, hist);
  if (int rc = check_launch("k_exp_hist")) return rc;
  unsigned long long h[256];
  cudaError_t e = cudaMemcpyAsync(h, hist, sizeof h, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_bf16p_codebook: %s", cudaGetErrorString(e));
  int ord[256];
  for (int i = 0; i < 256; ++i) ord[i] = i;
  std::stable_sort(ord, ord + 256, [&](int a, int b) { return h[a] > h[b]; });
  for (int i = 0; i < 8; ++i) cb8[i] = (uint8_t)ord[i];
  return G4_OK;
}

static Codebook make_cb(const uint8_t* cb8) { Codebook c; std::memcpy(c.e, cb8, 8); return c; }

extern "C" int g4_bf16p_count(const uint16_t* E, int N, int K, const uint8_t* cb8, long long* exc_ptr, void* ws,
                              size_t ws_bytes, long long* total, void* stream) {
  G4_REQUIRE(E && cb8 && exc_ptr && ws && total && N > 0 && K > 0 && K % 32 == 0, "g4_bf16p_count: bad arguments");
  if (ws_bytes < sizeof(long long) * (size_t)N) return set_error(G4_ERR_NOMEM, "g4_bf16p_count: workspace < 8*N bytes");
  cudaStream_t st = as_stream(stream);
  long long* cnt = static_cast<long long*>(ws);
  k_bf16p_count<<<N, 256, 0, st>>>(E, K, make_cb(cb8), cnt);
  if (int rc = check_launch("k_bf16p_count")) return rc;
  k_scan_rows<<<1, 1024, 0, st>>>(cnt, N, exc_ptr);
  if (int rc = check_launch("k_scan_rows")) return rc;
  cudaError_t e = cudaMemcpyAsync(total, exc_ptr + N, sizeof(long long), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_bf16p_count: %s", cudaGetErrorString(e));
  return G4_OK;
}

extern "C" int g4_bf16p_pack(const uint16_t* E, int N, int K, const uint8_t* cb8, uint8_t* data,
                             const long long* exc_ptr, uint16_t* exc_col, float* exc_delta, void* stream) {
  G4_REQUIRE(E && cb8 && data && exc_ptr && N > 0 && K > 0 && K % 32 == 0, "g4_bf16p_pack: bad arguments");
  G4_REQUIRE(aligned(data, 4), "g4_bf16p_pack: data must be 4-byte aligned");
  const int G = K / 32;
  k_bf16p_fill<<<N, 64, sizeof(int) * G, as_stream(stream)>>>(E, K, make_cb(cb8), data, exc_ptr, exc_col, exc_delta);
  return check_launch("k_bf16p_fill");
}

static HeadPacked make_head(const uint8_t* data, const uint8_t* cb8, const long long* exc_ptr, const uint16_t* exc_col,
                            const float* exc_delta, int N, int K) {
  HeadPacked P;
  P.data = data; P.unp = nullptr; P.nib = nullptr; P.exc_ptr = exc_ptr; P.exc_col = exc_col; P.exc_delta = exc_delta; P.N = N; P.K = K;
  std::memcpy(&P.cb_lo, cb8, 4);
  std::memcpy(&P.cb_hi, cb8 + 4, 4);
  return P;
}

// The packed head as a 2D byte tensor [N][rowb] with boxes of [kBtRows][kBtBox]; cached per
// (address, N, K).  False when the driver entry point or the encoding is unavailable.
static bool head_tmap(const HeadPacked& P, CUtensorMap* out) {
  static std::mutex mu;
  struct Entry { const void* ptr; int N, K; CUtensorMap map; };
  static Entry cache[8];
  static int used = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].ptr == P.data && cache[i].N == P.N && cache[i].K == P.K) { *out = cache[i].map; return true; }
  const uint64_t rowb = (uint64_t)(P.K / 32) * 44;
  CUtensorMap m;
  if (!encode_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, P.data, rowb, (uint64_t)P.N, rowb, kBtBox, kBtRows,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
    return false;
  if (used < 8) cache[used++] = Entry{P.data, P.N, P.K, m};
  *out = m;
  return true;
}

// ---- unpacked layout of the packed head (64 bytes per group): the 32 weights as bf16p::pack
// represents them (codebook exponent, before the exception patches) stored as bf16, in the order
// that the two threads of a row consume them: bytes 32h..32h+31 hold half h's 16 weights, octets
// in chain order 0, 2, 1, 3, elements 8o+4h..8o+4h+3 within an octet.  The GEMV then turns each
// 32-bit word into two floats with one shift and one mask, instead of decoding exponent codes.
__device__ __forceinline__ uint32_t bf16p_bits(const uint32_t* w, int e, uint32_t cb_lo, uint32_t cb_hi) {
  const uint32_t idx = ((w[8] >> e) & 1u) | (((w[9] >> e) & 1u) << 1) | (((w[10] >> e) & 1u) << 2);
  const uint32_t ex = __byte_perm(cb_lo, cb_hi, idx) & 0xFFu;
  const uint32_t sm = (w[e >> 2] >> (8 * (e & 3))) & 0xFFu;
  return ((sm & 0x80u) << 8) | (ex << 7) | (sm & 0x7Fu);
}
__global__ void k_bf16u_pack(const uint8_t* __restrict__ data, long long ngroups, uint32_t cb_lo, uint32_t cb_hi,
                             uint8_t* __restrict__ out) {
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ngroups) return;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(data + g * 44);  // 4-byte aligned (44 = 4 * 11)
  uint32_t w[11];
#pragma unroll
  for (int i = 0; i < 11; ++i) w[i] = src[i];
  uint32_t* dst = reinterpret_cast<uint32_t*>(out + g * 64);
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int oi = 0; oi < 4; ++oi) {
      const int o8 = (oi == 1) ? 2 : (oi == 2 ? 1 : oi);
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        const int e = 8 * o8 + 4 * h + 2 * pr;
        dst[8 * h + 2 * oi + pr] = bf16p_bits(w, e, cb_lo, cb_hi) | (bf16p_bits(w, e + 1, cb_lo, cb_hi) << 16);
      }
    }
}

// ---- split-nibble layout of the packed head (48 bytes per group, two arrays): sm [N][G/4][2][4][16]
// holds the 32 sign/mantissa bytes of bf16p::pack, per block of 4 groups first the half-0 parts of
// the 4 groups, then the half-1 parts (so that the 16-byte loads of 4 rows x 2 halves land on 8
// distinct bank quads under the 128-byte swizzle), half h's 16 bytes of a group in the order that
// half consumes them (octets in chain order 0, 2, 1, 3; elements 8o+4h..8o+4h+3 within an octet: one
// 32-bit word per octet quad); codes [N][G][16] holds the same weights' 3-bit exponent codes as
// nibbles, half h's 16 at byte 8h (word w of a half: quads 2w and 2w+1, nibble k of a quad = its
// weight k).  A quad's
// four codes are one byte-permute selector over the 8-entry codebook: two permutes give the four
// weights' bf16 high-byte exponent bits (e >> 1) and low-byte bit ((e & 1) << 7), two masked merges
// add the sign and mantissa, and two permutes interleave the bytes into the two bf16 pairs that the
// unpacked layout stores, so the values are those of k_bf16u_rows_tma.  11% more bytes than bf16p
// (44 per group), 25% fewer than the unpacked copy (64).
__global__ void k_bf16n_pack(const uint8_t* __restrict__ data, long long ngroups, uint8_t* __restrict__ sm_out,
                             uint8_t* __restrict__ code_out) {
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ngroups) return;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(data + g * 44);  // 4-byte aligned (44 = 4 * 11)
  uint32_t w[11];
#pragma unroll
  for (int i = 0; i < 11; ++i) w[i] = src[i];
  uint8_t* smb = sm_out + (g >> 2) * 128 + (g & 3) * 16;  // + 64 h: half h's part
  uint32_t* cd = reinterpret_cast<uint32_t*>(code_out + g * 16);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t cw[2] = {0u, 0u};
#pragma unroll
    for (int oi = 0; oi < 4; ++oi) {
      const int o8 = (oi == 1) ? 2 : (oi == 2 ? 1 : oi);
      uint32_t smw = 0u, code = 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = 8 * o8 + 4 * h + k;
        const uint32_t idx = ((w[8] >> e) & 1u) | (((w[9] >> e) & 1u) << 1) | (((w[10] >> e) & 1u) << 2);
        smw |= ((w[e >> 2] >> (8 * (e & 3))) & 0xFFu) << (8 * k);
        code |= idx << (4 * k);
      }
      reinterpret_cast<uint32_t*>(smb + 64 * h)[oi] = smw;
      cw[oi >> 1] |= code << (16 * (oi & 1));
    }
    cd[2 * h] = cw[0];
    cd[2 * h + 1] = cw[1];
  }
}

// Two bf16 pairs (weights 0, 1 and 2, 3 of a quad) from its sign/mantissa word and code selector.
__device__ __forceinline__ void bf16n_quad(uint32_t smw, uint32_t sel, uint32_t cbh_lo, uint32_t cbh_hi, uint32_t cbl_lo,
                                           uint32_t cbl_hi, uint32_t& w0, uint32_t& w1) {
  const uint32_t hi4 = (smw & 0x80808080u) | __byte_perm(cbh_lo, cbh_hi, sel);
  const uint32_t lo4 = (smw & 0x7F7F7F7Fu) | __byte_perm(cbl_lo, cbl_hi, sel);
  w0 = __byte_perm(lo4, hi4, 0x5140);
  w1 = __byte_perm(lo4, hi4, 0x7362);
}

// Exact-head GEMV over the split-nibble layout, fed by the TMA, two threads per row (the arithmetic
// of k_bf16u_rows_tma): per pipeline item two tensor-map loads bring 4 groups of 128 rows, the
// sign/mantissa bytes as a [128][128 B] box under the 128-byte swizzle and the codes as a [128][64 B]
// box under the 64-byte swizzle (16-byte chunk c of row r lands at c ^ ((r >> 1) & 3)), into one of
// kBnNS stages of 24 KB.
constexpr int kBnRows = 128, kBnThreads = 256, kBnNS = 3;
constexpr int kBnSm = kBnRows * 128, kBnStage = kBnSm + kBnRows * 64;  // 4 groups per item
__host__ __device__ inline size_t head_nib_smem(int M, int K) {
  return 1024 + 128 + (size_t)kBnNS * kBnStage + (size_t)K * ((M + 1) / 2) * 8;
}

// Exact-head GEMV over the unpacked layout, fed by the TMA, two threads per row (as
// k_bf16p_rows_tma, same values): per pipeline item two tensor-map loads bring 4 groups (2 boxes
// of 128 bytes) of 128 rows under the 128-byte swizzle (16-byte chunk u of row r lands at chunk
// u ^ (r & 7)), so the half-row loads of a 16-byte phase hit distinct bank quads.  Two stages of
// 32 KB hold as many bytes in flight as four of 16 KB, with half the CTA barriers per byte.
constexpr int kBuRows = 128, kBuThreads = 256, kBuNS = 2, kBuBox = 128, kBuBoxes = 2;  // 4 groups per item
constexpr int kBuStage = kBuBoxes * kBuRows * kBuBox;
__host__ __device__ inline size_t head_unp_smem(int M, int K) {
  return 1024 + 128 + (size_t)kBuNS * kBuStage + (size_t)K * ((M + 1) / 2) * 8;
}

template <int M>
__global__ void __launch_bounds__(kBuThreads, 2) k_bf16u_rows_tma(const __grid_constant__ CUtensorMap tmap, HeadPacked P,
                                                                  const float* __restrict__ X, float* __restrict__ Y, int ldy,
                                                                  const int* __restrict__ gate) {
  constexpr int NP = (M + 1) / 2;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kBuNS];
  uint8_t* stages = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // 1024-byte aligned
  float2* xs = reinterpret_cast<float2*>(stages + (size_t)kBuNS * kBuStage);  // [K][NP]
  pdl_wait();
  pdl_trigger();
  if (gate != nullptr && *gate == 0) return;
  const int K = P.K, G = K >> 5, nch = G / (2 * kBuBoxes);
  const int nblk = (P.N + kBuRows - 1) / kBuRows;
  const int myblk = nblk > (int)blockIdx.x ? (nblk - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int nitems = myblk * nch;
  const int t = threadIdx.x, rl = t >> 1, half = t & 1;
  if (t == 0) {
    for (int b = 0; b < kBuNS; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i, int st) {  // thread 0
    const int blk = blockIdx.x + (i / nch) * gridDim.x, c = i % nch;
    mbar_expect_tx(&bars[st], (uint32_t)kBuStage);
#pragma unroll
    for (int b = 0; b < kBuBoxes; ++b)
      tma_load_2d(stages + (size_t)st * kBuStage + (size_t)b * kBuRows * kBuBox, &tmap, (c * kBuBoxes + b) * kBuBox,
                  blk * kBuRows, &bars[st]);
  };
  if (t == 0)
    for (int b = 0; b < kBuNS && b < nitems; ++b) issue(b, b);
  for (int i = t; i < K; i += kBuThreads) {
    float v[2 * NP];
#pragma unroll
    for (int m = 0; m < 2 * NP; ++m) v[m] = m < M ? X[(size_t)m * K + i] : 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) xs[(size_t)i * NP + p] = make_float2(v[2 * p], v[2 * p + 1]);
  }
  __syncthreads();
  const int hsh = 4 * half;
  float2 acc[4][NP];
  for (int i = 0; i < nitems; ++i) {
    const int st = i % kBuNS;
    const int blk = blockIdx.x + (i / nch) * gridDim.x, c = i % nch;
    const int n = blk * kBuRows + rl;
    if (!cta_wait(&bars[st], (uint32_t)(i / kBuNS) & 1u)) return;
    if (c == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int p = 0; p < NP; ++p) acc[j][p] = make_float2(0.f, 0.f);
    }
    const uint8_t* rowp = stages + (size_t)st * kBuStage + (size_t)rl * kBuBox;
    uint32_t wv[16 * kBuBoxes];  // this half's words of the item's groups (2 per box)
#pragma unroll
    for (int gg = 0; gg < 2 * kBuBoxes; ++gg)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int chunk = (gg & 1) * 4 + half * 2 + u;
        const uint4 t4 = *reinterpret_cast<const uint4*>(rowp + (size_t)(gg >> 1) * kBuRows * kBuBox + ((chunk ^ (rl & 7)) << 4));
        wv[8 * gg + 4 * u] = t4.x; wv[8 * gg + 4 * u + 1] = t4.y; wv[8 * gg + 4 * u + 2] = t4.z; wv[8 * gg + 4 * u + 3] = t4.w;
      }
    __syncthreads();  // every row has its words in registers: the stage can be refilled
    if (t == 0 && i + kBuNS < nitems) {
      fence_proxy_async_smem();
      issue(i + kBuNS, st);
    }
#pragma unroll
    for (int gg = 0; gg < 2 * kBuBoxes; ++gg) {
      const int g = c * 2 * kBuBoxes + gg;
      const float2* xg = xs + ((size_t)g * 32 + hsh) * NP;
#pragma unroll
      for (int oi = 0; oi < 4; ++oi) {
        const int o8 = (oi == 1) ? 2 : (oi == 2 ? 1 : oi);  // element octets in chain order 0, 2, 1, 3
        const uint32_t w0 = wv[8 * gg + 2 * oi], w1 = wv[8 * gg + 2 * oi + 1];
        const float wk[4] = {__uint_as_float(w0 << 16), __uint_as_float(w0 & 0xFFFF0000u), __uint_as_float(w1 << 16),
                             __uint_as_float(w1 & 0xFFFF0000u)};
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int p = 0; p < NP; ++p)
            acc[k][p] = __ffma2_rn(make_float2(wk[k], wk[k]), xg[(8 * o8 + k) * NP + p], acc[k][p]);
      }
    }
    if (c == nch - 1) {
      // lanes 4..7 come from the other half; fadd is commutative, so both halves hold
      // ((v0 + v4) + (v1 + v5)) + ((v2 + v6) + (v3 + v7)) bit for bit
      float y[2 * NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        float2 w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          w[k].x = __shfl_xor_sync(0xffffffffu, acc[k][p].x, 1);
          w[k].y = __shfl_xor_sync(0xffffffffu, acc[k][p].y, 1);
        }
        y[2 * p] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][p].x, w[0].x), __fadd_rn(acc[1][p].x, w[1].x)),
                             __fadd_rn(__fadd_rn(acc[2][p].x, w[2].x), __fadd_rn(acc[3][p].x, w[3].x)));
        y[2 * p + 1] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][p].y, w[0].y), __fadd_rn(acc[1][p].y, w[1].y)),
                                 __fadd_rn(__fadd_rn(acc[2][p].y, w[2].y), __fadd_rn(acc[3][p].y, w[3].y)));
      }
      if (n < P.N) {
        float yo[NP];  // this half's activation rows 2p + half
#pragma unroll
        for (int p = 0; p < NP; ++p) yo[p] = half ? y[2 * p + 1] : y[2 * p];
        for (long long e = P.exc_ptr[n]; e < P.exc_ptr[n + 1]; ++e) {  // CSR order, unfused (bf16_exp3_head.h:103)
          const float dl = P.exc_delta[e];
          const int col = P.exc_col[e];
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            const float2 xv = xs[(size_t)col * NP + p];
            yo[p] = __fadd_rn(yo[p], __fmul_rn(dl, half ? xv.y : xv.x));
          }
        }
#pragma unroll
        for (int p = 0; p < NP; ++p)
          if (2 * p + half < M) Y[(size_t)(2 * p + half) * ldy + n] = yo[p];
      }
    }
  }
}

template <int M>
__global__ void __launch_bounds__(kBnThreads, 2) k_bf16n_rows_tma(const __grid_constant__ CUtensorMap tsm,
                                                                  const __grid_constant__ CUtensorMap tcode, HeadPacked P,
                                                                  const float* __restrict__ X, float* __restrict__ Y, int ldy,
                                                                  const int* __restrict__ gate) {
  constexpr int NP = (M + 1) / 2;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kBnNS];
  uint8_t* stages = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // 1024-byte aligned
  float2* xs = reinterpret_cast<float2*>(stages + (size_t)kBnNS * kBnStage);  // [K][NP]
  pdl_wait();
  pdl_trigger();
  if (gate != nullptr && *gate == 0) return;
  const int K = P.K, G = K >> 5, nch = G / 4;
  const int nblk = (P.N + kBnRows - 1) / kBnRows;
  const int myblk = nblk > (int)blockIdx.x ? (nblk - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int nitems = myblk * nch;
  const int t = threadIdx.x, rl = t >> 1, half = t & 1;
  // codebook bytes split into the bf16 high-byte bits (e >> 1) and low-byte bit ((e & 1) << 7)
  const uint32_t cbh_lo = (P.cb_lo >> 1) & 0x7F7F7F7Fu, cbh_hi = (P.cb_hi >> 1) & 0x7F7F7F7Fu;
  const uint32_t cbl_lo = (P.cb_lo << 7) & 0x80808080u, cbl_hi = (P.cb_hi << 7) & 0x80808080u;
  if (t == 0) {
    for (int b = 0; b < kBnNS; ++b) mbar_init(&bars[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i, int st) {  // thread 0
    const int blk = blockIdx.x + (i / nch) * gridDim.x, c = i % nch;
    uint8_t* sb = stages + (size_t)st * kBnStage;
    mbar_expect_tx(&bars[st], (uint32_t)kBnStage);
    tma_load_2d(sb, &tsm, c * 128, blk * kBnRows, &bars[st]);
    tma_load_2d(sb + kBnSm, &tcode, c * 64, blk * kBnRows, &bars[st]);
  };
  if (t == 0)
    for (int b = 0; b < kBnNS && b < nitems; ++b) issue(b, b);
  for (int i = t; i < K; i += kBnThreads) {
    float v[2 * NP];
#pragma unroll
    for (int m = 0; m < 2 * NP; ++m) v[m] = m < M ? X[(size_t)m * K + i] : 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) xs[(size_t)i * NP + p] = make_float2(v[2 * p], v[2 * p + 1]);
  }
  __syncthreads();
  const int hsh = 4 * half;
  float2 acc[4][NP];
  for (int i = 0; i < nitems; ++i) {
    const int st = i % kBnNS;
    const int blk = blockIdx.x + (i / nch) * gridDim.x, c = i % nch;
    const int n = blk * kBnRows + rl;
    if (!cta_wait(&bars[st], (uint32_t)(i / kBnNS) & 1u)) return;
    if (c == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int p = 0; p < NP; ++p) acc[j][p] = make_float2(0.f, 0.f);
    }
    const uint8_t* smrow = stages + (size_t)st * kBnStage + (size_t)rl * 128;
    const uint8_t* cdrow = stages + (size_t)st * kBnStage + kBnSm + (size_t)rl * 64;
    uint32_t smv[16], cdv[8];  // this half's sign/mantissa words and code words of the item's 4 groups
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) {
      const uint4 s4 = *reinterpret_cast<const uint4*>(smrow + (((gg + 4 * half) ^ (rl & 7)) << 4));
      smv[4 * gg] = s4.x; smv[4 * gg + 1] = s4.y; smv[4 * gg + 2] = s4.z; smv[4 * gg + 3] = s4.w;
      const uint2 c2 = *reinterpret_cast<const uint2*>(cdrow + ((gg ^ ((rl >> 1) & 3)) << 4) + 8 * half);
      cdv[2 * gg] = c2.x; cdv[2 * gg + 1] = c2.y;
    }
    __syncthreads();  // every row has its words in registers: the stage can be refilled
    if (t == 0 && i + kBnNS < nitems) {
      fence_proxy_async_smem();
      issue(i + kBnNS, st);
    }
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) {
      const int g = c * 4 + gg;
      const float2* xg = xs + ((size_t)g * 32 + hsh) * NP;
#pragma unroll
      for (int oi = 0; oi < 4; ++oi) {
        const int o8 = (oi == 1) ? 2 : (oi == 2 ? 1 : oi);  // element octets in chain order 0, 2, 1, 3
        const uint32_t cw = cdv[2 * gg + (oi >> 1)];
        uint32_t w0, w1;
        bf16n_quad(smv[4 * gg + oi], (oi & 1) ? (cw >> 16) : (cw & 0xFFFFu), cbh_lo, cbh_hi, cbl_lo, cbl_hi, w0, w1);
        const float wk[4] = {__uint_as_float(w0 << 16), __uint_as_float(w0 & 0xFFFF0000u), __uint_as_float(w1 << 16),
                             __uint_as_float(w1 & 0xFFFF0000u)};
        // the quad's activations: 4 x NP consecutive pairs, 2 x NP 16-byte loads
        const float4* x4 = reinterpret_cast<const float4*>(xg + 8 * o8 * NP);
        float4 xv[2 * NP];
#pragma unroll
        for (int j = 0; j < 2 * NP; ++j) xv[j] = x4[j];
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            const int f = k * NP + p;
            const float2 xp = (f & 1) ? make_float2(xv[f >> 1].z, xv[f >> 1].w) : make_float2(xv[f >> 1].x, xv[f >> 1].y);
            acc[k][p] = __ffma2_rn(make_float2(wk[k], wk[k]), xp, acc[k][p]);
          }
      }
    }
    if (c == nch - 1) {
      // lanes 4..7 come from the other half; both halves hold the same hsum8 (as k_bf16u_rows_tma)
      float y[2 * NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        float2 w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          w[k].x = __shfl_xor_sync(0xffffffffu, acc[k][p].x, 1);
          w[k].y = __shfl_xor_sync(0xffffffffu, acc[k][p].y, 1);
        }
        y[2 * p] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][p].x, w[0].x), __fadd_rn(acc[1][p].x, w[1].x)),
                             __fadd_rn(__fadd_rn(acc[2][p].x, w[2].x), __fadd_rn(acc[3][p].x, w[3].x)));
        y[2 * p + 1] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][p].y, w[0].y), __fadd_rn(acc[1][p].y, w[1].y)),
                                 __fadd_rn(__fadd_rn(acc[2][p].y, w[2].y), __fadd_rn(acc[3][p].y, w[3].y)));
      }
      if (n < P.N) {
        float yo[NP];  // this half's activation rows 2p + half
#pragma unroll
        for (int p = 0; p < NP; ++p) yo[p] = half ? y[2 * p + 1] : y[2 * p];
        for (long long e = P.exc_ptr[n]; e < P.exc_ptr[n + 1]; ++e) {  // CSR order, unfused (bf16_exp3_head.h:103)
          const float dl = P.exc_delta[e];
          const int col = P.exc_col[e];
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            const float2 xv = xs[(size_t)col * NP + p];
            yo[p] = __fadd_rn(yo[p], __fmul_rn(dl, half ? xv.y : xv.x));
          }
        }
#pragma unroll
        for (int p = 0; p < NP; ++p)
          if (2 * p + half < M) Y[(size_t)(2 * p + half) * ldy + n] = yo[p];
      }
    }
  }
}

// The split-nibble head as two 2D byte tensors, [N][G*32] in [128][128 B] boxes under the 128-byte
// swizzle and [N][G*16] in [128][64 B] boxes under the 64-byte swizzle; cached per (address, N, K).
static bool head_nib_tmaps(const HeadPacked& P, CUtensorMap* tsm, CUtensorMap* tcode) {
  static std::mutex mu;
  struct Entry { const void* ptr; int N, K; CUtensorMap ms, mc; };
  static Entry cache[8];
  static int used = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].ptr == P.nib && cache[i].N == P.N && cache[i].K == P.K) {
      *tsm = cache[i].ms;
      *tcode = cache[i].mc;
      return true;
    }
  const uint64_t G = (uint64_t)P.K / 32;
  const uint8_t* codes = P.nib + (size_t)P.N * G * 32;
  CUtensorMap ms, mc;
  if (!encode_tmap_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT8, P.nib, G * 32, (uint64_t)P.N, G * 32, 128, kBnRows,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&mc, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, G * 16, (uint64_t)P.N, G * 16, 64, kBnRows,
                      CU_TENSOR_MAP_SWIZZLE_64B))
    return false;
  if (used < 8) cache[used++] = Entry{P.nib, P.N, P.K, ms, mc};
  *tsm = ms;
  *tcode = mc;
  return true;
}

// The unpacked head as a 2D byte tensor [N][G*64] with boxes of [kBuRows][kBuBox] under the
// 128-byte swizzle; cached per (address, N, K).
static bool head_unp_tmap(const HeadPacked& P, CUtensorMap* out) {
  static std::mutex mu;
  struct Entry { const void* ptr; int N, K; CUtensorMap map; };
  static Entry cache[8];
  static int used = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].ptr == P.unp && cache[i].N == P.N && cache[i].K == P.K) { *out = cache[i].map; return true; }
  const uint64_t rowb = (uint64_t)(P.K / 32) * 64;
  CUtensorMap m;
  if (!encode_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, P.unp, rowb, (uint64_t)P.N, rowb, kBuBox, kBuRows,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return false;
  if (used < 8) cache[used++] = Entry{P.unp, P.N, P.K, m};
  *out = m;
  return true;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

template <int M>
static int launch_head_gemv(const HeadPacked& P, const float* X, float* Y, int ldy, const int* gate, cudaStream_t st) {
  const char* hv = getenv("G4_HEAD_GEMV");  // "direct" / "octet" select other variants (experiments)
  CUtensorMap tm, tm2;
  const size_t nsmem = head_nib_smem(M, P.K);
  if (P.nib != nullptr && P.K % 128 == 0 && aligned(P.nib, 16) && nsmem <= 113 * 1024 && head_nib_tmaps(P, &tm, &tm2)) {
    cudaFuncSetAttribute(k_bf16n_rows_tma<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)nsmem);
    cudaFuncSetAttribute(k_bf16n_rows_tma<M>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);  // 2 CTAs per SM
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_bf16n_rows_tma<M>, kBnThreads, nsmem) != cudaSuccess || occ < 1)
      occ = 1;
    const int nblk = (P.N + kBnRows - 1) / kBnRows;
    return launch("k_bf16n_rows_tma", k_bf16n_rows_tma<M>, dim3(std::min(nblk, num_sms() * occ)), dim3(kBnThreads), nsmem,
                  st, tm, tm2, P, X, Y, ldy, gate);
  }
  if (P.nib != nullptr && P.data == nullptr && P.unp == nullptr)
    return set_error(G4_ERR_UNSUPPORTED, "bf16p split-nibble GEMV: K=%d (a multiple of 128 and a 16-byte aligned head needed)", P.K);
  const size_t usmem = head_unp_smem(M, P.K);
  if (P.unp != nullptr && P.K % (64 * kBuBoxes) == 0 && aligned(P.unp, 16) && usmem <= 113 * 1024 && head_unp_tmap(P, &tm)) {
    cudaFuncSetAttribute(k_bf16u_rows_tma<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)usmem);
    cudaFuncSetAttribute(k_bf16u_rows_tma<M>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);  // 2 CTAs per SM
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_bf16u_rows_tma<M>, kBuThreads, usmem) != cudaSuccess || occ < 1)
      occ = 1;
    const int nblk = (P.N + kBuRows - 1) / kBuRows;
    return launch("k_bf16u_rows_tma", k_bf16u_rows_tma<M>, dim3(std::min(nblk, num_sms() * occ)), dim3(kBuThreads), usmem,
                  st, tm, P, X, Y, ldy, gate);
  }
  if (P.data == nullptr)
    return set_error(G4_ERR_UNSUPPORTED, "bf16p unpacked GEMV: K=%d (a multiple of 64 and a 16-byte aligned head needed)", P.K);
  const size_t tsmem = head_tma_smem(M, P.K);
  if (!hv && P.K % 128 == 0 && (P.K / 32) * 44 % 16 == 0 && aligned(P.data, 16) && tsmem <= 227 * 1024 && head_tmap(P, &tm)) {
    cudaFuncSetAttribute(k_bf16p_rows_tma<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsmem);
    cudaFuncSetAttribute(k_bf16p_rows_tma<M>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);  // 2 CTAs per SM
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_bf16p_rows_tma<M>, kBtThreads, tsmem) != cudaSuccess || occ < 1)
      occ = 1;
    const int nblk = (P.N + kBtRows - 1) / kBtRows;
    return launch("k_bf16p_rows_tma", k_bf16p_rows_tma<M>, dim3(std::min(nblk, num_sms() * occ)), dim3(kBtThreads), tsmem,
                  st, tm, P, X, Y, ldy, gate);
  }
  const size_t rsmem = head_rows_smem(M, P.K);
  if (P.K % 128 == 0 && rsmem <= 100 * 1024 && aligned(P.data, 16) && !(hv && hv[0] == 'o')) {
    if (rsmem > 40 * 1024) cudaFuncSetAttribute(k_bf16p_rows<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsmem);
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_bf16p_rows<M>, kBrThreads, rsmem) != cudaSuccess || occ < 1)
      occ = 1;
    const int nblk = (P.N + kBrThreads - 1) / kBrThreads;
    return launch("k_bf16p_rows", k_bf16p_rows<M>, dim3(std::min(nblk, num_sms() * occ)), dim3(kBrThreads), rsmem, st, P,
                  X, Y, ldy, gate);
  }
  const size_t smem = head_smem_bytes(M, P.K);
  if (P.K % 256 == 0 && smem <= 227 * 1024 && aligned(P.data, 16)) {
    cudaFuncSetAttribute(k_bf16p_gemv_staged<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int nblk = (P.N + kHeadBlkRows - 1) / kHeadBlkRows;
    return launch("k_bf16p_gemv_staged", k_bf16p_gemv_staged<M>, dim3(std::min(nblk, num_sms())), dim3(256), smem, st, P,
                  X, Y, ldy, gate);
  }
  return launch("k_bf16p_gemv", k_bf16p_gemv<M>, dim3((P.N + 31) / 32), dim3(256), 0, st, P, X, Y, ldy, gate);
}
static int head_gemv(const HeadPacked& P, const float* X, int M, float* Y, int ldy, const int* gate, cudaStream_t st) {
  switch (M) {
    case 1: return launch_head_gemv<1>(P, X, Y, ldy, gate, st);
    case 2: return launch_head_gemv<2>(P, X, Y, ldy, gate, st);
    case 3: return launch_head_gemv<3>(P, X, Y, ldy, gate, st);
    default: return launch_head_gemv<4>(P, X, Y, ldy, gate, st);
  }
}

extern "C" int g4_bf16p_gemm(const uint8_t* data, const uint8_t* cb8, const long long* exc_ptr, const uint16_t* exc_col,
                             const float* exc_delta, int N, int K, const float* X, int M, float* Y, int ldy,
                             void* stream) {
  G4_REQUIRE(data && cb8 && exc_ptr && X && Y && N > 0 && K > 0 && K % 32 == 0 && M >= 1 && M <= 4 && ldy >= N,
             "g4_bf16p_gemm: bad arguments N=%d K=%d M=%d", N, K, M);
  return head_gemv(make_head(data, cb8, exc_ptr, exc_col, exc_delta, N, K), X, M, Y, ldy, nullptr, as_stream(stream));
}

extern "C" int g4_bf16p_unpack(const uint8_t* data, const uint8_t* cb8, int N, int K, uint8_t* unp, void* stream) {
  G4_REQUIRE(data && cb8 && unp, "g4_bf16p_unpack: null pointer");
  G4_REQUIRE(N > 0 && K > 0 && K % 32 == 0, "g4_bf16p_unpack: bad shape N=%d K=%d", N, K);
  G4_REQUIRE(aligned(data, 4) && aligned(unp, 16), "g4_bf16p_unpack: data 4-byte, unp 16-byte aligned");
  const long long ng = (long long)N * (K / 32);
  uint32_t cb_lo, cb_hi;
  std::memcpy(&cb_lo, cb8, 4);
  std::memcpy(&cb_hi, cb8 + 4, 4);
  k_bf16u_pack<<<(unsigned)((ng + 255) / 256), 256, 0, as_stream(stream)>>>(data, ng, cb_lo, cb_hi, unp);
  return check_launch("k_bf16u_pack");
}

extern "C" size_t g4_bf16p_nib_bytes(int N, int K) { return (size_t)N * (size_t)(K / 32) * 48; }

extern "C" int g4_bf16p_nib_pack(const uint8_t* data, int N, int K, uint8_t* nib, void* stream) {
  G4_REQUIRE(data && nib, "g4_bf16p_nib_pack: null pointer");
  G4_REQUIRE(N > 0 && K > 0 && K % 128 == 0, "g4_bf16p_nib_pack: bad shape N=%d K=%d (K % 128 == 0)", N, K);
  G4_REQUIRE(aligned(data, 4) && aligned(nib, 16), "g4_bf16p_nib_pack: data 4-byte, nib 16-byte aligned");
  const long long ng = (long long)N * (K / 32);
  k_bf16n_pack<<<(unsigned)((ng + 255) / 256), 256, 0, as_stream(stream)>>>(data, ng, nib, nib + (size_t)ng * 32);
  return check_launch("k_bf16n_pack");
}

extern "C" int g4_bf16p_nib_gemm(const uint8_t* nib, const uint8_t* cb8, const long long* exc_ptr, const uint16_t* exc_col,
                                 const float* exc_delta, int N, int K, const float* X, int M, float* Y, int ldy,
                                 void* stream) {
  G4_REQUIRE(nib && cb8 && exc_ptr && X && Y, "g4_bf16p_nib_gemm: null pointer");
  G4_REQUIRE(M >= 1 && M <= 4 && N > 0 && K > 0 && K % 128 == 0 && ldy >= N, "g4_bf16p_nib_gemm: bad shape M=%d N=%d K=%d",
             M, N, K);
  HeadPacked P = make_head(nullptr, cb8, exc_ptr, exc_col, exc_delta, N, K);
  P.nib = nib;
  return head_gemv(P, X, M, Y, ldy, nullptr, as_stream(stream));
}

extern "C" int g4_bf16p_unpacked_gemm(const uint8_t* unp, const long long* exc_ptr, const uint16_t* exc_col,
                                      const float* exc_delta, int N, int K, const float* X, int M, float* Y, int ldy,
                                      void* stream) {
  G4_REQUIRE(unp && exc_ptr && X && Y, "g4_bf16p_unpacked_gemm: null pointer");
  G4_REQUIRE(M >= 1 && M <= 4 && N > 0 && K > 0 && K % 64 == 0 && ldy >= N,
             "g4_bf16p_unpacked_gemm: bad shape M=%d N=%d K=%d", M, N, K);
  const uint8_t zero_cb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  HeadPacked P = make_head(nullptr, zero_cb, exc_ptr, exc_col, exc_delta, N, K);
  P.unp = unp;
  return head_gemv(P, X, M, Y, ldy, nullptr, as_stream(stream));
}

static int pick(const float* Y, int M, int N, int ldy, int* slots, int* out, const int* gate, cudaStream_t st) {
  if (int rc_ = launch("k_pick_init", k_pick_init, dim3(1), dim3(32), 0, st, slots, M)) return rc_;
  if (int rc_ = launch("k_pick_max", k_pick_max, dim3(dim3(296, M)), dim3(256), 0, st, Y, N, ldy, slots, gate)) return rc_;
  if (int rc_ = launch("k_pick_idx", k_pick_idx, dim3(dim3(296, M)), dim3(256), 0, st, Y, N, ldy, slots, gate)) return rc_;
  if (out) if (int rc_ = launch("k_pick_out", k_pick_out, dim3(1), dim3(32), 0, st, slots, M, out, gate)) return rc_;
  return check_launch("head pick");
}

extern "C" int g4_head_argmax(const float* Y, int M, int N, int ldy, int* out_idx, void* ws, size_t ws_bytes,
                              void* stream) {
  G4_REQUIRE(Y && out_idx && ws && M >= 1 && M <= 16 && N > 0 && ldy >= N, "g4_head_argmax: bad arguments");
  G4_NEED_INIT("g4_head_argmax");
  if (ws_bytes < sizeof(int) * 2 * (size_t)M) return set_error(G4_ERR_NOMEM, "g4_head_argmax: workspace < 8*M bytes");
  return pick(Y, M, N, ldy, static_cast<int*>(ws), out_idx, nullptr, as_stream(stream));
}

extern "C" int g4_screen_build(const uint16_t* E, int N, int K, uint8_t* W4p, uint16_t* S4, float* coef, void* stream) {
  G4_REQUIRE(E && W4p && S4 && coef && N > 0 && K > 0 && K % 32 == 0, "g4_screen_build: bad arguments");
  G4_REQUIRE(aligned(W4p, 16), "g4_screen_build: W4p must be 16-byte aligned");
  k_screen_build<<<N, 64, sizeof(float) * (K / 32), as_stream(stream)>>>(E, K, W4p, S4, coef);
  return check_launch("k_screen_build");
}

extern "C" size_t g4_head_screen_ws_bytes(int M, int N, int lim) { return screen_ws_layout(M, N, lim, nullptr, nullptr); }

extern "C" int g4_head_screen(const uint8_t* W4p, const uint16_t* S4, const float* coef, const uint8_t* data,
                              const uint8_t* cb8, const long long* exc_ptr, const uint16_t* exc_col,
                              const float* exc_delta, int N, int K, const float* H, int M, int lim, int* out_idx,
                              int* out_nsurv, void* ws, size_t ws_bytes, void* stream) {
  return head_screen_impl(W4p, S4, coef, data, nullptr, cb8, exc_ptr, exc_col, exc_delta, N, K, H, M, lim, out_idx,
                          out_nsurv, ws, ws_bytes, stream);
}

// The screen with the fallback head GEMV over the unpacked copy of the head when unp is set
// (the rescoring of survivors reads the bf16p rows).
int g4::head_screen_impl(const uint8_t* W4p, const uint16_t* S4, const float* coef, const uint8_t* data, const uint8_t* unp,
                         const uint8_t* cb8, const long long* exc_ptr, const uint16_t* exc_col, const float* exc_delta,
                         int N, int K, const float* H, int M, int lim, int* out_idx, int* out_nsurv, void* ws,
                         size_t ws_bytes, void* stream, int* policy, const uint8_t* nib) {
  G4_REQUIRE(W4p && S4 && coef && data && cb8 && exc_ptr && H && out_idx && out_nsurv && ws,
             "g4_head_screen: null pointer");
  G4_REQUIRE(M >= 1 && M <= 4 && N > 0 && K > 0 && K % 256 == 0 && lim > 0, "g4_head_screen: bad shape M=%d N=%d K=%d", M,
             N, K);
  G4_NEED_INIT("g4_head_screen");
  const size_t need = screen_ws_layout(M, N, lim, nullptr, nullptr);
  if (ws_bytes < need) return set_error(G4_ERR_NOMEM, "g4_head_screen: workspace %zu < %zu bytes", ws_bytes, need);
  G4_REQUIRE(aligned(ws, 256), "g4_head_screen: workspace must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  ScreenWs w;
  screen_ws_layout(M, N, lim, &w, static_cast<char*>(ws));
  w.pol = policy;
  HeadPacked P = make_head(data, cb8, exc_ptr, exc_col, exc_delta, N, K);
  P.unp = unp;
  P.nib = nib;
  if (int rc_ = launch("k_screen_init", k_screen_init, dim3(M), dim3(32), 0, st, H, K, M, w)) return rc_;
  if (int rc = check_launch("k_screen_init")) return rc;
  if (int rc = w4g32_gemm_gated(W4p, S4, H, M, N, K, w.s, N, policy ? policy + 1 : nullptr, st)) return rc;
  if (int rc_ = launch("k_screen_L", k_screen_L, dim3(dim3(296, M)), dim3(256), 0, st, coef, N, w)) return rc_;
  if (int rc_ = launch("k_screen_thr", k_screen_thr, dim3(1), dim3(32), 0, st, M, w)) return rc_;
  if (int rc_ = launch("k_screen_collect", k_screen_collect, dim3(dim3(296, M)), dim3(256), 0, st, coef, N, lim, w)) return rc_;
  if (int rc_ = launch("k_screen_rescore", k_screen_rescore, dim3(dim3((lim + 31) / 32, M)), dim3(256), 0, st, P, H, lim, w)) return rc_;
  if (int rc_ = launch("k_screen_pick", k_screen_pick, dim3(M), dim3(256), 0, st, lim, w, out_idx, out_nsurv)) return rc_;
  if (int rc = check_launch("screen")) return rc;
  // fallback: full exact head for all rows, gated on the device flag
  if (int rc = head_gemv(P, H, M, w.s, N, w.fb, st)) return rc;
  if (int rc = pick(w.s, M, N, N, w.slots, nullptr, w.fb, st)) return rc;
  if (int rc_ = launch("k_screen_fb_out", k_screen_fb_out, dim3(1), dim3(32), 0, st, w.slots, M, w, out_idx)) return rc_;
  return check_launch("k_screen_fb_out");
}

// ---- vocab-parallel screen phases (one shard of N rows of the head on this device)
extern "C" int g4_head_screen_shard_bound(const uint8_t* W4p, const uint16_t* S4, const float* coef, int N, int K,
                                          const float* H, int M, int lim, float* L_out, void* ws, size_t ws_bytes,
                                          void* stream) {
  G4_REQUIRE(W4p && S4 && coef && H && L_out && ws, "g4_head_screen_shard_bound: null pointer");
  G4_REQUIRE(M >= 1 && M <= 4 && N > 0 && K > 0 && K % 256 == 0 && lim > 0, "g4_head_screen_shard_bound: bad shape");
  G4_NEED_INIT("g4_head_screen_shard_bound");
  const size_t need = screen_ws_layout(M, N, lim, nullptr, nullptr);
  if (ws_bytes < need) return set_error(G4_ERR_NOMEM, "g4_head_screen_shard_bound: workspace %zu < %zu bytes", ws_bytes, need);
  G4_REQUIRE(aligned(ws, 256), "g4_head_screen_shard_bound: workspace must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  ScreenWs w;
  screen_ws_layout(M, N, lim, &w, static_cast<char*>(ws));
  if (int rc_ = launch("k_screen_init", k_screen_init, dim3(M), dim3(32), 0, st, H, K, M, w)) return rc_;
  if (int rc = g4_w4g32_gemm(W4p, S4, H, nullptr, M, N, K, w.s, N, stream)) return rc;
  if (int rc_ = launch("k_screen_L", k_screen_L, dim3(dim3(296, M)), dim3(256), 0, st, coef, N, w)) return rc_;
  if (int rc_ = launch("k_shard_L_out", k_shard_L_out, dim3(1), dim3(32), 0, st, w, M, L_out)) return rc_;
  return check_launch("g4_head_screen_shard_bound");
}

extern "C" int g4_head_screen_shard_select(const float* coef, const uint8_t* data, const uint8_t* unp, const uint8_t* cb8,
                                           const long long* exc_ptr, const uint16_t* exc_col, const float* exc_delta,
                                           int N, int K, const float* H, int M, int lim, const float* L,
                                           float* vmax_out, int* out_nsurv, void* ws, size_t ws_bytes, void* stream) {
  G4_REQUIRE(coef && data && cb8 && exc_ptr && H && L && vmax_out && out_nsurv && ws,
             "g4_head_screen_shard_select: null pointer");
  G4_REQUIRE(M >= 1 && M <= 4 && N > 0 && K > 0 && K % 256 == 0 && lim > 0, "g4_head_screen_shard_select: bad shape");
  const size_t need = screen_ws_layout(M, N, lim, nullptr, nullptr);
  if (ws_bytes < need) return set_error(G4_ERR_NOMEM, "g4_head_screen_shard_select: workspace %zu < %zu bytes", ws_bytes, need);
  cudaStream_t st = as_stream(stream);
  ScreenWs w;
  screen_ws_layout(M, N, lim, &w, static_cast<char*>(ws));
  HeadPacked P = make_head(data, cb8, exc_ptr, exc_col, exc_delta, N, K);
  P.unp = unp;
  if (int rc_ = launch("k_shard_set_L", k_shard_set_L, dim3(1), dim3(32), 0, st, L, M, w)) return rc_;
  if (int rc_ = launch("k_screen_thr", k_screen_thr, dim3(1), dim3(32), 0, st, M, w)) return rc_;
  if (int rc_ = launch("k_screen_collect", k_screen_collect, dim3(dim3(296, M)), dim3(256), 0, st, coef, N, lim, w)) return rc_;
  if (int rc_ = launch("k_screen_rescore", k_screen_rescore, dim3(dim3((lim + 31) / 32, M)), dim3(256), 0, st, P, H, lim, w)) return rc_;
  // fallback: the shard's full exact head and its max, gated on the device flag
  if (int rc = head_gemv(P, H, M, w.s, N, w.fb, st)) return rc;
  if (int rc_ = launch("k_pick_init", k_pick_init, dim3(1), dim3(32), 0, st, w.slots, M)) return rc_;
  if (int rc_ = launch("k_pick_max", k_pick_max, dim3(dim3(296, M)), dim3(256), 0, st, w.s, N, N, w.slots, w.fb)) return rc_;
  if (int rc_ = launch("k_shard_vmax", k_shard_vmax, dim3(M), dim3(256), 0, st, lim, w, w.slots, vmax_out, out_nsurv)) return rc_;
  return check_launch("g4_head_screen_shard_select");
}

extern "C" int g4_head_screen_shard_pick(int N, int M, int lim, int row0, const float* gmax, int* idx_out, void* ws,
                                         size_t ws_bytes, void* stream) {
  G4_REQUIRE(gmax && idx_out && ws, "g4_head_screen_shard_pick: null pointer");
  G4_REQUIRE(M >= 1 && M <= 4 && N > 0 && lim > 0 && row0 >= 0, "g4_head_screen_shard_pick: bad shape");
  const size_t need = screen_ws_layout(M, N, lim, nullptr, nullptr);
  if (ws_bytes < need) return set_error(G4_ERR_NOMEM, "g4_head_screen_shard_pick: workspace %zu < %zu bytes", ws_bytes, need);
  ScreenWs w;
  screen_ws_layout(M, N, lim, &w, static_cast<char*>(ws));
  if (int rc_ = launch("k_shard_pick", k_shard_pick, dim3(M), dim3(1024), 0, as_stream(stream), gmax, lim, w, N, row0, idx_out))
    return rc_;
  return check_launch("k_shard_pick");
}
