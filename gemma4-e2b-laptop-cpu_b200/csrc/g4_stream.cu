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
constexpr int kSegNS = 6;                                       // ring slots
constexpr int kSegKmax = 8192;
constexpr int kSegRow = 2048;                                   // hidden width handled by the prologues

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
      __nanosleep(64);
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

// ------------------------------------------------------------------------- rows in registers
// Thread t (< 256) owns float4 blocks t and t + 256 of each of the M rows (elements 4f..4f+3).
template <int M>
struct Rows {
  float4 v[M][2];
};

// Exponent keys for the exactness test (see rows_rms): bytes (kmax, 255 - kmin) of the nonzero
// elements' biased exponents; a value that is not bf16-valued or not finite fails the test.
__device__ __forceinline__ uint32_t seg_ekeys(float x) {
  const uint32_t b = __float_as_uint(x) & 0x7FFFFFFFu;
  const uint32_t e = max(b >> 23, 1u);
  const uint32_t key = ((b & 0xFFFFu) != 0u || e == 255u) ? ((255u << 8) | 254u) : ((e << 8) | (255u - e));
  return b == 0u ? 0u : key;
}

// RMS scales of M rows of n (<= 2048) elements in the reference's order (ss_avx2, :326-343): per
// row the sum of squares in double over 16 partials (element j to partial j % 16, each in element
// order), combined ((p_b + p_4+b) + (p_8+b + p_12+b)), then (t0 + t2) + (t1 + t3);
// r = 1 / sqrtf((float)(ss / n) + 1e-6).  A partial whose elements are bf16-valued with nonzero
// exponents spanning at most 15 is an exact sum in double in any order (every square is a multiple
// of 2^(2 e_min - 268) and 128 of them stay below 2^53 such units), so it is summed as a tree;
// any other partial runs the sequential chain over xs (the rows in shared memory, stride n).
template <int M>
__device__ void rows_rms(const Rows<M>& rw, const float* xs, int n, SegShared& sh, float (&r)[M]) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, nf = n >> 2;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    double d[4] = {0.0, 0.0, 0.0, 0.0};
    uint32_t k01 = 0u, k23 = 0u;
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (t + 256 * k < nf) {
        const float c[4] = {rw.v[m][k].x, rw.v[m][k].y, rw.v[m][k].z, rw.v[m][k].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) { const double x = c[e]; d[e] = fma(x, x, d[e]); }
        k01 = __vmaxu4(k01, seg_ekeys(c[0]) | (seg_ekeys(c[1]) << 16));
        k23 = __vmaxu4(k23, seg_ekeys(c[2]) | (seg_ekeys(c[3]) << 16));
      }
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
    double p8[8];
    uint32_t kw = 0u;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) {
      p8[ww] = sh.part[ww][m][p];
      kw = __vmaxu4(kw, sh.keys[ww][m][p >> 1]);
    }
    double s = ((p8[0] + p8[1]) + (p8[2] + p8[3])) + ((p8[4] + p8[5]) + (p8[6] + p8[7]));
    const uint32_t kk = (kw >> (16 * (p & 1))) & 0xFFFFu;
    const int kmax = (int)(kk >> 8), kmin = 255 - (int)(kk & 0xFFu);
    if (kmax - kmin > 15) {
      s = 0.0;
      const float* xr = xs + (size_t)m * n;
      for (int i = p; i < n; i += 16) { const double x = xr[i]; s = fma(x, x, s); }
    }
    sh.chain[m][p] = s;
  }
  consumer_sync();
#pragma unroll
  for (int m = 0; m < M; ++m) {
    double tb[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) tb[b] = (sh.chain[m][b] + sh.chain[m][4 + b]) + (sh.chain[m][8 + b] + sh.chain[m][12 + b]);
    const double ss = (tb[0] + tb[2]) + (tb[1] + tb[3]);
    const double mean = (n & (n - 1)) == 0 ? ss * (1.0 / (double)n) : ss / (double)n;
    r[m] = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)mean, 1e-6f)));
  }
}

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

// ------------------------------------------------------------------------------------ kernel
struct SegSmem {
  uint8_t* slots;   // kSegNS x kSegSlot
  int8_t* q;        // [M][K + 16] int8 activations
  float* sx;        // [M][256]
  int32_t* sm;      // [M][256]
  float* rows;      // [M][2048] rows for the RMS chains
  float* gub;       // [8 teams][M][16] gate/up outputs of a round
};

// One team's chain rows: thread j -> (tile row r = j % R, activation row m = j / R).
template <int M>
__device__ __forceinline__ float tile_chain(const uint8_t* slot, int K, int R, int r, int m, const SegSmem& S) {
  const int G = K >> 5;
  const int rs = (K >> 1) + kSegRowPad;
  const uint8_t* wrow = slot + (size_t)r * rs;
  const uint16_t* srow = reinterpret_cast<const uint16_t*>(slot + kSegScaleOff) + (size_t)r * G;
  const int8_t* xq = S.q + (size_t)m * (K + 16);
  const float* sxm = S.sx + m * 256;
  const int32_t* smm = S.sm + m * 256;
  float row = 0.f;
#pragma unroll 4
  for (int g = 0; g < G; ++g) {
    const uint4 wv = *reinterpret_cast<const uint4*>(wrow + (size_t)g * 16);
    const int4 qa = *reinterpret_cast<const int4*>(xq + (size_t)g * 32);
    const int4 qb = *reinterpret_cast<const int4*>(xq + (size_t)g * 32 + 16);
    int a0 = -8 * smm[g], a1 = 0;
    a0 = __dp4a((int)(wv.x & 0x0F0F0F0Fu), qa.x, a0);
    a1 = __dp4a((int)(wv.y & 0x0F0F0F0Fu), qa.y, a1);
    a0 = __dp4a((int)(wv.z & 0x0F0F0F0Fu), qa.z, a0);
    a1 = __dp4a((int)(wv.w & 0x0F0F0F0Fu), qa.w, a1);
    a0 = __dp4a((int)((wv.x >> 4) & 0x0F0F0F0Fu), qb.x, a0);
    a1 = __dp4a((int)((wv.y >> 4) & 0x0F0F0F0Fu), qb.y, a1);
    a0 = __dp4a((int)((wv.z >> 4) & 0x0F0F0F0Fu), qb.z, a0);
    a1 = __dp4a((int)((wv.w >> 4) & 0x0F0F0F0Fu), qb.w, a1);
    const float s = __fmul_rn(bf2f(srow[g]), sxm[g]);
    row = fmaf((float)(a0 + a1), s, row);  // the integer dot is exact in any order
  }
  return row;
}

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

// Wait for a ring slot to fill (team-wide poll, bounded).
__device__ __forceinline__ bool slot_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait(bar, parity);
}

template <int M>
__device__ bool gemv_stage(const SegMatDev& mt, int stage_tiles_base, int& ring, float* Y, int ldy, int half_rows,
                           const SegSmem& S, SegShared& sh, bool geglu, int8_t* aq, float* asx, int32_t* asum) {
  const int G = gridDim.x, c = blockIdx.x, t = threadIdx.x;
  constexpr int MT = M == 3 ? 4 : M;  // team slots per tile row (teams stay warp-aligned)
  const int R = mt.R, tsz = R * MT;
  const int nteams = kSegConsumers / tsz;
  const int team = t / tsz, j = t % tsz, r = j % R, m = j / R;
  const int nunits = seg_units(mt, c, G);
  const int ntl = nunits * mt.tpu;  // this CTA's tiles of the stage, in ring order
  bool ok = true;
  for (int base = 0; base < ntl; base += nteams) {
    const int i = base + team;  // the team's tile in this round
    float val = 0.f;
    int n0 = -1;
    if (team < nteams && i < ntl) {
      const int slot = (ring + i) % kSegNS;
      const uint32_t par = (uint32_t)(((ring + i) / kSegNS) & 1);
      if (!slot_wait(&sh.full[slot], par)) ok = false;
      const int u = seg_unit(mt, c, G, i / mt.tpu), tj = i % mt.tpu;
      n0 = seg_tile_row(mt, u, tj, half_rows);
      if (ok && m < M) val = tile_chain<M>(S.slots + (size_t)slot * kSegSlot, mt.K, R, r, m, S);
      // the team has read its slot: one elected thread frees it
      if (tsz >= 32) {
        asm volatile("bar.sync %0, %1;" ::"r"(2 + team), "r"(tsz) : "memory");
        if (j == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sh.empty[slot])) : "memory");
      } else {
        const unsigned mask = ((1u << tsz) - 1u) << (t & 31 & ~(tsz - 1));
        __syncwarp(mask);
        if (j == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sh.empty[slot])) : "memory");
      }
      if (!geglu && ok && m < M) Y[(size_t)m * ldy + n0 + r] = val;
      if (geglu && m < M) S.gub[((size_t)team * 4 + m) * 16 + r] = val;
    }
    if (geglu) {
      // GeGLU of the round's units (teams 4k..4k+3 hold gate rows 0-15, 16-31, up rows 0-15,
      // 16-31 of one unit): act = r16(r16(gelu(r16 g)) * r16 u), then the 32-group quantisation
      consumer_sync();
      const int w = t >> 5, lane = t & 31;
      const int units_round = nteams / 4;
      for (int pi = w; pi < units_round * M; pi += 8) {
        const int ur = pi / M, mm = pi % M;
        const int i0 = base + 4 * ur;
        if (i0 >= ntl) continue;
        const int u = seg_unit(mt, c, G, i0 / 4);
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
  ring += ntl;
  (void)stage_tiles_base;
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
  for (int k = ring - 1; k >= 0 && k >= ring - kSegNS; --k) mbar_wait(&sh.full[k % kSegNS], (uint32_t)((k / kSegNS) & 1));
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
  S.rows = reinterpret_cast<float*>(S.sm + M * 256);
  S.gub = S.rows + (size_t)M * kSegRow;
  const int t = threadIdx.x;
  const int H = p.H, nf = H >> 2;
  if (t == 0) {
    for (int i = 0; i < kSegNS; ++i) { mbar_init(&sh.full[i], 1); mbar_init(&sh.empty[i], 1); }
    fence_mbar_init();
    sh.flag = 0;
  }
  __syncthreads();
  // the matrices of this launch, in stage order
  SegMatDev mats[4];
  int half[4] = {0, 0, 0, 0};
  int nm = 0, i_o = -1, i_gu = -1, i_dn = -1, i_qkv = -1;
  if (p.do_mlp) {
    i_o = nm;  mats[nm++] = SegMatDev{p.o.w, p.o.s, p.o.N, p.o.K, 16, p.o.N / 16, 1, 0};
    i_gu = nm; half[nm] = p.I; mats[nm++] = SegMatDev{p.gu.w, p.gu.s, p.gu.N, p.gu.K, 16, p.gu.N / 16, 4, 37};
    i_dn = nm; mats[nm++] = SegMatDev{p.down.w, p.down.s, p.down.N, p.down.K, 4, p.down.N / 4, 1, 74};
  }
  if (p.do_qkv) { i_qkv = nm; mats[nm++] = SegMatDev{p.qkv.w, p.qkv.s, p.qkv.N, p.qkv.K, 16, p.qkv.N / 16, 1, 111}; }
  if (t >= kSegConsumers) {  // producer warp: weights are read-only, no wait on earlier kernels
    seg_producer(mats, nm, half, S, sh, p.abort_flag);
    return;
  }
  pdl_wait();
  pdl_trigger();
  const unsigned G = gridDim.x;
  int ring = 0;
  bool ok = true;
  int bar = 0;
  float r1[M], r2[M];
  Rows<M> A, B;
  auto load_rows = [&](Rows<M>& dst, const float* src, bool round) {
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int f = t + 256 * k;
        float4 v = f < nf ? ldcg4(src + (size_t)m * H + 4 * f) : make_float4(0.f, 0.f, 0.f, 0.f);
        dst.v[m][k] = round ? r16x4(v) : v;
      }
  };
  auto stash = [&](const Rows<M>& src) {  // the rows for the RMS chains
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int f = t + 256 * k;
        if (f < nf) reinterpret_cast<float4*>(S.rows + (size_t)m * H)[f] = src.v[m][k];
      }
  };
  auto quant_rows = [&](const Rows<M>& y) {
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int f = t + 256 * k;
        if (f < nf) quant4_smem(y.v[m][k], f, m, S.q, H + 16, S.sx, S.sm);  // warp-uniform (nf % 64 == 0)
      }
  };
  auto store_rows = [&](float* dst, const Rows<M>& src) {
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int f = t + 256 * k;
        if (f < nf) reinterpret_cast<float4*>(dst + (size_t)m * H)[f] = src.v[m][k];
      }
  };
  auto weights4 = [&](const float* w, int k) {
    const int f = t + 256 * k;
    return f < nf ? __ldg(reinterpret_cast<const float4*>(w) + f) : make_float4(0.f, 0.f, 0.f, 0.f);
  };

  if (p.do_mlp) {
    // ---- S1: o projection of the attention output (quantised by the attention kernel)
    load_act<M>(p.att_q, p.att_sx, p.att_sum, p.o.K, S);
    consumer_sync();
    ok = gemv_stage<M>(mats[i_o], 0, ring, p.o_out, p.H, 0, S, sh, false, nullptr, nullptr, nullptr) && ok;
    ok = grid_barrier(p.bar + bar++, p.abort_flag, G, ok, sh);
    // ---- S2: o = r16(o); x = r16(x + r16((o*r)*w_post)); mlp_in = r16((x*r')*w_pre), quantised;
    //          then gate/up with GeGLU and the down projection's quantisation
    if (ok) {
      load_rows(A, p.o_out, true);
      load_rows(B, p.x_a, false);
      stash(A);
      consumer_sync();
      rows_rms<M>(A, S.rows, H, sh, r1);
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int k = 0; k < 2; ++k) B.v[m][k] = resid4(B.v[m][k], A.v[m][k], r1[m], weights4(p.w_post_attn, k));
      consumer_sync();
      stash(B);
      if (blockIdx.x == 0) store_rows(p.x_b, B);
      consumer_sync();
      rows_rms<M>(B, S.rows, H, sh, r2);
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int k = 0; k < 2; ++k) A.v[m][k] = r16x4(scale4(B.v[m][k], r2[m], weights4(p.w_pre_ff, k)));
      quant_rows(A);
      consumer_sync();
      ok = gemv_stage<M>(mats[i_gu], 0, ring, nullptr, 0, p.I, S, sh, true, p.act_q, p.act_sx, p.act_sum) && ok;
    }
    ok = grid_barrier(p.bar + bar++, p.abort_flag, G, ok, sh);
    // ---- S3: down projection
    if (ok) {
      load_act<M>(p.act_q, p.act_sx, p.act_sum, p.down.K, S);
      consumer_sync();
      ok = gemv_stage<M>(mats[i_dn], 0, ring, p.down_out, p.H, 0, S, sh, false, nullptr, nullptr, nullptr) && ok;
    }
    ok = grid_barrier(p.bar + bar++, p.abort_flag, G, ok, sh);
    // ---- S4: o = r16(down); x = r16(x + r16((o*r)*w_post_ff)) (layer scalar 1); then the next
    //          layer's input norm (x*r')*w_in, quantised, or the final norm (rounded) into hbuf
    if (ok) {
      load_rows(A, p.down_out, true);
      load_rows(B, p.x_b, false);
      stash(A);
      consumer_sync();
      rows_rms<M>(A, S.rows, H, sh, r1);
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int k = 0; k < 2; ++k) B.v[m][k] = resid4(B.v[m][k], A.v[m][k], r1[m], weights4(p.w_post_ff, k));
      consumer_sync();
      stash(B);
      if (blockIdx.x == 0) store_rows(p.x_a, B);
      consumer_sync();
      rows_rms<M>(B, S.rows, H, sh, r2);
      if (!p.do_qkv) {  // final norm, rounded (:1402)
        if (blockIdx.x == 0) {
#pragma unroll
          for (int m = 0; m < M; ++m)
#pragma unroll
            for (int k = 0; k < 2; ++k) A.v[m][k] = r16x4(scale4(B.v[m][k], r2[m], weights4(p.w_next, k)));
          store_rows(p.hbuf, A);
        }
      } else {
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
          for (int k = 0; k < 2; ++k) A.v[m][k] = scale4(B.v[m][k], r2[m], weights4(p.w_next, k));
        quant_rows(A);
      }
      consumer_sync();
    }
  } else if (p.do_qkv) {
    // ---- first launch of a pass: x = r16(E[tok] * sqrt(H)) (:1264), a = (x*r)*w_in, quantised
    const int* toks = p.toks;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const uint16_t* er = p.E + (size_t)__ldcg(toks + m) * H;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int f = t + 256 * k;
        if (f < nf) {
          const uint2 b = __ldg(reinterpret_cast<const uint2*>(er) + f);
          B.v[m][k] = make_float4(r16(__fmul_rn(bf2f(b.x & 0xFFFFu), p.sqrtH)), r16(__fmul_rn(bf2f(b.x >> 16), p.sqrtH)),
                                  r16(__fmul_rn(bf2f(b.y & 0xFFFFu), p.sqrtH)), r16(__fmul_rn(bf2f(b.y >> 16), p.sqrtH)));
        } else {
          B.v[m][k] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    stash(B);
    if (blockIdx.x == 0) store_rows(p.x_a, B);
    consumer_sync();
    rows_rms<M>(B, S.rows, H, sh, r2);
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int k = 0; k < 2; ++k) A.v[m][k] = scale4(B.v[m][k], r2[m], weights4(p.w_next, k));
    quant_rows(A);
    consumer_sync();
  }
  if (p.do_qkv) {
    // ---- qkv projection of the next layer
    if (ok) ok = gemv_stage<M>(mats[i_qkv], 0, ring, p.qkv_out, p.qkv.N, 0, S, sh, false, nullptr, nullptr, nullptr) && ok;
    ok = grid_barrier(p.bar + bar++, p.abort_flag, G, ok, sh);
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
        double s = 0.0;  // lanes 0..15: partial `lane` (elements lane, lane + 16, ... in order)
        if (lane < 16)
          for (int i = lane; i < HD; i += 16) { const double d = __ldcg(src + i); s = fma(d, d, s); }
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
  (void)ok;
}

}  // namespace g4

using namespace g4;

namespace g4 {
size_t seg_smem_bytes(int M) {
  return (size_t)kSegNS * kSegSlot + (size_t)M * (kSegKmax + 16) + (size_t)M * 256 * 8 + (size_t)M * kSegRow * 4 +
         (size_t)8 * 4 * 16 * 4;
}

int seg_check(const SegParams& p) {
  const bool shapes = p.H == 2048 && p.HD == 256 && p.NQ == 8 && p.QD == 2048 && (!p.do_mlp || (p.o.N == p.H && p.o.K == p.QD &&
                      p.gu.N == 2 * p.I && p.gu.K == p.H && p.down.N == p.H && p.down.K == p.I && p.I == 8192)) &&
                      (!p.do_qkv || (p.qkv.N == p.QD + 2 * p.HD && p.qkv.K == p.H));
  if (!shapes || p.M < 2 || p.M > 4) return set_error(G4_ERR_UNSUPPORTED, "segment kernel: unsupported shape");
  return G4_OK;
}

// Launch with one CTA per SM; the grid barriers need every CTA resident at once, which the
// cooperative attribute makes the driver guarantee (a launch it cannot place fails instead of
// hanging).  Programmatic dependent launch lets the producer's weight stream start under the
// previous kernel when the engine records a pass.
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
    // attribute sets tried in order: cooperative + programmatic, cooperative, ordinary
    cudaError_t e = cudaErrorUnknown;
    for (int variant = pdl_enabled() ? 0 : 1; variant < 3; ++variant) {
      cudaLaunchAttribute at[2];
      int na = 0;
      if (variant <= 1) {
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
