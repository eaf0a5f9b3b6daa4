// Row-wise kernels of the decoder layer (norms, RoPE, KV write, residual adds, GeGLU), the
// embedding, the non-split attention paths used for prefill and short contexts, the drafter's
// candidate scoring, and the seeded weight generator.  Each follows the rounding points of the
// reference's fwd (gemma4_engine.cpp:1262-1404) operation for operation.
#include "g4_layers.cuh"
#include "g4_api.h"

namespace g4 {

// ---- RMS scale in the reference's order: sum of squares in double over 16 partial sums
// (element i + 4a + b goes to partial (a, b), i in steps of 16), combined as ss_avx2 does
// (gemma4_engine.cpp:326-343); r = 1 / sqrtf((float)(ss / n) + eps).  Block-wide, >= 16 threads;
// every thread gets r.
__device__ float block_rms_scale(const float* __restrict__ x, int n, double* red) {
  if (threadIdx.x < 16) {
    double s = 0;
    int i = 0;
    for (; i + 128 <= n; i += 128) {  // 8 loads in flight, then the chain in element order
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = x[i + 16 * u + threadIdx.x];
#pragma unroll
      for (int u = 0; u < 8; ++u) { const double d = v[u]; s = fma(d, d, s); }
    }
    for (; i < n; i += 16) { const double d = x[i + threadIdx.x]; s = fma(d, d, s); }
    red[threadIdx.x] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double t[4];
    for (int b = 0; b < 4; ++b) t[b] = (red[b] + red[4 + b]) + (red[8 + b] + red[12 + b]);
    const double ss = (t[0] + t[2]) + (t[1] + t[3]);
    red[16] = (double)__fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(ss / (double)n), 1e-6f)));
  }
  __syncthreads();
  const float r = (float)red[16];
  __syncthreads();
  return r;
}

// Copy a row into shared memory (float4 when n % 4 == 0 and both ends are 16-byte aligned).
__device__ __forceinline__ void stage_row(float* dst, const float* __restrict__ src, int n) {
  if ((n & 3) == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
    for (int i = threadIdx.x; i < (n >> 2); i += blockDim.x)
      reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}


// y[m] = (x[m]*r)*w, optionally rounded to bf16 (rms / rms_prep_x, :344-352, :365-381).
__global__ void k_rmsnorm(const float* __restrict__ x, const float* __restrict__ w, int n, float* __restrict__ y, int round) {
  pdl_wait();
  pdl_trigger();
  __shared__ double red[17];
  const float* xm = x + (size_t)blockIdx.x * n;
  float* ym = y + (size_t)blockIdx.x * n;
  const float r = block_rms_scale(xm, n, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(xm[i], r), w[i]);
    ym[i] = round ? r16(v) : v;
  }
}

// x[m] = r16(E[tok[m]] * sqrt(H))   (embed, :1264)
__global__ void k_embed(const uint16_t* __restrict__ E, const int* __restrict__ toks, int H, float sqrtH, float* __restrict__ x) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const uint16_t* er = E + (size_t)toks[m] * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) x[(size_t)m * H + i] = r16(__fmul_rn(bf2f(er[i]), sqrtH));
}

// q/k/v after the qkv projection (:1290-1303, :1314-1323).  Block (m, part): part < nq is query
// head `part`: rms_r16 with q_norm, then RoPE (fp32, not rounded); part == nq is k: rms_r16 with
// k_norm, RoPE, bf16 store at cache position pos0+m; part == nq+1 is v: rms_r16 without weight,
// bf16 store.  RoPE (rope_avx2 :394-402): h[j] = fma(u, c, -(w*s)), h[j+hd/2] = fma(w, c, u*s).
__global__ void k_qkv_post(const float* __restrict__ qkv, int ldqkv, int nq, int hd, int pos0,
                           const int* __restrict__ dpos, const float* __restrict__ qn, const float* __restrict__ kn,
                           const float* __restrict__ cosT, const float* __restrict__ sinT, uint16_t* __restrict__ Kc,
                           uint16_t* __restrict__ Vc, float* __restrict__ qdst, int ldq) {
  pdl_wait();
  pdl_trigger();
  __shared__ double red[17];
  __shared__ __align__(16) float hbuf[512];
  if (dpos) pos0 += *dpos;  // position read on the device (captured decode steps)
  const int m = blockIdx.x, part = blockIdx.y, pos = pos0 + m, hh = hd >> 1;
  const float* src = qkv + (size_t)m * ldqkv + (size_t)part * hd;  // q heads, then k, then v
  float* dst = qdst + (size_t)m * ldq + (size_t)part * hd;
  const float* w = part < nq ? qn : (part == nq ? kn : nullptr);
  stage_row(hbuf, src, hd);
  __syncthreads();
  const float r = block_rms_scale(hbuf, hd, red);
  for (int i = threadIdx.x; i < hd; i += blockDim.x) {
    const float v = w ? __fmul_rn(__fmul_rn(hbuf[i], r), w[i]) : __fmul_rn(hbuf[i], r);
    hbuf[i] = r16(v);
  }
  __syncthreads();
  if (part == nq + 1) {
    for (int i = threadIdx.x; i < hd; i += blockDim.x) Vc[(size_t)pos * hd + i] = (uint16_t)f2bf(hbuf[i]);
    return;
  }
  const float* cs = cosT + (size_t)pos * hh;
  const float* sn = sinT + (size_t)pos * hh;
  for (int j = threadIdx.x; j < hh; j += blockDim.x) {
    const float u = hbuf[j], ww = hbuf[j + hh], c = cs[j], s = sn[j];
    const float a = fmaf(u, c, -__fmul_rn(ww, s));
    const float b = fmaf(ww, c, __fmul_rn(u, s));
    if (part == nq) {
      Kc[(size_t)pos * hd + j] = (uint16_t)f2bf(a);
      Kc[(size_t)pos * hd + j + hh] = (uint16_t)f2bf(b);
    } else {
      dst[j] = a;
      dst[j + hh] = b;
    }
  }
}

// Warp-per-head variant of k_qkv_post (same values): block = row m, warp w = part w (q heads, then
// k, then v), hd a multiple of 64 and at most 512.  Lanes 0..15 run the 16 ordered partial sums of
// the RMS (lane c: elements c, c+16, ... in order, from global memory); the reference's combine
// ((p_b + p_4+b) + (p_8+b + p_12+b)), then (t0 + t2) + (t1 + t3), is done by shuffles (fadd is
// commutative, so each sum pairs the same operands); lane l owns elements j = l + 32k (k < hd/64)
// and j + hd/2, the RoPE pairs.  The norm weights and the RoPE rows (positions read on the device
// come from the host-written control word) are loaded before the wait on the previous kernel.
__global__ void __launch_bounds__(512) k_qkv_post_w(const float* __restrict__ qkv, int ldqkv, int nq, int hd, int pos0,
                                                    const int* __restrict__ dpos, const float* __restrict__ qn,
                                                    const float* __restrict__ kn, const float* __restrict__ cosT,
                                                    const float* __restrict__ sinT, uint16_t* __restrict__ Kc,
                                                    uint16_t* __restrict__ Vc, float* __restrict__ qdst, int ldq) {
  constexpr int kMaxPer = 8;  // hd / 64
  const int m = blockIdx.x, part = threadIdx.x >> 5, lane = threadIdx.x & 31, hh = hd >> 1, per = hd >> 6;
  if (dpos) pos0 += *dpos;
  const int pos = pos0 + m;
  const float* w = part < nq ? qn : (part == nq ? kn : nullptr);
  float wl[kMaxPer], wh[kMaxPer], cs[kMaxPer], sn[kMaxPer];
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int j = lane + 32 * k;
    const bool in = k < per;
    wl[k] = (in && w) ? w[j] : 1.f;
    wh[k] = (in && w) ? w[j + hh] : 1.f;
    cs[k] = (in && part <= nq) ? cosT[(size_t)pos * hh + j] : 0.f;
    sn[k] = (in && part <= nq) ? sinT[(size_t)pos * hh + j] : 0.f;
  }
  pdl_wait();  // the weights and tables above are read-only; the row comes from the previous kernel
  pdl_trigger();
  const float* src = qkv + (size_t)m * ldqkv + (size_t)part * hd;
  float xl[kMaxPer], xh[kMaxPer];
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int j = lane + 32 * k;
    xl[k] = k < per ? src[j] : 0.f;
    xh[k] = k < per ? src[j + hh] : 0.f;
  }
  double s = 0.0;  // partial lane (lanes 0..15): elements lane, lane + 16, ... in order
  if (lane < 16) {
    int i = lane;
    for (; i + 112 < hd; i += 128) {  // 8 loads ahead of the chain
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = src[i + 16 * u];
#pragma unroll
      for (int u = 0; u < 8; ++u) { const double d = v[u]; s = fma(d, d, s); }
    }
    for (; i < hd; i += 16) { const double d = src[i]; s = fma(d, d, s); }
  }
  double u = s + __shfl_down_sync(FULL, s, 4);   // lanes 0-3, 8-11: p_b + p_4+b and p_8+b + p_12+b
  double t = u + __shfl_down_sync(FULL, u, 8);   // lanes 0-3: t_b
  double v2 = t + __shfl_down_sync(FULL, t, 2);  // lanes 0, 1: t0 + t2, t1 + t3
  double ss = v2 + __shfl_down_sync(FULL, v2, 1);
  ss = __shfl_sync(FULL, ss, 0);
  const double mean = (hd & (hd - 1)) == 0 ? ss * (1.0 / (double)hd) : ss / (double)hd;
  const float r = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)mean, 1e-6f)));
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    if (k >= per) break;
    const int j = lane + 32 * k;
    const float a = w ? r16(__fmul_rn(__fmul_rn(xl[k], r), wl[k])) : r16(__fmul_rn(xl[k], r));
    const float b = w ? r16(__fmul_rn(__fmul_rn(xh[k], r), wh[k])) : r16(__fmul_rn(xh[k], r));
    if (part == nq + 1) {
      Vc[(size_t)pos * hd + j] = (uint16_t)f2bf(a);
      Vc[(size_t)pos * hd + j + hh] = (uint16_t)f2bf(b);
      continue;
    }
    const float ra = fmaf(a, cs[k], -__fmul_rn(b, sn[k]));
    const float rb = fmaf(b, cs[k], __fmul_rn(a, sn[k]));
    if (part == nq) {
      Kc[(size_t)pos * hd + j] = (uint16_t)f2bf(ra);
      Kc[(size_t)pos * hd + j + hh] = (uint16_t)f2bf(rb);
    } else {
      float* dst = qdst + (size_t)m * ldq + (size_t)part * hd;
      dst[j] = ra;
      dst[j + hh] = rb;
    }
  }
}

// Query-only variant for the drafter (and any caller whose k/v are not written): heads of q in
// place, rms_r16 with q_norm then RoPE at position pos.
__global__ void k_q_post(float* __restrict__ q, int hd, int pos, const int* __restrict__ dpos, const float* __restrict__ qn,
                         const float* __restrict__ cosT, const float* __restrict__ sinT) {
  pdl_wait();
  pdl_trigger();
  __shared__ double red[17];
  __shared__ __align__(16) float hbuf[512];
  if (dpos) pos += *dpos;
  const int h = blockIdx.x, hh = hd >> 1;
  float* src = q + (size_t)h * hd;
  stage_row(hbuf, src, hd);
  __syncthreads();
  const float r = block_rms_scale(hbuf, hd, red);
  for (int i = threadIdx.x; i < hd; i += blockDim.x) hbuf[i] = r16(__fmul_rn(__fmul_rn(hbuf[i], r), qn[i]));
  __syncthreads();
  const float* cs = cosT + (size_t)pos * hh;
  const float* sn = sinT + (size_t)pos * hh;
  for (int j = threadIdx.x; j < hh; j += blockDim.x) {
    const float u = hbuf[j], ww = hbuf[j + hh], c = cs[j], s = sn[j];
    src[j] = fmaf(u, c, -__fmul_rn(ww, s));
    src[j + hh] = fmaf(ww, c, __fmul_rn(u, s));
  }
}

// After o_proj (:1358-1361): o = r16(o); x = r16(x + r16((o*r)*w_post_attn)); then the pre-MLP
// input mlp_in = r16((x*r')*w_pre_ff) (rms_prep_x with rounding, :1360).
__global__ void k_post_attn(float* __restrict__ o, float* __restrict__ x, const float* __restrict__ w_post,
                            const float* __restrict__ w_pre, float* __restrict__ mlp_in, int n) {
  pdl_wait();
  pdl_trigger();
  __shared__ double red[17];
  float* om = o + (size_t)blockIdx.x * n;
  float* xm = x + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) om[i] = r16(om[i]);
  __syncthreads();
  const float r = block_rms_scale(om, n, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    xm[i] = r16(__fadd_rn(xm[i], r16(__fmul_rn(__fmul_rn(om[i], r), w_post[i]))));
  __syncthreads();
  const float r2 = block_rms_scale(xm, n, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) mlp_in[(size_t)blockIdx.x * n + i] = r16(__fmul_rn(__fmul_rn(xm[i], r2), w_pre[i]));
}

// After down_proj (:1375-1378) and the layer scalar (:1395): o = r16(o);
// x = r16(x + r16((o*r)*w_post_ff)); x = r16(x * scalar).
__global__ void k_post_ff(float* __restrict__ o, float* __restrict__ x, const float* __restrict__ w_post, float scalar, int n) {
  pdl_wait();
  pdl_trigger();
  __shared__ double red[17];
  float* om = o + (size_t)blockIdx.x * n;
  float* xm = x + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) om[i] = r16(om[i]);
  __syncthreads();
  const float r = block_rms_scale(om, n, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = r16(__fadd_rn(xm[i], r16(__fmul_rn(__fmul_rn(om[i], r), w_post[i]))));
    xm[i] = r16(__fmul_rn(v, scalar));
  }
}

// GeGLU: act = r16(r16(gelu(r16 g)) * r16 u), gate in columns [0, I), up in [I, 2I) (:1370).
__global__ void k_act(const float* __restrict__ gu, int I, int M, float* __restrict__ act) {
  pdl_wait();
  pdl_trigger();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)M * I) return;
  const int m = (int)(idx / I), i = (int)(idx % I);
  const float g = r16(gu[(size_t)m * 2 * I + i]), u = r16(gu[(size_t)m * 2 * I + I + i]);
  act[idx] = r16(__fmul_rn(r16(gelu(g)), u));
}

// o_drafter residual (:1548): x = r16(x + r16((o*r)*w)) after o = r16(o); no second norm.
__global__ void k_resid_norm(float* __restrict__ o, float* __restrict__ x, const float* __restrict__ w, int n) {
  pdl_wait();
  pdl_trigger();
  __shared__ double red[17];
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = r16(o[i]);
  __syncthreads();
  const float r = block_rms_scale(o, n, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = r16(__fadd_rn(x[i], r16(__fmul_rn(__fmul_rn(o[i], r), w[i]))));
}

// ---- fused row kernels: one block (256 threads) per activation row, rows up to kRowMax wide and a
// multiple of 256.  Thread t owns the float4 blocks f = t + 256k (elements 4f..4f+3) and keeps them
// in registers from load to store; the row also goes to shared memory for the sequential fallback
// of the RMS sum.  When qo.q is set the kernel writes the W4A8 quantisation of its output row for
// the next linear (the values of g4_w4a8_quant).  They compute the values of the unfused kernels.
constexpr int kRowMax = 2048;
constexpr int kF4 = kRowMax / 1024;  // float4 blocks per thread

struct RmsScratch {
  double part[8][16];     // per warp and partial: the warp's share of the partial sum
  uint32_t keys[8][8];    // per warp: exponent keys of two partials per word (see row_rms_scale)
  double chain[16];       // the 16 partial sums
};

// Exponent keys of x for the exactness test of row_rms_scale, packed as the bytes of a max-reduced
// word: (kmax, 255 - kmin) of the nonzero elements' biased exponents (subnormals as 1; a value that
// is not bf16-valued or not finite counts as kmax 255, kmin 1, which fails the test).
__device__ __forceinline__ uint32_t ekeys(float x) {
  const uint32_t b = __float_as_uint(x) & 0x7FFFFFFFu;
  const uint32_t e = max(b >> 23, 1u);
  const uint32_t key = ((b & 0xFFFFu) != 0u || e == 255u) ? ((255u << 8) | 254u) : ((e << 8) | (255u - e));
  return b == 0u ? 0u : key;
}

// RMS scale of a row held as float4 blocks, in the reference's order (gemma4_engine.cpp:326-343):
// the sum of squares in double over 16 partials (element j to partial j % 16, each partial in
// element order), combined as ((p_b + p_4+b) + (p_8+b + p_12+b)) for b = 0..3, then
// (t0 + t2) + (t1 + t3); r = 1 / sqrtf((float)(ss / n) + eps).
// A partial is summed as a tree when that is exact: if its elements are bf16-valued and the biased
// exponents of its nonzero elements span at most 15, every squared element is an integer multiple
// of u = 2^(2 e_min - 268) and any sum of at most 128 of them is below 2^(2 e_max - 245) =
// 2^(23 + 2 span) u <= 2^53 u, hence exact in double; the sequential sum then equals the exact sum,
// as does any other order.  Other partials take the sequential chain over xs (the row in shared
// memory, written before the call).  Needs blockDim 256, n <= 2048; every thread gets r.
__device__ float row_rms_scale(const float4 (&v)[kF4], const float* xs, int n, RmsScratch& sc) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, nf = n >> 2;
  double d[4] = {0.0, 0.0, 0.0, 0.0};  // partials 4 (t % 4) + e
  uint32_t k01 = 0u, k23 = 0u;         // keys of partials e = 0, 1 and 2, 3 (two bytes each)
#pragma unroll
  for (int k = 0; k < kF4; ++k)
    if (t + 256 * k < nf) {
      const float c[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) { const double x = c[e]; d[e] = fma(x, x, d[e]); }
      k01 = __vmaxu4(k01, ekeys(c[0]) | (ekeys(c[1]) << 16));
      k23 = __vmaxu4(k23, ekeys(c[2]) | (ekeys(c[3]) << 16));
    }
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {  // lanes with equal lane % 4 hold the same partials
#pragma unroll
    for (int e = 0; e < 4; ++e) d[e] += __shfl_xor_sync(FULL, d[e], o);
    k01 = __vmaxu4(k01, __shfl_xor_sync(FULL, k01, o));
    k23 = __vmaxu4(k23, __shfl_xor_sync(FULL, k23, o));
  }
  if (lane < 4) {
#pragma unroll
    for (int e = 0; e < 4; ++e) sc.part[w][4 * lane + e] = d[e];
    sc.keys[w][2 * lane] = k01;
    sc.keys[w][2 * lane + 1] = k23;
  }
  __syncthreads();
  if (t < 16) {
    double p8[8];
    uint32_t kw = 0u;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) {
      p8[ww] = sc.part[ww][t];
      kw = __vmaxu4(kw, sc.keys[ww][t >> 1]);
    }
    // exact on the fast path (any order), replaced by the chain otherwise: a tree
    double s = ((p8[0] + p8[1]) + (p8[2] + p8[3])) + ((p8[4] + p8[5]) + (p8[6] + p8[7]));
    const uint32_t kk = (kw >> (16 * (t & 1))) & 0xFFFFu;  // this partial's (kmax, 255 - kmin)
    const int kmax = (int)(kk >> 8), kmin = 255 - (int)(kk & 0xFFu);
    if (kmax - kmin > 15) {  // the chain may round: the sequential sum in element order, 8 loads ahead
      s = 0.0;
      int i = t;
      for (; i + 112 < n; i += 128) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = xs[i + 16 * u];
#pragma unroll
        for (int u = 0; u < 8; ++u) { const double x = v[u]; s = fma(x, x, s); }
      }
      for (; i < n; i += 16) { const double x = xs[i]; s = fma(x, x, s); }
    }
    sc.chain[t] = s;
  }
  __syncthreads();
  double tb[4];
#pragma unroll
  for (int b = 0; b < 4; ++b) tb[b] = (sc.chain[b] + sc.chain[4 + b]) + (sc.chain[8 + b] + sc.chain[12 + b]);
  const double ss = (tb[0] + tb[2]) + (tb[1] + tb[3]);
  const double mean = (n & (n - 1)) == 0 ? ss * (1.0 / (double)n) : ss / (double)n;  // equal for a power of two
  return __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)mean, 1e-6f)));
}

__device__ __forceinline__ float4 f4_r16(float4 a) { return make_float4(r16(a.x), r16(a.y), r16(a.z), r16(a.w)); }
__device__ __forceinline__ float4 f4_load(const float* p, int f) { return reinterpret_cast<const float4*>(p)[f]; }
__device__ __forceinline__ void f4_store(float* p, int f, float4 a) { reinterpret_cast<float4*>(p)[f] = a; }
// (a * r) * w per element
__device__ __forceinline__ float4 f4_scale(float4 a, float r, float4 w) {
  return make_float4(__fmul_rn(__fmul_rn(a.x, r), w.x), __fmul_rn(__fmul_rn(a.y, r), w.y),
                     __fmul_rn(__fmul_rn(a.z, r), w.z), __fmul_rn(__fmul_rn(a.w, r), w.w));
}
// r16(x + r16((o * r) * w)) per element
__device__ __forceinline__ float4 f4_resid(float4 x, float4 o, float r, float4 w) {
  const float4 u = f4_r16(f4_scale(o, r, w));
  return f4_r16(make_float4(__fadd_rn(x.x, u.x), __fadd_rn(x.y, u.y), __fadd_rn(x.z, u.z), __fadd_rn(x.w, u.w)));
}

// quant_group32 of one float4 block per thread: a group of 32 is the 8 consecutive lanes holding
// its blocks; all 32 lanes of the warp call it together.
__device__ __forceinline__ void quant_f4(float4 y, int f, int m, int n, const QuantOut& qo) {
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
    const int32_t r = (v > -2147483648.f && v < 2147483648.f) ? __float2int_rn(v) : INT32_MIN;
    tot += r;
    const int32_t r16v = r < -32768 ? -32768 : (r > 32767 ? 32767 : r);
    const int32_t q = r16v < -128 ? -128 : (r16v > 127 ? 127 : r16v);
    packed |= ((uint32_t)q & 0xFFu) << (8 * e);
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) tot += __shfl_xor_sync(FULL, tot, o);
  reinterpret_cast<uint32_t*>(qo.q + (size_t)m * n)[f] = packed;
  if ((threadIdx.x & 7) == 0) {
    const int G = n >> 5;
    qo.sx[(size_t)m * G + (f >> 3)] = s;
    qo.sum[(size_t)m * G + (f >> 3)] = tot;
  }
}

// y[m] = (x[m]*r)*w, optionally rounded to bf16 (rms / rms_prep_x, :344-352, :365-381).
__global__ void __launch_bounds__(256) k_norm_q(const float* __restrict__ x, const float* __restrict__ w, int n,
                                                float* __restrict__ y, int round, QuantOut qo) {
  __shared__ __align__(16) float xs[kRowMax];
  __shared__ RmsScratch sc;
  const int m = blockIdx.x, t = threadIdx.x, nf = n >> 2;
  float4 wv[kF4], v[kF4];
#pragma unroll
  for (int k = 0; k < kF4; ++k) wv[k] = t + 256 * k < nf ? f4_load(w, t + 256 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
  pdl_wait();  // the norm weights above are read-only; the row comes from the previous kernel
  pdl_trigger();
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const int f = t + 256 * k;
    v[k] = f < nf ? f4_load(x + (size_t)m * n, f) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (f < nf) f4_store(xs, f, v[k]);
  }
  const float r = row_rms_scale(v, xs, n, sc);
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const int f = t + 256 * k;
    if (f < nf) {  // warp-uniform (nf is a multiple of 64)
      float4 yv = f4_scale(v[k], r, wv[k]);
      if (round) yv = f4_r16(yv);
      f4_store(y + (size_t)m * n, f, yv);
      if (qo.q) quant_f4(yv, f, m, n, qo);
    }
  }
}

// After o_proj (:1358-1361) with the pre-MLP input quantised: o = r16(o);
// x = r16(x + r16((o*r)*w_post)); mlp_in = r16((x*r')*w_pre).
__global__ void __launch_bounds__(256) k_post_attn_q(const float* __restrict__ o, float* __restrict__ x,
                                                     const float* __restrict__ w_post, const float* __restrict__ w_pre,
                                                     float* __restrict__ mlp_in, int n, QuantOut qo) {
  __shared__ __align__(16) float os[kRowMax];
  __shared__ __align__(16) float xs[kRowMax];
  __shared__ RmsScratch sc1, sc2;
  const int m = blockIdx.x, t = threadIdx.x, nf = n >> 2;
  float* xm = x + (size_t)m * n;
  float4 wa[kF4], wb[kF4], ov[kF4], xv[kF4];
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const bool in = t + 256 * k < nf;
    wa[k] = in ? f4_load(w_post, t + 256 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
    wb[k] = in ? f4_load(w_pre, t + 256 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  pdl_wait();  // the norm weights above are read-only; the rows come from earlier kernels
  pdl_trigger();
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const int f = t + 256 * k;
    const bool in = f < nf;
    ov[k] = in ? f4_r16(f4_load(o + (size_t)m * n, f)) : make_float4(0.f, 0.f, 0.f, 0.f);
    xv[k] = in ? f4_load(xm, f) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (in) f4_store(os, f, ov[k]);
  }
  const float r = row_rms_scale(ov, os, n, sc1);
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const int f = t + 256 * k;
    if (f < nf) {
      xv[k] = f4_resid(xv[k], ov[k], r, wa[k]);
      f4_store(xm, f, xv[k]);
      f4_store(xs, f, xv[k]);
    }
  }
  const float r2 = row_rms_scale(xv, xs, n, sc2);
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const int f = t + 256 * k;
    if (f < nf) {  // warp-uniform
      const float4 yv = f4_r16(f4_scale(xv[k], r2, wb[k]));
      f4_store(mlp_in + (size_t)m * n, f, yv);
      if (qo.q) quant_f4(yv, f, m, n, qo);
    }
  }
}

// Residual after the MLP (or the drafter's attention / MLP), then the next norm:
//   o = r16(o); x = r16(x + r16((o*r)*w_post)); if (scalar != 0) x = r16(x*scalar)
//   (k_post_ff / k_resid_norm + k_scale_round); then, when w_next is set,
//   a = (x*r')*w_next (rounded when round_next) and its quantisation.  a may alias o.
__global__ void __launch_bounds__(256) k_resid_norm_q(const float* o, float* __restrict__ x,
                                                      const float* __restrict__ w_post, float scalar, int n,
                                                      const float* __restrict__ w_next, float* a,
                                                      int round_next, QuantOut qo) {
  __shared__ __align__(16) float os[kRowMax];
  __shared__ __align__(16) float xs[kRowMax];
  __shared__ RmsScratch sc1, sc2;
  const int m = blockIdx.x, t = threadIdx.x, nf = n >> 2;
  float* xm = x + (size_t)m * n;
  float4 wa[kF4], wb[kF4], ov[kF4], xv[kF4];
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const bool in = t + 256 * k < nf;
    wa[k] = in ? f4_load(w_post, t + 256 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
    wb[k] = (in && w_next != nullptr) ? f4_load(w_next, t + 256 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  pdl_wait();  // the norm weights above are read-only; the rows come from earlier kernels
  pdl_trigger();
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const int f = t + 256 * k;
    const bool in = f < nf;
    ov[k] = in ? f4_r16(f4_load(o + (size_t)m * n, f)) : make_float4(0.f, 0.f, 0.f, 0.f);
    xv[k] = in ? f4_load(xm, f) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (in) f4_store(os, f, ov[k]);
  }
  const float r = row_rms_scale(ov, os, n, sc1);
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const int f = t + 256 * k;
    if (f < nf) {
      float4 v = f4_resid(xv[k], ov[k], r, wa[k]);
      if (scalar != 0.f) v = f4_r16(make_float4(__fmul_rn(v.x, scalar), __fmul_rn(v.y, scalar), __fmul_rn(v.z, scalar),
                                                __fmul_rn(v.w, scalar)));
      xv[k] = v;
      f4_store(xm, f, v);
      f4_store(xs, f, v);
    }
  }
  if (w_next == nullptr) return;
  const float r2 = row_rms_scale(xv, xs, n, sc2);
#pragma unroll
  for (int k = 0; k < kF4; ++k) {
    const int f = t + 256 * k;
    if (f < nf) {  // warp-uniform
      float4 yv = f4_scale(xv[k], r2, wb[k]);
      if (round_next) yv = f4_r16(yv);
      f4_store(a + (size_t)m * n, f, yv);
      if (qo.q) quant_f4(yv, f, m, n, qo);
    }
  }
}

// GeGLU with the down-projection input quantised: one warp per 32-group of a row (I % 32 == 0,
// blockDim 256, grid M*I/256).
__global__ void __launch_bounds__(256) k_act_q(const float* __restrict__ gu, int I, int M, float* __restrict__ act,
                                               QuantOut qo) {
  pdl_wait();
  pdl_trigger();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)M * I) return;  // warp-uniform (M*I is a multiple of 32)
  const int m = (int)(idx / I), i = (int)(idx % I);
  const float g = r16(gu[(size_t)m * 2 * I + i]), u = r16(gu[(size_t)m * 2 * I + I + i]);
  const float v = r16(__fmul_rn(r16(gelu(g)), u));
  act[idx] = v;
  if (qo.q) {
    int8_t qv;
    float sx;
    int32_t tot;
    quant_group32(v, qv, sx, tot);
    qo.q[idx] = qv;
    if ((threadIdx.x & 31) == 0) {
      qo.sx[idx >> 5] = sx;
      qo.sum[idx >> 5] = tot;
    }
  }
}

// elementwise helpers
__global__ void k_round(float* __restrict__ p, long long n) {
  pdl_wait();
  pdl_trigger();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = r16(p[i]);
}
__global__ void k_scale_round(float* __restrict__ p, long long n, float s) {
  pdl_wait();
  pdl_trigger();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = r16(__fmul_rn(p[i], s));
}
// drafter input [r16(E[tok]*sqrt(H)) | h]
__global__ void k_draft_in(const uint16_t* __restrict__ E, const int* __restrict__ tok, const float* __restrict__ h, int H,
                           float sqrtH, float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const uint16_t* er = E + (size_t)(*tok) * H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) {
    out[i] = r16(__fmul_rn(bf2f(er[i]), sqrtH));
    out[H + i] = h[i];
  }
}

// ---- non-split attention (prefill blocks and short contexts), one block per (row m, head h).
// Keys lo..pos in order, pos = pos0+m, lo = pos-511 clamped for sliding layers.
//   variant 0 (attn_tile, :1061-1083): scores by the 16-partial dot (s0/s1 of stride 16 and hsum),
//     weights exp8(s - max), den in key order, O = fma(w, v, O), out = r16(O * (1/den)).
//   variant 1 (per-(m,h) path, :1337-1355): scores by the 8-partial dot (stride 8, hsum),
//     weights expf(s - max) (correctly rounded here), den in key order, O = fma(w/den, v, O),
//     out = r16(O).
__global__ void __launch_bounds__(256) k_attn_rows(const uint16_t* __restrict__ Kc, const uint16_t* __restrict__ Vc,
                                                   const float* __restrict__ q, int ldq, int nh, int hd, int pos0,
                                                   int window, int variant, float* __restrict__ out, int ldo,
                                                   int blk_fn, int blk) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sc[];
  __shared__ float s_red[32];
  const int m = blockIdx.x, h = blockIdx.y;
  const int pos = pos0 + m, lo = window > 0 ? max(0, pos - (window - 1)) : 0, len = pos - lo + 1;
  if (variant < 0) {  // rows of full prefill blocks of blk rows starting at position blk_fn: the block's choice
    const int b0 = pos - (pos - blk_fn) % blk;
    variant = (blk >= 4 && b0 + blk > 64) ? 0 : 1;
  }
  const float* qh = q + (size_t)m * ldq + (size_t)h * hd;
  const int hw = threadIdx.x >> 4, c = threadIdx.x & 15;
  // scores: one half-warp per key; the two half-warps of a warp take keys pb and pb+1
  float qr[32];
  if (variant == 0) {
#pragma unroll
    for (int i = 0; i < 32; ++i) qr[i] = (i < (hd >> 4)) ? qh[c + 16 * i] : 0.f;
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) qr[i] = (c < 8 && i < (hd >> 3)) ? qh[c + 8 * i] : 0.f;
  }
  for (int pb = lo + (hw & ~1); pb <= pos; pb += 16) {
    const int p = min(pb + (hw & 1), pos);
    const uint16_t* kr = Kc + (size_t)p * hd;
    float acc = 0.f, s;
    if (variant == 0) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < (hd >> 4)) acc = fmaf(qr[i], bf2f(kr[c + 16 * i]), acc);
      s = hsum8_octet(__fadd_rn(acc, __shfl_xor_sync(FULL, acc, 8)));
    } else {
      if (c < 8) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < (hd >> 3)) acc = fmaf(qr[i], bf2f(kr[c + 8 * i]), acc);
      }
      s = hsum8_octet(acc);
    }
    if (c == 0 && pb + (hw & 1) <= pos) sc[p - lo] = s;
  }
  __syncthreads();
  float mx = -1e30f;
  for (int i = threadIdx.x; i < len; i += blockDim.x) mx = fmaxf(mx, sc[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = -1e30f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, s_red[i]);
  __syncthreads();
  for (int i = threadIdx.x; i < len; i += blockDim.x) {
    const float d = __fsub_rn(sc[i], mx);
    sc[i] = variant == 0 ? exp8(d) : exp_cr(d);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // the in-order sum, 8 loads in flight ahead of the chain
    float den = 0.f;
    int i = 0;
    for (; i + 8 <= len; i += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = sc[i + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) den = __fadd_rn(den, v[u]);
    }
    for (; i < len; ++i) den = __fadd_rn(den, sc[i]);
    s_red[0] = den;
  }
  __syncthreads();
  const float den = s_red[0];
  if (variant == 1) {
    for (int i = threadIdx.x; i < len; i += blockDim.x) sc[i] = __fdiv_rn(sc[i], den);
    __syncthreads();
  }
  const float inv = __fdiv_rn(1.0f, den);
  for (int i = threadIdx.x; i < hd; i += blockDim.x) {
    float o = 0.f;
    const uint16_t* vp = Vc + (size_t)lo * hd + i;
    int p = 0;
    for (; p + 8 <= len; p += 8) {  // 8 V loads in flight ahead of the in-order chain
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = bf2f(vp[(size_t)(p + u) * hd]);
#pragma unroll
      for (int u = 0; u < 8; ++u) o = fmaf(sc[p + u], v[u], o);
    }
    for (; p < len; ++p) o = fmaf(sc[p], bf2f(vp[(size_t)p * hd]), o);
    out[(size_t)m * ldo + (size_t)h * hd + i] = variant == 0 ? r16(__fmul_rn(o, inv)) : r16(o);
  }
}

// ---- prefill attention with fewer instructions per key (the values of k_attn_rows, variant < 0).
// Scores (attn_tile rows): eight lanes per key, lane l running chains 2l and 2l+1 (elements 2l+16i
// and 2l+1+16i, one 32-bit load per i), then v_j = chain j + chain j+8 (xor 4) and the hsum
// ((v0+v4)+(v1+v5))+((v2+v6)+(v3+v7)) by xor 2 and xor 1: the chains and the order of k_attn_rows.
// O: thread t runs dims 2t and 2t+1 (one 32-bit V load per key, the weights of 4 keys per 16-byte
// shared load), each over the keys in order.  Rows of per-row blocks (variant 1) run as in
// k_attn_rows.  blockDim 256, hd <= 256, hd % 16 == 0; dynamic shared memory len_max floats.
__global__ void __launch_bounds__(256) k_attn_rows2(const uint16_t* __restrict__ Kc, const uint16_t* __restrict__ Vc,
                                                    const float* __restrict__ q, int ldq, int nh, int hd, int pos0,
                                                    int window, float* __restrict__ out, int ldo, int blk_fn, int blk) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float sc[];
  __shared__ float s_red[32];
  const int m = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int pos = pos0 + m, lo = window > 0 ? max(0, pos - (window - 1)) : 0, len = pos - lo + 1;
  const int b0 = pos - (pos - blk_fn) % blk;
  const int variant = (blk >= 4 && b0 + blk > 64) ? 0 : 1;
  const float* qh = q + (size_t)m * ldq + (size_t)h * hd;
  if (variant == 0) {
    const int l = tid & 7, kq = tid >> 3;  // 32 keys per pass of the block
    float qa[16], qb[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      qa[i] = i < (hd >> 4) ? qh[2 * l + 16 * i] : 0.f;
      qb[i] = i < (hd >> 4) ? qh[2 * l + 1 + 16 * i] : 0.f;
    }
    for (int pb = lo; pb <= pos; pb += 32) {
      const int p = min(pb + kq, pos);
      const uint32_t* kr = reinterpret_cast<const uint32_t*>(Kc + (size_t)p * hd) + l;
      float aa = 0.f, ab = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < (hd >> 4)) {
          const uint32_t w = kr[8 * i];
          aa = fmaf(qa[i], __uint_as_float(w << 16), aa);
          ab = fmaf(qb[i], __uint_as_float(w & 0xFFFF0000u), ab);
        }
      const float va = __fadd_rn(aa, __shfl_xor_sync(FULL, aa, 4)), vb = __fadd_rn(ab, __shfl_xor_sync(FULL, ab, 4));
      const float pa = __fadd_rn(va, __shfl_xor_sync(FULL, va, 2)), pbv = __fadd_rn(vb, __shfl_xor_sync(FULL, vb, 2));
      const float s1 = __fadd_rn(pa, pbv);
      const float s = __fadd_rn(s1, __shfl_xor_sync(FULL, s1, 1));
      if (l == 0 && pb + kq <= pos) sc[p - lo] = s;
    }
  } else {
    const int hw = tid >> 4, c = tid & 15;
    float qr[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) qr[i] = (c < 8 && i < (hd >> 3)) ? qh[c + 8 * i] : 0.f;
    for (int pb = lo + (hw & ~1); pb <= pos; pb += 16) {
      const int p = min(pb + (hw & 1), pos);
      const uint16_t* kr = Kc + (size_t)p * hd;
      float acc = 0.f;
      if (c < 8) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < (hd >> 3)) acc = fmaf(qr[i], bf2f(kr[c + 8 * i]), acc);
      }
      const float s = hsum8_octet(acc);
      if (c == 0 && pb + (hw & 1) <= pos) sc[p - lo] = s;
    }
  }
  __syncthreads();
  float mx = -1e30f;
  for (int i = tid; i < len; i += blockDim.x) mx = fmaxf(mx, sc[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if ((tid & 31) == 0) s_red[tid >> 5] = mx;
  __syncthreads();
  mx = -1e30f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, s_red[i]);
  __syncthreads();
  for (int i = tid; i < len; i += blockDim.x) {
    const float d = __fsub_rn(sc[i], mx);
    sc[i] = variant == 0 ? exp8(d) : exp_cr(d);
  }
  __syncthreads();
  if (tid == 0) {  // the in-order sum, 8 loads in flight ahead of the chain
    float den = 0.f;
    int i = 0;
    for (; i + 8 <= len; i += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = sc[i + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) den = __fadd_rn(den, v[u]);
    }
    for (; i < len; ++i) den = __fadd_rn(den, sc[i]);
    s_red[0] = den;
  }
  __syncthreads();
  const float den = s_red[0];
  if (variant == 1) {
    for (int i = tid; i < len; i += blockDim.x) sc[i] = __fdiv_rn(sc[i], den);
    __syncthreads();
  }
  const float inv = __fdiv_rn(1.0f, den);
  for (int t2 = tid; 2 * t2 < hd; t2 += blockDim.x) {
    float o0 = 0.f, o1 = 0.f;
    const uint32_t* vp = reinterpret_cast<const uint32_t*>(Vc + (size_t)lo * hd) + t2;
    const int hw2 = hd >> 1;  // 32-bit words per V row
    int p = 0;
    for (; p + 8 <= len; p += 8) {  // 8 V loads in flight ahead of the in-order chains
      uint32_t v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = vp[(size_t)(p + u) * hw2];
      const float4 wa = *reinterpret_cast<const float4*>(sc + p);
      const float4 wb = *reinterpret_cast<const float4*>(sc + p + 4);
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        o0 = fmaf(w[u], __uint_as_float(v[u] << 16), o0);
        o1 = fmaf(w[u], __uint_as_float(v[u] & 0xFFFF0000u), o1);
      }
    }
    for (; p < len; ++p) {
      const uint32_t v = vp[(size_t)p * hw2];
      o0 = fmaf(sc[p], __uint_as_float(v << 16), o0);
      o1 = fmaf(sc[p], __uint_as_float(v & 0xFFFF0000u), o1);
    }
    float* op = out + (size_t)m * ldo + (size_t)h * hd + 2 * t2;
    op[0] = variant == 0 ? r16(__fmul_rn(o0, inv)) : r16(o0);
    op[1] = variant == 0 ? r16(__fmul_rn(o1, inv)) : r16(o1);
  }
}

// ---- prefill attention, R consecutive query rows of one head per block.  The rows of a prefill
// chunk share their keys (global layers: 0..pos; sliding: a window that moves by one per row), so a
// block takes rows m0..m0+R-1 (positions pos0+m0..) of head h over the union of their key ranges
// [lo_0, pos_{R-1}]: every K row it loads feeds R score chains, every V element R O chains, and the
// R in-order weight sums run side by side.  Per (row, head) the values are k_attn_rows's with
// variant < 0: scores in the variant's lane order, the row max, exp8 / the correctly rounded exp,
// the in-order sum, O per dim over the row's keys in order, rounded to bf16.  Keys outside a row's
// range get weight +0 in its O chain, which leaves the chain bit-exact: it starts at +0, an FMA of
// a zero weight adds a signed zero to it (x + (-0) = x, and +0 + -0 = +0 under round-to-nearest),
// and the chain can never hold -0 (it starts at +0 and an exact zero sum rounds to +0).  A group
// whose rows take different variants runs its rows one at a time.  blockDim 256, hd <= 256, hd % 16
// == 0; dynamic shared memory R * span floats, span = len_max + R - 1.
template <int R>
__global__ void __launch_bounds__(256) k_attn_rows_multi(const uint16_t* __restrict__ Kc, const uint16_t* __restrict__ Vc,
                                                         const float* __restrict__ q, int ldq, int nh, int hd, int pos0,
                                                         int Mrows, int window, float* __restrict__ out, int ldo,
                                                         int blk_fn, int blk, int span) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sc[];  // [R][span]
  __shared__ float s_red[8][R];
  __shared__ float s_mx[R], s_den[R];
  const int m_first = blockIdx.x * R, h = blockIdx.y, tid = threadIdx.x;
  const int nr_all = min(R, Mrows - m_first);
  auto variant_of = [&](int m) {
    const int pos = pos0 + m;
    const int b0 = pos - (pos - blk_fn) % blk;
    return (blk >= 4 && b0 + blk > 64) ? 0 : 1;
  };
  bool uniform = true;
  for (int r = 1; r < nr_all; ++r) uniform = uniform && variant_of(m_first + r) == variant_of(m_first);
  const int groups = uniform ? 1 : nr_all;
  for (int gi = 0; gi < groups; ++gi) {
    const int m0 = m_first + (uniform ? 0 : gi), nr = uniform ? nr_all : 1;
    const int variant = variant_of(m0);
    const int pos_lo = pos0 + m0, pos_hi = pos_lo + nr - 1;
    const int lo_min = window > 0 ? max(0, pos_lo - (window - 1)) : 0;
    const int sp = pos_hi - lo_min + 1;  // keys of the union (<= span)
    int lo_r[R], hi_r[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int pr = pos_lo + min(r, nr - 1);
      lo_r[r] = (window > 0 ? max(0, pr - (window - 1)) : 0) - lo_min;
      hi_r[r] = r < nr ? pr - lo_min : -1;  // rows past nr own no keys
    }
    // scores: one half-warp per key, the two half-warps of a warp take keys pb and pb+1
    const int hw = tid >> 4, c = tid & 15;
    if (variant == 0) {
      float qr[R][16];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float* qh = q + (size_t)(m0 + min(r, nr - 1)) * ldq + (size_t)h * hd;
#pragma unroll
        for (int i = 0; i < 16; ++i) qr[r][i] = (i < (hd >> 4)) ? qh[c + 16 * i] : 0.f;
      }
      for (int pb = (hw & ~1); pb < sp; pb += 16) {
        const int j = min(pb + (hw & 1), sp - 1);
        const uint16_t* kr = Kc + (size_t)(lo_min + j) * hd;
        float kv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) kv[i] = (i < (hd >> 4)) ? bf2f(kr[c + 16 * i]) : 0.f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (i < (hd >> 4)) acc = fmaf(qr[r][i], kv[i], acc);
          const float s = hsum8_octet(__fadd_rn(acc, __shfl_xor_sync(FULL, acc, 8)));
          if (c == 0 && pb + (hw & 1) < sp && j >= lo_r[r] && j <= hi_r[r]) sc[r * span + j] = s;
        }
      }
    } else {
      float qr[32];  // variant 1 groups are single rows or rows of one block below position 64
      for (int r = 0; r < nr; ++r) {
        const float* qh = q + (size_t)(m0 + r) * ldq + (size_t)h * hd;
#pragma unroll
        for (int i = 0; i < 32; ++i) qr[i] = (c < 8 && i < (hd >> 3)) ? qh[c + 8 * i] : 0.f;
        for (int pb = (hw & ~1); pb < sp; pb += 16) {
          const int j = min(pb + (hw & 1), sp - 1);
          const uint16_t* kr = Kc + (size_t)(lo_min + j) * hd;
          float acc = 0.f;
          if (c < 8) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < (hd >> 3)) acc = fmaf(qr[i], bf2f(kr[c + 8 * i]), acc);
          }
          const float s = hsum8_octet(acc);
          if (c == 0 && pb + (hw & 1) < sp && j >= lo_r[r] && j <= hi_r[r]) sc[r * span + j] = s;
        }
      }
    }
    __syncthreads();
    // row maxima over each row's keys
    float mx[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      mx[r] = -1e30f;
      if (r < nr)
        for (int j = lo_r[r] + tid; j <= hi_r[r]; j += blockDim.x) mx[r] = fmaxf(mx[r], sc[r * span + j]);
#pragma unroll
      for (int o = 16; o; o >>= 1) mx[r] = fmaxf(mx[r], __shfl_xor_sync(FULL, mx[r], o));
      if ((tid & 31) == 0) s_red[tid >> 5][r] = mx[r];
    }
    __syncthreads();
    if (tid < R) {
      float v = -1e30f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v = fmaxf(v, s_red[w][tid]);
      s_mx[tid] = v;
    }
    __syncthreads();
    // weights; +0 outside each row's keys (and for rows past nr)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float m_r = s_mx[r];
      for (int j = tid; j < sp; j += blockDim.x) {
        const bool in = j >= lo_r[r] && j <= hi_r[r];
        const float d = in ? __fsub_rn(sc[r * span + j], m_r) : 0.f;
        sc[r * span + j] = in ? (variant == 0 ? exp8(d) : exp_cr(d)) : 0.f;
      }
    }
    __syncthreads();
    if (tid < nr) {  // the in-order sums, one thread per row, 8 loads in flight ahead of each chain
      const float* w = sc + tid * span;
      float den = 0.f;
      int j = lo_r[tid];
      for (; j + 8 <= hi_r[tid] + 1; j += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = w[j + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) den = __fadd_rn(den, v[u]);
      }
      for (; j <= hi_r[tid]; ++j) den = __fadd_rn(den, w[j]);
      s_den[tid] = den;
    }
    __syncthreads();
    if (variant == 1) {
      for (int r = 0; r < nr; ++r)
        for (int j = lo_r[r] + tid; j <= hi_r[r]; j += blockDim.x) sc[r * span + j] = __fdiv_rn(sc[r * span + j], s_den[r]);
      __syncthreads();
    }
    // O: thread i runs dim i of the R rows over the union's keys in order, 8 V loads in flight
    for (int i = tid; i < hd; i += blockDim.x) {
      float o[R];
#pragma unroll
      for (int r = 0; r < R; ++r) o[r] = 0.f;
      const uint16_t* vp = Vc + (size_t)lo_min * hd + i;
      int p = 0;
      for (; p + 8 <= sp; p += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = bf2f(vp[(size_t)(p + u) * hd]);
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int r = 0; r < R; ++r) o[r] = fmaf(sc[r * span + p + u], v[u], o[r]);
      }
      for (; p < sp; ++p) {
        const float v = bf2f(vp[(size_t)p * hd]);
#pragma unroll
        for (int r = 0; r < R; ++r) o[r] = fmaf(sc[r * span + p], v, o[r]);
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r < nr) {
          const float den = s_den[r];
          out[(size_t)(m0 + r) * ldo + (size_t)h * hd + i] = variant == 0 ? r16(__fmul_rn(o[r], __fdiv_rn(1.0f, den))) : r16(o[r]);
        }
    }
    __syncthreads();  // the next single-row pass reuses the shared arrays
  }
}

int attn_rows_multi(int R, const uint16_t* Kc, const uint16_t* Vc, const float* q, int ldq, int nh, int hd, int pos0,
                    int Mrows, int window, int len_max, float* out, int ldo, int blk_fn, int blk, cudaStream_t st) {
  const int span = len_max + R - 1;
  const size_t smem = sizeof(float) * (size_t)R * span;
  if (hd > 256 || hd % 16 != 0 || smem > 200 * 1024 || (R != 4 && R != 8))
    return set_error(G4_ERR_UNSUPPORTED, "prefill attention: R=%d hd=%d span=%d", R, hd, span);
  auto go = [&](auto kern) -> int {
    if (smem > 40 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return launch("k_attn_rows_multi", kern, dim3((Mrows + R - 1) / R, nh), dim3(256), smem, st, Kc, Vc, q, ldq, nh, hd,
                  pos0, Mrows, window, out, ldo, blk_fn, blk, span);
  };
  return R == 4 ? go(k_attn_rows_multi<4>) : go(k_attn_rows_multi<8>);
}

// ---- prefill attention, four query heads of one row per block (they share the KV head: one read of
// each K and V row serves four heads).  The values are k_attn_rows's, per (row, head): scores in the
// variant's lane order (variant 0, attn_tile :1061-1083: two 8-lane chains of stride 16; variant 1,
// :1337-1355: one 8-lane chain of stride 8), the row max, exp8 (0) or the correctly rounded exp (1),
// the in-order sum of the weights, and O per dim over the keys in order (variant 1 first divides
// each weight by the sum, variant 0 scales O by its inverse), rounded to bf16.  The variant of a row
// is its prefill block's (full blocks of blk rows from position blk_fn).  Block (row, head quad),
// 256 threads; dynamic shared memory 4 x len_max floats.
constexpr int kApHeads = 4;
__global__ void __launch_bounds__(288) k_attn_prefill(const uint16_t* __restrict__ Kc, const uint16_t* __restrict__ Vc,
                                                      const float* __restrict__ q, int ldq, int hd, int pos0, int window,
                                                      int blk_fn, int blk, float* __restrict__ out, int ldo) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sc[];  // [kApHeads][len]
  __shared__ float s_mx[kApHeads], s_den[kApHeads];
  const int m = blockIdx.x, h0 = blockIdx.y * kApHeads;
  const int pos = pos0 + m, lo = window > 0 ? max(0, pos - (window - 1)) : 0, len = pos - lo + 1;
  const int b0 = pos - (pos - blk_fn) % blk;
  const int variant = (blk >= 4 && b0 + blk > 64) ? 0 : 1;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  // scores (threads 0-255): half-warp hw runs (head hw % 4, key slot hw / 4) dots in the variant's order
  if (t < 256) {
    const int hw = t >> 4, c = t & 15, hh = hw & 3, slot = hw >> 2;
    const float* qh = q + (size_t)m * ldq + (size_t)(h0 + hh) * hd;
    float qr[32];
    if (variant == 0) {
#pragma unroll
      for (int i = 0; i < 32; ++i) qr[i] = (i < (hd >> 4)) ? qh[c + 16 * i] : 0.f;
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) qr[i] = (c < 8 && i < (hd >> 3)) ? qh[c + 8 * i] : 0.f;
    }
    float* sh = sc + (size_t)hh * len;
    for (int pb = 0; pb < len; pb += 4) {
      const int pi = min(pb + slot, len - 1);
      const uint16_t* kr = Kc + (size_t)(lo + pi) * hd;
      float acc = 0.f, s;
      if (variant == 0) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < (hd >> 4)) acc = fmaf(qr[i], bf2f(kr[c + 16 * i]), acc);
        s = hsum8_octet(__fadd_rn(acc, __shfl_xor_sync(FULL, acc, 8)));
      } else {
        if (c < 8) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < (hd >> 3)) acc = fmaf(qr[i], bf2f(kr[c + 8 * i]), acc);
        }
        s = hsum8_octet(acc);
      }
      if (c == 0 && pb + slot < len) sh[pb + slot] = s;
    }
  }
  __syncthreads();
  if (wid < kApHeads) {  // per-head max (order-free)
    const float* sh = sc + (size_t)wid * len;
    float mx = -1e30f;
    for (int i = lane; i < len; i += 32) mx = fmaxf(mx, sh[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    if (lane == 0) s_mx[wid] = mx;
  }
  __syncthreads();
  for (int i = t; i < kApHeads * len; i += blockDim.x) {
    const int hq = i / len;
    const float d = __fsub_rn(sc[i], s_mx[hq]);
    sc[i] = variant == 0 ? exp8(d) : exp_cr(d);
  }
  __syncthreads();
  // the in-order sums of the weights: lanes 0-3 of warp 8, one head each (variant 0: while warps
  // 0-7 run the O chains; variant 1 divides by them first)
  auto sums = [&]() {
    if (wid == 8 && lane < kApHeads) {
      const float* sh = sc + (size_t)lane * len;
      float den = 0.f;
      int i = 0;
      for (; i + 8 <= len; i += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = sh[i + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) den = __fadd_rn(den, v[u]);
      }
      for (; i < len; ++i) den = __fadd_rn(den, sh[i]);
      s_den[lane] = den;
    }
  };
  if (variant == 1) {
    sums();
    __syncthreads();
    for (int i = t; i < kApHeads * len; i += blockDim.x) sc[i] = __fdiv_rn(sc[i], s_den[i / len]);
    __syncthreads();
  }
  // O (threads 0-255): thread per dim, the four heads' chains together (one V load, four FMAs)
  float o[kApHeads] = {0.f, 0.f, 0.f, 0.f};
  if (t < 256 && t < hd) {
    const uint16_t* vp = Vc + (size_t)lo * hd + t;
    int p = 0;
    for (; p + 8 <= len; p += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = bf2f(vp[(size_t)(p + u) * hd]);
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int hq = 0; hq < kApHeads; ++hq) o[hq] = fmaf(sc[(size_t)hq * len + p + u], v[u], o[hq]);
    }
    for (; p < len; ++p) {
      const float v = bf2f(vp[(size_t)p * hd]);
#pragma unroll
      for (int hq = 0; hq < kApHeads; ++hq) o[hq] = fmaf(sc[(size_t)hq * len + p], v, o[hq]);
    }
  } else if (variant == 0) {
    sums();
  }
  __syncthreads();  // the sums are ready
  if (t < 256 && t < hd) {
#pragma unroll
    for (int hq = 0; hq < kApHeads; ++hq) {
      const float r = variant == 0 ? r16(__fmul_rn(o[hq], __fdiv_rn(1.0f, s_den[hq]))) : r16(o[hq]);
      out[(size_t)m * ldo + (size_t)(h0 + hq) * hd + t] = r;
    }
  }
}

// ---- drafter candidates (dcand_task :675-722): score c = hsum(a + b) of the two 8-lane chains
// of stride 16 (the same shape as the attention score), against the tied embedding; then the
// first maximum in candidate order (:1557-1558).  One half-warp per candidate.
__global__ void k_cand_scores(const uint16_t* __restrict__ E, const int* __restrict__ cand, int nc, const float* __restrict__ dh,
                              int H, float* __restrict__ score) {
  pdl_wait();
  pdl_trigger();
  const int hw = (blockIdx.x * blockDim.x + threadIdx.x) >> 4, c = threadIdx.x & 15;
  const int base = hw & ~1;  // warp-uniform
  if (base >= nc) return;
  const int k = min(hw, nc - 1);
  const uint16_t* er = E + (size_t)cand[k] * H;
  float acc = 0.f;
#pragma unroll 16
  for (int i = c; i < H; i += 16) acc = fmaf(__ldg(dh + i), bf2f(__ldg(er + i)), acc);
  const float s = hsum8_octet(__fadd_rn(acc, __shfl_xor_sync(FULL, acc, 8)));
  if (c == 0 && hw < nc) score[hw] = s;
}
// Top-T centroids by score (stable: ties keep the lower centroid first, as the insertion sort of
// :1554-1555 does) and the candidate list cand[t*per + j] = perm((top t)*per + j).
__global__ void __launch_bounds__(256) k_topk_cand(const float* __restrict__ score, int n, int T, int per, int vocab,
                                                   int* __restrict__ cand) {
  pdl_wait();
  pdl_trigger();
  // block of 32 scores (one per lane); the 8 warps each count the higher-ranked scores in one
  // eighth of the list, and the partial ranks are summed (rank = #(s_j > v) + #(s_j == v, j < i))
  extern __shared__ float s[];
  __shared__ int part[8][32];
  for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = score[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + lane;
  const float v = i < n ? s[i] : 0.f;
  const int span = (n + 7) / 8, j0 = w * span, j1 = min(n, j0 + span);
  int rank = 0;
#pragma unroll 8
  for (int j = j0; j < j1; ++j) rank += (s[j] > v) || (s[j] == v && j < i);
  part[w][lane] = rank;
  __syncthreads();
  __shared__ int rk[32];
  if (w == 0) {
    int r = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) r += part[k][lane];
    rk[lane] = (i < n) ? r : 0x7FFFFFFF;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 32 * per; e += blockDim.x) {
    const int l = e / per, k = e % per, r = rk[l];
    if (r < T) cand[r * per + k] = (int)perm_token((uint32_t)((blockIdx.x * 32 + l) * per + k), (uint32_t)vocab);
  }
}
// first argmax in candidate order -> *best (one block)
__global__ void k_cand_best(const float* __restrict__ score, const int* __restrict__ cand, int nc, int* __restrict__ best) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[32];
  __shared__ int si[32];
  float bv = -1e30f;
  int bi = 0x7FFFFFFF;
  for (int i = threadIdx.x; i < nc; i += blockDim.x)
    if (score[i] > bv) { bv = score[i]; bi = i; }  // per thread: increasing i, strict > keeps the first
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, bv, o);
    const int oi = __shfl_xor_sync(FULL, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    *best = bi < nc ? cand[bi] : -1;
  }
}

// ---- seeded weights ("g4-e2b-synth v1", g4_model.cuh)
__global__ void k_gen_w4(uint64_t seed, uint64_t id, long long nbytes, uint8_t* __restrict__ out) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes; i += (long long)gridDim.x * blockDim.x)
    out[i] = (uint8_t)(wh(seed, id, (uint64_t)i) & 0xFF);
}
__global__ void k_gen_scales(uint64_t seed, uint64_t id, long long n, uint16_t* __restrict__ out) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = (uint16_t)f2bf(__fmul_rn(fabsf(wnorm(wh(seed, id, (uint64_t)i))), 0.01f));
}
__global__ void k_gen_norm(uint64_t seed, uint64_t id, int n, float mul, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = bf2f(f2bf(__fmul_rn(__fadd_rn(1.0f, __fmul_rn(0.1f, wnorm(wh(seed, id, (uint64_t)i)))), mul)));
}
// Per-layer inputs (the int8 branch of gemma4_engine.cpp:1270-1288): block (row m, layer l), 256
// threads, one per input of the layer: p = r16(pr * s1) (s1 = 1/sqrt(H)), its RMS norm with the
// per_layer_projection_norm weights (rms, not rounded), plus the token's table row times 16 rounded
// to bf16, times 2^-0.5.
__global__ void __launch_bounds__(256) k_ple_in(const float* __restrict__ pr, const int* __restrict__ toks,
                                                const uint16_t* __restrict__ table, const float* __restrict__ wn, float s1,
                                                int NL, float* __restrict__ pli) {
  pdl_wait();
  pdl_trigger();
  __shared__ float xs[256];
  __shared__ double red[17];
  const int m = blockIdx.x, l = blockIdx.y, i = threadIdx.x;
  const size_t NP = (size_t)NL * 256, off = (size_t)m * NP + (size_t)l * 256 + i;
  const float p = r16(__fmul_rn(pr[off], s1));
  xs[i] = p;
  __syncthreads();
  const float r = block_rms_scale(xs, 256, red);
  const float pj = __fmul_rn(__fmul_rn(p, r), wn[i]);
  const float pe = r16(__fmul_rn(bf2f(table[(size_t)toks[m] * NP + (size_t)l * 256 + i]), 16.0f));
  pli[off] = __fmul_rn(__fadd_rn(pj, pe), 0.70710678118f);
}

// The per-layer input gate (the int8 branch of :1381-1384): block = row m, 256 threads:
// g2 = r16(r16(gelu(r16 pgv)) * r16(pli of layer l)), and its W4A8 quantisation (qo.q set) for the
// per_layer_projection.
__global__ void __launch_bounds__(256) k_ple_gate(const float* __restrict__ pgv, const float* __restrict__ pli, int l, int NL,
                                                  float* __restrict__ g2, QuantOut qo) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x, i = threadIdx.x;
  const float g = r16(pgv[(size_t)m * 256 + i]);
  const float v = r16(__fmul_rn(r16(gelu(g)), r16(pli[(size_t)m * NL * 256 + (size_t)l * 256 + i])));
  g2[(size_t)m * 256 + i] = v;
  if (qo.q) {
    int8_t q;
    float sx;
    int32_t tot;
    quant_group32(v, q, sx, tot);
    qo.q[(size_t)m * 256 + i] = q;
    if ((i & 31) == 0) {
      qo.sx[(size_t)m * 8 + (i >> 5)] = sx;
      qo.sum[(size_t)m * 8 + (i >> 5)] = tot;
    }
  }
}

// bf16 table of n values mul * r (the per-layer embedding table; the embedding is k_gen_embed).
__global__ void k_gen_bf16(uint64_t seed, uint64_t id, long long n, float mul, uint16_t* __restrict__ out) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = (uint16_t)f2bf(__fmul_rn(mul, wnorm(wh(seed, id, (uint64_t)i))));
}

__global__ void k_gen_embed(uint64_t seed, long long n, uint16_t* __restrict__ out) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = (uint16_t)f2bf(__fmul_rn(0.02f, wnorm(wh(seed, T_EMBED, (uint64_t)i))));
}

}  // namespace g4

extern "C" int g4_rmsnorm(const float* x, const float* w, int M, int n, float* y, int round, int8_t* q, float* sx,
                          int32_t* sum, void* stream) {
  using namespace g4;
  G4_REQUIRE(x && w && y && (q == nullptr || (sx && sum)), "g4_rmsnorm: null pointer");
  G4_REQUIRE(M >= 1 && n >= 256 && n <= kRowMax && n % 256 == 0, "g4_rmsnorm: unsupported shape M=%d n=%d", M, n);
  G4_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(y, 16) && (q == nullptr || aligned(q, 4)),
             "g4_rmsnorm: x, w and y must be 16-byte aligned, q 4-byte aligned");
  if (int rc = launch("k_norm_q", k_norm_q, dim3(M), dim3(256), 0, as_stream(stream), x, w, n, y, round,
                      QuantOut{q, sx, sum}))
    return rc;
  return check_launch("k_norm_q");
}
