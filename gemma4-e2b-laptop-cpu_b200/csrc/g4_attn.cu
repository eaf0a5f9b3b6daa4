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

namespace g4 {

struct AttnDesc {
  int M, nh, hd, kmin, kmax, T;
  int pos[4], lo[4];
};

__device__ __forceinline__ bool allowed(const AttnDesc& d, int m, int p) { return p >= d.lo[m] && p <= d.pos[m]; }
__device__ __forceinline__ int chunk_lo(const AttnDesc& d, int t) {
  const int len = d.kmax - d.kmin + 1;
  return d.kmin + (int)((long long)t * len / d.T);
}

// Workspace layout (floats): S [len][M][nh] scores then weights, AM [T][M][nh], AL [T][M][nh],
// AO [T][M][nh][hd].
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

// ---- scores.  Block = 256 threads = 16 half-warps; half-warp (m, h) pairs are spread over the
// blocks' y dimension.  Each block walks KB keys; K rows come from L1/L2 (each row is read by the
// M*nh half-warps of the key).  q for the half-warp's (m, h) stays in registers (16 floats/lane).
constexpr int kScoreKeys = 32;
__global__ void __launch_bounds__(256) k_attn_scores(const uint16_t* __restrict__ Kc, const float* __restrict__ q,
                                                     AttnDesc d, float* __restrict__ ws) {
  const AttnWs w = attn_ws(ws, d);
  const int hw = threadIdx.x >> 4, c = threadIdx.x & 15;
  const int mh = blockIdx.y * 16 + hw;  // (m, h) pair of this half-warp
  const bool live_mh = mh < d.M * d.nh;
  const int m = live_mh ? mh / d.nh : 0, h = live_mh ? mh % d.nh : 0;
  const int steps = d.hd >> 4;  // <= 32 (hd <= 512)
  float qr[32];
  const float* qh = q + ((size_t)m * d.nh + h) * d.hd;
#pragma unroll
  for (int i = 0; i < 32; ++i) qr[i] = (i < steps) ? qh[c + 16 * i] : 0.f;
  const int p0 = d.kmin + blockIdx.x * kScoreKeys;
  const int p1 = min(p0 + kScoreKeys, d.kmax + 1);
  for (int p = p0; p < p1; ++p) {
    const uint16_t* kr = Kc + (size_t)p * d.hd;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < steps) acc = fmaf(qr[i], bf2f(__ldg(kr + c + 16 * i)), acc);
    // t_l = s0_l + s1_l (lanes l and l+8 of the half-warp), then the 8-lane hsum tree.
    const float t = __fadd_rn(acc, __shfl_xor_sync(FULL, acc, 8));
    const float sc = hsum8_octet(t);
    if (c == 0 && live_mh && allowed(d, m, p)) w.S[((size_t)(p - d.kmin) * d.M + m) * d.nh + h] = sc;
  }
}

// ---- chunk statistics: one warp per (t, m, h).  max is order-free; the weights exp8(s - max)
// are elementwise; their sum runs in key order in lane 0 (a batch of 32 keys at a time).
__global__ void __launch_bounds__(256) k_attn_stats(AttnDesc d, float* __restrict__ ws) {
  const AttnWs w = attn_ws(ws, d);
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (wid >= d.T * d.M * d.nh) return;
  const int t = wid / (d.M * d.nh), m = (wid / d.nh) % d.M, h = wid % d.nh;
  const int c0 = chunk_lo(d, t), c1 = chunk_lo(d, t + 1);
  float mx = -1e30f;
  for (int p = c0 + lane; p < c1; p += 32)
    if (allowed(d, m, p)) mx = fmaxf(mx, w.S[((size_t)(p - d.kmin) * d.M + m) * d.nh + h]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  float l8 = 0.f;
  for (int pb = c0; pb < c1; pb += 32) {
    const int p = pb + lane;
    float wt = 0.f;
    const bool ok = p < c1 && allowed(d, m, p);
    if (ok) {
      float* sp = &w.S[((size_t)(p - d.kmin) * d.M + m) * d.nh + h];
      wt = exp8(__fsub_rn(*sp, mx));
      *sp = wt;
    }
    const unsigned okm = __ballot_sync(FULL, ok);
    for (int k = 0; k < 32; ++k) {  // lane 0 adds the batch in key order
      const float v = __shfl_sync(FULL, wt, k);
      if ((okm >> k) & 1u) l8 = __fadd_rn(l8, v);
    }
  }
  if (lane == 0) {
    const size_t ix = ((size_t)t * d.M + m) * d.nh + h;
    w.AM[ix] = mx;
    w.AL[ix] = (d.lo[m] > d.pos[m]) ? 0.0f : l8;
  }
}

// ---- O accumulation: block = (chunk t, 32-dim slice); thread = (m, h, dim).  Each thread runs
// its fma chain over the chunk's keys in order; a warp shares (m, h), so the weight load is a
// broadcast and the V loads are one 64-byte row segment shared by all warps of the block.
__global__ void __launch_bounds__(1024) k_attn_accum(const uint16_t* __restrict__ Vc, AttnDesc d,
                                                     float* __restrict__ ws) {
  const AttnWs w = attn_ws(ws, d);
  const int t = blockIdx.x, i = blockIdx.y * 32 + (threadIdx.x & 31);
  const int mh = threadIdx.x >> 5;
  if (mh >= d.M * d.nh || i >= d.hd) return;
  const int m = mh / d.nh, h = mh % d.nh;
  const int c0 = chunk_lo(d, t), c1 = chunk_lo(d, t + 1);
  const int a = max(c0, d.lo[m]), b = min(c1 - 1, d.pos[m]);
  float o = 0.f;
  const float* wp = w.S + (size_t)m * d.nh + h;
  const size_t wstride = (size_t)d.M * d.nh;
#pragma unroll 4
  for (int p = a; p <= b; ++p) o = fmaf(wp[(size_t)(p - d.kmin) * wstride], bf2f(__ldg(Vc + (size_t)p * d.hd + i)), o);
  w.AO[(((size_t)t * d.M + m) * d.nh + h) * d.hd + i] = o;
}

// ---- merge: thread per (m, h, dim).  M0 = max of the chunk maxima with L > 0; sc_t =
// expf(M_t - M0) (correctly rounded here); l = sum L_t*sc_t in double (each product exact);
// out = r16((sum_t fma(O_t, sc_t)) * (float)(1/l)).
__global__ void __launch_bounds__(256) k_attn_merge(AttnDesc d, const float* __restrict__ ws, float* __restrict__ out) {
  const AttnWs w = attn_ws(const_cast<float*>(ws), d);
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= d.M * d.nh * d.hd) return;
  const int i = idx % d.hd, mh = idx / d.hd, m = mh / d.nh, h = mh % d.nh;
  float M0 = -1e30f;
  for (int t = 0; t < d.T; ++t) {
    const size_t ix = ((size_t)t * d.M + m) * d.nh + h;
    if (w.AL[ix] > 0) M0 = fmaxf(M0, w.AM[ix]);
  }
  double l = 0;
  float acc = 0.f;
  for (int t = 0; t < d.T; ++t) {
    const size_t ix = ((size_t)t * d.M + m) * d.nh + h;
    if (!(w.AL[ix] > 0)) continue;
    const float sc = exp_cr(__fsub_rn(w.AM[ix], M0));
    l = fma((double)w.AL[ix], (double)sc, l);
    acc = fmaf(w.AO[ix * d.hd + i], sc, acc);
  }
  const float inv = (float)(1.0 / l);
  out[idx] = r16(__fmul_rn(acc, inv));
}

}  // namespace g4

G4_STATUS_READER(attn)

using namespace g4;

static int fill_desc(AttnDesc& d, int M, int nh, int hd, const int* pos, const int* lo, int kmin, int kmax, int T) {
  G4_REQUIRE(M >= 1 && M <= 4 && nh >= 1 && nh <= 8 && hd >= 16 && hd <= 512 && hd % 32 == 0 && T >= 1 && T <= 64,
             "attention: unsupported shape M=%d nh=%d hd=%d T=%d", M, nh, hd, T);
  G4_REQUIRE(pos && lo && kmin >= 0 && kmax >= kmin, "attention: bad key range [%d, %d]", kmin, kmax);
  d.M = M; d.nh = nh; d.hd = hd; d.kmin = kmin; d.kmax = kmax; d.T = T;
  for (int m = 0; m < 4; ++m) { d.pos[m] = m < M ? pos[m] : -1; d.lo[m] = m < M ? lo[m] : 0; }
  for (int m = 0; m < M; ++m)
    G4_REQUIRE(lo[m] >= kmin && pos[m] <= kmax, "attention: row %d range [%d, %d] outside [%d, %d]", m, lo[m], pos[m],
               kmin, kmax);
  return G4_OK;
}

extern "C" size_t g4_attn_splitkv_ws_bytes(int M, int nh, int hd, int kmin, int kmax, int T) {
  return sizeof(float) * attn_ws_floats(M, nh, hd, kmax - kmin + 1, T);
}

extern "C" int g4_attn_splitkv(const uint16_t* Kc, const uint16_t* Vc, const float* q, const int* pos, const int* lo,
                               int M, int nh, int hd, int kmin, int kmax, int T, float* out, void* ws, size_t ws_bytes,
                               void* stream) {
  G4_REQUIRE(Kc && Vc && q && out && ws, "g4_attn_splitkv: null pointer");
  AttnDesc d;
  if (int rc = fill_desc(d, M, nh, hd, pos, lo, kmin, kmax, T)) return rc;
  const size_t need = g4_attn_splitkv_ws_bytes(M, nh, hd, kmin, kmax, T);
  if (ws_bytes < need) return set_error(G4_ERR_NOMEM, "g4_attn_splitkv: workspace %zu < %zu bytes", ws_bytes, need);
  G4_REQUIRE(aligned(ws, 16), "g4_attn_splitkv: workspace must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  float* w = static_cast<float*>(ws);
  const int len = kmax - kmin + 1;
  k_attn_scores<<<dim3((len + kScoreKeys - 1) / kScoreKeys, (M * nh + 15) / 16), 256, 0, st>>>(Kc, q, d, w);
  if (int rc = check_launch("k_attn_scores")) return rc;
  k_attn_stats<<<(T * M * nh * 32 + 255) / 256, 256, 0, st>>>(d, w);
  if (int rc = check_launch("k_attn_stats")) return rc;
  k_attn_accum<<<dim3(T, (hd + 31) / 32), M * nh * 32, 0, st>>>(Vc, d, w);
  if (int rc = check_launch("k_attn_accum")) return rc;
  k_attn_merge<<<(M * nh * hd + 255) / 256, 256, 0, st>>>(d, w, out);
  return check_launch("k_attn_merge");
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
// cudaGetSymbolAddress, looked up once per device (with that device current) by the first call on
// it, so make that first call before any stream capture.  All calls on a device share the array
// and it keeps the previous call's contents; every word a call reads is written earlier in the
// same call, so nothing needs clearing, but two calls whose kernels overlap on the GPU (two
// streams, or two host threads) race on it and must be serialised by the caller.
constexpr size_t kAttnNoAllocFloats = (size_t)8192 * 4 * 8 + 2 * (size_t)8 * 4 * 8 + (size_t)8 * 4 * 8 * 256;
static __device__ __align__(256) float g_attn_scratch[kAttnNoAllocFloats];

#include <mutex>
static std::mutex g_attn_scratch_mu;
static float* g_attn_scratch_dev[128];

static int attn_scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "g4_attn_splitkv_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return set_error(G4_ERR_UNSUPPORTED, "g4_attn_splitkv_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lk(g_attn_scratch_mu);
  if (g_attn_scratch_dev[dev] == nullptr) {
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
  if (int rc = fill_desc(d, M, nh, hd, pos, lo, kmin, kmax, T)) return rc;
  const int len = kmax - kmin + 1;
  if (hd > 256 || T > 8 || len > 8192 || attn_ws_floats(M, nh, hd, len, T) > kAttnNoAllocFloats)
    return set_error(G4_ERR_UNSUPPORTED,
                     "g4_attn_splitkv_noalloc: M=%d nh=%d hd=%d T=%d keys=%d exceed the fixed scratch "
                     "(hd <= 256, T <= 8, keys <= 8192); use g4_attn_splitkv with a workspace",
                     M, nh, hd, T, len);
  float* w = nullptr;
  if (int rc = attn_scratch_for_current_device(&w)) return rc;
  cudaStream_t st = as_stream(stream);
  k_attn_scores<<<dim3((len + kScoreKeys - 1) / kScoreKeys, (M * nh + 15) / 16), 256, 0, st>>>(Kc, q, d, w);
  if (int rc = check_launch("k_attn_scores")) return rc;
  k_attn_stats<<<(T * M * nh * 32 + 255) / 256, 256, 0, st>>>(d, w);
  if (int rc = check_launch("k_attn_stats")) return rc;
  k_attn_accum<<<dim3(T, (hd + 31) / 32), M * nh * 32, 0, st>>>(Vc, d, w);
  if (int rc = check_launch("k_attn_accum")) return rc;
  k_attn_merge<<<(M * nh * hd + 255) / 256, 256, 0, st>>>(d, w, out);
  return check_launch("k_attn_merge");
}
