// W4A8 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a) for prefill-sized M.
//
// The reference's int8 path (w4a8::tile<MT>, w4a8_avx2.h:46-60) computes, per (activation row m,
// weight row n), the exact integer dot of every 32-group g, a32 = sum t*xq - 8*sum xq with
// t = q + 8 in [0, 15], and then the fp32 chain row = fma(float(a32), sw[n,g]*sx[m,g], row) over
// the groups in order.  Here the integer dots come from tcgen05.mma.kind::i8 with s8 weights
// (q = t - 8, so the product sum is sum (t - 8) xq = a32, exact in int32) and s8 activations: one
// MMA of K = 32 per group writes that group's 128 x 128 dot block into a tensor-memory buffer, and
// the epilogue warps run the fp32 chain group by group from tensor memory.  The chain keeps the
// reference's order, so results are bit-identical to the GEMV path (g4_w4a8_gemm).
//
// CTA tile: 128 activation rows x 128 weight rows.  Warp roles: warps 0-15 epilogue (warp w reads
// tensor-memory lanes 32*(w%4).. and columns 32*(w/4)..; the epilogue is CUDA-core work, so it gets
// as many warps as the register file allows), warp 16 the TMA producer (one thread), warp 17 the
// MMA issuer (one thread; the warp also allocates tensor memory).  A pipeline stage is
// 4 groups (128 bytes of K): the A and B tiles [128][128 B] by 2D tensor-map loads under the 128-byte
// swizzle (the canonical K-major SW128 layout of the MMA's shared-memory descriptors), plus the 4
// groups' activation scales (transposed [G][Mpad]) and weight scales (transposed [G][N]) by bulk
// copies.  Tensor memory holds 4 buffers of 128 columns (int32), one per group of a stage.
// No cluster multicast; every copy reads this GPU's own memory.
#include "g4_api.h"
#include "g4_async.cuh"
#include "g4_common.cuh"
#include "g4_tc.h"
#include <mutex>

namespace g4 {

// warps 0 .. kTcEpi-1: epilogue (4 per tensor-memory lane quarter, kTcCols columns each); then the
// TMA producer warp and the MMA warp
constexpr int kTcEpi = 16;
constexpr int kTcCols = 128 * 4 / kTcEpi;            // columns per epilogue warp
constexpr int kTcProd = kTcEpi, kTcMma = kTcEpi + 1;
constexpr int kTcThreads = (kTcEpi + 2) * 32;
constexpr int kTcNS = 4;
constexpr int kTcTileA = 128 * 128;            // bytes
constexpr int kTcTileB = 128 * 128;
constexpr int kTcSx = 4 * 128 * 4;             // 4 groups x 128 rows fp32
constexpr int kTcSw = 4 * 128 * 4;             // 4 groups x 128 cols, the bf16 scales as fp32
constexpr int kTcStage = 36 * 1024;            // A + B + sx + sw, rounded to 1 KB (swizzle atoms)
constexpr int kTcSmem = kTcNS * kTcStage + 1024;

struct TcShared {
  uint64_t full[kTcNS], empty[kTcNS], accf[4], acce[4], drain;
  uint32_t tmem;
  int abort;
  int issued;  // stages the producer issued
};

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte-swizzled shared-memory matrix descriptor (SBO = 1024 bytes between 8-row
// groups, LBO unused for swizzled K-major layouts, version 1, layout type SWIZZLE_128B = 2).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}
// Instruction descriptor: D s32, A and B s8, both K-major, M = 128, N = 128.
constexpr uint32_t kTcIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

// D (+)= A x B: accumulate = 1 adds the products to what tensor memory holds.
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :
      : "r"(tmem_d), "l"(da), "l"(db), "r"(kTcIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
// The int32 word 0x4B400000 (the float 1.5 x 2^23) into 32 columns of this warp's tensor-memory lanes,
// as four 8-column stores (one 8-register source range instead of 32 registers holding the bias).
constexpr uint32_t kTcBias = 0x4B400000u;
__device__ __forceinline__ void tc_st_bias32(uint32_t taddr) {
  const uint32_t b = kTcBias;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr + 8u * k),
                 "r"(b)
                 : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait; on expiry the CTA's abort flag and the device status word are set.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, TcShared& sh) {
  if (sh.abort) return false;
  if (mbar_wait(bar, parity)) return true;
  atomicOr(&g_dev_status, kStatusTimeout);
  sh.abort = 1;
  return false;
}

__global__ void __launch_bounds__(kTcThreads, 1)
k_w4a8_tc(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, const float* __restrict__ sxT,
          int Mpad, const float* __restrict__ swT, int M, int N, int K, float* __restrict__ Y, int ldy) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ TcShared sh;
  uint8_t* stages = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // 1 KB aligned (swizzle atoms)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128, m0 = blockIdx.y * 128;
  const int G = K >> 5, nst = G >> 2;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcNS; ++i) { mbar_init(&sh.full[i], 1); mbar_init(&sh.empty[i], 1 + kTcEpi); }
    for (int i = 0; i < 4; ++i) { mbar_init(&sh.accf[i], 1); mbar_init(&sh.acce[i], kTcEpi); }
    mbar_init(&sh.drain, 1);
    fence_mbar_init();
    sh.abort = 0;
    sh.issued = 0;
  }
  if (warp == kTcMma) {  // tensor memory: 512 columns = 4 buffers x 128
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem)), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  pdl_wait();
  pdl_trigger();

  if (warp == kTcProd) {
    if (lane == 0) {  // producer
      int s = 0;
      for (; s < nst && !sh.abort; ++s) {
        const int st = s % kTcNS;
        if (s >= kTcNS && !tc_wait(&sh.empty[st], (uint32_t)(((s / kTcNS) - 1) & 1), sh)) break;
        uint8_t* sb = stages + (size_t)st * kTcStage;
        mbar_expect_tx(&sh.full[st], (uint32_t)(kTcTileA + kTcTileB + kTcSx + kTcSw));
        tma_load_2d(sb, &ta, s * 128, m0, &sh.full[st]);
        tma_load_2d(sb + kTcTileA, &tb, s * 128, n0, &sh.full[st]);
        for (int j = 0; j < 4; ++j) {
          bulk_g2s(sb + kTcTileA + kTcTileB + j * 512, sxT + (size_t)(4 * s + j) * Mpad + m0, 512, &sh.full[st]);
          bulk_g2s(sb + kTcTileA + kTcTileB + kTcSx + j * 512, swT + (size_t)(4 * s + j) * N + n0, 512, &sh.full[st]);
        }
        sh.issued = s + 1;
      }
    }
  } else if (warp == kTcMma) {
    if (lane == 0) {  // MMA issuer: per group one K = 32 MMA added into buffer j (which holds the bias)
      for (int s = 0; s < nst; ++s) {
        const int st = s % kTcNS;
        if (!tc_wait(&sh.full[st], (uint32_t)((s / kTcNS) & 1), sh)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(stages + (size_t)st * kTcStage), b0 = a0 + kTcTileA;
        bool ok = true;
        for (int j = 0; j < 4; ++j) {
          // phase s of acce[j]: the epilogue has read buffer j's previous dots and stored the bias again
          // (phase 0: the first bias)
          if (!tc_wait(&sh.acce[j], (uint32_t)(s & 1), sh)) { ok = false; break; }
          tc_fence_after();
          tc_mma(tmem + 128u * j, sw128_desc(a0 + 32u * j), sw128_desc(b0 + 32u * j), 1u);
          tc_commit(&sh.accf[j]);
        }
        if (!ok) break;
        tc_commit(&sh.empty[st]);  // the stage's tiles are free once its MMAs have completed
      }
    }
  } else {
    // epilogue: warp w -> tensor-memory lanes 32 (w % 4).. (tile rows), columns kTcCols (w / 4)..
    const int q = warp & 3, h = warp >> 2;
    const int row = 32 * q + lane;
    float2 acc[kTcCols / 2];  // columns 2c, 2c+1: the chains advance in pairs through packed fp32 operations
#pragma unroll
    for (int c = 0; c < kTcCols / 2; ++c) acc[c] = make_float2(0.f, 0.f);
    // every buffer starts at the bias 1.5 x 2^23 (as an int32 word), which the MMAs add the group's
    // dots to, so the read-back word is the float 1.5 x 2^23 + a32 (exact: |a32| <= 32 x 8 x 128)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int half = 0; half < kTcCols / 32; ++half)
        tc_st_bias32(tmem + ((uint32_t)(32 * q) << 16) + 128u * j + (uint32_t)(kTcCols * h) + 32u * half);
    }
    tc_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int j = 0; j < 4; ++j) arrive(&sh.acce[j]);
    bool ok = true;
    for (int s = 0; s < nst && ok; ++s) {
      const int st = s % kTcNS;
      const uint8_t* sb = stages + (size_t)st * kTcStage;
      const float* sxs = reinterpret_cast<const float*>(sb + kTcTileA + kTcTileB);
      const float* sws = reinterpret_cast<const float*>(sb + kTcTileA + kTcTileB + kTcSx);
      for (int j = 0; j < 4; ++j) {
        if (!tc_wait(&sh.accf[j], (uint32_t)(s & 1), sh)) { ok = false; break; }
        tc_fence_after();
        const float sx = sxs[j * 128 + row];
        const float* sw = sws + j * 128 + kTcCols * h;
#pragma unroll
        for (int half = 0; half < kTcCols / 32; ++half) {
          uint32_t r[32];
          const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + 128u * j + (uint32_t)(kTcCols * h) + 32u * half;
          tc_ld32(ta, r);
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const float4 wlo = *reinterpret_cast<const float4*>(sw + 32 * half + 8 * c8);
            const float4 whi = *reinterpret_cast<const float4*>(sw + 32 * half + 8 * c8 + 4);
            const float2 wv[4] = {make_float2(wlo.x, wlo.y), make_float2(wlo.z, wlo.w), make_float2(whi.x, whi.y),
                                  make_float2(whi.z, whi.w)};
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int c2 = 16 * half + 4 * c8 + v;  // columns 2 c2, 2 c2 + 1
              // the group's integer dots as floats: 1.5 x 2^23 + a32 was formed by the MMA (exact in
              // the mantissa, |a32| < 2^22), so the subtraction is exact
              const float2 a = __fadd2_rn(make_float2(__uint_as_float(r[8 * c8 + 2 * v]), __uint_as_float(r[8 * c8 + 2 * v + 1])),
                                          make_float2(-12582912.0f, -12582912.0f));
              acc[c2] = __ffma2_rn(a, __fmul2_rn(wv[v], make_float2(sx, sx)), acc[c2]);
            }
          }
          tc_st_bias32(ta);  // the bias back for the next stage's MMA (completed before acce[j] below)
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive(&sh.acce[j]);
      }
      __syncwarp();
      if (lane == 0) arrive(&sh.empty[st]);  // this warp has read the stage's scales
    }
    const int m = m0 + row;
    if (ok && m < M) {
      float* yr = Y + (size_t)m * ldy + n0 + kTcCols * h;
#pragma unroll
      for (int c = 0; c < kTcCols / 2; c += 2)
        *reinterpret_cast<float4*>(yr + 2 * c) = make_float4(acc[c].x, acc[c].y, acc[c + 1].x, acc[c + 1].y);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (sh.abort) {  // a wait gave up: before the CTA frees anything, let its own copies and MMAs finish
    if (warp == kTcProd && lane == 0) {
      for (int k = sh.issued > kTcNS ? sh.issued - kTcNS : 0; k < sh.issued; ++k)
        if (!mbar_wait(&sh.full[k % kTcNS], (uint32_t)((k / kTcNS) & 1))) atomicOr(&g_dev_status, kStatusInflight);
    } else if (warp == kTcMma && lane == 0) {
      tc_commit(&sh.drain);
      if (!mbar_wait(&sh.drain, 0)) atomicOr(&g_dev_status, kStatusInflight);
    }
    tc_fence_before();
    __syncthreads();
  }
  if (warp == kTcMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

// ------------------------------------------------------------------------------- helpers
// Device-layout W4 (per 32-group byte b = element b | element 16+b << 4, see g4_w4_pack) -> s8
// weights q = t - 8 in natural element order, [N][K].  One thread per group.
__global__ void k_w8_expand(const uint8_t* __restrict__ Wp, long long groups, int8_t* __restrict__ W8) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= groups) return;
  const uint4 v = reinterpret_cast<const uint4*>(Wp)[i];
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t lo[4], hi[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    // nibble t in [0, 15] -> t - 8 as s8: (t + 0x78) ^ 0x80 per byte = t - 8 (mod 256)
    lo[k] = ((w[k] & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
    hi[k] = (((w[k] >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
  }
  uint4* dst = reinterpret_cast<uint4*>(W8) + 2 * i;
  dst[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  dst[1] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
}

// [R][C] -> [C][ldo] transposes (rows past R are left as they are: zeroed by the caller); the bf16
// weight scales are widened to fp32 on the way (exact), so the epilogue reads them as floats.
__global__ void k_transpose_bf2f(const uint16_t* __restrict__ in, int R, int C, float* __restrict__ out, int ldo) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)R * C) return;
  const int r = (int)(i / C), c = (int)(i % C);
  out[(size_t)c * ldo + r] = __uint_as_float((uint32_t)in[i] << 16);
}
__global__ void k_transpose_f32(const float* __restrict__ in, int R, int C, float* __restrict__ out, int ldo) {
  pdl_wait();
  pdl_trigger();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)R * C) return;
  const int r = (int)(i / C), c = (int)(i % C);
  out[(size_t)c * ldo + r] = in[i];
}

}  // namespace g4

G4_STATUS_READER(tc)

using namespace g4;

namespace g4 {

int tc_expand_weights(const uint8_t* Wp, const uint16_t* S, int N, int K, int8_t* W8, float* swT, cudaStream_t st) {
  if (N % 128 != 0 || K % 128 != 0) return set_error(G4_ERR_UNSUPPORTED, "tensor-core W4A8: N and K must be multiples of 128");
  const long long groups = (long long)N * (K / 32);
  k_w8_expand<<<(unsigned)((groups + 255) / 256), 256, 0, st>>>(Wp, groups, W8);
  const long long ns = (long long)N * (K / 32);
  k_transpose_bf2f<<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(S, N, K / 32, swT, N);
  return check_launch("tc_expand_weights");
}

int tc_transpose_sx(const float* sx, int M, int G, float* sxT, int Mpad, cudaStream_t st) {
  const long long n = (long long)M * G;
  if (Mpad > M && cudaMemsetAsync(sxT, 0, sizeof(float) * (size_t)G * Mpad, st) != cudaSuccess)
    return set_error(G4_ERR_CUDA, "tc_transpose_sx: memset");
  if (int rc = launch("k_transpose_f32", k_transpose_f32, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, sx, M, G, sxT, Mpad))
    return rc;
  return check_launch("k_transpose_f32");
}

// Tensor maps of the A (activations [M][K]) and B (weights [N][K]) operands, cached by pointer.
static bool tc_tmap(const void* base, uint64_t K, uint64_t rows, CUtensorMap* out) {
  static std::mutex mu;
  struct Entry { const void* p; uint64_t K, rows; CUtensorMap m; };
  static Entry cache[256];
  static int used = 0, next = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].p == base && cache[i].K == K && cache[i].rows == rows) { *out = cache[i].m; return true; }
  CUtensorMap m;
  if (!encode_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, K, rows, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return false;
  const int slot = used < 256 ? used++ : (next++ % 256);
  cache[slot] = Entry{base, K, rows, m};
  *out = m;
  return true;
}

int tc_gemm(const int8_t* A, int M, int K, const float* sxT, int Mpad, const int8_t* W8, const float* swT, int N, float* Y,
            int ldy, cudaStream_t st) {
  if (M < 1 || N % 128 != 0 || K % 128 != 0 || Mpad < (M + 127) / 128 * 128 || ldy < N)
    return set_error(G4_ERR_UNSUPPORTED, "tensor-core W4A8: unsupported shape M=%d N=%d K=%d", M, N, K);
  if (!aligned(A, 16) || !aligned(W8, 16) || !aligned(sxT, 16) || !aligned(swT, 16) || !aligned(Y, 16) || ldy % 4 != 0)
    return set_error(G4_ERR_INVALID, "tensor-core W4A8: operands must be 16-byte aligned");
  CUtensorMap ta, tb;
  if (!tc_tmap(A, (uint64_t)K, (uint64_t)M, &ta) || !tc_tmap(W8, (uint64_t)K, (uint64_t)N, &tb))
    return set_error(G4_ERR_UNSUPPORTED, "tensor-core W4A8: tensor maps unavailable");
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_w4a8_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    attr = true;
  }
  if (int rc = launch("k_w4a8_tc", k_w4a8_tc, dim3(N / 128, (M + 127) / 128), dim3(kTcThreads), (size_t)kTcSmem, st, ta, tb,
                      sxT, Mpad, swT, M, N, K, Y, ldy))
    return rc;
  return check_launch("k_w4a8_tc");
}

}  // namespace g4

size_t g4_w4a8_gemm_tc_ws_bytes(int M, int N, int K) {
  const size_t Mpad = (size_t)(M + 127) / 128 * 128;
  return (size_t)N * K + 256 + (size_t)(K / 32) * N * 4 + 256 + (size_t)(K / 32) * Mpad * 4 + 256;
}

extern "C" int g4_w4a8_gemm_tc(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx, int M, int N, int K,
                               float* Y, int ldy, void* ws, size_t ws_bytes, void* stream) {
  G4_REQUIRE(Wp && S && q && sx && Y && ws, "g4_w4a8_gemm_tc: null pointer");
  G4_REQUIRE(M >= 1 && N % 128 == 0 && K % 128 == 0 && ldy >= N, "g4_w4a8_gemm_tc: unsupported shape M=%d N=%d K=%d", M, N, K);
  G4_REQUIRE(ws_bytes >= g4_w4a8_gemm_tc_ws_bytes(M, N, K), "g4_w4a8_gemm_tc: workspace too small");
  G4_REQUIRE(aligned(ws, 256) && aligned(q, 16) && aligned(Y, 16) && aligned(Wp, 16), "g4_w4a8_gemm_tc: misaligned operand");
  cudaStream_t st = as_stream(stream);
  const int Mpad = (M + 127) / 128 * 128, G = K / 32;
  uint8_t* p = static_cast<uint8_t*>(ws);
  int8_t* W8 = reinterpret_cast<int8_t*>(p);
  p += ((size_t)N * K + 255) / 256 * 256;
  float* swT = reinterpret_cast<float*>(p);
  p += ((size_t)G * N * 4 + 255) / 256 * 256;
  float* sxT = reinterpret_cast<float*>(p);
  if (int rc = tc_expand_weights(Wp, S, N, K, W8, swT, st)) return rc;
  if (int rc = tc_transpose_sx(sx, M, G, sxT, Mpad, st)) return rc;
  return tc_gemm(q, M, K, sxT, Mpad, W8, swT, N, Y, ldy, st);
}
