// Shared device helpers for the g4 kernels (sm_100a).
//
// The library is compiled with -fmad=false: every fused multiply-add is written out with
// fmaf(), every other product and sum is rounded on its own, so each kernel reproduces the fp32
// operation order of the reference it names, instruction by instruction.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace g4 {

constexpr unsigned FULL = 0xffffffffu;

// bf16 bits -> fp32 (exact), fp32 -> bf16 round-to-nearest-even with NaN quieting
// (gemma4_engine.cpp:33-35), and the round trip r16 (rbf8, :37-42).
__device__ __forceinline__ float bf2f(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ uint32_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (u >> 16) | 0x40u;
  u += 0x7fffu + ((u >> 16) & 1u);
  return u >> 16;
}
__device__ __forceinline__ float r16(float f) { return bf2f(f2bf(f)); }

// Programmatic dependent launch (see launch() in g4_api.h): pdl_wait() returns once the grid this
// kernel depends on has completed and its writes are visible (at once for an ordinary launch);
// pdl_trigger() allows the next dependent grid to begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// %globaltimer: a nanosecond clock shared by every SM of the device.
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Exact small-integer to float: 0x4B000000 | t is the float 2^23 + t for 0 <= t < 2^23.
__device__ __forceinline__ float u4f(uint32_t t) { return __fsub_rn(__uint_as_float(0x4B000000u | t), 8388608.0f); }

// W4A8 quantisation of one 32-group, lane i owning element x (w4a8_avx2.h:30-42): amax,
// sx = amax/127, inv = sx > 0 ? 1/sx : 0, r = RNE(x*inv) (x86 cvtps_epi32: out of range or NaN ->
// INT32_MIN), tot = sum of the unsaturated r, q = r saturated to int16 then int8.  All 32 lanes.
__device__ __forceinline__ void quant_group32(float x, int8_t& q, float& sx, int32_t& tot) {
  float amax = fabsf(x);
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, o));
  const float s = __fdiv_rn(amax, 127.0f);
  const float inv = s > 0.f ? __frcp_rn(s) : 0.0f;  // = __fdiv_rn(1.0f, s): both correctly rounded
  const float v = __fmul_rn(x, inv);
  const int32_t r = (v > -2147483648.f && v < 2147483648.f) ? __float2int_rn(v) : INT32_MIN;
  int32_t t = r;
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(FULL, t, o);
  const int32_t r16v = r < -32768 ? -32768 : (r > 32767 ? 32767 : r);
  q = (int8_t)(r16v < -128 ? -128 : (r16v > 127 ? 127 : r16v));
  sx = s;
  tot = t;
}

// Destination of a fused W4A8 quantisation: rows of q [M][K], sx and sum [M][K/32] (NULL q = none).
struct QuantOut {
  int8_t* q;
  float* sx;
  int32_t* sum;
};

// Horizontal sum over the 8 consecutive lanes of an octet (lane j holds v_j), in the order of the
// AVX2 hsum (w4g32_avx2.h:41-44): ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)).  Every lane of the octet
// ends with the same value; all 32 lanes of the warp must call it together.
__device__ __forceinline__ float hsum8_octet(float v) {
  const float a = __fadd_rn(v, __shfl_xor_sync(FULL, v, 4));
  const float b = __fadd_rn(a, __shfl_xor_sync(FULL, a, 1));
  return __fadd_rn(b, __shfl_xor_sync(FULL, b, 2));
}

// The reference's Cephes-style exp (gemma4_engine.cpp:43-53), restated operation for operation.
__device__ __forceinline__ float exp8(float x) {
  x = fminf(fmaxf(x, -87.3f), 88.3f);
  const float fx = floorf(fmaf(x, 1.44269504088896341f, 0.5f));
  x = fmaf(-fx, 0.693359375f, x);
  x = fmaf(-fx, -2.12194440e-4f, x);
  const float z = __fmul_rn(x, x);
  float y = 1.9875691500E-4f;
  y = fmaf(y, x, 1.3981999507E-3f);
  y = fmaf(y, x, 8.3334519073E-3f);
  y = fmaf(y, x, 4.1665795894E-2f);
  y = fmaf(y, x, 1.6666665459E-1f);
  y = fmaf(y, x, 5.0000001201E-1f);
  y = fmaf(y, z, __fadd_rn(x, 1.0f));
  const uint32_t n = (uint32_t)(((int)fx + 127) << 23);
  return __fmul_rn(y, __uint_as_float(n));
}

// tanh-GELU of the reference (gelu8, gemma4_engine.cpp:54-60), IEEE division.
__device__ __forceinline__ float gelu(float x) {
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float u = __fmul_rn(0.7978845608028654f, fmaf(0.044715f, x3, x));
  const float e = exp8(__fmul_rn(2.0f, u));
  const float th = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(e, 1.0f)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, th));
}

// Correctly rounded expf: the double-precision exp (error below one double ulp) rounded once
// to float.  glibc's expf, which the reference calls in attn_merge, agrees with it except in
// roughly 6 of 10^4 random arguments, where they differ by one float ulp.
__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }

}  // namespace g4
