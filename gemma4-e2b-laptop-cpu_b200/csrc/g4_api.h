// Host-side helpers shared by the C-ABI entry points: thread-local error message and the checks
// every entry point runs before it launches anything.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include "g4.h"
#include <atomic>
#include <utility>

namespace g4 {
int set_error(int code, const char* fmt, ...);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
// After a launch: turn a launch error into G4_ERR_CUDA with the kernel's name.
int check_launch(const char* what);
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
struct QuantOut;
// Programmatic dependent launch.  While pdl_enabled() is set on this host thread (the engine sets
// it while it records a decode round into a CUDA graph), launch() gives kernels the programmatic
// stream serialisation attribute: such a kernel may start while its predecessor on the stream is
// still running, and its pdl_wait() (g4_common.cuh) blocks until that predecessor has finished and
// its writes are visible.  Every kernel launched this way calls pdl_wait() before it touches
// anything an earlier kernel writes, so only read-only prologues (weight prefetches, barrier set-up)
// overlap the previous kernel.  Otherwise launch() is an ordinary <<<>>> launch.
// A 2D tiled tensor map over a row-major [outer][inner] array (row stride stride_bytes), boxes of
// [box_outer][box_inner] elements, for cp.async.bulk.tensor loads (cuTensorMapEncodeTiled, reached
// through the runtime's driver entry point).  False when the driver lacks it or rejects the map.
bool encode_tmap_2d(CUtensorMap* out, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);
bool& pdl_enabled();
// Set when g4_device_status() has seen the in-flight bit (bit 1) and cleared by its reset: while
// set, launch() refuses every kernel, since a CTA's shared or tensor memory may have been written
// after that CTA ended.
std::atomic<bool>& inflight_fault();
// Kernels started through launch() on this host thread (the engine counts its launches with it).
long long& launch_count();
template <typename... KArgs, typename... Args>
inline int launch(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                  Args&&... args) {
  if (inflight_fault().load(std::memory_order_relaxed))
    return set_error(G4_ERR_TIMEOUT, "%s: refused: a kernel ended with copies in flight (device status bit 1); "
                                     "reset the device status first", what);
  cudaError_t e;
  if (pdl_enabled()) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  } else {
    kern<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  ++launch_count();
  return G4_OK;
}

// Split-KV attention whose key ranges are computed on the device from a position (g4_attn.cu); the
// output rows are also quantised for a W4A8 linear when qo.q is set.  zeroed_counters (may be NULL):
// M*nh ints that are 0 on entry, reserved for such calls (they are 0 again when the call
// completes); with them no counter reset is enqueued.
// g4_head_screen with the fallback GEMV over the unpacked copy of the head (unp, may be NULL).
int head_screen_impl(const uint8_t* W4p, const uint16_t* S4, const float* coef, const uint8_t* data, const uint8_t* unp,
                     const uint8_t* cb8, const long long* exc_ptr, const uint16_t* exc_col, const float* exc_delta, int N,
                     int K, const float* H, int M, int lim, int* out_idx, int* out_nsurv, void* ws, size_t ws_bytes,
                     void* stream, int* policy = nullptr, const uint8_t* nib = nullptr);
// The W4G32 GEMV of the head screen, skipped on the device while *skip != 0 (skip may be NULL).
// Only the TMA-fed variant reads the flag; shapes it does not serve run ungated.
int w4g32_gemm_gated(const uint8_t* Wp, const uint16_t* S, const float* X, int M, int N, int K, float* Y, int ldy,
                     const int* skip, cudaStream_t st);
int attn_splitkv_dev(const uint16_t* Kc, const uint16_t* Vc, const float* q, int M, int nh, int hd, const int* dP,
                     int base_add, int q_add, int window, int max_len, int T, float* out, void* ws, size_t ws_bytes,
                     cudaStream_t st, QuantOut qo, int* zeroed_counters = nullptr);
}  // namespace g4

#define G4_REQUIRE(cond, ...) \
  do { if (!(cond)) return ::g4::set_error(G4_ERR_INVALID, __VA_ARGS__); } while (0)
