// Host-side helpers shared by the C-ABI entry points: thread-local error message and the checks
// every entry point runs before it launches anything.
#pragma once
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include "g4.h"

namespace g4 {
int set_error(int code, const char* fmt, ...);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
// After a launch: turn a launch error into G4_ERR_CUDA with the kernel's name.
int check_launch(const char* what);
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
struct QuantOut;
// Split-KV attention whose key ranges are computed on the device from a position (g4_attn.cu); the
// output rows are also quantised for a W4A8 linear when qo.q is set.
int attn_splitkv_dev(const uint16_t* Kc, const uint16_t* Vc, const float* q, int M, int nh, int hd, const int* dP,
                     int base_add, int q_add, int window, int max_len, int T, float* out, void* ws, size_t ws_bytes,
                     cudaStream_t st, QuantOut qo);
}  // namespace g4

#define G4_REQUIRE(cond, ...) \
  do { if (!(cond)) return ::g4::set_error(G4_ERR_INVALID, __VA_ARGS__); } while (0)
