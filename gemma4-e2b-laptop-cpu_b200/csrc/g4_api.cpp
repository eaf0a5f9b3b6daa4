// Error reporting and version for the C ABI (include/g4.h).
#include "g4_api.h"
#include <cstring>
#include <cudaTypedefs.h>
#include <mutex>

namespace g4 {
static thread_local char g_msg[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof g_msg, fmt, ap);
  va_end(ap);
  return code;
}

bool encode_tmap_2d(CUtensorMap* out, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return fn(out, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

long long& launch_count() {
  static thread_local long long n = 0;
  return n;
}

bool& pdl_enabled() {
  static thread_local bool on = false;
  return on;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(G4_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return G4_OK;
}
}  // namespace g4

extern "C" const char* g4_last_error(void) { return g4::g_msg; }
extern "C" int g4_abi_version(void) { return 7; }

namespace g4 {
unsigned status_read_linear(bool reset);
unsigned status_read_attn(bool reset);
unsigned status_read_head(bool reset);
unsigned status_read_tc(bool reset);
unsigned status_read_stream(bool reset);
std::atomic<bool>& inflight_fault() {
  static std::atomic<bool> f{false};
  return f;
}
}

// OR of the device status words of all kernel files on the current device; reset clears them.
extern "C" int g4_device_status(unsigned* out, int reset) {
  if (!out) return g4::set_error(G4_ERR_INVALID, "g4_device_status: null pointer");
  unsigned v = 0;
  v |= g4::status_read_linear(reset != 0);
  v |= g4::status_read_attn(reset != 0);
  v |= g4::status_read_head(reset != 0);
  v |= g4::status_read_tc(reset != 0);
  v |= g4::status_read_stream(reset != 0);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return g4::set_error(G4_ERR_CUDA, "g4_device_status: %s", cudaGetErrorString(e));
  // bit 1: memory of a CTA that ended may have been written after it ended; nothing is launched
  // through this library until the status is reset
  if (reset) g4::inflight_fault().store(false);
  else if (v & 2u) g4::inflight_fault().store(true);
  *out = v;
  return G4_OK;
}
