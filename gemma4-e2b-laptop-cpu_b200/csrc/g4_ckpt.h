// A checkpoint in the reference's format (model.safetensors, read through the reference's index
// file or the safetensors header), memory-mapped read-only.  Used by g4_ckpt.cpp (parsing, the
// C ABI) and by the engine's loader (g4_engine.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "g4.h"

namespace g4 {

// One tensor: dtype as the safetensors header names it ("BF16", "I32", ...), the absolute byte
// offset in the file, its byte count and shape (the fields of one index line, make_index.py).
struct CkTensor {
  std::string dtype;
  size_t off = 0, nbytes = 0;
  std::vector<long long> shape;
};

// The target model's tensor names (the reference's q4 / bfvec / bfp keys,
// gemma4_engine.cpp:1222-1231): layer l's are "layers.<l>." + suffix.
std::string ck_layer(int l, const char* suffix);

}  // namespace g4

struct g4_checkpoint {
  std::string path;
  int fd = -1;
  const uint8_t* base = nullptr;
  size_t size = 0;
  std::map<std::string, g4::CkTensor> t;
  const g4::CkTensor* find(const std::string& name) const {
    auto it = t.find(name);
    return it == t.end() ? nullptr : &it->second;
  }
};

namespace g4 {
// Loader helpers for the engine (sizes checked against the expected shapes; G4_OK or an error with
// the tensor's name in the message).  Each copy is made on stream st and has completed when the
// helper returns: a plain cudaMemcpy from pageable memory may return before its transfer lands, and
// it is not ordered with the engine's non-blocking stream.
// A stack of int4 matrices ("<name>.weight_packed", "<name>.weight_scale"; rows[i] rows each, K
// columns): the reference-layout bytes into w_dev (then packed by the caller), the bf16 scales
// into s_dev.
int ck_load_lin(const g4_checkpoint* ck, const std::vector<std::pair<std::string, int>>& parts, int K, uint8_t* w_dev,
                uint16_t* s_dev, cudaStream_t st);
// A bf16 vector of n elements as fp32 (exact) into dev.
int ck_load_vec(const g4_checkpoint* ck, const std::string& name, int n, float* dev, cudaStream_t st);
// A bf16 matrix [rows][cols] as is into dev.
int ck_load_bf16(const g4_checkpoint* ck, const std::string& name, long long rows, long long cols, uint16_t* dev,
                 cudaStream_t st);
// A bf16 scalar ("layers.<l>.layer_scalar"); 1.0 when the tensor is absent.
int ck_load_scalar(const g4_checkpoint* ck, const std::string& name, float* out);
}  // namespace g4
