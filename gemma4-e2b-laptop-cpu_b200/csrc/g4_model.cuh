// The synthetic Gemma-style E2B model of BASELINE.json configs[4] and its seeded weights.
//
// Architecture (the reference's decoder layer, gemma4_engine.cpp:1256-1404, without the per-layer
// embeddings and KV sharing that the synthetic config drops): hidden 2048, 30 layers (layer l is
// global when l % 5 == 4, else sliding with a 512-token window), 8 query heads and 1 KV head of
// dim 256, RoPE theta 1e6 (global) / 1e4 (sliding) over the full head, GeGLU MLP 8192, RMSNorm
// eps 1e-6, tied 262,144-token head with softcap 30, layer_scalar 1.  The 1/sqrt(256) softmax
// scale is folded into the q_norm weights.
//
// MTP drafter (the reference's structure, draft_step :1534-1563, at the target's width): input
// [emb(tok)*sqrt(H) | h] (4096) -> pre_projection -> 4 q-only layers (3 sliding, 1 global; 8
// heads of 256 attending the target's KV of its last sliding / last global layer up to P) ->
// norm -> post_projection (next h) and 2,048 centroid scores -> top 32 centroids x 128 tokens ->
// candidates scored against the tied embedding -> argmax.  Every linear is int4 W4G32; the
// drafter's run with int8 activations (W4A8) at M = 1.
//
// Weights (generator "g4-e2b-synth v1", counter-based so that every implementation reproduces
// the same bytes): h(id, i) = splitmix64(seed * 0x100000001B3 ^ (id << 40) ^ i);
//   int4 weight byte i (reference layout)  = h & 0xFF
//   unit "normal" r(h) = (float)(four 16-bit fields of h summed - 131070) * 2.642868e-5f
//   W4 scale i  = bf16(|r| * 0.01)        norm weight i = bf16(1 + 0.1 r) (q_norm: bf16((1 + 0.1 r) / 16))
//   embedding i = bf16(0.02 r)            token ordering: perm(i) = (i * 0x9E3779B1 + 12345) mod vocab
#pragma once
#include <cstdint>

namespace g4 {

struct ModelDims {
  int H = 2048, NL = 30, NQ = 8, HD = 256, I = 8192, V = 262144, WINDOW = 512;
  int DL = 4, DCENT = 2048, DTOP = 32, DPER = 128;  // drafter layers, centroids, top centroids, tokens per centroid
  int OWN = 0;  // KV owners: layers [0, OWN) own a KV cache (0 = all)
  int IS = 0;   // MLP width of the KV-shared layers (0 = I)
  int mlp_of(int l) const { return (!owns(l) && IS > 0) ? IS : I; }
  int mlp_max() const { return IS > I ? IS : I; }
  bool global_layer(int l) const { return l % 5 == 4; }
  bool owns(int l) const { return OWN <= 0 || l < OWN; }
  // the layer whose KV cache layer l reads (owner_of, gemma4_engine.cpp:1251): itself, or the last
  // owner of its type; -1 when there is none
  int owner_of(int l) const {
    if (owns(l)) return l;
    for (int j = OWN - 1; j >= 0; --j)
      if (global_layer(j) == global_layer(l)) return j;
    return -1;
  }
};

// tensor ids
enum : uint64_t {
  T_Q = 0, T_K = 1, T_V = 2, T_O = 3, T_GATE = 4, T_UP = 5, T_DOWN = 6,
  T_IN_LN = 8, T_POST_ATTN = 9, T_PRE_FF = 10, T_POST_FF = 11, T_QN = 12, T_KN = 13,
  T_PG = 7, T_PP = 14, T_POST_PLE = 15,  // per-layer input gate, projection and post norm (PLE)
  T_SCALES = 0x100000,
  T_EMBED = 1000, T_FNORM = 1001, T_PLE = 1002, T_PLPROJ = 1003, T_PLNORM = 1004,
  T_DPRE = 2000, T_DPOST = 2001, T_DCENT = 2002, T_DNORM = 2003,
};
__host__ __device__ inline uint64_t layer_id(int l, uint64_t what) { return 16ull * (uint64_t)l + what; }
__host__ __device__ inline uint64_t dlayer_id(int l, uint64_t what) { return 2100ull + 16ull * (uint64_t)l + what; }

__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t wh(uint64_t seed, uint64_t id, uint64_t i) {
  return splitmix64((seed * 0x100000001B3ull) ^ (id << 40) ^ i);
}
__host__ __device__ inline float wnorm(uint64_t h) {
  const int s = (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48) - 131070;
  return (float)s * 2.642868e-5f;
}
// vocab is a power of two and the multiplier is odd, so this is a permutation of [0, vocab)
__host__ __device__ inline uint32_t perm_token(uint32_t i, uint32_t vocab) { return (uint32_t)(((uint64_t)i * 0x9E3779B1ull + 12345ull) & (uint64_t)(vocab - 1)); }

}  // namespace g4
