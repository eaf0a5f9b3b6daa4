// Declarations of the decoder-layer kernels (g4_layers.cu) used by the engine (g4_engine.cu).
#pragma once
#include "g4_common.cuh"
#include "g4_model.cuh"

namespace g4 {
__global__ void k_rmsnorm(const float* x, const float* w, int n, float* y, int round);
__global__ void k_embed(const uint16_t* E, const int* toks, int H, float sqrtH, float* x);
// dpos (device, may be NULL) is added to the position argument: pos0 / pos is then an offset.
// The rotated query heads go to qdst (row m at qdst + m*ldq; qdst = qkv, ldq = ldqkv for in place).
__global__ void k_qkv_post(const float* qkv, int ldqkv, int nq, int hd, int pos0, const int* dpos, const float* qn,
                           const float* kn, const float* cosT, const float* sinT, uint16_t* Kc, uint16_t* Vc,
                           float* qdst, int ldq);
__global__ void k_qkv_post_w(const float* qkv, int ldqkv, int nq, int hd, int pos0, const int* dpos, const float* qn,
                             const float* kn, const float* cosT, const float* sinT, uint16_t* Kc, uint16_t* Vc,
                             float* qdst, int ldq);
__global__ void k_q_post(float* q, int hd, int pos, const int* dpos, const float* qn, const float* cosT, const float* sinT);
__global__ void k_post_attn(float* o, float* x, const float* w_post, const float* w_pre, float* mlp_in, int n);
__global__ void k_post_ff(float* o, float* x, const float* w_post, float scalar, int n);
__global__ void k_act(const float* gu, int I, int M, float* act);
__global__ void k_resid_norm(float* o, float* x, const float* w, int n);
// Fused row kernels (one 256-thread block per row, rows up to kRowMax = 2048 wide) that also
// quantise their output for the next W4A8 linear when qo.q is set.
__global__ void k_norm_q(const float* x, const float* w, int n, float* y, int round, QuantOut qo);
__global__ void k_post_attn_q(const float* o, float* x, const float* w_post, const float* w_pre, float* mlp_in, int n,
                              QuantOut qo);
__global__ void k_resid_norm_q(const float* o, float* x, const float* w_post, float scalar, int n, const float* w_next,
                               float* a, int round_next, QuantOut qo);
__global__ void k_act_q(const float* gu, int I, int M, float* act, QuantOut qo);
__global__ void k_round(float* p, long long n);
__global__ void k_scale_round(float* p, long long n, float s);
__global__ void k_draft_in(const uint16_t* E, const int* tok, const float* h, int H, float sqrtH, float* out);
// variant < 0: each row takes the variant of its prefill block (full blocks of blk rows from position
// blk_fn), as fwd chooses per block (:1328-1355).
__global__ void k_attn_rows(const uint16_t* Kc, const uint16_t* Vc, const float* q, int ldq, int nh, int hd, int pos0,
                            int window, int variant, float* out, int ldo, int blk_fn = 0, int blk = 32);
// Prefill attention for rows of full prefill blocks with fewer instructions per key (grid (M, nh),
// 256 threads, hd <= 256, hd % 16 == 0, dynamic shared memory len_max floats): the values of
// k_attn_rows with variant < 0.
__global__ void k_attn_rows2(const uint16_t* Kc, const uint16_t* Vc, const float* q, int ldq, int nh, int hd, int pos0,
                             int window, float* out, int ldo, int blk_fn, int blk);
// Prefill attention for rows of full prefill blocks, R consecutive rows of one head per block (grid
// (ceil(Mrows / R), nh), 256 threads, hd <= 256, dynamic shared memory R * span floats with span =
// len_max + R - 1): the values of k_attn_rows with variant < 0.
// Returns G4_ERR_UNSUPPORTED (nothing launched) when the shape does not fit.
int attn_rows_multi(int R, const uint16_t* Kc, const uint16_t* Vc, const float* q, int ldq, int nh, int hd, int pos0,
                    int Mrows, int window, int len_max, float* out, int ldo, int blk_fn, int blk, cudaStream_t st);
// Prefill attention for rows of full prefill blocks, four query heads per block (grid (M, nh / 4),
// 288 threads, hd <= 256, dynamic shared memory 4 * len_max floats): the values of k_attn_rows with variant < 0.
__global__ void k_attn_prefill(const uint16_t* Kc, const uint16_t* Vc, const float* q, int ldq, int hd, int pos0, int window,
                               int blk_fn, int blk, float* out, int ldo);
__global__ void k_cand_scores(const uint16_t* E, const int* cand, int nc, const float* dh, int H, float* score);
__global__ void k_topk_cand(const float* score, int n, int T, int per, int vocab, int* cand);
__global__ void k_cand_best(const float* score, const int* cand, int nc, int* best);
__global__ void k_gen_w4(uint64_t seed, uint64_t id, long long nbytes, uint8_t* out);
__global__ void k_gen_scales(uint64_t seed, uint64_t id, long long n, uint16_t* out);
__global__ void k_gen_norm(uint64_t seed, uint64_t id, int n, float mul, float* out);
__global__ void k_gen_embed(uint64_t seed, long long n, uint16_t* out);
__global__ void k_gen_bf16(uint64_t seed, uint64_t id, long long n, float mul, uint16_t* out);
// Per-layer embeddings (grid (M, NL) / M, 256 threads; 256 inputs per layer).
__global__ void k_ple_in(const float* pr, const int* toks, const uint16_t* table, const float* wn, float s1, int NL,
                         float* pli);
__global__ void k_ple_gate(const float* pgv, const float* pli, int l, int NL, float* g2, QuantOut qo);
}  // namespace g4
