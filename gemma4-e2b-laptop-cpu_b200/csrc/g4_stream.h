// Host interface of the persistent layer-segment kernel (g4_stream.cu), used by the engine.
#pragma once
#include <cstddef>
#include <cuda_runtime.h>
#include <stdint.h>

namespace g4 {

struct SegLin {  // one int4 matrix in the device layout of g4_w4_pack
  const uint8_t* w;
  const uint16_t* s;
  int N, K;
};

// One launch: do_mlp runs layer l's o projection, post-attention residual + pre-MLP norm, gate/up
// + GeGLU and down projection, post-MLP residual; do_qkv then runs the next layer's input norm (or,
// without do_mlp, the embedding and layer 0's input norm), its qkv projection and q/k/v post
// (norms, RoPE, KV write).  do_mlp without do_qkv ends with the final norm into hbuf.
struct SegParams {
  int M, H, I, QD, HD, NQ;
  int do_mlp, do_qkv;
  SegLin o, gu, down, qkv;
  // layer l (do_mlp)
  const int8_t* att_q;
  const float* att_sx;
  const int32_t* att_sum;
  float* o_out;
  const float *w_post_attn, *w_pre_ff, *w_post_ff;
  int8_t* act_q;
  float* act_sx;
  int32_t* act_sum;
  float* down_out;
  // residual stream: x_a at entry and exit, x_b in between
  float *x_a, *x_b;
  // next layer input norm (or the final norm when !do_qkv) and its outputs
  const float* w_next;
  float* hbuf;
  float* qkv_out;
  const float *qn, *kn, *cosT, *sinT;
  uint16_t *Kc, *Vc;
  float* qs;
  int ldq;
  const int* dpos;  // device position base (may be NULL): row m is at position *dpos + pos0 + m
  int pos0;
  // embedding (first launch of a pass)
  const uint16_t* E;
  const int* toks;
  float sqrtH;
  // grid barriers of this launch (4 counters, zero at launch) and the pass's abort flag
  unsigned* bar;
  unsigned* abort_flag;
  // stage timestamps (%globaltimer, may be NULL): [slot][first CTA, last CTA][kSegStamps]
  unsigned long long* trace;
  int trace_slot;
};
constexpr int kSegStamps = 24;

size_t seg_smem_bytes(int M);
int seg_check(const SegParams& p);
int seg_launch(const SegParams& p, cudaStream_t st);

}  // namespace g4
