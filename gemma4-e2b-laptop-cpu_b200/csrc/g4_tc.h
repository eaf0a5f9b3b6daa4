// Host interface of the tensor-core W4A8 GEMM (g4_tc.cu), used by the engine's prefill.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace g4 {
// Load-time operands: s8 weights (q = t - 8, natural element order) [N][K] and the bf16 group scales
// transposed [K/32][N] and widened to fp32, from a device-layout W4 matrix and its scales.  N, K
// multiples of 128.
int tc_expand_weights(const uint8_t* Wp, const uint16_t* S, int N, int K, int8_t* W8, float* swT, cudaStream_t st);
// Activation group scales [M][G] -> [G][Mpad] (rows past M zeroed).
int tc_transpose_sx(const float* sx, int M, int G, float* sxT, int Mpad, cudaStream_t st);
// Y[m][n] = the W4A8 row chains of activations A (int8 [M][K], scales sxT) against W8 / swT.
int tc_gemm(const int8_t* A, int M, int K, const float* sxT, int Mpad, const int8_t* W8, const float* swT, int N, float* Y,
            int ldy, cudaStream_t st);
}  // namespace g4
