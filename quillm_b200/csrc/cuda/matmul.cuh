#pragma once
#include "common.cuh"

namespace qmc {
// A[T,K] f32 -> int8 qs [T][nb*32] and fp32 block scales d [T][nb] (bit-exact Q8_0 quantization); with dT
// the scales also block-major, dT[b * ldT + t]
int launch_quantize_act(const float *x, int64_t T, int64_t K, int8_t *qs, float *d, cudaStream_t s,
                        float *dT = nullptr, int64_t ldT = 0);
int launch_matmul_q(int dtype, const void *W, const int8_t *aq, const float *ad, float *C, int64_t T, int64_t N,
                    int64_t K, cudaStream_t s);
int launch_gemm_f32(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, cudaStream_t s);
}  // namespace qmc
