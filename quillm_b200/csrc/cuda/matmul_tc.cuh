// Quantized-weight prefill contraction on the tensor cores (tcgen05.mma kind::i8); see matmul_tc.cu.
#pragma once
#include "common.cuh"

namespace qmc {
// row pitch (in floats) of the block-major activation scales the contraction reads: T rounded up to 4
int64_t matmul_tc_scale_ld(int64_t T);
// C[T][N] = rows of W (split-row layout, row stride wstride) against the Q8_0 activation blocks aq [T][nb*32]
// and their block-major scales adT[b * matmul_tc_scale_ld(T) + t] (launch_quantize_act with dT): row t
// equals qm_matvec(W, A[t]) bit for bit.  With C2, weight row 2i goes to C[t][i] and row 2i + 1 to C2[t][i]
// (an interleaved w1/w3 matrix feeding SwiGLU).  err: device error word for the bounded waits.
int launch_matmul_q_tc(int dtype, const void *Wsplit, int64_t wstride, const int8_t *aq, const float *adT, float *C,
                       float *C2, int64_t T, int64_t N, int64_t K, int *err, cudaStream_t s);
}  // namespace qmc
