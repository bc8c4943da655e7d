#pragma once
#include "common.cuh"

namespace qmc {
int launch_synth(uint64_t seed, uint64_t tid, int dtype, int64_t cols, int64_t r0, int64_t nr, int64_t c0, int64_t nc,
                 double stdv, void *out, cudaStream_t s);
int launch_fill(float *p, int64_t n, float v, cudaStream_t s);
}  // namespace qmc
