// Device-side sampler (temperature / top-k / top-p, the reference's xorshift64* stream).
#pragma once
#include "common.cuh"

namespace qmc {

// one draw from logits[n] (device) into *out (device); rng: the device-resident xorshift64* state,
// advanced unless the draw is greedy; p: n floats of scratch
int launch_sample(const float *logits, int n, float temperature, int top_k, float top_p, uint64_t *rng, float *p,
                  int32_t *out, cudaStream_t s);

}  // namespace qmc
