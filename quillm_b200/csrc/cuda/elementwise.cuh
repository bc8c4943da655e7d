#pragma once
#include "common.cuh"

namespace qmc {

constexpr int kMaxRopeHalf = 128;  // head_dim <= 256
// (cos, sin) per rotation pair for one position, computed on the host with the reference's double math
struct RopeRow {
    float v[2 * kMaxRopeHalf];
};

int launch_quantize_rows(int dtype, const float *x, void *out, int64_t rows, int64_t cols, cudaStream_t s);
int launch_dequantize_rows(int dtype, const void *in, float *y, int64_t rows, int64_t cols, cudaStream_t s);
int launch_embed(int dtype, const void *table, int64_t cols, const int *token, float *x, cudaStream_t s, bool pdl);
// argmax of x[0..n) into *out.  With step_ctr (device-resident generation), step s: *out becomes the
// next input token (forced[s+1] while s+1 < *forced_n, i.e. while the prompt lasts, else the argmax),
// the argmax of every step s >= *forced_n - 1 goes to tokens_out[s + 1 - *forced_n], *advance_pos and
// *step_ctr are incremented.
int launch_argmax(const float *x, int n, int *out, cudaStream_t s, bool pdl, int *advance_pos = nullptr,
                  const int *forced = nullptr, const int *forced_n = nullptr, int *step_ctr = nullptr,
                  int *tokens_out = nullptr, int tokens_cap = 0);
int launch_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps, cudaStream_t s);
int launch_softmax(float *x, int64_t n, cudaStream_t s);
int launch_rope(float *v, int64_t n_heads, int64_t hd, const RopeRow &cs, cudaStream_t s);
int launch_swiglu(float *g, const float *u, int64_t n, cudaStream_t s);
int launch_dot(int dtype, const void *w, const void *xq, int64_t n, float *out, cudaStream_t s);

// host: (cos, sin) of pos * theta^(-2i/hd) in double, rounded to float (src/ops.c:116-118)
void rope_row_host(int64_t pos, int64_t hd, float theta, float *out_cs);

}  // namespace qmc
