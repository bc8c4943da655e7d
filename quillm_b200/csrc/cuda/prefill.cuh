// Batched prompt forward (prefill): the T tokens of a prompt go through every layer together, each
// matrix applied once to all T rows (quantized weights: per-row Q8_0 activations and matmul_q, whose row
// t equals the reference's matvec of row t), with causal attention over the cache.
#pragma once
#include "common.cuh"

namespace qmc {

// x[t] = dequantized row tokens[t] of the embedding table (src/quant.c:65-94)
int launch_embed_rows(int dtype, const void *table, int64_t cols, const int *tokens, int64_t T, float *x, cudaStream_t s);
// out[t] = rmsnorm(x[t]) * w, per row as src/ops.c:93-98
int launch_rmsnorm_rows(const float *x, const float *w, float *out, int64_t T, int64_t n, float eps, cudaStream_t s);
// the Q8_0 blocks (qs [T][nb*32], scales d [T][nb] and, with dT, dT[b * ldT + t]) of rmsnorm(x[t]) * w: the
// same bits as launch_rmsnorm_rows followed by launch_quantize_act, in one pass; with `add` (not null) the
// residual x += add happens first and is written back (the same bits as launch_add before them)
int launch_rmsnorm_quant_rows(float *x, const float *add, const float *w, int64_t T, int64_t n, float eps, int8_t *qs,
                              float *d, float *dT, int64_t ldT, cudaStream_t s);
// the Q8_0 blocks of silu(g[t]) * u[t] (the SwiGLU rows, same bits as launch_swiglu then launch_quantize_act)
int launch_swiglu_quant_rows(const float *g, const float *u, int64_t T, int64_t n, int8_t *qs, float *d, float *dT,
                             int64_t ldT, cudaStream_t s);
// rows of qkv[T][Dq + 2 KVl] at positions pos0 + t: RoPE on the q pairs (in place) and the k pairs, then
// k and v stored in the layer's cache slots [pos][KVl] of float, or of __half when kv16
// (src/model.c:165-173, src/ops.c:114-126)
int launch_rope_kv_rows(float *qkv, int64_t T, int Dq, int KVl, int hd, int pos0, const float2 *rope, void *kc,
                        void *vc, bool kv16, cudaStream_t s);
// out[t][h*hd ..] = causal attention of query head h of row t over cache positions 0 .. pos0 + t
// (src/model.c:132-156), online softmax
int launch_attn_prefill(const float *qkv, int64_t T, int64_t ldq, int n_heads, int group, int hd, int KVl, int pos0,
                        float scale, const void *kc, const void *vc, bool kv16, float *out, cudaStream_t s);
// x += y over n floats (residual, src/model.c:179,186)
int launch_add(float *x, const float *y, int64_t n, cudaStream_t s);

}  // namespace qmc
