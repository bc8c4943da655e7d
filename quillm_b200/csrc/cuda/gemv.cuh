// Decode matvec (batch 1) over Q8_0 / Q4_0 / f32 weight rows with fused prologues and epilogues.
#pragma once
#include "common.cuh"

namespace qmc {

enum GemvEpi : int {
    EPI_STORE = 0,   // y[r] = v
    EPI_ADD = 1,     // y[r] += v            (residual add, src/model.c:179,186)
    EPI_QKV = 2,     // rows [0,Dq) -> q, [Dq,Dq+KVl) -> K-cache slot, rest -> V-cache slot; RoPE on q and k
    EPI_SWIGLU = 3,  // virtual row 2h = w1[h], 2h+1 = w3[h]; y[h] = silu(g) * u (src/ops.c:128-133)
    EPI_LOGITS = 4,  // y[r] = v, plus the greedy argmax: the last CTA advances the generation state
};

struct GemvArgs {
    int dtype = QMC_Q8_0;
    const void *W0 = nullptr;  // rows x row_bytes, 16-byte aligned
    const void *W1 = nullptr;  // EPI_SWIGLU: the w3 matrix (same shape as W0)
    int64_t rows = 0;          // rows of W0 (EPI_SWIGLU: rows of each matrix)
    int64_t K = 0;             // columns
    const float *x = nullptr;  // f32 input [K]
    const float *norm_w = nullptr;  // fused rmsnorm weight (src/ops.c:93-98), or null
    float eps = 1e-5f;
    int epi = EPI_STORE;
    float *y = nullptr;
    // EPI_QKV
    float *q = nullptr;
    void *kcache = nullptr, *vcache = nullptr;  // caches: layer base, [max_seq][KVl]
    int kv16 = 0;                               // caches hold fp16 (else fp32)
    int Dq = 0, KVl = 0, hd = 0;
    const float2 *rope = nullptr;  // [max_seq][hd/2] (cos, sin) rounded to float exactly as src/ops.c:116-118
    const int *pos = nullptr;      // device position
    // EPI_LOGITS: argmax key/ticket (zero between launches) and the generation state
    unsigned long long *amax_key = nullptr;
    int *amax_ctr = nullptr, *state = nullptr, *gen = nullptr;
    const int *forced = nullptr;
    int gen_cap = 0;
    // optional: also write the Q8_0 activation blocks (the qm_matvec xq scratch)
    void *xq_out = nullptr;
    int *err = nullptr;
};

// Launch on `stream`.  pdl: launch with programmatic stream serialization (the kernel issues its
// weight prefetch before waiting on the previous kernel).  grid_limit 0 = one CTA per SM.
int launch_gemv(const GemvArgs &a, cudaStream_t stream, bool pdl, int grid_limit = 0);

}  // namespace qmc
