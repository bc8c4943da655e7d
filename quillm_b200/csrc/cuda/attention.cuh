#pragma once
#include "common.cuh"

namespace qmc {

struct AttnPlan {
    int nsplit = 1, chunk_max = 1;
    size_t smem = 0;
    size_t part_floats = 0;  // scratch floats: n_kv_local * group * nsplit * (hd + 2)
};

AttnPlan plan_attention(int n_kv_local, int group, int hd, int max_seq, int num_sms);
// q [n_kv_local*group*hd] (RoPE applied), kc/vc: this layer's caches [max_seq][kvl] of float, or of
// __half when kv16; out like q.  cnt: n_kv_local ints, zero on entry, left zero on exit.
int launch_attention(const AttnPlan &a, const float *q, const void *kc, const void *vc, bool kv16, float *out,
                     float *part, int *cnt, const int *pos, int n_kv_local, int group, int hd, int kvl, cudaStream_t s,
                     bool pdl);

}  // namespace qmc
