// Row kernels of the batched prompt forward (prefill).  The matrices themselves go through matmul.cu
// (quantized weights) or gemm_f32; the driver is qmc_model_prefill in model.cu.
#include <algorithm>

#include "prefill.cuh"

namespace qmc {
namespace {

__global__ void embed_rows_kernel(int dtype, const uint8_t *__restrict__ table, int64_t cols,
                                  const int *__restrict__ tokens, float *__restrict__ x) {
    const int64_t t = blockIdx.x;
    const uint8_t *row = table + (int64_t)tokens[t] * row_bytes(dtype, cols);
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) x[t * cols + c] = deq_elem(dtype, row, c);
}

// one row per block: double sum of squares (squares of floats are exact in double), the block sum in a
// fixed order, inv = (float)(1 / sqrt(ss / n + eps)), out = (x * inv) * w with two float roundings
__global__ void rmsnorm_rows_kernel(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ out,
                                    int64_t n, float eps) {
    __shared__ double red[32];
    __shared__ float inv_s;
    const float *xr = x + (int64_t)blockIdx.x * n;
    float *yr = out + (int64_t)blockIdx.x * n;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    double ss = 0.0;
    for (int64_t i = t; i < n; i += blockDim.x) ss = fma((double)xr[i], (double)xr[i], ss);
    ss = warp_sum_d(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (t == 0) {
        double tot = 0.0;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) tot += red[k];
        inv_s = (float)(1.0 / sqrt(tot / (double)n + (double)eps));
    }
    __syncthreads();
    const float inv = inv_s;
    for (int64_t i = t; i < n; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// p0 = x0 c - x1 s ; p1 = x0 s + x1 c, each product and sum rounded separately (src/ops.c:121-123)
__device__ __forceinline__ void rope_rotate(float a, float b, float2 cs, float &o0, float &o1) {
    o0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    o1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
}

__global__ void rope_kv_rows_kernel(float *__restrict__ qkv, int Dq, int KVl, int hd, int pos0,
                                    const float2 *__restrict__ rope, void *__restrict__ kc, void *__restrict__ vc,
                                    bool kv16) {
    const int64_t t = blockIdx.x;
    const int pos = pos0 + (int)t;
    float *row = qkv + t * (int64_t)(Dq + 2 * KVl);
    const float2 *cs = rope + (int64_t)pos * (hd >> 1);
    for (int i = threadIdx.x; i < (Dq + KVl) >> 1; i += blockDim.x) {
        const int e = 2 * i;  // pair (e, e + 1) of q (e < Dq) or k
        float o0, o1;
        rope_rotate(row[e], row[e + 1], cs[(e % hd) >> 1], o0, o1);
        if (e < Dq) row[e] = o0, row[e + 1] = o1;
        else kv_st2(kc, kv16, (int64_t)pos * KVl + (e - Dq), o0, o1);
    }
    for (int i = threadIdx.x; i < KVl >> 1; i += blockDim.x)
        kv_st2(vc, kv16, (int64_t)pos * KVl + 2 * i, row[Dq + KVl + 2 * i], row[Dq + KVl + 2 * i + 1]);
}

// one warp per (query head, token): lane l holds q[l + 32 j] (j < 4, head_dim <= 128); the positions are
// walked 4 at a time with the 4 score reductions interleaved, online softmax (running max, sum, and
// accumulator rescaled when the max grows)
constexpr int kPfWarps = 4;  // tokens per block
template <typename KT>         // cache element: float or __half
__global__ void __launch_bounds__(32 * kPfWarps) attn_prefill_kernel(const float *__restrict__ qkv, int64_t T, int64_t ldq,
                                                                   int group, int hd, int KVl, int pos0, float scale,
                                                                   const KT *__restrict__ kc,
                                                                   const KT *__restrict__ vc, float *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * kPfWarps + (threadIdx.x >> 5);
    if (t >= T) return;
    const int h = blockIdx.y, kvh = h / group;
    const int npos = pos0 + (int)t + 1;
    float q[4], o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int d = lane + 32 * j;
        q[j] = d < hd ? qkv[t * ldq + (int64_t)h * hd + d] : 0.0f;
        o[j] = 0.0f;
    }
    const KT *kb = kc + (int64_t)kvh * hd, *vb = vc + (int64_t)kvh * hd;
    float m = -INFINITY, l = 0.0f;
    for (int p0 = 0; p0 < npos; p0 += 4) {
        float sc[4], v[4][4];  // the 4 positions' K and V rows are loaded together
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int p = p0 + c;
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int d = lane + 32 * j;
                const bool ok = p < npos && d < hd;
                if (ok) s = fmaf(q[j], kv_ld(kb + (int64_t)p * KVl + d), s);
                v[c][j] = ok ? kv_ld(vb + (int64_t)p * KVl + d) : 0.0f;
            }
            sc[c] = s;
        }
#pragma unroll
        for (int off = 16; off; off >>= 1)
#pragma unroll
            for (int c = 0; c < 4; c++) sc[c] += __shfl_xor_sync(0xffffffffu, sc[c], off);
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int p = p0 + c;
            if (p >= npos) break;
            const float s = sc[c] * scale;
            const float mn = fmaxf(m, s);
            const float corr = expf(m - mn), e = expf(s - mn);
            l = l * corr + e;
#pragma unroll
            for (int j = 0; j < 4; j++) o[j] = o[j] * corr + e * v[c][j];
            m = mn;
        }
    }
    const float rl = 1.0f / l;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int d = lane + 32 * j;
        if (d < hd) out[t * (int64_t)gridDim.y * hd + (int64_t)h * hd + d] = o[j] * rl;
    }
}

__global__ void add_kernel(float *__restrict__ x, const float *__restrict__ y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], y[i]);
}

int grid_for(int64_t n, int threads) { return (int)std::min<int64_t>((n + threads - 1) / threads, 148 * 16); }

}  // namespace

int launch_embed_rows(int dtype, const void *table, int64_t cols, const int *tokens, int64_t T, float *x, cudaStream_t s) {
    embed_rows_kernel<<<(unsigned)T, 256, 0, s>>>(dtype, (const uint8_t *)table, cols, tokens, x);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_rmsnorm_rows(const float *x, const float *w, float *out, int64_t T, int64_t n, float eps, cudaStream_t s) {
    rmsnorm_rows_kernel<<<(unsigned)T, 256, 0, s>>>(x, w, out, n, eps);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_rope_kv_rows(float *qkv, int64_t T, int Dq, int KVl, int hd, int pos0, const float2 *rope, void *kc,
                        void *vc, bool kv16, cudaStream_t s) {
    rope_kv_rows_kernel<<<(unsigned)T, 256, 0, s>>>(qkv, Dq, KVl, hd, pos0, rope, kc, vc, kv16);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_attn_prefill(const float *qkv, int64_t T, int64_t ldq, int n_heads, int group, int hd, int KVl, int pos0,
                        float scale, const void *kc, const void *vc, bool kv16, float *out, cudaStream_t s) {
    if (hd > 128) return set_error(QMC_EINVAL, "prefill attention: head_dim %d > 128", hd);
    dim3 grid((unsigned)((T + kPfWarps - 1) / kPfWarps), (unsigned)n_heads);
    if (kv16)
        attn_prefill_kernel<<<grid, 32 * kPfWarps, 0, s>>>(qkv, T, ldq, group, hd, KVl, pos0, scale, (const __half *)kc,
                                                           (const __half *)vc, out);
    else
        attn_prefill_kernel<<<grid, 32 * kPfWarps, 0, s>>>(qkv, T, ldq, group, hd, KVl, pos0, scale, (const float *)kc,
                                                           (const float *)vc, out);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_add(float *x, const float *y, int64_t n, cudaStream_t s) {
    add_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, y, n);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

}  // namespace qmc
