// Row kernels of the batched prompt forward (prefill).  The matrices themselves go through matmul.cu
// (quantized weights) or gemm_f32; the driver is qmc_model_prefill in model.cu.
#include <algorithm>

#include "actquant.cuh"
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

// rmsnorm of one row per block followed by its Q8_0 quantization, without the normalised row in memory:
// the same operations as rmsnorm_rows then quantize_act (inv from the double sum of squares, v = (x * inv)
// * w rounded twice, per 32-element block the reference's quantizer), so the blocks are bit-identical.
// With `add`, the row first takes the residual add x += add (written back; src/model.c:179,186).  Four
// threads per 32-element block, 8 elements each (quant_group<8>), blockDim / 4 blocks a round: a row of
// one round (n <= 8192 at 1024 threads) keeps its values in registers across the block sum, all loads in
// flight at once.
__global__ void rmsnorm_quant_rows_kernel(float *__restrict__ x, const float *__restrict__ add, const float *__restrict__ w,
                                          int64_t n, float eps, int8_t *__restrict__ qs, float *__restrict__ d,
                                          float *__restrict__ dT, int64_t ldT) {
    __shared__ double red[32];
    __shared__ float inv_s;
    const int64_t row = blockIdx.x;
    float *xr = x + row * n;
    const float *ar = add ? add + row * n : nullptr;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, j = t & 3;
    const int qb = blockDim.x >> 2;  // blocks per round
    const int64_t nb = nblocks(n);
    const int rounds = (int)((nb + qb - 1) / qb);
    float v[8];
    double ss = 0.0;
    for (int r = 0; r < rounds; r++) {
        const int64_t e0 = ((int64_t)r * qb + (t >> 2)) * 32 + 8 * j;
        load8_any(xr, e0, n, v);
        if (ar) {
            float a[8];
            load8_any(ar, e0, n, a);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                v[i] = __fadd_rn(v[i], a[i]);
                if (e0 + i < n) xr[e0 + i] = v[i];
            }
        }
#pragma unroll
        for (int i = 0; i < 8; i++) ss = fma((double)v[i], (double)v[i], ss);
    }
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
    for (int r = 0; r < rounds; r++) {
        const int64_t b = (int64_t)r * qb + (t >> 2), e0 = b * 32 + 8 * j;
        if (rounds > 1) load8_any(xr, e0, n, v);  // this thread's own values (the add written back above)
        float wv[8];
        load8_any(w, e0, n, wv);
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(v[i], inv), wv[i]);
        uint32_t q[2];
        int sum;
        float sc;
        quant_group<8>(v, q, sum, sc);
        if (b < nb) {
            *(uint2 *)(qs + (row * nb + b) * 32 + 8 * j) = make_uint2(q[0], q[1]);
            if (j == 0) {
                d[row * nb + b] = sc;
                if (dT) dT[b * ldT + row] = sc;
            }
        }
    }
}

// h = silu(g) * u over T rows of n (the SwiGLU of src/ops.c:128-133, same roundings as swiglu_kernel)
// straight into its Q8_0 blocks (quant_rows_quads), h never stored
__global__ void swiglu_quant_rows_kernel(const float *__restrict__ g, const float *__restrict__ u, int64_t T, int64_t n,
                                         int8_t *__restrict__ qs, float *__restrict__ d, float *__restrict__ dT,
                                         int64_t ldT) {
    quant_rows_quads(
        T, n,
        [&](int64_t t, int64_t e0, float (&v)[8]) {
            float gv[8], uv[8];
            load8_any(g + t * n, e0, n, gv);
            load8_any(u + t * n, e0, n, uv);
#pragma unroll
            for (int i = 0; i < 8; i++)
                v[i] = e0 + i < n ? __fmul_rn(__fdiv_rn(gv[i], __fadd_rn(1.0f, expf(-gv[i]))), uv[i]) : 0.0f;
        },
        qs, d, dT, ldT);
}

// p0 = x0 c - x1 s ; p1 = x0 s + x1 c, each product and sum rounded separately (src/ops.c:121-123)
__device__ __forceinline__ void rope_rotate(float a, float b, float2 cs, float &o0, float &o1) {
    o0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    o1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
}

// one thread per value pair of a row: RoPE on the q / k pairs (k to its cache slot), v copied to its slot
__global__ void rope_kv_rows_kernel(float *__restrict__ qkv, int Dq, int KVl, int hd, int pos0,
                                    const float2 *__restrict__ rope, void *__restrict__ kc, void *__restrict__ vc,
                                    bool kv16) {
    const int64_t t = blockIdx.y;
    const int pos = pos0 + (int)t;
    float *row = qkv + t * (int64_t)(Dq + 2 * KVl);
    const int i = (int)blockIdx.x * blockDim.x + threadIdx.x, nrot = (Dq + KVl) >> 1;
    if (i < nrot) {
        const int e = 2 * i;  // pair (e, e + 1) of q (e < Dq) or k
        float o0, o1;
        rope_rotate(row[e], row[e + 1], rope[(int64_t)pos * (hd >> 1) + ((e % hd) >> 1)], o0, o1);
        if (e < Dq) row[e] = o0, row[e + 1] = o1;
        else kv_st2(kc, kv16, (int64_t)pos * KVl + (e - Dq), o0, o1);
    } else if (i < nrot + (KVl >> 1)) {
        const int e = 2 * (i - nrot);
        kv_st2(vc, kv16, (int64_t)pos * KVl + e, row[Dq + KVl + e], row[Dq + KVl + e + 1]);
    }
}

// Causal attention of a tile of kQT query tokens of one head: the head's K and V rows are staged through
// shared memory kPT positions at a time and shared by the tile's tokens.  Each warp owns kQT / 4 tokens.
// Per token and position tile, lane p scores position p (its dot over head_dim, K transposed in shared
// memory so lane p reads its own column), the warp updates the online softmax once for the tile (max,
// one rescale of the running sum and accumulator), and lane l accumulates head dimensions 4l .. 4l + 3
// over the tile's positions.  Rows are zero-padded to a multiple of 4 dimensions in shared memory.
// QT (query tokens per block: 8, 16 or 32) only groups the tokens: every token's arithmetic is the same
// whatever the tile, so the launch takes the largest tile that still gives every SM two blocks (short
// prompts run many small tiles, long ones share each staged K/V tile among 32 tokens).
constexpr int kPT = 32;  // positions per staged tile (one per lane)
// four consecutive cache elements (16-byte aligned for float, 8-byte for __half)
__device__ __forceinline__ float4 kv_ld4(const float *p) { return __ldcg((const float4 *)p); }
__device__ __forceinline__ float4 kv_ld4(const __half *p) {
    const uint2 r = __ldcg((const uint2 *)p);
    const float2 a = __half22float2(*(const __half2 *)&r.x), b = __half22float2(*(const __half2 *)&r.y);
    return make_float4(a.x, a.y, b.x, b.y);
}
template <typename KT, int QT>     // cache element: float or __half; query tokens per block
__global__ void __launch_bounds__(128, 2) attn_prefill_kernel(const float *__restrict__ qkv, int64_t T, int64_t ldq, int group,
                                                           int hd, int KVl, int pos0, float scale,
                                                           const KT *__restrict__ kc, const KT *__restrict__ vc,
                                                           float *__restrict__ out) {
    extern __shared__ __align__(16) float smf[];
    const int hd4 = (hd + 3) & ~3;
    float *Kt = smf;                 // [hd4 / 4][kPT][4]: dims 4c .. 4c + 3 of position p at (c * kPT + p) * 4
    float *Vs = Kt + hd4 * kPT;      // [kPT][hd4]
    float *Qs = Vs + kPT * hd4;      // [QT][hd4]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int h = blockIdx.y, kvh = h / group;
    const int64_t tq0 = (int64_t)blockIdx.x * QT;
    const int nq = (int)(T - tq0 < QT ? T - tq0 : QT);
    for (int i = tid; i < QT * hd4; i += 128) {
        const int r = i / hd4, d = i % hd4;
        Qs[i] = (r < nq && d < hd) ? qkv[(tq0 + r) * ldq + (int64_t)h * hd + d] : 0.0f;
    }
    constexpr int TW = QT / 4;  // tokens per warp
    float m[TW], l[TW], o[TW][4];
#pragma unroll
    for (int j = 0; j < TW; j++) {
        m[j] = -INFINITY, l[j] = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) o[j][i] = 0.0f;
    }
    const int last = pos0 + (int)tq0 + nq - 1;  // the tile's last token sees positions 0 .. last
    const bool vec = (hd & 3) == 0 && (KVl & 3) == 0;  // 4-dimension groups stay aligned in the cache
    const KT *kb = kc + (int64_t)kvh * hd, *vb = vc + (int64_t)kvh * hd;
    for (int p0 = 0; p0 <= last; p0 += kPT) {
        __syncthreads();  // the previous tile's K/V (and, first time, nothing) are no longer read
        if (vec) {  // 4 dimensions per load; K positions vary fastest (conflict-free transposed stores)
            for (int i = tid; i < kPT * (hd4 / 4); i += 128) {
                const int pp = i % kPT, c = i / kPT, pos = p0 + pp;
                *(float4 *)(Kt + (c * kPT + pp) * 4) = pos <= last ? kv_ld4(kb + (int64_t)pos * KVl + 4 * c)
                                                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
            for (int i = tid; i < kPT * (hd4 / 4); i += 128) {
                const int c = i % (hd4 / 4), pp = i / (hd4 / 4), pos = p0 + pp;
                *(float4 *)(Vs + pp * hd4 + 4 * c) = pos <= last ? kv_ld4(vb + (int64_t)pos * KVl + 4 * c)
                                                                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        } else {
            for (int i = tid; i < kPT * hd4; i += 128) {
                const int pp = i / hd4, d = i % hd4, pos = p0 + pp;
                const bool ok = pos <= last && d < hd;
                Kt[((d >> 2) * kPT + pp) * 4 + (d & 3)] = ok ? kv_ld(kb + (int64_t)pos * KVl + d) : 0.0f;
                Vs[pp * hd4 + d] = ok ? kv_ld(vb + (int64_t)pos * KVl + d) : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < TW; j++) {
            const int r = warp * TW + j;  // query token of the tile
            if (r >= nq) break;
            const int lim = pos0 + (int)tq0 + r;  // causal: positions 0 .. lim
            if (p0 > lim) continue;
            const float *q = Qs + r * hd4;
            float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four independent chains, summed at the end
            for (int c = 0; c < hd4 / 4; c++) {
                const float4 kv4 = *(const float4 *)(Kt + (c * kPT + lane) * 4);
                const float4 q4 = *(const float4 *)(q + 4 * c);
                s4[0] = fmaf(q4.x, kv4.x, s4[0]);
                s4[1] = fmaf(q4.y, kv4.y, s4[1]);
                s4[2] = fmaf(q4.z, kv4.z, s4[2]);
                s4[3] = fmaf(q4.w, kv4.w, s4[3]);
            }
            float sc = (s4[0] + s4[1]) + (s4[2] + s4[3]);
            sc = p0 + lane <= lim ? sc * scale : -INFINITY;
            float mx = sc;
#pragma unroll
            for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[j], mx);
            const float corr = expf(m[j] - mn), e = expf(sc - mn);  // e = 0 past the causal limit
            float es = e;
#pragma unroll
            for (int off = 16; off; off >>= 1) es += __shfl_xor_sync(0xffffffffu, es, off);
            l[j] = l[j] * corr + es;
            m[j] = mn;
#pragma unroll
            for (int i = 0; i < 4; i++) o[j][i] *= corr;
            const bool own = 4 * lane < hd4;  // this lane holds head dimensions
            for (int pp = 0; pp < kPT; pp++) {
                const float ep = __shfl_sync(0xffffffffu, e, pp);  // every lane takes part
                if (own) {
                    const float4 v4 = *(const float4 *)(Vs + pp * hd4 + 4 * lane);
                    o[j][0] = fmaf(ep, v4.x, o[j][0]);
                    o[j][1] = fmaf(ep, v4.y, o[j][1]);
                    o[j][2] = fmaf(ep, v4.z, o[j][2]);
                    o[j][3] = fmaf(ep, v4.w, o[j][3]);
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < TW; j++) {
        const int r = warp * TW + j;
        if (r >= nq) break;
        const float rl = 1.0f / l[j];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int d = 4 * lane + i;
            if (d < hd) out[(tq0 + r) * (int64_t)gridDim.y * hd + (int64_t)h * hd + d] = o[j][i] * rl;
        }
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

int launch_rmsnorm_quant_rows(float *x, const float *add, const float *w, int64_t T, int64_t n, float eps, int8_t *qs,
                              float *d, float *dT, int64_t ldT, cudaStream_t s) {
    // four threads per block: one round up to 8192 elements
    const int threads = (int)std::min<int64_t>(1024, std::max<int64_t>(32, (nblocks(n) * 4 + 31) / 32 * 32));
    rmsnorm_quant_rows_kernel<<<(unsigned)T, threads, 0, s>>>(x, add, w, n, eps, qs, d, dT, ldT);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_swiglu_quant_rows(const float *g, const float *u, int64_t T, int64_t n, int8_t *qs, float *d, float *dT,
                             int64_t ldT, cudaStream_t s) {
    const int64_t grid = (T * nblocks(n) * 4 + 255) / 256;  // a thread per 8 elements (the loop covers the rest)
    swiglu_quant_rows_kernel<<<(int)(grid < 65535 ? grid : 65535), 256, 0, s>>>(g, u, T, n, qs, d, dT, ldT);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_rope_kv_rows(float *qkv, int64_t T, int Dq, int KVl, int hd, int pos0, const float2 *rope, void *kc,
                        void *vc, bool kv16, cudaStream_t s) {
    if (T > 65535) return set_error(QMC_EINVAL, "prefill rope: %lld rows exceed the grid", (long long)T);
    const int pairs = ((Dq + KVl) >> 1) + (KVl >> 1);
    rope_kv_rows_kernel<<<dim3((unsigned)((pairs + 255) / 256), (unsigned)T), 256, 0, s>>>(qkv, Dq, KVl, hd, pos0, rope, kc,
                                                                                         vc, kv16);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

template <int QT>
int launch_attn_prefill_t(const float *qkv, int64_t T, int64_t ldq, int n_heads, int group, int hd, int KVl, int pos0,
                          float scale, const void *kc, const void *vc, bool kv16, float *out, int dev, cudaStream_t s) {
    const int hd4 = (hd + 3) & ~3;
    const size_t smem = (size_t)(hd4 * kPT + kPT * hd4 + QT * hd4) * 4;
    dim3 grid((unsigned)((T + QT - 1) / QT), (unsigned)n_heads);
    static bool attr_done[64];
    if (!attr_done[dev]) {  // the largest tile set (head_dim 128)
        const int most = (2 * 128 * kPT + QT * 128) * 4;
        QMC_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<__half, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, most));
        QMC_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<float, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, most));
        attr_done[dev] = true;
    }
    if (kv16) {
        attn_prefill_kernel<__half, QT><<<grid, 128, smem, s>>>(qkv, T, ldq, group, hd, KVl, pos0, scale,
                                                               (const __half *)kc, (const __half *)vc, out);
    } else {
        attn_prefill_kernel<float, QT><<<grid, 128, smem, s>>>(qkv, T, ldq, group, hd, KVl, pos0, scale,
                                                              (const float *)kc, (const float *)vc, out);
    }
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_attn_prefill(const float *qkv, int64_t T, int64_t ldq, int n_heads, int group, int hd, int KVl, int pos0,
                        float scale, const void *kc, const void *vc, bool kv16, float *out, cudaStream_t s) {
    if (hd > 128) return set_error(QMC_EINVAL, "prefill attention: head_dim %d > 128", hd);
    int dev = 0;
    QMC_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(QMC_EINVAL, "prefill attention: device %d out of range", dev);
    const DevCtx *c = ctx();
    const int64_t want = 2 * (int64_t)(c ? c->num_sms : 148);  // blocks
    if ((T + 31) / 32 * n_heads >= want)
        return launch_attn_prefill_t<32>(qkv, T, ldq, n_heads, group, hd, KVl, pos0, scale, kc, vc, kv16, out, dev, s);
    if ((T + 15) / 16 * n_heads >= want)
        return launch_attn_prefill_t<16>(qkv, T, ldq, n_heads, group, hd, KVl, pos0, scale, kc, vc, kv16, out, dev, s);
    return launch_attn_prefill_t<8>(qkv, T, ldq, n_heads, group, hd, KVl, pos0, scale, kc, vc, kv16, out, dev, s);
}

int launch_add(float *x, const float *y, int64_t n, cudaStream_t s) {
    add_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, y, n);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

}  // namespace qmc
