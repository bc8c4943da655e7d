// Decode attention over the device-resident fp32 KV cache (src/model.c:132-156), split over positions.
//
// Batch-1 decode has only n_kv_heads (x group) heads, far fewer than the 148 SMs, so each KV head's
// positions 0..pos are split into `nsplit` chunks, one CTA each (flash-decoding).  A CTA computes the
// scores q.k * scale of all `group` query heads sharing its KV head (GQA: K/V read once), a local max
// m, l = sum exp(s - m) and o = sum exp(s - m) v, and stores (m, l, o) to scratch.  The last CTA to
// finish a KV head (atomic ticket) merges the splits: out = sum_j e^(m_j-M) o_j / sum_j e^(m_j-M) l_j.
// Equal to the reference's softmax-then-weighted-sum up to float rounding.
#include "attention.cuh"

namespace qmc {
namespace {

constexpr int AT = 128;  // threads per CTA (4 warps)
constexpr int MAXW = 8;  // head_dim / 32 upper bound (head_dim <= 256)

struct AParams {
    const float *q, *kc, *vc;
    float *out, *part;
    int *cnt;
    const int *pos;
    int hd, group, kvl, nsplit, chunk_max;
    float scale;
};

__global__ void __launch_bounds__(AT) attn_decode_kernel(const AParams p) {
    extern __shared__ __align__(16) float sm[];
    const int g0 = blockIdx.x, split = blockIdx.y;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int hd = p.hd, G = p.group, nw = (hd + 31) >> 5;
    float *qs = sm;                               // [G][hd]
    float *sc = qs + G * hd;                      // [G][chunk_max]
    float *red = sc + G * p.chunk_max;            // [4][G][hd]
    float *ml = red + 4 * G * hd;                 // [G][2]
    pdl_wait();
    const int npos = *p.pos + 1;
    const int chunk = (npos + p.nsplit - 1) / p.nsplit;
    const int t0 = split * chunk;
    const int t1 = min(npos, t0 + chunk);
    const int n = max(0, t1 - t0);
    const float *kbase = p.kc + (int64_t)g0 * hd, *vbase = p.vc + (int64_t)g0 * hd;

    for (int i = t; i < G * hd; i += AT) qs[i] = p.q[(int64_t)g0 * G * hd + i];
    __syncthreads();

    // scores: warp per position, lanes across head_dim
    for (int j = warp; j < n; j += AT / 32) {
        const float *kr = kbase + (int64_t)(t0 + j) * p.kvl;
        float kv[MAXW];
#pragma unroll
        for (int m = 0; m < MAXW; m++) kv[m] = (m < nw && lane + 32 * m < hd) ? kr[lane + 32 * m] : 0.0f;
        for (int g = 0; g < G; g++) {
            float s = 0.0f;
#pragma unroll
            for (int m = 0; m < MAXW; m++)
                if (m < nw && lane + 32 * m < hd) s = fmaf(kv[m], qs[g * hd + lane + 32 * m], s);
            s = warp_sum(s);
            if (lane == 0) sc[g * p.chunk_max + j] = s * p.scale;
        }
    }
    __syncthreads();
    // softmax statistics per head: warp g % 4
    for (int g = warp; g < G; g += AT / 32) {
        float mx = -INFINITY;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[g * p.chunk_max + j]);
        mx = warp_max(mx);
        float l = 0.0f;
        for (int j = lane; j < n; j += 32) {
            const float e = n ? expf(sc[g * p.chunk_max + j] - mx) : 0.0f;
            sc[g * p.chunk_max + j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) ml[2 * g] = mx, ml[2 * g + 1] = l;
    }
    __syncthreads();
    // o = sum_j e_j v_j: warp per position subset, lanes across head_dim
    {
        float acc[8][MAXW];
        const int GG = G < 8 ? G : 8;
        for (int g0b = 0; g0b < G; g0b += 8) {
#pragma unroll
            for (int g = 0; g < 8; g++)
#pragma unroll
                for (int m = 0; m < MAXW; m++) acc[g][m] = 0.0f;
            for (int j = warp; j < n; j += AT / 32) {
                const float *vr = vbase + (int64_t)(t0 + j) * p.kvl;
                float vv[MAXW];
#pragma unroll
                for (int m = 0; m < MAXW; m++) vv[m] = (m < nw && lane + 32 * m < hd) ? vr[lane + 32 * m] : 0.0f;
#pragma unroll
                for (int g = 0; g < 8; g++)
                    if (g0b + g < G) {
                        const float e = sc[(g0b + g) * p.chunk_max + j];
#pragma unroll
                        for (int m = 0; m < MAXW; m++) acc[g][m] = fmaf(e, vv[m], acc[g][m]);
                    }
            }
#pragma unroll
            for (int g = 0; g < 8; g++)
                if (g0b + g < G)
#pragma unroll
                    for (int m = 0; m < MAXW; m++)
                        if (m < nw && lane + 32 * m < hd) red[(warp * G + g0b + g) * hd + lane + 32 * m] = acc[g][m];
        }
        (void)GG;
    }
    __syncthreads();
    for (int i = t; i < G * hd; i += AT) {
        const float o = red[i] + red[G * hd + i] + red[2 * G * hd + i] + red[3 * G * hd + i];
        const int g = i / hd, d = i % hd;
        float *dst = p.part + ((int64_t)(g0 * G + g) * p.nsplit + split) * (hd + 2);
        dst[2 + d] = o;
        if (d == 0) dst[0] = ml[2 * g], dst[1] = ml[2 * g + 1];
    }
    // last CTA of this KV head merges the splits
    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (t == 0) {
        const int ticket = atomicAdd(&p.cnt[g0], 1);
        is_last = ticket == p.nsplit - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int i = t; i < G * hd; i += AT) {
        const int g = i / hd, d = i % hd;
        const float *base = p.part + (int64_t)(g0 * G + g) * p.nsplit * (hd + 2);
        float M = -INFINITY;
        for (int s = 0; s < p.nsplit; s++) M = fmaxf(M, base[s * (hd + 2)]);
        float num = 0.0f, den = 0.0f;
        for (int s = 0; s < p.nsplit; s++) {
            const float *ps = base + s * (hd + 2);
            const float w = ps[1] > 0.0f ? expf(ps[0] - M) : 0.0f;
            num = fmaf(w, ps[2 + d], num);
            den = fmaf(w, ps[1], den);
        }
        p.out[(int64_t)(g0 * G + g) * hd + d] = num / den;
    }
    if (t == 0) p.cnt[g0] = 0;
    pdl_launch_dependents();
}

}  // namespace

AttnPlan plan_attention(int n_kv_local, int group, int hd, int max_seq, int num_sms) {
    AttnPlan a;
    int ns = (2 * num_sms + n_kv_local - 1) / n_kv_local;
    const int min_for_smem = (max_seq + 511) / 512;  // chunk <= 512 positions
    if (ns < min_for_smem) ns = min_for_smem;
    if (ns > max_seq) ns = max_seq;
    if (ns < 1) ns = 1;
    a.nsplit = ns;
    a.chunk_max = (max_seq + ns - 1) / ns;
    a.smem = (size_t)(group * hd + group * a.chunk_max + 4 * group * hd + 2 * group) * 4;
    a.part_floats = (size_t)n_kv_local * group * ns * (hd + 2);
    (void)hd;
    return a;
}

int launch_attention(const AttnPlan &a, const float *q, const float *kc, const float *vc, float *out, float *part,
                     int *cnt, const int *pos, int n_kv_local, int group, int hd, int kvl, cudaStream_t s, bool pdl) {
    if (hd > 32 * MAXW || (hd & 1)) return set_error(QMC_EINVAL, "attention: head_dim %d unsupported", hd);
    AParams p{q, kc, vc, out, part, cnt, pos, hd, group, kvl, a.nsplit, a.chunk_max, 1.0f / sqrtf((float)hd)};
    if (a.smem > 48 * 1024)
        QMC_CUDA(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)a.smem));
    cudaLaunchConfig_t c = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    c.gridDim = dim3(n_kv_local, a.nsplit);
    c.blockDim = dim3(AT);
    c.dynamicSmemBytes = a.smem;
    c.stream = s;
    c.attrs = pdl ? attr : nullptr;
    c.numAttrs = pdl ? 1 : 0;
    QMC_CUDA(cudaLaunchKernelEx(&c, attn_decode_kernel, p));
    return QMC_OK;
}

}  // namespace qmc
