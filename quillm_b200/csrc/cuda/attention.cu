// Decode attention over the device-resident KV cache (fp32 as src/model.c:132-156, or fp16), split over
// positions.
//
// Batch-1 decode has only n_kv_heads (x group) heads, far fewer than the 148 SMs, so each KV head's
// positions 0..pos are split into `nsplit` chunks, one CTA each, and the nsplit CTAs of a head form one
// thread-block cluster.  In a CTA every warp walks its positions once, reading K_t and V_t together
// (coalesced, lanes across head_dim) with an online softmax per query head of the GQA group (K/V read
// once for the whole group): running max m, l = sum e^(s-m), o = sum e^(s-m) v.  Warps merge in shared
// memory; the cluster's rank-0 CTA then merges the nsplit partial (m, l, o) through distributed shared
// memory and writes out = sum_j e^(m_j-M) o_j / sum_j e^(m_j-M) l_j.  Equal to the reference's
// softmax-then-weighted-sum up to float rounding; no global scratch and no atomics.
#include <cooperative_groups.h>

#include "attention.cuh"

namespace cg = cooperative_groups;

namespace qmc {
namespace {

constexpr int AT = 128;  // threads per CTA (4 warps)
constexpr int GMAX = 8;  // query heads per CTA (a larger GQA group spans several CTAs)

struct AParams {
    const float *q;
    const void *kc, *vc;  // float or __half elements
    float *out;
    const int *pos;
    int hd, group, gsplit, kvl, nsplit;
    float scale;
};

template <int MAXW, typename KT>
__global__ void __launch_bounds__(AT) attn_decode_kernel(const AParams p) {
    extern __shared__ __align__(16) float sm[];
    cg::cluster_group cluster = cg::this_cluster();
    const int kvh = blockIdx.x / p.gsplit, gs = blockIdx.x % p.gsplit, split = blockIdx.y;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int hd = p.hd, h0 = gs * GMAX, G = min(GMAX, p.group - h0);
    const int stride = hd + 2;
    float *wpart = sm;                      // [4 warps][G][hd + 2]   per-warp (m, l, o)
    float *cpart = sm + 4 * GMAX * stride;  // [G][hd + 2]            this CTA's merged (m, l, o)
    pdl_wait();
    const int npos = *p.pos + 1;
    const int chunk = (npos + p.nsplit - 1) / p.nsplit;
    const int t0 = split * chunk, t1 = min(npos, t0 + chunk);
    const int64_t hq = (int64_t)kvh * p.group + h0;  // first query head of this CTA
    const KT *kb = (const KT *)p.kc + (int64_t)kvh * hd, *vb = (const KT *)p.vc + (int64_t)kvh * hd;

    float q[GMAX][MAXW], o[GMAX][MAXW], m[GMAX], l[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int w = 0; w < MAXW; w++) {
            const int d = lane + 32 * w;
            q[g][w] = (g < G && d < hd) ? p.q[(hq + g) * hd + d] : 0.0f;
            o[g][w] = 0.0f;
        }
    }
    for (int tt = t0 + warp; tt < t1; tt += AT / 32) {
        float k[MAXW], v[MAXW];
#pragma unroll
        for (int w = 0; w < MAXW; w++) {
            const int d = lane + 32 * w;
            k[w] = d < hd ? kv_ld(kb + (int64_t)tt * p.kvl + d) : 0.0f;
            v[w] = d < hd ? kv_ld(vb + (int64_t)tt * p.kvl + d) : 0.0f;
        }
#pragma unroll
        for (int g = 0; g < GMAX; g++) {
            if (g < G) {
                float s = 0.0f;
#pragma unroll
                for (int w = 0; w < MAXW; w++) s = fmaf(k[w], q[g][w], s);
                s = warp_sum(s) * p.scale;
                const float mn = fmaxf(m[g], s);
                const float corr = expf(m[g] - mn), e = expf(s - mn);
                l[g] = l[g] * corr + e;
#pragma unroll
                for (int w = 0; w < MAXW; w++) o[g][w] = o[g][w] * corr + e * v[w];
                m[g] = mn;
            }
        }
    }
#pragma unroll
    for (int g = 0; g < GMAX; g++) {
        if (g < G) {
            float *dst = wpart + (warp * GMAX + g) * stride;
            if (lane == 0) dst[0] = m[g], dst[1] = l[g];
#pragma unroll
            for (int w = 0; w < MAXW; w++)
                if (lane + 32 * w < hd) dst[2 + lane + 32 * w] = o[g][w];
        }
    }
    __syncthreads();
    for (int i = t; i < G * hd; i += AT) {  // merge the 4 warps
        const int g = i / hd, d = i % hd;
        float M = -INFINITY;
        for (int w = 0; w < 4; w++) M = fmaxf(M, wpart[(w * GMAX + g) * stride]);
        float lo = 0.0f, oo = 0.0f;
        for (int w = 0; w < 4; w++) {
            const float *src = wpart + (w * GMAX + g) * stride;
            const float c = src[1] > 0.0f ? expf(src[0] - M) : 0.0f;
            lo = fmaf(c, src[1], lo);
            oo = fmaf(c, src[2 + d], oo);
        }
        float *dst = cpart + g * stride;
        if (d == 0) dst[0] = M, dst[1] = lo;
        dst[2 + d] = oo;
    }
    cluster.sync();  // every split's merged partial is visible cluster-wide
    if (split == 0) {
        for (int i = t; i < G * hd; i += AT) {
            const int g = i / hd, d = i % hd;
            float M = -INFINITY;
            for (int r = 0; r < p.nsplit; r++) M = fmaxf(M, cluster.map_shared_rank(cpart, r)[g * stride]);
            float num = 0.0f, den = 0.0f;
            for (int r = 0; r < p.nsplit; r++) {
                const float *src = cluster.map_shared_rank(cpart, r) + g * stride;
                const float c = src[1] > 0.0f ? expf(src[0] - M) : 0.0f;
                den = fmaf(c, src[1], den);
                num = fmaf(c, src[2 + d], num);
            }
            p.out[(hq + g) * hd + d] = num / den;
        }
    }
    pdl_launch_dependents();
    cluster.sync();  // rank 0 has finished reading the other CTAs' shared memory
}

template <int MAXW, typename KT>
int launch_t(const AttnPlan &a, const AParams &p, int n_kv_local, cudaStream_t s, bool pdl) {
    auto fn = attn_decode_kernel<MAXW, KT>;
    QMC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    cudaLaunchConfig_t c = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = a.nsplit;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    c.gridDim = dim3(n_kv_local * p.gsplit, a.nsplit);
    c.blockDim = dim3(AT);
    c.dynamicSmemBytes = a.smem;
    c.stream = s;
    c.attrs = attr;
    c.numAttrs = pdl ? 2 : 1;
    QMC_CUDA(cudaLaunchKernelEx(&c, fn, p));
    return QMC_OK;
}

}  // namespace

AttnPlan plan_attention(int n_kv_local, int group, int hd, int max_seq, int num_sms) {
    AttnPlan a;
    const int gsplit = (group + GMAX - 1) / GMAX;
    int ns = (2 * num_sms + n_kv_local * gsplit - 1) / (n_kv_local * gsplit);
    if (ns > 16) ns = 16;
    if (ns > max_seq) ns = max_seq;
    if (ns < 1) ns = 1;
    a.nsplit = ns;
    a.chunk_max = (max_seq + ns - 1) / ns;
    a.smem = (size_t)(5 * GMAX * (hd + 2)) * 4;
    a.part_floats = 0;
    return a;
}

template <typename KT>
int launch_kt(const AttnPlan &a, const AParams &p, int n_kv_local, int hd, cudaStream_t s, bool pdl) {
    if (hd <= 32) return launch_t<1, KT>(a, p, n_kv_local, s, pdl);
    if (hd <= 64) return launch_t<2, KT>(a, p, n_kv_local, s, pdl);
    if (hd <= 128) return launch_t<4, KT>(a, p, n_kv_local, s, pdl);
    return launch_t<8, KT>(a, p, n_kv_local, s, pdl);
}

int launch_attention(const AttnPlan &a, const float *q, const void *kc, const void *vc, bool kv16, float *out,
                     float *part, int *cnt, const int *pos, int n_kv_local, int group, int hd, int kvl, cudaStream_t s,
                     bool pdl) {
    (void)part;
    (void)cnt;
    if (hd > 256 || (hd & 1)) return set_error(QMC_EINVAL, "attention: head_dim %d unsupported", hd);
    AParams p{q, kc, vc, out, pos, hd, group, (group + GMAX - 1) / GMAX, kvl, a.nsplit, 1.0f / sqrtf((float)hd)};
    return kv16 ? launch_kt<__half>(a, p, n_kv_local, hd, s, pdl) : launch_kt<float>(a, p, n_kv_local, hd, s, pdl);
}

}  // namespace qmc
