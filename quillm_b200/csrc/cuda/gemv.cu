// Decode matvec kernels (batch 1, HBM-bound).
//
// Quantized weights (Q8_0 34-byte / Q4_0 18-byte AoS blocks, exactly the file bytes) stream through a
// ring of shared-memory stages filled by 1-D bulk async copies (cp.async.bulk, completion on an
// mbarrier).  The copies for the first stages are issued before the activation prologue, so weight
// traffic overlaps the (dependent) activation work; with programmatic dependent launch they even
// overlap the previous kernel's tail.
//
// Work split: each CTA owns a contiguous range of rows; a "pass" covers P rows.  Thread t owns the
// fixed K-segment t % S (4 blocks = 128 activations) of row slot t / S, so its quantized activations
// (int8 words, block scale, block sum) are loaded once into registers and reused for every row.
// Per block: aligned 32-bit shared loads + funnel shifts realign the 2-byte-aligned block, dp4a
// computes the integer block dot, then s += (float)acc * (dW * dX) as the reference does
// (src/kernels_scalar.c:12-34).  Q4_0 uses sum_i (n_i - 8) x_i = sum_i n_i x_i - 8 sum_i x_i with the
// nibbles n_i fed to dp4a unchanged against even/odd-permuted activations.
#include <stdio.h>

#include "gemv.cuh"

namespace qmc {
namespace {

constexpr int NT = 256;
constexpr int SEGB = 4;  // blocks per thread segment

struct KParams {
    const uint8_t *W0, *W1;
    int64_t w_bytes;  // readable bytes of W0 (and of W1)
    int64_t vrows;    // virtual rows
    int K, nb, rb, S, P;
    int stage_bytes, nstages, part_stride;
    int xoff_q, xoff_d, xoff_s, red_off, rowv_off, misc_off;  // shared-memory offsets
    const float *x, *norm_w;
    float eps;
    int epi;
    float *y, *q, *kcache, *vcache;
    int Dq, KVl, hd;
    const float2 *rope;
    const int *pos;
    uint8_t *xq_out;
    int *err;
};

// ---------------------------------------------------------------- staging (one thread)
struct CopyPlan {
    int64_t a0;       // 16-aligned global start
    uint32_t tma;     // bytes by bulk copy from a0
    int64_t tail0;    // plain byte copy [tail0, end)
    int64_t end;
};
__device__ __forceinline__ CopyPlan plan_copy(int64_t start, int64_t len, int64_t w_bytes) {
    CopyPlan c;
    c.a0 = start & ~(int64_t)15;
    int64_t e16 = (start + len + 15) & ~(int64_t)15, lim = w_bytes & ~(int64_t)15;
    int64_t te = e16 < lim ? e16 : lim;
    if (te < c.a0) te = c.a0;
    c.tma = (uint32_t)(te - c.a0);
    c.tail0 = te;
    c.end = start + len;
    return c;
}

__device__ void issue_stage(const KParams &p, uint8_t *stage, uint64_t *bar, int64_t vr0, int64_t n) {
    const uint8_t *src[2];
    uint8_t *dst[2];
    CopyPlan cp[2];
    int parts;
    if (p.W1) {  // paired matrices: virtual rows 2h, 2h+1 -> W0[h], W1[h]
        int64_t h0 = vr0 >> 1, nh = n >> 1;
        parts = 2;
        src[0] = p.W0, src[1] = p.W1;
        dst[0] = stage, dst[1] = stage + p.part_stride;
        cp[0] = cp[1] = plan_copy(h0 * p.rb, nh * p.rb, p.w_bytes);
    } else {
        parts = 1;
        src[0] = p.W0, dst[0] = stage;
        cp[0] = plan_copy(vr0 * p.rb, n * p.rb, p.w_bytes);
    }
    uint32_t tx = 0;
    for (int i = 0; i < parts; i++) {
        for (int64_t b = cp[i].tail0; b < cp[i].end; b++) dst[i][b - cp[i].a0] = src[i][b];
        tx += cp[i].tma;
    }
    fence_proxy_async();
    mbar_arrive_tx(bar, tx);
    for (int i = 0; i < parts; i++)
        if (cp[i].tma) bulk_g2s(dst[i], src[i] + cp[i].a0, cp[i].tma, bar);
}

// ---------------------------------------------------------------- per-block dots from shared memory
// 2-byte aligned block at bp: read aligned words, realign with funnel shifts (shift 32 selects `hi`).
template <int NW>
__device__ __forceinline__ void load_words(const uint8_t *bp, uint32_t (&w)[NW], uint32_t &sh) {
    const uint32_t a = smem_u32(bp);
    const uint32_t *wp = (const uint32_t *)(bp - (a & 3u));
    sh = (a & 3u) * 8u;  // 0 or 16
#pragma unroll
    for (int i = 0; i < NW; i++) w[i] = wp[i];
}

__device__ __forceinline__ float dot_q8_block(const uint8_t *bp, const uint32_t (&xw)[8], float xd) {
    uint32_t w[9], sh;
    load_words<9>(bp, w, sh);
    const uint32_t dbits = __funnelshift_r(w[0], w[1], sh) & 0xffffu;
    int acc = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) acc = __dp4a((int)__funnelshift_rc(w[i], w[i + 1], 16u + sh), (int)xw[i], acc);
    return (float)acc * (h2f(dbits) * xd);
}

__device__ __forceinline__ float dot_q4_block(const uint8_t *bp, const uint32_t (&xe)[4], const uint32_t (&xo)[4],
                                              float xd, int xs) {
    uint32_t w[5], sh;
    load_words<5>(bp, w, sh);
    const uint32_t dbits = __funnelshift_r(w[0], w[1], sh) & 0xffffu;
    int acc = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t qw = __funnelshift_rc(w[i], w[i + 1], 16u + sh);
        acc = __dp4a((int)(qw & 0x0f0f0f0fu), (int)xe[i], acc);
        acc = __dp4a((int)((qw >> 4) & 0x0f0f0f0fu), (int)xo[i], acc);
    }
    acc -= 8 * xs;
    return (float)acc * (h2f(dbits) * xd);
}

// ---------------------------------------------------------------- epilogues
__device__ __forceinline__ void rope_pair(float a, float b, float2 cs, float &o0, float &o1) {
    // p0 = x0 c - x1 s ; p1 = x0 s + x1 c, each product and sum rounded separately (src/ops.c:121-123)
    o0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    o1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
}

__device__ __forceinline__ void epi_pair(const KParams &p, int64_t vr, float a, float b, int pos) {
    if (p.epi == EPI_SWIGLU) {
        p.y[vr >> 1] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), b);
        return;
    }
    // EPI_QKV: vr is even; rows vr, vr+1 form one RoPE pair inside a head
    if (vr < p.Dq + p.KVl) {
        const int i = (int)(vr % p.hd) >> 1;
        float o0, o1;
        rope_pair(a, b, p.rope[(int64_t)pos * (p.hd >> 1) + i], o0, o1);
        float *dst = vr < p.Dq ? p.q + vr : p.kcache + (int64_t)pos * p.KVl + (vr - p.Dq);
        dst[0] = o0;
        dst[1] = o1;
    } else {
        float *dst = p.vcache + (int64_t)pos * p.KVl + (vr - p.Dq - p.KVl);
        dst[0] = a;
        dst[1] = b;
    }
}

__device__ __forceinline__ void epi_row(const KParams &p, int64_t r, float v) {
    if (p.epi == EPI_ADD) p.y[r] += v;
    else p.y[r] = v;
}

// ---------------------------------------------------------------- shared prologue: rmsnorm + quantize
// Writes int8 activations, fp32 block scales and int block sums into shared memory (warp per block).
// With norm_w: out = x * inv * w, inv = (float)(1 / sqrt(sum_double(x^2)/n + eps)) (src/ops.c:93-98).
__device__ void prologue_quant(const KParams &p, uint8_t *sm) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float *misc = (float *)(sm + p.misc_off);
    float inv = 1.0f;
    if (p.norm_w) {
        double ss = 0.0;
        for (int i = t; i < p.K; i += NT) ss += (double)p.x[i] * (double)p.x[i];
        ss = warp_sum_d(ss);
        double *dred = (double *)(sm + p.red_off);
        if (lane == 0) dred[warp] = ss;
        __syncthreads();
        if (t == 0) {
            double s = 0.0;
            for (int w = 0; w < NT / 32; w++) s += dred[w];
            misc[0] = (float)(1.0 / sqrt(s / (double)p.K + (double)p.eps));
        }
        __syncthreads();
        inv = misc[0];
    }
    int8_t *xq = (int8_t *)(sm + p.xoff_q);
    float *xd = (float *)(sm + p.xoff_d);
    int *xs = (int *)(sm + p.xoff_s);
    for (int b = warp; b < p.nb; b += NT / 32) {
        const int i = b * 32 + lane;
        float v = 0.0f;
        if (i < p.K) {
            v = p.x[i];
            if (p.norm_w) v = __fmul_rn(__fmul_rn(v, inv), p.norm_w[i]);
        }
        float dd;
        uint32_t dh;
        const int qv = quant_lane(v, 127.0f, -127, 127, &dd, &dh);
        xq[i] = (int8_t)qv;
        const int bs = __reduce_add_sync(0xffffffffu, qv);
        if (lane == 0) {
            xd[b] = dd;
            xs[b] = bs;
        }
        if (p.xq_out) {
            uint8_t *blk = p.xq_out + (int64_t)b * kQ8Bytes;
            blk[2 + lane] = (uint8_t)(int8_t)qv;
            if (lane == 0) {
                blk[0] = (uint8_t)(dh & 0xff);
                blk[1] = (uint8_t)(dh >> 8);
            }
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(NT, 1) gemv_q_kernel(const KParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *bars = (uint64_t *)(sm + (int64_t)p.nstages * p.stage_bytes);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const bool paired = (p.epi == EPI_QKV || p.epi == EPI_SWIGLU);
    const int64_t unit = paired ? 2 : 1;
    const int64_t U = (p.vrows + unit - 1) / unit;
    const int64_t r0 = ((int64_t)blockIdx.x * U / gridDim.x) * unit;
    int64_t r1 = ((int64_t)(blockIdx.x + 1) * U / gridDim.x) * unit;
    if (r1 > p.vrows) r1 = p.vrows;
    const int npass = (int)((r1 - r0 + p.P - 1) / p.P);

    if (t == 0) {
        for (int s = 0; s < p.nstages; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (t == 0)  // weights do not depend on the previous kernel: prefetch before waiting on it
        for (int s = 0; s < p.nstages && s < npass; s++) {
            const int64_t v0 = r0 + (int64_t)s * p.P;
            issue_stage(p, sm + (int64_t)s * p.stage_bytes, &bars[s], v0, min((int64_t)p.P, r1 - v0));
        }
    pdl_wait();
    prologue_quant(p, sm);
    __syncthreads();
    pdl_launch_dependents();

    // this thread's segment of the activations, in registers
    const int seg = t % p.S, slot = t / p.S;
    constexpr int BS = DT == QMC_Q8_0 ? kQ8Bytes : kQ4Bytes;
    uint32_t xa[SEGB][8];
    float xdd[SEGB];
    int xsum[SEGB];
    {
        const uint32_t *xq32 = (const uint32_t *)(sm + p.xoff_q);
        const float *xd = (const float *)(sm + p.xoff_d);
        const int *xs = (const int *)(sm + p.xoff_s);
#pragma unroll
        for (int k = 0; k < SEGB; k++) {
            const int b = seg * SEGB + k;
            uint32_t n[8];
#pragma unroll
            for (int i = 0; i < 8; i++) n[i] = b < p.nb ? xq32[b * 8 + i] : 0u;
            if (DT == QMC_Q4_0) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    xa[k][i] = __byte_perm(n[2 * i], n[2 * i + 1], 0x6420);      // elements 8i, +2, +4, +6
                    xa[k][4 + i] = __byte_perm(n[2 * i], n[2 * i + 1], 0x7531);  // elements 8i+1, +3, +5, +7
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) xa[k][i] = n[i];
            }
            xdd[k] = b < p.nb ? xd[b] : 0.0f;
            xsum[k] = b < p.nb ? xs[b] : 0;
        }
    }
    const int pos = (p.epi == EPI_QKV) ? *p.pos : 0;
    float *red = (float *)(sm + p.red_off);
    float *rowv = (float *)(sm + p.rowv_off);

    for (int pass = 0; pass < npass; pass++) {
        const int st = pass % p.nstages;
        const uint32_t par = (uint32_t)(pass / p.nstages) & 1u;
        const int64_t v0 = r0 + (int64_t)pass * p.P;
        const int nrows = (int)min((int64_t)p.P, r1 - v0);
        const bool ok = mbar_wait(&bars[st], par);
        float part = 0.0f;
        if (ok && slot < nrows) {
            const uint8_t *stage = sm + (int64_t)st * p.stage_bytes;
            const uint8_t *rowp;
            if (p.W1) {
                const int64_t h0 = v0 >> 1;
                rowp = stage + (slot & 1) * p.part_stride + ((h0 * p.rb) & 15) + (int64_t)(slot >> 1) * p.rb;
            } else {
                rowp = stage + ((v0 * p.rb) & 15) + (int64_t)slot * p.rb;
            }
#pragma unroll
            for (int k = 0; k < SEGB; k++) {
                const int b = seg * SEGB + k;
                if (b < p.nb) {
                    if (DT == QMC_Q8_0) {
                        part += dot_q8_block(rowp + b * BS, *(const uint32_t(*)[8]) & xa[k][0], xdd[k]);
                    } else {
                        part += dot_q4_block(rowp + b * BS, *(const uint32_t(*)[4]) & xa[k][0],
                                             *(const uint32_t(*)[4]) & xa[k][4], xdd[k], xsum[k]);
                    }
                }
            }
        }
        red[(pass & 1) * NT + t] = part;
        if (__syncthreads_or(!ok)) {
            if (t == 0) raise_error(p.err, kErrMbarTimeout);
            break;
        }
        if (t == 0 && pass + p.nstages < npass) {
            const int64_t vn = r0 + (int64_t)(pass + p.nstages) * p.P;
            issue_stage(p, sm + (int64_t)st * p.stage_bytes, &bars[st], vn, min((int64_t)p.P, r1 - vn));
        }
        for (int s = warp; s < nrows; s += NT / 32) {
            float v = 0.0f;
            for (int i = lane; i < p.S; i += 32) v += red[(pass & 1) * NT + s * p.S + i];
            v = warp_sum(v);
            if (lane == 0) rowv[(pass & 1) * NT + s] = v;
        }
        __syncthreads();
        const float *rv = rowv + (pass & 1) * NT;
        if (paired) {
            for (int i = t; i < (nrows >> 1); i += NT) epi_pair(p, v0 + 2 * i, rv[2 * i], rv[2 * i + 1], pos);
        } else {
            for (int i = t; i < nrows; i += NT) epi_row(p, v0 + i, rv[i]);
        }
    }
}

// ---------------------------------------------------------------- f32 weights (small models)
// Warp per row (or per row pair), activations (optionally normalised) staged in shared memory.
__global__ void __launch_bounds__(NT) gemv_f32_kernel(const KParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    float *xs = (float *)sm;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const bool paired = (p.epi == EPI_QKV || p.epi == EPI_SWIGLU);
    const int64_t unit = paired ? 2 : 1;
    const int64_t U = (p.vrows + unit - 1) / unit;
    const int64_t u0 = (int64_t)blockIdx.x * U / gridDim.x, u1 = (int64_t)(blockIdx.x + 1) * U / gridDim.x;
    pdl_wait();
    float inv = 1.0f;
    if (p.norm_w) {
        double ss = 0.0;
        for (int i = t; i < p.K; i += NT) ss += (double)p.x[i] * (double)p.x[i];
        ss = warp_sum_d(ss);
        __shared__ double dred[NT / 32];
        __shared__ float sinv;
        if (lane == 0) dred[warp] = ss;
        __syncthreads();
        if (t == 0) {
            double s = 0.0;
            for (int w = 0; w < NT / 32; w++) s += dred[w];
            sinv = (float)(1.0 / sqrt(s / (double)p.K + (double)p.eps));
        }
        __syncthreads();
        inv = sinv;
    }
    for (int i = t; i < p.K; i += NT) xs[i] = p.norm_w ? __fmul_rn(__fmul_rn(p.x[i], inv), p.norm_w[i]) : p.x[i];
    __syncthreads();
    pdl_launch_dependents();
    const int pos = (p.epi == EPI_QKV) ? *p.pos : 0;
    for (int64_t u = u0 + warp; u < u1; u += NT / 32) {
        float v[2] = {0.0f, 0.0f};
        for (int j = 0; j < (int)unit; j++) {
            const int64_t vr = u * unit + j;
            const float *row = p.W1 ? (const float *)((j ? p.W1 : p.W0) + (vr >> 1) * p.rb)
                                    : (const float *)(p.W0 + vr * p.rb);
            float acc = 0.0f;
            for (int i = lane; i < p.K; i += 32) acc = fmaf(row[i], xs[i], acc);
            v[j] = warp_sum(acc);
        }
        if (lane == 0) {
            if (paired) epi_pair(p, u * 2, v[0], v[1], pos);
            else epi_row(p, u, v[0]);
        }
    }
}

int g_attr_done[2] = {0, 0};

}  // namespace

int launch_gemv(const GemvArgs &a, cudaStream_t stream, bool pdl, int grid_limit) {
    DevCtx *c = ctx();
    if (!c) return QMC_ECUDA;
    if (a.rows <= 0 || a.K <= 0) return set_error(QMC_EINVAL, "gemv: empty shape");
    if (a.dtype != QMC_F32 && a.dtype != QMC_Q8_0 && a.dtype != QMC_Q4_0)
        return set_error(QMC_EINVAL, "gemv: bad dtype %d", a.dtype);
    if (((uintptr_t)a.W0 & 15) || ((uintptr_t)a.W1 & 15))
        return set_error(QMC_EINVAL, "gemv: weights must be 16-byte aligned");
    const bool paired = a.epi == EPI_QKV || a.epi == EPI_SWIGLU;
    KParams p{};
    p.W0 = (const uint8_t *)a.W0;
    p.W1 = (const uint8_t *)a.W1;
    p.rb = (int)row_bytes(a.dtype, a.K);
    p.w_bytes = a.rows * (int64_t)p.rb;
    p.vrows = a.epi == EPI_SWIGLU ? 2 * a.rows : a.rows;
    if (paired && (p.vrows & 1)) return set_error(QMC_EINVAL, "gemv: paired epilogue needs an even row count");
    p.K = (int)a.K;
    p.nb = (int)nblocks(a.K);
    p.x = a.x;
    p.norm_w = a.norm_w;
    p.eps = a.eps;
    p.epi = a.epi;
    p.y = a.y;
    p.q = a.q;
    p.kcache = a.kcache;
    p.vcache = a.vcache;
    p.Dq = a.Dq;
    p.KVl = a.KVl;
    p.hd = a.hd;
    p.rope = a.rope;
    p.pos = a.pos;
    p.xq_out = (uint8_t *)a.xq_out;
    p.err = a.err ? a.err : c->err;

    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    cfg.blockDim = dim3(NT);
    cfg.stream = stream;
    const int64_t units = paired ? p.vrows / 2 : p.vrows;
    int grid = grid_limit > 0 ? grid_limit : c->num_sms;

    if (a.dtype == QMC_F32) {
        if (a.xq_out) return set_error(QMC_EINVAL, "gemv: f32 weights take no xq");
        if (p.K > 48 * 1024) return set_error(QMC_EINVAL, "gemv: f32 K too large");
        p.S = 1;
        p.P = 1;
        size_t smem = (size_t)p.K * 4;
        if (smem > 48 * 1024) QMC_CUDA(cudaFuncSetAttribute(gemv_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        if (units < grid) grid = (int)units;
        cfg.gridDim = dim3(grid);
        cfg.dynamicSmemBytes = smem;
        QMC_CUDA(cudaLaunchKernelEx(&cfg, gemv_f32_kernel, p));
        return QMC_OK;
    }

    p.S = (p.nb + SEGB - 1) / SEGB;
    if (p.S > NT) return set_error(QMC_EINVAL, "gemv: K=%lld exceeds %d", (long long)a.K, NT * SEGB * 32);
    p.P = NT / p.S;
    if (paired) p.P &= ~1;
    if (p.P < 1 || (paired && p.P < 2)) return set_error(QMC_EINVAL, "gemv: K too large for a paired epilogue");
    if (p.W1) {
        p.part_stride = (int)(((int64_t)(p.P / 2) * p.rb + 32 + 127) & ~(int64_t)127);
        p.stage_bytes = 2 * p.part_stride;
    } else {
        p.part_stride = 0;
        p.stage_bytes = (int)(((int64_t)p.P * p.rb + 32 + 127) & ~(int64_t)127);
    }
    // activation area + reduction buffers, then the stage ring
    const int xq_bytes = ((p.nb * 32 + 127) / 128) * 128;
    const int xd_bytes = ((p.nb * 4 + 127) / 128) * 128;
    const int red_bytes = 2 * NT * 4, rowv_bytes = 2 * NT * 4, misc_bytes = 128;
    const int fixed = xq_bytes + 2 * xd_bytes + red_bytes + rowv_bytes + misc_bytes;
    const int budget = 100 * 1024;
    int ns = budget / p.stage_bytes;
    ns = ns < 2 ? 2 : (ns > 8 ? 8 : ns);
    p.nstages = ns;
    const int bar_off = ns * p.stage_bytes;
    const int base = bar_off + ((ns * 8 + 127) / 128) * 128;
    p.xoff_q = base;
    p.xoff_d = p.xoff_q + xq_bytes;
    p.xoff_s = p.xoff_d + xd_bytes;
    p.red_off = p.xoff_s + xd_bytes;
    p.rowv_off = p.red_off + red_bytes;
    p.misc_off = p.rowv_off + rowv_bytes;
    const size_t smem = (size_t)p.misc_off + misc_bytes;
    (void)fixed;
    if (smem > c->max_smem_optin) return set_error(QMC_EINVAL, "gemv: %zu bytes of shared memory needed", smem);
    const int which = a.dtype == QMC_Q8_0 ? 0 : 1;
    if (!g_attr_done[which]) {
        if (which == 0)
            QMC_CUDA(cudaFuncSetAttribute(gemv_q_kernel<QMC_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)c->max_smem_optin));
        else
            QMC_CUDA(cudaFuncSetAttribute(gemv_q_kernel<QMC_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)c->max_smem_optin));
        g_attr_done[which] = 1;
    }
    if (units < grid) grid = (int)units;
    cfg.gridDim = dim3(grid);
    cfg.dynamicSmemBytes = smem;
    if (a.dtype == QMC_Q8_0) QMC_CUDA(cudaLaunchKernelEx(&cfg, gemv_q_kernel<QMC_Q8_0>, p));
    else QMC_CUDA(cudaLaunchKernelEx(&cfg, gemv_q_kernel<QMC_Q4_0>, p));
    return QMC_OK;
}

}  // namespace qmc
