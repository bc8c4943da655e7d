// Decode matvec kernels (batch 1, HBM-bound).
//
// Weights (Q8_0 34-byte / Q4_0 18-byte AoS blocks, exactly the file bytes) stream through a ring of
// shared-memory stages filled by 1-D bulk async copies (cp.async.bulk, completion on an mbarrier).
// Warp-specialised: one producer warp issues the copies (the first ring-full before it even waits on
// the previous kernel, so weight traffic overlaps the dependent activation prologue and, under
// programmatic dependent launch, the previous kernel's tail); 16 consumer warps read the stages and
// release them through per-stage "empty" mbarriers.  No CTA-wide barrier runs inside the stream loop.
//
// Work split: a CTA owns a contiguous range of units (a unit is one row, or the row pair of the RoPE /
// SwiGLU epilogues) and one consumer warp owns each unit of a 16-unit row group.  Rows are streamed in
// K-chunks of C blocks (one bulk copy per row chunk), so a stage stays near 18 KB whatever the row
// length; a warp accumulates its row across the chunk stages and reduces once, at the row's end.
// Activations are quantized once per CTA into shared memory (int8, fp32 scale, block sum).  Per block:
// aligned 32-bit shared loads + funnel shifts realign the 2-byte-aligned block, dp4a forms the integer
// block dot, s += (float)acc * (dW * dX) as in the reference (src/kernels_scalar.c:12-34).  Q4_0 uses
// sum (n_i - 8) x_i = sum n_i x_i - 8 sum x_i with nibbles fed to dp4a against even/odd-permuted
// activations.
#include <stdio.h>

#include "gemv.cuh"

namespace qmc {
namespace {

constexpr int NCW = 16;              // consumer warps
constexpr int NT = (NCW + 1) * 32;   // + one producer warp
constexpr int CH = 4096;             // activation staging chunk (floats)
constexpr int kStageBudget = 24 * 1024;
constexpr int kCoResidentSmem = 112 * 1024;  // two CTAs (this kernel and the next) per SM

struct KParams {
    const uint8_t *W0, *W1;
    int64_t w_bytes;  // readable bytes of W0 (and of W1)
    int64_t units;    // rows, or row pairs for the paired epilogues
    int K, nb, rb;
    int urows;        // rows per unit in shared memory (2 for QKV pairs and for SwiGLU's w1/w3 rows)
    int chunked;      // 1: per-row chunk copies (row bytes % 16 == 0); 0: whole rows, one copy per stage
    int C, nchunks, slot_bytes;  // blocks per chunk, chunks per row, bytes per row slot (chunked mode)
    int stage_bytes, nstages;
    int off_bars, off_xq, off_xds, off_xs, off_red;  // shared-memory offsets
    const float *x, *norm_w;
    float eps;
    int epi;
    float *y, *q, *kcache, *vcache;
    int Dq, KVl, hd;
    const float2 *rope;
    const int *pos;
    uint8_t *xq_out;
    unsigned long long *amax_key;
    int *amax_ctr, *state, *gen;
    const int *forced;
    int gen_cap;
    int *err;
};

// ---------------------------------------------------------------- staging (producer lane)
struct CopyPlan {
    int64_t a0, tail0, end;
    uint32_t tma;
};
__device__ __forceinline__ CopyPlan plan_copy(int64_t start, int64_t len, int64_t w_bytes) {
    CopyPlan c;
    c.a0 = start & ~(int64_t)15;
    const int64_t e16 = (start + len + 15) & ~(int64_t)15, lim = w_bytes & ~(int64_t)15;
    int64_t te = e16 < lim ? e16 : lim;
    if (te < c.a0) te = c.a0;
    c.tma = (uint32_t)(te - c.a0);
    c.tail0 = te;
    c.end = start + len;
    return c;
}

// source row `i` (0..urows-1) of unit u
__device__ __forceinline__ const uint8_t *unit_row(const KParams &p, int64_t u, int i) {
    if (p.W1) return (i ? p.W1 : p.W0) + u * p.rb;
    return p.W0 + (u * p.urows + i) * p.rb;
}

// stage k of a CTA whose units start at u0: row group k / nchunks, chunk k % nchunks
__device__ void issue_stage(const KParams &p, uint8_t *stage, uint64_t *bar, int64_t u0, int64_t u1, int k) {
    const int64_t ua = u0 + (int64_t)(k / p.nchunks) * NCW;
    const int64_t n = min((int64_t)NCW, u1 - ua);
    constexpr int BS_Q8 = kQ8Bytes;
    const int BS = p.rb / p.nb == BS_Q8 ? kQ8Bytes : kQ4Bytes;
    if (p.chunked) {
        const int c = k % p.nchunks, cb0 = c * p.C, cb1 = min(p.nb, cb0 + p.C);
        const uint32_t bytes = (uint32_t)((cb1 - cb0) * BS);
        mbar_arrive_tx(bar, bytes * (uint32_t)(n * p.urows));
        for (int64_t j = 0; j < n; j++)
            for (int i = 0; i < p.urows; i++)
                bulk_g2s(stage + (j * p.urows + i) * p.slot_bytes, unit_row(p, ua + j, i) + (int64_t)cb0 * BS, bytes, bar);
        return;
    }
    // whole rows: contiguous units (two runs for SwiGLU's separate matrices), 16-byte lines + tail bytes
    const uint8_t *src[2];
    uint8_t *dst[2];
    CopyPlan cp[2];
    int parts = 1;
    if (p.W1) {
        parts = 2;
        src[0] = p.W0, src[1] = p.W1;
        dst[0] = stage, dst[1] = stage + p.stage_bytes / 2;
        cp[0] = cp[1] = plan_copy(ua * p.rb, n * p.rb, p.w_bytes);
    } else {
        src[0] = p.W0, dst[0] = stage;
        cp[0] = plan_copy(ua * p.urows * p.rb, n * p.urows * p.rb, p.w_bytes);
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

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------- per-block dots from shared memory
template <int NW>
__device__ __forceinline__ void load_words(const uint8_t *bp, uint32_t (&w)[NW], uint32_t &sh) {
    const uint32_t a = smem_u32(bp);
    const uint32_t *wp = (const uint32_t *)(bp - (a & 3u));
    sh = (a & 3u) * 8u;  // 0 or 16
#pragma unroll
    for (int i = 0; i < NW; i++) w[i] = wp[i];
}

// 32 activation bytes of block b as 8 words; quarter-warps alternate halves to stay conflict-free
__device__ __forceinline__ void load_x(const uint8_t *xq, int b, int lane, uint32_t (&xw)[8]) {
    const uint4 *p = (const uint4 *)(xq + (int64_t)b * 32);
    const int h = (lane >> 2) & 1;
    const uint4 a = p[h], c = p[h ^ 1];
    const uint4 lo = h ? c : a, hi = h ? a : c;
    xw[0] = lo.x, xw[1] = lo.y, xw[2] = lo.z, xw[3] = lo.w, xw[4] = hi.x, xw[5] = hi.y, xw[6] = hi.z, xw[7] = hi.w;
}

template <int DT>
__device__ __forceinline__ float block_dot(const uint8_t *bp, const uint32_t (&xw)[8], float xd, int xs) {
    if (DT == QMC_Q8_0) {
        uint32_t w[9], sh;
        load_words<9>(bp, w, sh);
        const uint32_t dbits = __funnelshift_r(w[0], w[1], sh) & 0xffffu;
        int acc = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) acc = __dp4a((int)__funnelshift_rc(w[i], w[i + 1], 16u + sh), (int)xw[i], acc);
        return (float)acc * (h2f(dbits) * xd);
    } else {
        uint32_t w[5], sh;
        load_words<5>(bp, w, sh);
        const uint32_t dbits = __funnelshift_r(w[0], w[1], sh) & 0xffffu;
        int acc = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t qw = __funnelshift_rc(w[i], w[i + 1], 16u + sh);
            acc = __dp4a((int)(qw & 0x0f0f0f0fu), (int)xw[i], acc);          // even elements
            acc = __dp4a((int)((qw >> 4) & 0x0f0f0f0fu), (int)xw[4 + i], acc);  // odd elements
        }
        acc -= 8 * xs;
        return (float)acc * (h2f(dbits) * xd);
    }
}

// ---------------------------------------------------------------- epilogues
__device__ __forceinline__ void rope_pair(float a, float b, float2 cs, float &o0, float &o1) {
    // p0 = x0 c - x1 s ; p1 = x0 s + x1 c, each product and sum rounded separately (src/ops.c:121-123)
    o0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    o1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
}

__device__ __forceinline__ void epilogue(const KParams &p, int64_t unit, float a, float b, int pos) {
    if (p.epi == EPI_STORE || p.epi == EPI_LOGITS) {
        p.y[unit] = a;
    } else if (p.epi == EPI_ADD) {
        p.y[unit] += a;
    } else if (p.epi == EPI_SWIGLU) {
        p.y[unit] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), b);
    } else {  // EPI_QKV: rows 2u, 2u+1 are one RoPE pair inside a head
        const int64_t vr = 2 * unit;
        float o0 = a, o1 = b;
        float *dst;
        if (vr < p.Dq + p.KVl) {
            rope_pair(a, b, p.rope[(int64_t)pos * (p.hd >> 1) + (int)((vr % p.hd) >> 1)], o0, o1);
            dst = vr < p.Dq ? p.q + vr : p.kcache + (int64_t)pos * p.KVl + (vr - p.Dq);
        } else {
            dst = p.vcache + (int64_t)pos * p.KVl + (vr - p.Dq - p.KVl);
        }
        dst[0] = o0;
        dst[1] = o1;
    }
}

// ---------------------------------------------------------------- prologue: rmsnorm + quantize
// x is staged through shared memory in CH-float chunks with wide independent loads; with norm_w the
// values become x * inv * w, inv = (float)(1 / sqrt(sum_double(x^2)/n + eps)) (src/ops.c:93-98).
// Quantized activations go to shared memory: int8 (Q4_0: even elements then odd elements per block),
// and (fp32 scale, int block sum) pairs.
__device__ __forceinline__ void stage_chunk(float *xs, const float *src, int c0, int n) {
    const int t = threadIdx.x;
    if (((uintptr_t)(src + c0) & 15) == 0) {
        const int n4 = n >> 2;
        const float4 *s4 = (const float4 *)(src + c0);
        for (int i = t; i < n4; i += NT) ((float4 *)xs)[i] = s4[i];
        for (int i = (n4 << 2) + t; i < n; i += NT) xs[i] = src[c0 + i];
    } else {
        for (int i = t; i < n; i += NT) xs[i] = src[c0 + i];
    }
}

template <int DT>
__device__ void prologue_quant(const KParams &p, uint8_t *sm) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float *xs = (float *)(sm + p.off_xs);
    float *red = (float *)(sm + p.off_red);
    uint8_t *xq = sm + p.off_xq;
    int2 *xds = (int2 *)(sm + p.off_xds);
    const int nchunk = (p.K + CH - 1) / CH;
    float inv = 1.0f;
    if (p.norm_w) {
        double ss = 0.0;
        for (int c = 0; c < nchunk; c++) {
            const int c0 = c * CH, n = min(CH, p.K - c0);
            if (nchunk > 1) __syncthreads();
            stage_chunk(xs, p.x, c0, n);
            __syncthreads();
            for (int i = t; i < n; i += NT) ss += (double)xs[i] * (double)xs[i];
        }
        ss = warp_sum_d(ss);
        double *dred = (double *)red;
        __syncthreads();
        if (lane == 0) dred[warp] = ss;
        __syncthreads();
        if (t == 0) {
            double s = 0.0;
            for (int w = 0; w < NT / 32; w++) s += dred[w];
            red[2 * NT / 32] = (float)(1.0 / sqrt(s / (double)p.K + (double)p.eps));
        }
        __syncthreads();
        inv = red[2 * NT / 32];
    }
    for (int c = 0; c < nchunk; c++) {
        const int c0 = c * CH, n = min(CH, p.K - c0);
        if (!(p.norm_w && nchunk == 1)) {  // single-chunk norm: x is still staged
            __syncthreads();
            stage_chunk(xs, p.x, c0, n);
        }
        __syncthreads();
        const int b0 = c0 / 32, nbc = (n + 31) / 32;
        for (int bb = warp; bb < nbc; bb += NT / 32) {
            const int b = b0 + bb, i = bb * 32 + lane;
            float v = 0.0f;
            if (i < n) {
                v = xs[i];
                if (p.norm_w) v = __fmul_rn(__fmul_rn(v, inv), p.norm_w[c0 + i]);
            }
            float dd;
            uint32_t dh;
            const int qv = quant_lane(v, 127.0f, -127, 127, &dd, &dh);
            const int pos_in_block = DT == QMC_Q4_0 ? ((lane & 1) ? 16 : 0) + (lane >> 3) * 4 + ((lane & 7) >> 1) : lane;
            xq[b * 32 + pos_in_block] = (uint8_t)(int8_t)qv;
            const int bs = __reduce_add_sync(0xffffffffu, qv);
            if (lane == 0) xds[b] = make_int2(__float_as_int(dd), bs);
            if (p.xq_out) {
                uint8_t *blk = p.xq_out + (int64_t)b * kQ8Bytes;
                blk[2 + lane] = (uint8_t)(int8_t)qv;
                if (lane == 0) blk[0] = (uint8_t)(dh & 0xff), blk[1] = (uint8_t)(dh >> 8);
            }
        }
    }
    __syncthreads();
}

// EPI_LOGITS tail (consumer warps only): CTA max of the warps' keys, one atomicMax per CTA, and the
// last CTA to finish (ticket) turns the global maximum into the next token and resets key and ticket.
__device__ void logits_argmax(const KParams &p, uint8_t *sm, unsigned long long best, int warp, int lane) {
    unsigned long long *keys = (unsigned long long *)(sm + p.off_red);
    if (lane == 0) keys[warp] = best;
    asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
    if (warp == 0 && lane == 0) {
        unsigned long long k = 0;
        for (int w = 0; w < NCW; w++) k = max(k, keys[w]);
        if (k) atomicMax(p.amax_key, k);
        __threadfence();
        if (atomicAdd(p.amax_ctr, 1) == (int)gridDim.x - 1) {
            __threadfence();
            const unsigned long long g = atomicExch(p.amax_key, 0ull);
            int bi = argmax_index(g);
            const float x0 = *(volatile float *)p.y;
            if (x0 != x0) bi = 0;  // a NaN in slot 0 is never replaced by the reference
            advance_state(bi, p.state, p.forced, p.gen, p.gen_cap);
            *p.amax_ctr = 0;
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(NT, 2) gemv_q_kernel(const KParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *full = (uint64_t *)(sm + p.off_bars), *empty = full + p.nstages;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t u0 = (int64_t)blockIdx.x * p.units / gridDim.x;
    const int64_t u1 = (int64_t)(blockIdx.x + 1) * p.units / gridDim.x;
    const int nst = (int)((u1 - u0 + NCW - 1) / NCW) * p.nchunks;  // stages this CTA streams

    if (t == 0) {
        for (int s = 0; s < p.nstages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == NCW && lane == 0)  // weights do not depend on the previous kernel: prefetch first
        for (int k = 0; k < p.nstages && k < nst; k++) issue_stage(p, sm + (int64_t)k * p.stage_bytes, &full[k], u0, u1, k);
    pdl_wait();
    prologue_quant<DT>(p, sm);
    pdl_launch_dependents();

    if (warp == NCW) {  // producer: refill each stage once its consumers released it
        if (lane == 0) {
            for (int k = p.nstages; k < nst; k++) {
                const int s = k % p.nstages;
                if (!mbar_wait(&empty[s], (uint32_t)((k / p.nstages) - 1) & 1u)) {
                    raise_error(p.err, kErrMbarTimeout);
                    break;
                }
                issue_stage(p, sm + (int64_t)s * p.stage_bytes, &full[s], u0, u1, k);
            }
        }
        return;
    }

    constexpr int BS = DT == QMC_Q8_0 ? kQ8Bytes : kQ4Bytes;
    const uint8_t *xq = sm + p.off_xq;
    const int2 *xds = (const int2 *)(sm + p.off_xds);
    const int pos = p.epi == EPI_QKV ? *p.pos : 0;
    const bool two = p.urows == 2;
    float a0 = 0.0f, a1 = 0.0f;
    unsigned long long best = 0;
    for (int k = 0; k < nst; k++) {
        const int s = k % p.nstages, c = k % p.nchunks;
        if (!mbar_wait(&full[s], (uint32_t)(k / p.nstages) & 1u)) {
            if (lane == 0) raise_error(p.err, kErrMbarTimeout);
            return;
        }
        const int64_t ua = u0 + (int64_t)(k / p.nchunks) * NCW, unit = ua + warp;
        if (unit < u1) {
            const uint8_t *stage = sm + (int64_t)s * p.stage_bytes;
            const uint8_t *r0, *r1;
            int cb0, cb1;
            if (p.chunked) {
                r0 = stage + (int64_t)warp * p.urows * p.slot_bytes;
                r1 = r0 + p.slot_bytes;
                cb0 = c * p.C;
                cb1 = min(p.nb, cb0 + p.C);
                r0 -= (int64_t)cb0 * BS;  // index blocks by their row position
                r1 -= (int64_t)cb0 * BS;
            } else if (p.W1) {
                const int64_t off = (ua * p.rb) & 15;
                r0 = stage + off + (int64_t)warp * p.rb;
                r1 = stage + p.stage_bytes / 2 + off + (int64_t)warp * p.rb;
                cb0 = 0, cb1 = p.nb;
            } else {
                r0 = stage + ((ua * p.urows * p.rb) & 15) + (int64_t)warp * p.urows * p.rb;
                r1 = r0 + p.rb;
                cb0 = 0, cb1 = p.nb;
            }
            for (int b = cb0 + lane; b < cb1; b += 32) {
                uint32_t xw[8];
                load_x(xq, b, lane, xw);
                const int2 ds = xds[b];
                const float xd = __int_as_float(ds.x);
                a0 += block_dot<DT>(r0 + b * BS, xw, xd, ds.y);
                if (two) a1 += block_dot<DT>(r1 + b * BS, xw, xd, ds.y);
            }
            if (c == p.nchunks - 1) {  // row complete
                a0 = warp_sum(a0);
                if (two) a1 = warp_sum(a1);
                if (lane == 0) {
                    epilogue(p, unit, a0, a1, pos);
                    if (p.epi == EPI_LOGITS && a0 == a0) best = max(best, argmax_key(a0, (int)unit));
                }
                a0 = a1 = 0.0f;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (p.epi == EPI_LOGITS) logits_argmax(p, sm, best, warp, lane);
}

// ---------------------------------------------------------------- f32 weights (small models)
// Warp per unit, activations (optionally normalised) staged in shared memory.
__global__ void __launch_bounds__(256) gemv_f32_kernel(const KParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    float *xs = (float *)sm;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t u0 = (int64_t)blockIdx.x * p.units / gridDim.x, u1 = (int64_t)(blockIdx.x + 1) * p.units / gridDim.x;
    pdl_wait();
    for (int i = t; i < p.K; i += 256) xs[i] = p.x[i];
    __syncthreads();
    if (p.norm_w) {
        __shared__ double dred[8];
        __shared__ float sinv;
        double ss = 0.0;
        for (int i = t; i < p.K; i += 256) ss += (double)xs[i] * (double)xs[i];
        ss = warp_sum_d(ss);
        if (lane == 0) dred[warp] = ss;
        __syncthreads();
        if (t == 0) {
            double s = 0.0;
            for (int w = 0; w < 8; w++) s += dred[w];
            sinv = (float)(1.0 / sqrt(s / (double)p.K + (double)p.eps));
        }
        __syncthreads();
        for (int i = t; i < p.K; i += 256) xs[i] = __fmul_rn(__fmul_rn(xs[i], sinv), p.norm_w[i]);
        __syncthreads();
    }
    pdl_launch_dependents();
    const int pos = p.epi == EPI_QKV ? *p.pos : 0;
    for (int64_t u = u0 + warp; u < u1; u += 8) {
        float v[2] = {0.0f, 0.0f};
        for (int j = 0; j < (p.W1 ? 2 : p.urows); j++) {
            const float *row = p.W1 ? (const float *)((j ? p.W1 : p.W0) + u * p.rb)
                                    : (const float *)(p.W0 + (u * p.urows + j) * p.rb);
            float acc = 0.0f;
            for (int i = lane; i < p.K; i += 32) acc = fmaf(row[i], xs[i], acc);
            v[j] = warp_sum(acc);
        }
        if (lane == 0) epilogue(p, u, v[0], v[1], pos);
    }
}

bool g_attr_done[64][2];

}  // namespace

int launch_gemv(const GemvArgs &a, cudaStream_t stream, bool pdl, int grid_limit) {
    DevCtx *c = ctx();
    if (!c) return QMC_ECUDA;
    if (a.rows <= 0 || a.K <= 0) return set_error(QMC_EINVAL, "gemv: empty shape");
    if (a.dtype != QMC_F32 && a.dtype != QMC_Q8_0 && a.dtype != QMC_Q4_0)
        return set_error(QMC_EINVAL, "gemv: bad dtype %d", a.dtype);
    if (((uintptr_t)a.W0 & 15) || ((uintptr_t)a.W1 & 15))
        return set_error(QMC_EINVAL, "gemv: weights must be 16-byte aligned");
    KParams p{};
    p.W0 = (const uint8_t *)a.W0;
    p.W1 = (const uint8_t *)a.W1;
    p.rb = (int)row_bytes(a.dtype, a.K);
    p.w_bytes = a.rows * (int64_t)p.rb;
    p.urows = (a.epi == EPI_QKV || (a.epi == EPI_SWIGLU && !a.W1)) ? 2 : 1;
    if (a.epi == EPI_SWIGLU && !a.W1) return set_error(QMC_EINVAL, "gemv: SwiGLU needs the w3 matrix");
    if (a.epi == EPI_SWIGLU) p.urows = 1;
    if (a.epi == EPI_QKV && (a.rows & 1)) return set_error(QMC_EINVAL, "gemv: QKV rows must be even");
    p.units = a.epi == EPI_QKV ? a.rows / 2 : a.rows;
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
    p.amax_key = a.amax_key;
    p.amax_ctr = a.amax_ctr;
    p.state = a.state;
    p.gen = a.gen;
    p.forced = a.forced;
    p.gen_cap = a.gen_cap;
    if (a.epi == EPI_LOGITS && (a.dtype == QMC_F32 || !a.amax_key || !a.amax_ctr || !a.state))
        return set_error(QMC_EINVAL, "gemv: the fused argmax needs quantized weights and its state buffers");
    p.err = a.err ? a.err : c->err;

    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    cfg.stream = stream;
    int grid = grid_limit > 0 ? grid_limit : c->num_sms;
    if (p.units < grid) grid = (int)p.units;
    cfg.gridDim = dim3(grid);

    if (a.dtype == QMC_F32) {
        if (a.xq_out) return set_error(QMC_EINVAL, "gemv: f32 weights take no xq");
        if (p.K > 48 * 1024) return set_error(QMC_EINVAL, "gemv: f32 K too large");
        const size_t smem = (size_t)p.K * 4;
        if (smem > 48 * 1024)
            QMC_CUDA(cudaFuncSetAttribute(gemv_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = smem;
        QMC_CUDA(cudaLaunchKernelEx(&cfg, gemv_f32_kernel, p));
        return QMC_OK;
    }

    // stage = 16 units x (urows rows) x (C blocks); rows whose byte length is a multiple of 16 stream as
    // per-row chunk copies, others as whole contiguous rows
    p.urows = (a.epi == EPI_QKV || a.epi == EPI_SWIGLU) ? 2 : 1;
    const int BS = a.dtype == QMC_Q8_0 ? kQ8Bytes : kQ4Bytes;
    p.chunked = (p.nb % 8) == 0;
    if (p.chunked) {
        p.C = 256;
        while (p.C > 32 && (int64_t)NCW * p.urows * p.C * BS > kStageBudget) p.C /= 2;
        if (p.C > p.nb) p.C = (p.nb + 31) / 32 * 32;
        p.nchunks = (p.nb + p.C - 1) / p.C;
        p.slot_bytes = p.C * BS;  // multiple of 16 (C is a multiple of 8 blocks)
        p.stage_bytes = (int)(((int64_t)NCW * p.urows * p.slot_bytes + 127) & ~(int64_t)127);
    } else {
        p.C = p.nb;
        p.nchunks = 1;
        p.slot_bytes = 0;
        const int64_t part = ((int64_t)NCW * (p.W1 ? 1 : p.urows) * p.rb + 48 + 127) & ~(int64_t)127;
        p.stage_bytes = (int)(p.W1 ? 2 * part : part);
    }
    const int xq_bytes = ((p.nb * 32 + 127) / 128) * 128, xds_bytes = ((p.nb * 8 + 127) / 128) * 128;
    const int fixed = xq_bytes + xds_bytes + CH * 4 + 2 * NT * 4 + 256;
    // prefer a footprint that lets the next kernel's CTA co-reside (its weight prefetch then overlaps this
    // kernel's tail); very long rows fall back to the whole shared memory of the SM
    int ns = (kCoResidentSmem - fixed - 256) / p.stage_bytes;
    if (ns < 3) ns = ((int)c->max_smem_optin - fixed - 256) / p.stage_bytes;
    if (ns > 6) ns = 6;
    if (ns < 2) return set_error(QMC_EINVAL, "gemv: K=%lld needs more shared memory than a CTA has", (long long)a.K);
    p.nstages = ns;
    p.off_bars = ns * p.stage_bytes;
    p.off_xq = p.off_bars + ((2 * ns * 8 + 127) / 128) * 128;
    p.off_xds = p.off_xq + xq_bytes;
    p.off_xs = p.off_xds + xds_bytes;
    p.off_red = p.off_xs + CH * 4;
    const size_t smem = (size_t)p.off_red + 2 * NT * 4 + 256;
    const int which = a.dtype == QMC_Q8_0 ? 0 : 1;
    if (!g_attr_done[c->device][which]) {
        if (which == 0)
            QMC_CUDA(cudaFuncSetAttribute(gemv_q_kernel<QMC_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)c->max_smem_optin));
        else
            QMC_CUDA(cudaFuncSetAttribute(gemv_q_kernel<QMC_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)c->max_smem_optin));
        g_attr_done[c->device][which] = true;
    }
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    if (a.dtype == QMC_Q8_0) QMC_CUDA(cudaLaunchKernelEx(&cfg, gemv_q_kernel<QMC_Q8_0>, p));
    else QMC_CUDA(cudaLaunchKernelEx(&cfg, gemv_q_kernel<QMC_Q4_0>, p));
    return QMC_OK;
}

}  // namespace qmc
