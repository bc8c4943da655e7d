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
// SwiGLU epilogues).  A stage is R whole units copied by ONE bulk copy of ~16-20 KB (many small copies
// per stage cost ~50 TMA cycles each and halve the stream rate).  The 16 consumer warps form 4 groups
// of 4 and group j owns stages j, j+4, j+8, ...: each stage's processing is a chain of dependent
// steps (~0.3-0.5 us even for trivial work), and with all warps on every stage that chain gated every
// refill (measured 2.4-2.8 TB/s); four stages in flight through four groups hide it.  Inside a group a
// warp owns whole units when a stage has >= 4 of them, otherwise g = 4/R warps share a unit's blocks and
// meet in shared memory behind a group-local named barrier.  Activations are quantized once per CTA into
// shared memory (int8 in a bank-swizzled layout, fp32 scale, block sum).  Per block: aligned 32-bit
// shared loads + funnel shifts realign the 2-byte-aligned block, dp4a forms the integer block dot and
// s += (float)acc * (dW * dX) as in the reference (src/kernels_scalar.c:12-34).  Q4_0 feeds the low
// nibbles (x 1) and the masked high nibbles (x 16, unsigned) to dp4a against even/odd-permuted
// activations and removes the offset with sum (n_i - 8) x_i = sum n_i x_i - 8 sum x_i.  The footprint
// stays under ~112 KB of shared memory and 60 registers so the next kernel's CTA can co-reside.
#include <stdio.h>

#include <algorithm>

#include "actquant.cuh"
#include "gemv.cuh"

namespace qmc {
namespace {

constexpr int NCW = 16;              // consumer warps
constexpr int NG = 4, GW = 4;        // consumer groups x warps per group (NG * GW == NCW)
constexpr int NT = (NCW + 1) * 32;   // + one producer warp
constexpr int kStageTarget = 16 * 1024;
constexpr int kCoResidentSmem = 112 * 1024;  // two CTAs (this kernel and the next) per SM
// Matrices of at least this many bytes take the whole shared memory of the SM for their ring (up to
// kDeepStages stages): streaming dominates their launch, and ~74 KB in flight per SM (the co-resident
// footprint) cannot cover the loaded copy latency at the SM's share of the HBM bandwidth.
constexpr int64_t kDeepBytes = 48ll << 20;
constexpr int kDeepStages = 3 * NG;

struct KParams {
    const uint8_t *W0, *W1;
    int64_t w_bytes;  // readable bytes of W0 (and of W1)
    int64_t units;    // rows, or row pairs for the paired epilogues
    int K, nb, rb;
    int urows;        // rows per unit (2 for QKV pairs and for SwiGLU's w1/w3 rows)
    int R, g;         // units per stage; warps per unit (g = 4 / R when R < 4, else 1)
    int stage_bytes, part_bytes, nstages;  // part_bytes: offset of the w3 copy inside a SwiGLU stage
    int off_bars, off_xq, off_xds, off_red;  // shared-memory offsets
    const float *x, *norm_w;
    float eps;
    int epi;
    float *y, *q;
    void *kcache, *vcache;
    int kv16;
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

// stage k of a CTA whose units start at u0: units [u0 + kR, u0 + kR + R) as one contiguous copy (two for
// SwiGLU's separate w1/w3 matrices), 16-byte lines by bulk copy plus tail bytes by plain stores
__device__ void issue_stage(const KParams &p, uint8_t *stage, uint64_t *bar, int64_t u0, int64_t u1, int k,
                            uint64_t pol) {
    const int64_t ua = u0 + (int64_t)k * p.R;
    const int64_t n = min((int64_t)p.R, u1 - ua);
    const uint8_t *src[2];
    uint8_t *dst[2];
    CopyPlan cp[2];
    int parts = 1;
    if (p.W1) {
        parts = 2;
        src[0] = p.W0, src[1] = p.W1;
        dst[0] = stage, dst[1] = stage + p.part_bytes;
        cp[0] = cp[1] = plan_copy(ua * p.rb, n * p.rb, p.w_bytes);
    } else {
        src[0] = p.W0, dst[0] = stage;
        cp[0] = plan_copy(ua * p.urows * p.rb, n * p.urows * p.rb, p.w_bytes);
    }
    uint32_t tx = 0;
    bool plain = false;
    for (int i = 0; i < parts; i++) {
        for (int64_t b = cp[i].tail0; b < cp[i].end; b++) dst[i][b - cp[i].a0] = src[i][b];
        plain |= cp[i].tail0 < cp[i].end;
        tx += cp[i].tma;
    }
    // only bytes stored by this thread need ordering against the async copies into the same stage; an
    // unconditional proxy fence here serialises the ring (measured: ~2 TB/s instead of ~7 TB/s)
    if (plain) fence_proxy_async();
    mbar_arrive_tx(bar, tx);
    for (int i = 0; i < parts; i++)
        if (cp[i].tma) bulk_g2s_hint(dst[i], src[i] + cp[i].a0, cp[i].tma, bar, pol);
}

__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
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

// 32 activation bytes of block b as 8 words (stored with the xswz bank swizzle of actquant.cuh)
__device__ __forceinline__ void load_x(const uint8_t *xq, int b, uint32_t (&xw)[8]) {
    const uint8_t *p = xq + (int64_t)b * 32;
    const int sw = xswz(b);
    const uint4 lo = *(const uint4 *)(p + sw), hi = *(const uint4 *)(p + (sw ^ 16));
    xw[0] = lo.x, xw[1] = lo.y, xw[2] = lo.z, xw[3] = lo.w, xw[4] = hi.x, xw[5] = hi.y, xw[6] = hi.z, xw[7] = hi.w;
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {  // unsigned a bytes x signed b bytes
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
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
        int lo = 0, hi16 = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t qw = __funnelshift_rc(w[i], w[i + 1], 16u + sh);
            lo = __dp4a((int)(qw & 0x0f0f0f0fu), (int)xw[i], lo);      // even elements
            hi16 = dp4a_us(qw & 0xf0f0f0f0u, xw[4 + i], hi16);         // odd elements, x16
        }
        const int acc = lo + (hi16 >> 4) - 8 * xs;
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
        if (vr < p.Dq + p.KVl) rope_pair(a, b, p.rope[(int64_t)pos * (p.hd >> 1) + (int)((vr % p.hd) >> 1)], o0, o1);
        if (vr < p.Dq) {
            p.q[vr] = o0;
            p.q[vr + 1] = o1;
        } else if (vr < p.Dq + p.KVl) {
            kv_st2(p.kcache, p.kv16, (int64_t)pos * p.KVl + (vr - p.Dq), o0, o1);
        } else {
            kv_st2(p.vcache, p.kv16, (int64_t)pos * p.KVl + (vr - p.Dq - p.KVl), o0, o1);
        }
    }
}

// ---------------------------------------------------------------- prologue: rmsnorm + quantize
// The consumer warps quantize the activations, four threads per block (8 elements each; quant_block<8>),
// NCW * 8 blocks a round: the values
// come straight from global memory into registers, and the next round's loads are issued before the
// current round is quantized.  With norm_w the values become x * inv * w, inv = (float)(1 / sqrt(
// sum_double(x^2)/n + eps)) (src/ops.c:93-98); a row of one round keeps x in registers across the block
// sum, longer rows take a first pass for the sum.  Quantized activations go to shared memory (int8
// blocks, Q4_0 with even elements then odd ones, and (fp32 scale, int block sum) pairs); CTA 0 also
// writes the Q8_0 blocks to xq_out.  x and norm_w are caller pointers: vector loads only where the 8
// elements are in range and 16-byte aligned (load8_any).
constexpr int QE = 8;              // elements per thread
constexpr int NCT = NCW * 32;      // consumer threads (the prologue's)
constexpr int QB = NCT / 4;        // blocks per round
constexpr int kBarPrologue = 14;   // named barrier of the consumer threads (1..8: unit groups, 15: argmax)
template <int DT>
__device__ void prologue_quant(const KParams &p, uint8_t *sm) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, qd = t >> 2, j = t & 3;
    float *red = (float *)(sm + p.off_red);
    uint8_t *xq = sm + p.off_xq;
    int2 *xds = (int2 *)(sm + p.off_xds);
    uint8_t *aos = p.xq_out && blockIdx.x == 0 ? p.xq_out : nullptr;  // every CTA holds the same blocks
    const int rounds = (p.nb + QB - 1) / QB;
    auto at = [&](int r) { return (int64_t)(r * QB + qd) * 32 + QE * j; };
    float v[QE], nx[QE];
    float inv = 1.0f;
    if (p.norm_w) {
        double ss = 0.0;
        for (int r = 0; r < rounds; r++) {
            load8_any(p.x, at(r), p.K, v);
#pragma unroll
            for (int i = 0; i < QE; i++) ss += (double)v[i] * (double)v[i];
        }
        ss = warp_sum_d(ss);
        double *dred = (double *)red;
        if (lane == 0) dred[warp] = ss;
        named_sync(kBarPrologue, NCT);
        if (t == 0) {
            double tot = 0.0;
            for (int w = 0; w < NCW; w++) tot += dred[w];
            red[2 * NT / 32] = (float)(1.0 / sqrt(tot / (double)p.K + (double)p.eps));
        }
        named_sync(kBarPrologue, NCT);
        inv = red[2 * NT / 32];
        if (rounds > 1) load8_any(p.x, at(0), p.K, v);  // one round: x is still in v
    } else {
        load8_any(p.x, at(0), p.K, v);
    }
    for (int r = 0; r < rounds; r++) {
        if (r + 1 < rounds) load8_any(p.x, at(r + 1), p.K, nx);
        if (p.norm_w) {
            float w[QE];
            load8_any(p.norm_w, at(r), p.K, w);
#pragma unroll
            for (int i = 0; i < QE; i++) v[i] = __fmul_rn(__fmul_rn(v[i], inv), w[i]);
        }
        const int b = r * QB + qd;
        quant_block<QE>(DT == QMC_Q4_0, xq, xds, b, j, b < p.nb, v, aos);
#pragma unroll
        for (int i = 0; i < QE; i++) v[i] = nx[i];
    }
    named_sync(kBarPrologue, NCT);
}

// EPI_LOGITS tail (consumer warps only): CTA max of the warps' keys, one atomicMax per CTA, and the
// last CTA to finish (ticket) turns the global maximum into the next token and resets key and ticket.
__device__ void logits_argmax(const KParams &p, uint8_t *sm, unsigned long long best, int warp, int lane) {
    unsigned long long *keys = (unsigned long long *)(sm + p.off_red + 4 * NCW * 4);
    if (lane == 0) keys[warp] = best;
    named_sync(15, NCW * 32);  // ids 1..8 belong to the unit groups
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
    const int nst = (int)((u1 - u0 + p.R - 1) / p.R);  // stages this CTA streams

    if (t == 0) {
        for (int s = 0; s < p.nstages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    // each weight byte is read once: its lines are the first L2 evicts, so the activations (the previous
    // kernel's output) and the other operands stay in L2 across a chain of matvecs
    const uint64_t pol = l2_evict_first_policy();
    // The producer warp takes no part in the activation prologue: its first copies may wait for room in
    // the copy queue, and a prologue barrier that included it would hold every consumer warp behind them.
    // Weights do not depend on the previous kernel, so the ring fills before (and while) it finishes.
    if (warp == NCW) {
        if (lane == 0) {
            for (int k = 0; k < p.nstages && k < nst; k++)
                issue_stage(p, sm + (int64_t)k * p.stage_bytes, &full[k], u0, u1, k, pol);
            int k = min(p.nstages, nst);  // stages issued so far; refill each once its consumers release it
            for (; k < nst; k++) {
                const int s = k % p.nstages;
                if (!mbar_wait(&empty[s], (uint32_t)((k / p.nstages) - 1) & 1u)) {
                    raise_error(p.err, kErrMbarTimeout);
                    break;
                }
                issue_stage(p, sm + (int64_t)s * p.stage_bytes, &full[s], u0, u1, k, pol);
            }
            // drain: the last copy of each slot may still be in flight; consumers that timed out will not
            // wait for it, and the CTA must not exit before it lands (bounded)
            const long long td = clock64();
            for (int j = max(0, k - p.nstages); j < k; j++)
                if (!mbar_wait_since(&full[j % p.nstages], (uint32_t)(j / p.nstages) & 1u, td)) {
                    raise_error(p.err, kErrMbarTimeout);
                    break;
                }
        }
        return;
    }

    pdl_wait();
    prologue_quant<DT>(p, sm);
    pdl_launch_dependents();

    constexpr int BS = DT == QMC_Q8_0 ? kQ8Bytes : kQ4Bytes;
    const uint8_t *xq = sm + p.off_xq;
    const int2 *xds = (const int2 *)(sm + p.off_xds);
    float2 *red = (float2 *)(sm + p.off_red);  // [2][NCW] partial sums of shared units, double-buffered
    const int pos = p.epi == EPI_QKV ? *p.pos : 0;
    const bool two = p.urows == 2;
    const int grp = warp / GW, wig = warp % GW;
    const int g = p.g, sub = wig % g, bstep = 32 * g;
    unsigned long long best = 0;
    // After a timeout a warp keeps running the loop (on stale stage data) so that every named barrier it
    // shares with other warps is still met, but waits for no more copies and releases no more slots:
    // the producer then never refills a slot whose copy may still be in flight.
    bool dead = false;
    for (int k = grp; k < nst; k += NG) {  // this group's stages
        const int s = k % p.nstages;
        if (!dead && __any_sync(0xffffffffu, !mbar_wait(&full[s], (uint32_t)(k / p.nstages) & 1u))) {
            dead = true;
            if (lane == 0) raise_error(p.err, kErrMbarTimeout);
        }
        const int64_t ua = u0 + (int64_t)k * p.R;
        const int n = (int)min((int64_t)p.R, u1 - ua);
        const uint8_t *stage = sm + (int64_t)s * p.stage_bytes;
        // g == 1: warp wig takes units wig, wig+4, ...; g > 1: the g warps of unit wig / g share it
        for (int i = g == 1 ? wig : wig / g; i < n; i += g == 1 ? GW : n) {
            const int64_t unit = ua + i;
            const uint8_t *r0, *r1;
            if (p.W1) {
                const int64_t off = (ua * p.rb) & 15;
                r0 = stage + off + (int64_t)i * p.rb;
                r1 = stage + p.part_bytes + off + (int64_t)i * p.rb;
            } else {
                r0 = stage + ((ua * p.urows * p.rb) & 15) + (int64_t)i * p.urows * p.rb;
                r1 = r0 + p.rb;
            }
            float a0 = 0.0f, a1 = 0.0f;
            for (int b = sub * 32 + lane; b < p.nb; b += bstep) {
                uint32_t xw[8];
                load_x(xq, b, xw);
                const int2 ds = xds[b];
                const float xd = __int_as_float(ds.x);
                a0 += block_dot<DT>(r0 + b * BS, xw, xd, ds.y);
                if (two) a1 += block_dot<DT>(r1 + b * BS, xw, xd, ds.y);
            }
            a0 = warp_sum(a0);
            if (two) a1 = warp_sum(a1);
            if (g > 1) {
                float2 *rb = red + ((k / NG) & 1) * NCW;
                if (lane == 0) rb[warp] = make_float2(a0, a1);
                named_sync(1 + grp * (GW / g) + i, 32 * g);  // ids 1..8: per (group, shared unit)
                if (sub == 0 && lane == 0) {
                    a0 = a1 = 0.0f;
                    for (int w = 0; w < g; w++) a0 += rb[warp + w].x, a1 += rb[warp + w].y;
                }
            }
            if (sub == 0 && lane == 0) {
                epilogue(p, unit, a0, a1, pos);
                if (p.epi == EPI_LOGITS && a0 == a0) best = max(best, argmax_key(a0, (int)unit));
            }
        }
        __syncwarp();
        if (lane == 0 && !dead) mbar_arrive(&empty[s]);
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
    p.kv16 = a.kv16;
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

    // stage = R whole units in one copy: the smallest power-of-two R (R * g = 16) whose stage reaches
    // kStageTarget bytes; very long units stream one per stage with all 16 warps on it
    p.urows = (a.epi == EPI_QKV || a.epi == EPI_SWIGLU) ? 2 : 1;
    const int64_t unit_bytes = (int64_t)p.urows * p.rb;
    p.R = 1;
    while (p.R < 64 && (int64_t)p.R * unit_bytes < kStageTarget) p.R *= 2;
    p.g = p.R >= GW ? 1 : GW / p.R;
    if (p.W1) {
        p.part_bytes = (int)(((int64_t)p.R * p.rb + 48 + 127) & ~(int64_t)127);
        p.stage_bytes = 2 * p.part_bytes;
    } else {
        p.part_bytes = 0;
        p.stage_bytes = (int)(((int64_t)p.R * unit_bytes + 48 + 127) & ~(int64_t)127);
    }
    const int xq_bytes = ((p.nb * 32 + 127) / 128) * 128, xds_bytes = ((p.nb * 8 + 127) / 128) * 128;
    const int fixed = xq_bytes + xds_bytes + 2 * NT * 4 + 256;  // red: 2 x 16 float2 + 16 keys
    // prefer a footprint that lets the next kernel's CTA co-reside (its weight prefetch then overlaps this
    // kernel's tail); very long rows fall back to the whole shared memory of the SM
    // nstages is a multiple of NG so every slot belongs to one group (slot s serves stages s, s + ns, ...,
    // all of group s % NG).  A slot shared by two groups breaks the parity waits: a group that runs one
    // ring lap ahead of the group before it sees the previous phase's parity as complete and reads a
    // slot whose copy has not landed.
    const bool deep = (int64_t)p.units * unit_bytes >= kDeepBytes;
    int ns = ((deep ? (int)c->max_smem_optin : kCoResidentSmem) - fixed - 256) / p.stage_bytes;
    if (ns < NG) ns = ((int)c->max_smem_optin - fixed - 256) / p.stage_bytes;
    ns = std::min(ns, deep ? kDeepStages : 2 * NG) / NG * NG;
    if (ns == 0) return set_error(QMC_EINVAL, "gemv: K=%lld needs more shared memory than a CTA has", (long long)a.K);
    p.nstages = ns;
    p.off_bars = ns * p.stage_bytes;
    p.off_xq = p.off_bars + ((2 * ns * 8 + 127) / 128) * 128;
    p.off_xds = p.off_xq + xq_bytes;
    p.off_red = p.off_xds + xds_bytes;
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
