// Persistent decode step: one cooperative launch of one CTA per SM runs the whole token step of
// src/model.c:158-191 -- embedding, L x {rmsnorm + QKV matvec + RoPE + KV store, attention, wo matvec +
// residual, rmsnorm + w1/w3 matvecs + SwiGLU, w2 matvec + residual}, final rmsnorm + output matvec +
// greedy argmax -- as a list of phases separated by grid barriers.
//
// Why one kernel: batch-1 decode streams every weight byte once and is bound by HBM, but a bulk copy
// takes ~3 us to land under load, so an SM needs ~130 KB in flight to draw its share of the bandwidth.
// Separate kernels per matvec cannot keep that: each boundary drains the pipeline, and co-residency
// with the next kernel caps the ring at half the shared memory.  Here one producer warp per CTA walks
// the weight stages of ALL phases in order through a ring of 15 (or 12, 9, 6, 3) slots in ~210 KB of shared
// memory and never waits on a grid barrier: while the consumers sit in a barrier, an activation
// prologue or the attention phase, the producer is already streaming the next matrices.
//
// Consumers: 12 warps in 3 groups; global stage g goes to group g % 3 and slot g % nslots (nslots is a
// multiple of 3, so a slot always serves one group and the parity waits stay one phase apart).  The
// units (rows, or the RoPE / SwiGLU row pairs) of a group's stages are dealt round-robin to its 4 warps
// and a warp works alone: lane l takes blocks l, l+32, ... of the row (the first four held in registers
// as Q8_0 activations for the whole phase), a warp sum forms the row dot and lane 0 runs the epilogue
// (RoPE + K/V store, residual add, SwiGLU, logits + argmax key).  No CTA or group barrier runs inside
// the stream loop.
//
// Weights are in the split-row layout (decode.cuh): aligned 16-byte shared loads per block, no realignment.
// Per block the arithmetic is the reference's (src/kernels_scalar.c:12-34): integer block dot (dp4a; Q4_0
// as low nibbles x 1 + masked high nibbles x 16 against even/odd activations, minus 8 * sum x), then
// s += (float)acc * (dW * dX).  Activations are quantized per phase by every CTA (bit-exact Q8_0,
// src/quant.c:33-53) after the fused rmsnorm (src/ops.c:93-98).
//
// Attention (src/model.c:132-156): (KV head, position segment) units over the CTAs; the 12 warps of a
// CTA walk the segment's positions with an online softmax per query head, merge in shared memory, and
// the last CTA of a head (ticket) merges the segments' (max, sum, acc) partials into the head's output.
//
// Every wait is bounded (mbarrier waits, the grid barrier): on expiry a thread raises the error word and
// continues without waiting, so the launch always ends; the host then reports QMC_ETIMEOUT.
#include <algorithm>

#include "decode.cuh"

namespace qmc {
namespace {

constexpr int NCW = 12;             // consumer warps (13 warps in all: at most 4 per SM sub-partition, so
                                    // each thread may hold 128 registers)
constexpr int NG = 3, GW = 4;       // groups x warps per group
constexpr int GT = GW * 32;         // threads per group
constexpr int NT = (NCW + 1) * 32;  // + the producer warp
constexpr int NCT = NCW * 32;       // consumer threads
constexpr int QPR = NCT / 2;        // activation blocks per prologue round (2 threads per block)
constexpr int XW = 4;               // activation blocks per lane kept in registers (the rest from shared)
constexpr int GMAX = kDecodeHeadsPerUnit;  // query heads per attention unit (a larger GQA group spans units)
constexpr int MAXW = 4;             // head_dim / 32 (head_dim <= 128)
constexpr int kMinAttnPos = 32;     // an attention segment spans at least this many positions
// named barriers: 0 = __syncthreads, 1..NG = the groups, kBarConsumers = all consumer warps
constexpr int kBarConsumers = NG + 1;
// shared scratch at off_red: prologue partial sums, argmax keys, grid-barrier flag
constexpr int kRedDred = 0, kRedKeys = 128;
constexpr int kRedFlag = kRedKeys + NCW * 8, kRedBytes = kRedFlag + 128;

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void split_units(int64_t units, int64_t &u0, int64_t &u1) {
    u0 = (int64_t)blockIdx.x * units / gridDim.x;
    u1 = (int64_t)(blockIdx.x + 1) * units / gridDim.x;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {  // unsigned a bytes x signed b bytes
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// ---------------------------------------------------------------- grid barrier (consumer threads)
// One monotonic arrival counter per step: barrier j is passed once (j + 1) * gridDim.x arrivals are seen.
// Thread 0 arrives with a release atomic after a CTA barrier (so the CTA's epilogue stores are ordered
// before it) and polls with acquire loads (bounded); the step's last CTA resets the counter for the next
// launch.  Activations written before a barrier are read after it with L2 (.cg) loads.
__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ bool grid_sync(const DecodeParams &p, uint8_t *sm, unsigned target, bool dead) {
    int *flag = (int *)(sm + p.off_red + kRedFlag);
    named_sync(kBarConsumers, NCT);
    if (threadIdx.x == 0) {
        int ok = 1;
        red_release_add(p.gbar, 1u);
        if (!dead) {
            const long long t0 = clock64();
            while ((int)(ld_acquire(p.gbar) - target) < 0)
                if (clock64() - t0 > kWaitCycles) {
                    raise_error(p.err, kErrFlagTimeout);
                    ok = 0;
                    break;
                }
        }
        *flag = ok;
    }
    named_sync(kBarConsumers, NCT);
    return *flag != 0;
}

// ---------------------------------------------------------------- producer
__device__ void producer(const DecodeParams &p, uint8_t *sm, uint64_t *full, uint64_t *empty) {
    unsigned gk = 0;
    for (int i = 0; i < p.nph; i++) {
        const DecodePhase &ph = p.ph[i];
        if (ph.kind == PH_ATTN) continue;
        int64_t u0, u1;
        split_units(ph.units, u0, u1);
        const int64_t ubytes = (int64_t)ph.urows * ph.rbytes;
        for (int64_t ua = u0; ua < u1; ua += ph.R, gk++) {
            const int s = (int)(gk % (unsigned)p.nslots);
            if (gk >= (unsigned)p.nslots && !mbar_wait(&empty[s], ((gk / p.nslots) - 1) & 1u)) {
                raise_error(p.err, kErrMbarTimeout);
                return;
            }
            const uint32_t bytes = (uint32_t)(min((int64_t)ph.R, u1 - ua) * ubytes);
            mbar_arrive_tx(&full[s], bytes);
            bulk_g2s(sm + (size_t)s * p.slot_bytes, ph.W + ua * ubytes, bytes, &full[s]);
        }
    }
}

// ---------------------------------------------------------------- prologue: input -> Q8_0 activations
// 16 elements e0..e0+15 of the phase input: the token's embedding row (dequantized as src/quant.c:65-94,
// one rounding) for the first phase, else the input vector; zero past K
__device__ __forceinline__ void fetch16(const DecodeParams &p, const DecodePhase &ph, const uint8_t *erow, int64_t e0,
                                        float (&v)[16]) {
    const int K = ph.K;
    if (e0 >= K) {  // pairs past the last block (their block and its scale lie outside the row)
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = 0.0f;
        return;
    }
    if (ph.embed) {
        const int64_t b = e0 >> 5;
        const int j0 = (int)(e0 & 31);
        if (p.dt_tok == QMC_F32) {
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = e0 + i < K ? ((const float *)erow)[e0 + i] : 0.0f;
        } else if (p.dt_tok == QMC_Q8_0) {
            const uint8_t *blk = erow + b * kQ8Bytes;
            const float d = h2f(blk[0] | (blk[1] << 8));
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = e0 + i < K ? d * (float)(int8_t)blk[2 + j0 + i] : 0.0f;
        } else {
            const uint8_t *blk = erow + b * kQ4Bytes;
            const float d = h2f(blk[0] | (blk[1] << 8));
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int k = j0 + i, byte = blk[2 + (k >> 1)];
                v[i] = e0 + i < K ? d * (float)(((k & 1) ? (byte >> 4) : (byte & 15)) - 8) : 0.0f;
            }
        }
        return;
    }
    const float *src = ph.in + e0;
    if (e0 + 16 <= K && !((uintptr_t)src & 15)) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 a = __ldcg((const float4 *)src + i);
            v[4 * i] = a.x, v[4 * i + 1] = a.y, v[4 * i + 2] = a.z, v[4 * i + 3] = a.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = e0 + i < K ? __ldcg(src + i) : 0.0f;
    }
}
__device__ __forceinline__ void fetch16_w(const float *w, int64_t e0, int K, float (&v)[16]) {
    if (e0 + 16 <= K && !((uintptr_t)(w + e0) & 15)) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 a = *((const float4 *)(w + e0) + i);
            v[4 * i] = a.x, v[4 * i + 1] = a.y, v[4 * i + 2] = a.z, v[4 * i + 3] = a.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = e0 + i < K ? w[e0 + i] : 0.0f;
    }
}

// activation block b is stored with its 16-byte halves swapped when bit 2 of b is set, so 8 threads
// loading consecutive blocks hit all 32 banks
__device__ __forceinline__ int xswz(int b) { return ((b >> 2) & 1) << 4; }

// Quotients v / sc for the quantizer (src/quant.c:47-50 divides, then rounds half to even).  |v / sc| <
// 256, so r = v * (1 / sc) lies within 4.6e-5 of the correctly rounded quotient and rounds to the same
// integer unless that quotient is within 4.6e-5 of a half-integer.  If any of the lane's 16 products is
// that close, the lane takes the IEEE divisions instead (rare); NaN and infinity give the same results
// on both paths.
__device__ __forceinline__ void quotients16(const float (&v)[16], float sc, float (&r)[16]) {
    const float rs = __frcp_rn(sc);
    bool near = false;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        r[i] = __fmul_rn(v[i], rs);
        near |= fabsf(__fsub_rn(r[i], floorf(r[i])) - 0.5f) < 1.0e-4f;
    }
    if (near) {
#pragma unroll
        for (int i = 0; i < 16; i++) r[i] = __fdiv_rn(v[i], sc);
    }
}

// Q8_0 of block b held by a lane pair (part j: elements 16j..16j+15), bit-exact with src/quant.c:33-53:
// amax ignores NaN, IEEE division for the scale, fp16 RNE scale, then the quantized elements.  All lanes
// call it (pair shuffles); `active` lanes store.  Q4_0 weights take the block's even elements in bytes
// 0-15 and odd elements in bytes 16-31.
__device__ __forceinline__ void quant_block(bool q4, uint8_t *xq, int2 *xds, int b, int j, bool active,
                                            const float (&v)[16]) {
    uint32_t ab = 0;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const float a = fabsf(v[i]);
        ab = max(ab, (a == a) ? __float_as_uint(a) : 0u);  // |v| bits order like floats; NaN -> 0
    }
    ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, 1));
    const float sc = h2f(f2h(__fdiv_rn(__uint_as_float(ab), 127.0f)));
    float qf[16];
    quotients16(v, sc, qf);
    uint32_t w[4] = {0u, 0u, 0u, 0u};  // Q8_0: bytes 16j.. in order; Q4_0: even | odd elements
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        float rq = rintf(qf[i]);
        rq = rq < -127.0f ? -127.0f : rq;
        rq = rq > 127.0f ? 127.0f : rq;
        const int q = sc != 0.0f ? (int)rq : 0;
        sum += q;
        const int k = q4 ? ((i & 1) ? 8 : 0) + (i >> 1) : i;  // byte index within this lane's 16
        w[k >> 2] |= (uint32_t)(q & 0xff) << (8 * (k & 3));
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    if (!active) return;
    uint8_t *blk = xq + (int64_t)b * 32;
    const int sw = xswz(b);
    if (!q4) {
        *(uint4 *)(blk + ((16 * j) ^ sw)) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        *(uint2 *)(blk + ((8 * j) ^ sw)) = make_uint2(w[0], w[1]);
        *(uint2 *)(blk + ((16 + 8 * j) ^ sw)) = make_uint2(w[2], w[3]);
    }
    if (j == 0) xds[b] = make_int2(__float_as_int(sc), sum);
}

// The phase input (optionally x * inv * w, inv = (float)(1 / sqrt(sum_double(x^2)/n + eps)),
// src/ops.c:93-98) quantized into shared memory by the consumer threads, two per block; the first
// phase's CTA 0 also stores the embedding into x.  The first round's x and w stay in registers.
__device__ void prologue(const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, int token) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, qd = t >> 1, j = t & 1;
    uint8_t *xq = sm + p.off_xq;
    int2 *xds = (int2 *)(sm + p.off_xds);
    const bool q4 = ph.dtype == QMC_Q4_0;
    const int K = ph.K, rounds = (ph.nb + QPR - 1) / QPR;
    const uint8_t *erow = ph.embed ? p.tok + (int64_t)token * row_bytes(p.dt_tok, K) : nullptr;
    const bool keep_x = ph.embed && blockIdx.x == 0;
    const float *nw = ph.norm_w;
    const int64_t e00 = (int64_t)qd * 32 + 16 * j;
    float v0[16], w0[16];
    fetch16(p, ph, erow, e00, v0);
    if (nw) fetch16_w(nw, e00, K, w0);
    float inv = 1.0f;
    if (nw) {
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < 16; i++) ss = fma((double)v0[i], (double)v0[i], ss);
        for (int r = 1; r < rounds; r++) {
            float v[16];
            fetch16(p, ph, erow, (int64_t)(r * QPR + qd) * 32 + 16 * j, v);
#pragma unroll
            for (int i = 0; i < 16; i++) ss = fma((double)v[i], (double)v[i], ss);
        }
        ss = warp_sum_d(ss);
        double *dred = (double *)(sm + p.off_red + kRedDred);
        if (lane == 0) dred[warp] = ss;
        named_sync(kBarConsumers, NCT);
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < NCW; w++) tot += dred[w];  // same order in every thread
        inv = (float)(1.0 / sqrt(tot / (double)K + (double)p.eps));
    }
    float v1[16], w1[16];
    for (int r = 0; r < rounds; r++) {
        const int b = r * QPR + qd;
        const int64_t e0 = (int64_t)b * 32 + 16 * j;
        if (r > 0) {
#pragma unroll
            for (int i = 0; i < 16; i++) v0[i] = v1[i], w0[i] = w1[i];
        }
        if (r + 1 < rounds) {  // next round's loads in flight while this one is quantized
            const int64_t e1 = e0 + (int64_t)QPR * 32;
            fetch16(p, ph, erow, e1, v1);
            if (nw) fetch16_w(nw, e1, K, w1);
        }
        if (keep_x) {
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (e0 + i < K) __stcg(p.x + e0 + i, v0[i]);
        }
        if (nw) {
#pragma unroll
            for (int i = 0; i < 16; i++) v0[i] = __fmul_rn(__fmul_rn(v0[i], inv), w0[i]);
        }
        quant_block(q4, xq, xds, b, j, b < ph.nb, v0);
    }
    named_sync(kBarConsumers, NCT);
}

// ---------------------------------------------------------------- matvec phases
template <int DT>
__device__ __forceinline__ float dot_split(const uint8_t *row, int sbytes, int b, const uint32_t (&xw)[8], float xd,
                                           int xs) {
    const float dw = h2f(*(const unsigned short *)(row + 2 * b));
    if (DT == QMC_Q8_0) {
        const uint4 a = *(const uint4 *)(row + sbytes + 32 * b), c = *(const uint4 *)(row + sbytes + 32 * b + 16);
        int acc = __dp4a((int)a.x, (int)xw[0], 0);
        acc = __dp4a((int)a.y, (int)xw[1], acc);
        acc = __dp4a((int)a.z, (int)xw[2], acc);
        acc = __dp4a((int)a.w, (int)xw[3], acc);
        acc = __dp4a((int)c.x, (int)xw[4], acc);
        acc = __dp4a((int)c.y, (int)xw[5], acc);
        acc = __dp4a((int)c.z, (int)xw[6], acc);
        acc = __dp4a((int)c.w, (int)xw[7], acc);
        return (float)acc * (dw * xd);
    } else {
        const uint4 a = *(const uint4 *)(row + sbytes + 16 * b);
        int lo = __dp4a((int)(a.x & 0x0f0f0f0fu), (int)xw[0], 0);  // even elements
        lo = __dp4a((int)(a.y & 0x0f0f0f0fu), (int)xw[1], lo);
        lo = __dp4a((int)(a.z & 0x0f0f0f0fu), (int)xw[2], lo);
        lo = __dp4a((int)(a.w & 0x0f0f0f0fu), (int)xw[3], lo);
        int hi16 = dp4a_us(a.x & 0xf0f0f0f0u, xw[4], 0);  // odd elements, x16
        hi16 = dp4a_us(a.y & 0xf0f0f0f0u, xw[5], hi16);
        hi16 = dp4a_us(a.z & 0xf0f0f0f0u, xw[6], hi16);
        hi16 = dp4a_us(a.w & 0xf0f0f0f0u, xw[7], hi16);
        const int acc = lo + (hi16 >> 4) - 8 * xs;
        return (float)acc * (dw * xd);
    }
}

__device__ __forceinline__ void load_x(const uint8_t *xq, const int2 *xds, int b, uint32_t (&xw)[8], float &xd,
                                       int &xs) {
    const uint8_t *p = xq + (int64_t)b * 32;
    const int sw = xswz(b);
    const uint4 lo = *(const uint4 *)(p + sw), hi = *(const uint4 *)(p + (sw ^ 16));
    xw[0] = lo.x, xw[1] = lo.y, xw[2] = lo.z, xw[3] = lo.w, xw[4] = hi.x, xw[5] = hi.y, xw[6] = hi.z, xw[7] = hi.w;
    const int2 ds = xds[b];
    xd = __int_as_float(ds.x);
    xs = ds.y;
}

__device__ __forceinline__ void rope_pair(float a, float b, float2 cs, float &o0, float &o1) {
    // p0 = x0 c - x1 s ; p1 = x0 s + x1 c, each product and sum rounded separately (src/ops.c:121-123)
    o0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
    o1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
}

// operand an epilogue lane needs besides the row sums, loaded before the unit.s dots so its latency is
// hidden: the RoPE (cos, sin) of a q/k pair, or the residual value of x
__device__ __forceinline__ float2 epilogue_operand(const DecodeParams &p, const DecodePhase &ph, int64_t unit, int pos) {
    if (ph.kind == PH_QKV) {
        const int64_t vr = 2 * unit;
        if (vr < p.Dq + p.KVl) return p.rope[(int64_t)pos * (p.hd >> 1) + (int)((vr % p.hd) >> 1)];
        return make_float2(0.0f, 0.0f);
    }
    if (ph.kind == PH_WO || ph.kind == PH_W2) return make_float2(__ldcg(ph.out + unit), 0.0f);
    return make_float2(0.0f, 0.0f);
}

__device__ __forceinline__ void epilogue(const DecodeParams &p, const DecodePhase &ph, int64_t unit, float a, float b,
                                         float2 opnd, int pos, unsigned long long &best) {
    switch (ph.kind) {
    case PH_QKV: {  // rows 2u, 2u+1: one RoPE pair of q or k, or two v values
        const int64_t vr = 2 * unit;
        float o0 = a, o1 = b;
        float *dst;
        if (vr < p.Dq + p.KVl) {
            rope_pair(a, b, opnd, o0, o1);
            dst = vr < p.Dq ? p.q + vr : ph.kc + (int64_t)pos * p.KVl + (vr - p.Dq);
        } else {
            dst = ph.vc + (int64_t)pos * p.KVl + (vr - p.Dq - p.KVl);
        }
        __stcg(dst, o0);
        __stcg(dst + 1, o1);
        break;
    }
    case PH_WO:
    case PH_W2: __stcg(ph.out + unit, opnd.x + a); break;  // residual (src/model.c:179,186)
    case PH_FFN: __stcg(ph.out + unit, __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), b)); break;  // src/ops.c:128-133
    default:  // PH_OUT
        __stcg(ph.out + unit, a);
        if (a == a) best = max(best, argmax_key(a, (int)unit));
        break;
    }
}

// one unit (a row, or a row pair when TWO) of a stage: this lane's blocks lane, lane + 32, ... (the first
// XW from registers), summed over the warp
template <int DT, bool TWO>
__device__ __forceinline__ void unit_dot(const uint8_t *r0, int rbytes, int sbytes, int nb, const uint8_t *xq,
                                         const int2 *xds, const uint32_t (&xw)[XW][8], const float (&xd)[XW],
                                         const int (&xs)[XW], float &a0, float &a1) {
    const int lane = threadIdx.x & 31;
    const uint8_t *r1 = r0 + rbytes;
    a0 = 0.0f, a1 = 0.0f;
    if (nb >= 32 * XW) {  // every register block is in the row: no per-block test
#pragma unroll
        for (int c = 0; c < XW; c++) {
            a0 += dot_split<DT>(r0, sbytes, lane + 32 * c, xw[c], xd[c], xs[c]);
            if (TWO) a1 += dot_split<DT>(r1, sbytes, lane + 32 * c, xw[c], xd[c], xs[c]);
        }
        for (int b = lane + 32 * XW; b < nb; b += 32) {
            uint32_t xr[8];
            float rd;
            int rs;
            load_x(xq, xds, b, xr, rd, rs);
            a0 += dot_split<DT>(r0, sbytes, b, xr, rd, rs);
            if (TWO) a1 += dot_split<DT>(r1, sbytes, b, xr, rd, rs);
        }
    } else {
#pragma unroll
        for (int c = 0; c < XW; c++) {
            const int b = lane + 32 * c;
            if (b < nb) {
                a0 += dot_split<DT>(r0, sbytes, b, xw[c], xd[c], xs[c]);
                if (TWO) a1 += dot_split<DT>(r1, sbytes, b, xw[c], xd[c], xs[c]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        a0 += __shfl_xor_sync(0xffffffffu, a0, o);
        if (TWO) a1 += __shfl_xor_sync(0xffffffffu, a1, o);
    }
}

// One matvec phase on this CTA's units.  Group grp takes the stages g with g % NG == grp; within the
// group the units of its stages are dealt round-robin to its 4 warps, so a warp works alone: its own
// row dots, its own warp sum, its own epilogue (lane 0), and one arrival on each of its group's stages.
template <int DT, bool TWO>
__device__ void run_matvec(const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, uint64_t *full, uint64_t *empty,
                           unsigned &gk, bool &dead, int pos, unsigned long long &best) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, grp = warp / GW, wig = warp % GW;
    const uint8_t *xq = sm + p.off_xq;
    const int2 *xds = (const int2 *)(sm + p.off_xds);
    const int nb = ph.nb, sbytes = ph.sbytes, rbytes = ph.rbytes, R = ph.R;
    constexpr int UR = TWO ? 2 : 1;
    uint32_t xw[XW][8];
    float xd[XW];
    int xs[XW];
#pragma unroll
    for (int c = 0; c < XW; c++) {
        const int b = lane + 32 * c;
        if (b < nb) {
            load_x(xq, xds, b, xw[c], xd[c], xs[c]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) xw[c][i] = 0;
            xd[c] = 0.0f, xs[c] = 0;
        }
    }
    int64_t u0, u1;
    split_units(ph.units, u0, u1);
    const int nst = (int)((u1 - u0 + R - 1) / R);
    int uoff = 0;  // units in this group's earlier stages of the phase
    for (int k = 0; k < nst; k++) {
        const unsigned g = gk + (unsigned)k;
        if ((int)(g % NG) != grp) continue;
        const int s = (int)(g % (unsigned)p.nslots);
        if (!dead && !mbar_wait(&full[s], (g / p.nslots) & 1u)) {
            dead = true;
            if (lane == 0) raise_error(p.err, kErrMbarTimeout);
        }
        const int64_t ua = u0 + (int64_t)k * R;
        const int n = (int)min((int64_t)R, u1 - ua);
        const uint8_t *stage = sm + (size_t)s * p.slot_bytes;
        if (!dead) {
            for (int i = (wig - uoff % GW + GW) % GW; i < n; i += GW) {
                // the epilogue operand is fetched first so its latency hides behind the dots
                const float2 opnd = lane == 0 ? epilogue_operand(p, ph, ua + i, pos) : make_float2(0.0f, 0.0f);
                float a0, a1;
                unit_dot<DT, TWO>(stage + (int64_t)i * UR * rbytes, rbytes, sbytes, nb, xq, xds, xw, xd, xs, a0, a1);
                if (lane == 0) epilogue(p, ph, ua + i, a0, a1, opnd, pos, best);
            }
        }
        uoff += n;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    gk += (unsigned)nst;
}

// ---------------------------------------------------------------- attention phase
__device__ void attention(const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, int pos) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int npos = pos + 1, nunit = p.nkv * p.gsplit;
    int nseg = min(p.maxseg, (npos + kMinAttnPos - 1) / kMinAttnPos);
    if (nseg < 1) nseg = 1;
    const bool active = (int)blockIdx.x < nunit * nseg;
    const int unit = active ? (int)blockIdx.x / nseg : 0, seg = active ? (int)blockIdx.x % nseg : 0;
    const int kvh = unit / p.gsplit, gs = unit % p.gsplit, h0 = gs * GMAX, G = min(GMAX, p.group - h0);
    const int hd = p.hd, stride = hd + 2;
    const int chunk = (npos + nseg - 1) / nseg, t0 = seg * chunk, t1 = active ? min(npos, t0 + chunk) : 0;
    const int64_t hq = (int64_t)kvh * p.group + h0;  // first query head of this unit
    const float *kb = ph.kc + (int64_t)kvh * hd, *vb = ph.vc + (int64_t)kvh * hd;

    float q[GMAX][MAXW], o[GMAX][MAXW], m[GMAX], l[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int w = 0; w < MAXW; w++) {
            const int d = lane + 32 * w;
            q[g][w] = (active && g < G && d < hd) ? __ldcg(p.q + (hq + g) * hd + d) : 0.0f;
            o[g][w] = 0.0f;
        }
    }
    // positions t0 + warp, + 12, ...; the next position's K and V rows are loaded before this one is used
    float kn[MAXW], vn[MAXW];
    int tt = t0 + warp;
#pragma unroll
    for (int w = 0; w < MAXW; w++) {
        const int d = lane + 32 * w;
        kn[w] = (tt < t1 && d < hd) ? __ldcg(kb + (int64_t)tt * p.KVl + d) : 0.0f;
        vn[w] = (tt < t1 && d < hd) ? __ldcg(vb + (int64_t)tt * p.KVl + d) : 0.0f;
    }
    for (; tt < t1; tt += NCW) {
        float k[MAXW], v[MAXW];
#pragma unroll
        for (int w = 0; w < MAXW; w++) k[w] = kn[w], v[w] = vn[w];
        const int tn = tt + NCW;
#pragma unroll
        for (int w = 0; w < MAXW; w++) {
            const int d = lane + 32 * w;
            kn[w] = (tn < t1 && d < hd) ? __ldcg(kb + (int64_t)tn * p.KVl + d) : 0.0f;
            vn[w] = (tn < t1 && d < hd) ? __ldcg(vb + (int64_t)tn * p.KVl + d) : 0.0f;
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
    // merge the warps: tree over shared memory (the activation area is free during attention)
    float *scr = (float *)(sm + p.off_xq);
    for (int n = NCW; n > 1;) {
        const int h = (n + 1) / 2;  // warps [h, n) hand their state to warps [0, n - h)
        if (warp >= h && warp < n) {
#pragma unroll
            for (int g = 0; g < GMAX; g++) {
                if (g < G) {
                    float *dst = scr + ((warp - h) * GMAX + g) * stride;
                    if (lane == 0) dst[0] = m[g], dst[1] = l[g];
#pragma unroll
                    for (int w = 0; w < MAXW; w++)
                        if (lane + 32 * w < hd) dst[2 + lane + 32 * w] = o[g][w];
                }
            }
        }
        named_sync(kBarConsumers, NCT);
        if (warp < n - h) {
#pragma unroll
            for (int g = 0; g < GMAX; g++) {
                if (g < G) {
                    const float *src = scr + (warp * GMAX + g) * stride;
                    const float m2 = src[0], l2 = src[1], M = fmaxf(m[g], m2);
                    const float c1 = l[g] > 0.0f ? expf(m[g] - M) : 0.0f, c2 = l2 > 0.0f ? expf(m2 - M) : 0.0f;
                    l[g] = l[g] * c1 + l2 * c2;
#pragma unroll
                    for (int w = 0; w < MAXW; w++)
                        if (lane + 32 * w < hd) o[g][w] = o[g][w] * c1 + src[2 + lane + 32 * w] * c2;
                    m[g] = M;
                }
            }
        }
        named_sync(kBarConsumers, NCT);
        n = h;
    }
    if (!active || warp != 0) return;
    if (nseg == 1) {
#pragma unroll
        for (int g = 0; g < GMAX; g++)
            if (g < G)
#pragma unroll
                for (int w = 0; w < MAXW; w++)
                    if (lane + 32 * w < hd) __stcg(p.xb + (hq + g) * hd + lane + 32 * w, o[g][w] / l[g]);
        return;
    }
    // segment partial -> global; the last segment of this unit merges them (src/model.c:141-153)
    float *part = p.apart + ((int64_t)unit * p.maxseg + seg) * GMAX * stride;
#pragma unroll
    for (int g = 0; g < GMAX; g++) {
        if (g < G) {
            if (lane == 0) __stcg(part + g * stride, m[g]), __stcg(part + g * stride + 1, l[g]);
#pragma unroll
            for (int w = 0; w < MAXW; w++)
                if (lane + 32 * w < hd) __stcg(part + g * stride + 2 + lane + 32 * w, o[g][w]);
        }
    }
    __threadfence();
    int tk = 0;
    if (lane == 0) tk = atomicAdd(p.acnt + unit, 1);
    tk = __shfl_sync(0xffffffffu, tk, 0);
    if (tk != nseg - 1) return;
    __threadfence();
    const float *base = p.apart + (int64_t)unit * p.maxseg * GMAX * stride;
    for (int g = 0; g < G; g++) {
        float M = -INFINITY;
        for (int sg = 0; sg < nseg; sg++) M = fmaxf(M, __ldcg(base + (sg * GMAX + g) * stride));
#pragma unroll
        for (int w = 0; w < MAXW; w++) {
            const int d = lane + 32 * w;
            if (d >= hd) continue;
            float num = 0.0f, den = 0.0f;
            for (int sg = 0; sg < nseg; sg++) {
                const float *src = base + (sg * GMAX + g) * stride;
                const float ls = __ldcg(src + 1);
                const float c = ls > 0.0f ? expf(__ldcg(src) - M) : 0.0f;
                den = fmaf(c, ls, den);
                num = fmaf(c, __ldcg(src + 2 + d), num);
            }
            __stcg(p.xb + (hq + g) * hd + d, num / den);
        }
    }
    if (lane == 0) atomicExch(p.acnt + unit, 0);
}

// ---------------------------------------------------------------- greedy argmax over the logits
__device__ void logits_argmax(const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, unsigned long long best) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long *keys = (unsigned long long *)(sm + p.off_red + kRedKeys);
#pragma unroll
    for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (lane == 0) keys[warp] = best;
    named_sync(kBarConsumers, NCT);
    if (threadIdx.x == 0) {
        unsigned long long k = 0;
        for (int w = 0; w < NCW; w++) k = max(k, keys[w]);
        if (k) atomicMax(p.amax_key, k);
        __threadfence();
        if (atomicAdd(p.amax_ctr, 1) == (int)gridDim.x - 1) {
            __threadfence();
            const unsigned long long gmax = atomicExch(p.amax_key, 0ull);
            int bi = argmax_index(gmax);
            const float x0 = __ldcg(ph.out);
            if (x0 != x0) bi = 0;  // a NaN in slot 0 is never replaced by the reference (src/sampler.c:27-32)
            advance_state(bi, p.state, p.forced, p.gen, p.gen_cap);
            *p.amax_ctr = 0;
            atomicExch(p.gbar, 0u);  // every CTA has passed the step's last grid barrier
        }
    }
}

__global__ void __launch_bounds__(NT, 1) decode_step_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *full = (uint64_t *)(sm + p.off_bars), *empty = full + p.nslots;
    const int t = threadIdx.x, warp = t >> 5;
    if (t == 0) {
        for (int s = 0; s < p.nslots; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    // every CTA reads the same state: an out-of-range position or token ends all of them before any
    // barrier or copy (the host validates what it passes in; this guards steps that continue from the
    // device's own position)
    const int token = __ldcg(p.state), pos = __ldcg(p.state + 1);
    if (pos < 0 || pos >= p.gen_cap || token < 0 || token >= p.vocab) {
        if (t == 0 && blockIdx.x == 0) raise_error(p.err, kErrBadState);
        return;
    }
    if (warp == NCW) {  // producer warp: weights only, never waits on the consumers' barriers
        if ((t & 31) == 0) producer(p, sm, full, empty);
        return;
    }
    unsigned gk = 0;
    bool dead = false;
    unsigned long long best = 0;
    for (int i = 0; i < p.nph; i++) {
        const DecodePhase &ph = p.ph[i];
        if (i > 0 && !grid_sync(p, sm, (unsigned)i * gridDim.x, dead)) dead = true;
        if (ph.kind == PH_ATTN) {
            attention(p, ph, sm, pos);
            continue;
        }
        prologue(p, ph, sm, token);
        const bool two = ph.urows == 2;
        if (ph.dtype == QMC_Q8_0) {
            if (two) run_matvec<QMC_Q8_0, true>(p, ph, sm, full, empty, gk, dead, pos, best);
            else run_matvec<QMC_Q8_0, false>(p, ph, sm, full, empty, gk, dead, pos, best);
        } else {
            if (two) run_matvec<QMC_Q4_0, true>(p, ph, sm, full, empty, gk, dead, pos, best);
            else run_matvec<QMC_Q4_0, false>(p, ph, sm, full, empty, gk, dead, pos, best);
        }
        if (ph.kind == PH_OUT) logits_argmax(p, ph, sm, best);
    }
}

__global__ void repack_split_kernel(int dtype, const uint8_t *__restrict__ aos, int64_t rows, int64_t K,
                                    uint8_t *__restrict__ dst, int64_t stride) {
    const int64_t nb = nblocks(K), sb = split_scale_bytes(K);
    const int BS = dtype == QMC_Q8_0 ? kQ8Bytes : kQ4Bytes, QB = BS - 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * nb; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / nb, b = i % nb;
        const uint8_t *s = aos + (r * nb + b) * BS;
        uint8_t *d = dst + r * stride;
        d[2 * b] = s[0];
        d[2 * b + 1] = s[1];
        for (int k = 0; k < QB; k++) d[sb + b * QB + k] = s[2 + k];
        if (b == nb - 1)
            for (int64_t z = 2 * nb; z < sb; z++) d[z] = 0;
    }
}

}  // namespace

int launch_repack_split(int dtype, const void *aos, int64_t rows, int64_t K, void *dst, int64_t dst_stride,
                        cudaStream_t s) {
    if (dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "repack: dtype %d is not quantized", dtype);
    if (rows <= 0) return QMC_OK;
    const int64_t work = rows * nblocks(K);
    const int grid = (int)std::min<int64_t>((work + 255) / 256, 65536);
    repack_split_kernel<<<grid, 256, 0, s>>>(dtype, (const uint8_t *)aos, rows, K, (uint8_t *)dst, dst_stride);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

bool plan_decode(int64_t max_unit_bytes, int nb_max, int hd, int group, size_t smem_optin, DecodePlan *out) {
    if (hd > 32 * MAXW) return false;
    auto r128 = [](int64_t b) { return (b + 127) / 128 * 128; };
    const int64_t act = r128((int64_t)nb_max * 32) + r128((int64_t)nb_max * 8);
    const int64_t tree = r128((int64_t)(NCW / 2) * GMAX * (hd + 2) * 4);  // [warps handing over][GMAX][hd + 2]
    (void)group;
    const int64_t scratch = std::max(act, tree);
    const int64_t fixed = 256 + scratch + kRedBytes;
    const int64_t avail = (int64_t)smem_optin - fixed;
    for (int ns : {5 * NG, 4 * NG, 3 * NG, 2 * NG, NG}) {
        const int64_t slot = (avail / ns) / 128 * 128;
        if (slot < max_unit_bytes) continue;
        DecodePlan d;
        d.nslots = ns;
        d.slot_bytes = (int)slot;
        d.off_bars = (int)(ns * slot);
        d.off_xq = d.off_bars + 256;
        d.off_xds = d.off_xq + (int)r128((int64_t)nb_max * 32);
        d.off_red = d.off_xq + (int)scratch;
        d.smem = (size_t)d.off_red + kRedBytes;
        *out = d;
        return true;
    }
    return false;
}

int launch_decode(const DecodeParams &p, const DecodePlan &plan, int grid, cudaStream_t s) {
    DevCtx *c = ctx();
    if (!c) return QMC_ECUDA;
    static bool attr_done[64];
    if (!attr_done[c->device]) {
        QMC_CUDA(cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)c->max_smem_optin));
        attr_done[c->device] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (the grid barriers need it)
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = s;
    QMC_CUDA(cudaLaunchKernelEx(&cfg, decode_step_kernel, p));
    return QMC_OK;
}

}  // namespace qmc
