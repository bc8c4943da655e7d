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
// CTA walk the segment's positions with an online softmax per query head and merge in shared memory;
// each segment's (max, sum, acc) partial goes to global memory and the wo phase's prologue merges the
// segments of a head while it quantizes the attention output (no extra barrier or ticket).
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
constexpr int kAttnChunk = 4;       // positions per warp whose K/V rows are loaded together
constexpr int kPartHead = kDecodePartHead;  // partial: (max, sum, 2 pad, acc[hd]), acc 16-byte aligned
constexpr int kFastSegs = 4;        // segment partials the wo prologue merges with all loads in flight
// named barriers: 0 = __syncthreads, 1..NG = the groups, kBarConsumers = all consumer warps
constexpr int kBarConsumers = NG + 1;
// shared scratch at off_red: prologue partial sums, argmax keys, grid-barrier flag
constexpr int kRedDred = 0, kRedKeys = 128;
constexpr int kRedFlag = kRedKeys + NCW * 8, kRedDesc = kRedFlag + 128;
constexpr int kRedBytes = kRedDesc + 2 * (int)sizeof(DecodePhase);  // + this and the next phase's descriptor
static_assert(sizeof(DecodePhase) % 16 == 0, "descriptors are copied in 16-byte chunks");

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
// Thread 0 arrives with a release reduction after a CTA barrier (so the CTA's epilogue stores are ordered
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

// ---------------------------------------------------------------- phase descriptors in shared memory
// The consumers read the current phase's descriptor from shared memory: the next one is copied there
// asynchronously (cp.async) while the current phase runs, so a phase start costs no global round trip.
__device__ __forceinline__ void desc_prefetch(const DecodePhase *src, DecodePhase *dst) {
    const int t = threadIdx.x;
    if (t < (int)(sizeof(DecodePhase) / 16))
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32((uint8_t *)dst + 16 * t)),
                     "l"((const uint8_t *)src + 16 * t)
                     : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void desc_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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
// number of position segments the attention phase splits each head into at position pos
__device__ __forceinline__ int attn_segments(const DecodeParams &p, int pos) {
    return max(1, min(p.maxseg, (pos + kMinAttnPos) / kMinAttnPos));
}

// segment partial (max, sum, 2 pad, acc[hd]) of query head hq
__device__ __forceinline__ const float *attn_part(const DecodeParams &p, int hq, int seg) {
    const int kvh = hq / p.group, r = hq % p.group, unit = kvh * p.gsplit + r / GMAX, g = r % GMAX;
    return p.apart + (((int64_t)unit * p.maxseg + seg) * GMAX + g) * (p.hd + kPartHead);
}

// 16 consecutive elements of the attention output, merged from the head's segment partials
// (src/model.c:141-153): out = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s, M the largest m_s
__device__ void attn_out16(const DecodeParams &p, int64_t e0, int K, int nseg, float (&v)[16]) {
    const int hd = p.hd;
    if ((hd & 15) == 0 && e0 + 16 <= K && nseg <= kFastSegs) {  // one head, few segments: loads at once
        const int hq = (int)(e0 / hd), d0 = (int)(e0 % hd);
        const float *head = attn_part(p, hq, 0), *src = head + kPartHead + d0;  // segment 0: (max, sum), acc
        const int64_t sstride = (int64_t)GMAX * (hd + kPartHead);
        float2 ml[kFastSegs];
        float4 o[kFastSegs][4];
#pragma unroll
        for (int sg = 0; sg < kFastSegs; sg++) {
            const bool ok = sg < nseg;
            ml[sg] = ok ? __ldcg((const float2 *)(head + sg * sstride)) : make_float2(-INFINITY, 0.0f);
#pragma unroll
            for (int i = 0; i < 4; i++)
                o[sg][i] = ok ? __ldcg((const float4 *)(src + sg * sstride) + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        float M = -INFINITY;
#pragma unroll
        for (int sg = 0; sg < kFastSegs; sg++) M = ml[sg].y > 0.0f ? fmaxf(M, ml[sg].x) : M;
        float den = 0.0f, num[16];
#pragma unroll
        for (int i = 0; i < 16; i++) num[i] = 0.0f;
#pragma unroll
        for (int sg = 0; sg < kFastSegs; sg++) {
            const float c = ml[sg].y > 0.0f ? expf(ml[sg].x - M) : 0.0f;
            den = fmaf(c, ml[sg].y, den);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                num[4 * i] = fmaf(c, o[sg][i].x, num[4 * i]);
                num[4 * i + 1] = fmaf(c, o[sg][i].y, num[4 * i + 1]);
                num[4 * i + 2] = fmaf(c, o[sg][i].z, num[4 * i + 2]);
                num[4 * i + 3] = fmaf(c, o[sg][i].w, num[4 * i + 3]);
            }
        }
        const float rden = 1.0f / den;
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = num[i] * rden;
        return;
    }
    for (int i = 0; i < 16; i++) {  // generic: element by element
        const int64_t e = e0 + i;
        if (e >= K) {
            v[i] = 0.0f;
            continue;
        }
        const int hq = (int)(e / hd), d = (int)(e % hd);
        float M = -INFINITY, den = 0.0f, num = 0.0f;
        for (int sg = 0; sg < nseg; sg++) {
            const float *src = attn_part(p, hq, sg);
            const float m = __ldcg(src), l = __ldcg(src + 1), o = __ldcg(src + kPartHead + d);
            if (l > 0.0f) {
                const float Mn = fmaxf(M, m);
                const float c0 = den > 0.0f ? expf(M - Mn) : 0.0f, c1 = expf(m - Mn);
                den = fmaf(den, c0, c1 * l);
                num = fmaf(num, c0, c1 * o);
                M = Mn;
            }
        }
        v[i] = num / den;
    }
}

// 16 elements e0..e0+15 of the phase input: the token's embedding row (dequantized as src/quant.c:65-94,
// one rounding) for the first phase, the merged attention output for wo, else the input vector; zero
// past K
__device__ __forceinline__ void fetch16(const DecodeParams &p, const DecodePhase &ph, const uint8_t *erow, int64_t e0,
                                        int nseg, float (&v)[16]) {
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
    if (ph.kind == PH_WO) {
        attn_out16(p, e0, K, nseg, v);
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

// x + kRound - kRound rounds |x| < 2^22 to the nearest integer, ties to even, in one round-to-nearest
// add; for |x| <= 127 the integer is also the low bits of x + kRound.  Used instead of rintf / floorf /
// float->int conversions, which issue at a fraction of the FMA pipe's rate.
constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
constexpr int kRoundBits = 0x4B400000;

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
        const float n = __fsub_rn(__fadd_rn(r[i], kRound), kRound);  // nearest integer
        near |= fabsf(__fsub_rn(r[i], n)) > 0.4999f;
    }
    if (near) {
#pragma unroll
        for (int i = 0; i < 16; i++) r[i] = __fdiv_rn(v[i], sc);
    }
}

// Q8_0 of block b held by a lane pair (part j: elements 16j..16j+15), bit-exact with src/quant.c:33-53:
// amax ignores NaN, IEEE division for the scale, fp16 RNE scale, then rint(v / scale) clamped to +-127
// (NaN -> 0, as the float->int conversion gives).  All lanes call it (pair shuffles); `active` lanes
// store.  Q4_0 weights take the block's even elements in bytes 0-15 and odd elements in bytes 16-31.
__device__ __forceinline__ void quant_block(bool q4, uint8_t *xq, int2 *xds, int b, int j, bool active,
                                            const float (&v)[16]) {
    uint32_t m[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {  // |v| bits order like floats; NaN -> 0
        const float a0 = fabsf(v[2 * i]), a1 = fabsf(v[2 * i + 1]);
        m[i] = max((a0 == a0) ? __float_as_uint(a0) : 0u, (a1 == a1) ? __float_as_uint(a1) : 0u);
    }
#pragma unroll
    for (int w = 4; w; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; i++) m[i] = max(m[i], m[i + w]);
    const uint32_t ab = max(m[0], __shfl_xor_sync(0xffffffffu, m[0], 1));
    const float sc = h2f(f2h(__fdiv_rn(__uint_as_float(ab), 127.0f)));
    float qf[16];
    quotients16(v, sc, qf);
    int q[16];
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const float c = fminf(fmaxf(qf[i], -127.0f), 127.0f);
        q[i] = (sc != 0.0f && qf[i] == qf[i]) ? __float_as_int(__fadd_rn(c, kRound)) - kRoundBits : 0;
    }
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 16; i += 4) sum += (q[i] + q[i + 1]) + (q[i + 2] + q[i + 3]);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    if (!active) return;
    auto pk = [&](int a, int b2, int c, int d) {
        return (uint32_t)(q[a] & 0xff) | ((uint32_t)(q[b2] & 0xff) << 8) | ((uint32_t)(q[c] & 0xff) << 16) |
               ((uint32_t)q[d] << 24);
    };
    uint8_t *blk = xq + (int64_t)b * 32;
    const int sw = xswz(b);
    if (!q4) {
        *(uint4 *)(blk + ((16 * j) ^ sw)) = make_uint4(pk(0, 1, 2, 3), pk(4, 5, 6, 7), pk(8, 9, 10, 11), pk(12, 13, 14, 15));
    } else {
        *(uint2 *)(blk + ((8 * j) ^ sw)) = make_uint2(pk(0, 2, 4, 6), pk(8, 10, 12, 14));
        *(uint2 *)(blk + ((16 + 8 * j) ^ sw)) = make_uint2(pk(1, 3, 5, 7), pk(9, 11, 13, 15));
    }
    if (j == 0) xds[b] = make_int2(__float_as_int(sc), sum);
}

// The phase input (optionally x * inv * w, inv = (float)(1 / sqrt(sum_double(x^2)/n + eps)),
// src/ops.c:93-98) quantized into shared memory by the consumer threads, two per block; the first
// phase's CTA 0 also stores the embedding into x.  The first round's x and w stay in registers.
__device__ void prologue(const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, int token, int pos) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, qd = t >> 1, j = t & 1;
    uint8_t *xq = sm + p.off_xq;
    int2 *xds = (int2 *)(sm + p.off_xds);
    const bool q4 = ph.dtype == QMC_Q4_0;
    const int K = ph.K, rounds = (ph.nb + QPR - 1) / QPR;
    const uint8_t *erow = ph.embed ? p.tok + (int64_t)token * row_bytes(p.dt_tok, K) : nullptr;
    const bool keep_x = ph.embed && blockIdx.x == 0;
    const float *nw = ph.norm_w;
    const int nseg = attn_segments(p, pos);
    const int64_t e00 = (int64_t)qd * 32 + 16 * j;
    float v0[16], w0[16];
    fetch16(p, ph, erow, e00, nseg, v0);
    if (nw) fetch16_w(nw, e00, K, w0);
    float inv = 1.0f;
    if (nw) {
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < 16; i++) ss = fma((double)v0[i], (double)v0[i], ss);
        for (int r = 1; r < rounds; r++) {
            float v[16];
            fetch16(p, ph, erow, (int64_t)(r * QPR + qd) * 32 + 16 * j, nseg, v);
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
        if (r * QPR + warp * 16 >= ph.nb) break;  // this warp's blocks (and later rounds') are past the row
        const int b = r * QPR + qd;
        const int64_t e0 = (int64_t)b * 32 + 16 * j;
        if (r > 0) {
#pragma unroll
            for (int i = 0; i < 16; i++) v0[i] = v1[i], w0[i] = w1[i];
        }
        if (r + 1 < rounds) {  // next round's loads in flight while this one is quantized
            const int64_t e1 = e0 + (int64_t)QPR * 32;
            fetch16(p, ph, erow, e1, nseg, v1);
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

// operand an epilogue lane needs besides the row sums, loaded before the unit's dots so its latency is
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
// row dots and warp sums, and one arrival on each of its group's stages.  Epilogues are deferred: lane
// k keeps the k-th pending unit's sums, and every 32 units (and at the end of the phase) all lanes run
// their epilogues at once, their operand loads (RoPE pairs, residual x) in flight together.
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
    float pa0 = 0.0f, pa1 = 0.0f;  // this lane's pending unit: sums and index
    int64_t punit = 0;
    int npend = 0;  // pending units in the warp (warp-uniform)
    auto flush = [&]() {
        if (lane < npend) {
            const float2 opnd = epilogue_operand(p, ph, punit, pos);
            epilogue(p, ph, punit, pa0, pa1, opnd, pos, best);
        }
        npend = 0;
    };
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
                float a0, a1;
                unit_dot<DT, TWO>(stage + (int64_t)i * UR * rbytes, rbytes, sbytes, nb, xq, xds, xw, xd, xs, a0, a1);
                if (lane == npend) pa0 = a0, pa1 = a1, punit = ua + i;
                if (++npend == 32) flush();
            }
        }
        uoff += n;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!dead) flush();
    gk += (unsigned)nst;
}

// ---------------------------------------------------------------- attention phase
__device__ void attention(const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, int pos) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int npos = pos + 1, nunit = p.nkv * p.gsplit;
    const int nseg = attn_segments(p, pos);
    const bool active = (int)blockIdx.x < nunit * nseg;
    const int unit = active ? (int)blockIdx.x / nseg : 0, seg = active ? (int)blockIdx.x % nseg : 0;
    const int kvh = unit / p.gsplit, gs = unit % p.gsplit, h0 = gs * GMAX, G = min(GMAX, p.group - h0);
    const int hd = p.hd, stride = hd + 2, ps = hd + kPartHead;
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
    // positions t0 + warp, + 12, ...: the K and V rows of up to kAttnChunk of them are loaded at once
    for (int tb = t0 + warp; tb < t1; tb += kAttnChunk * NCW) {
        float k[kAttnChunk][MAXW], v[kAttnChunk][MAXW];
#pragma unroll
        for (int c = 0; c < kAttnChunk; c++) {
            const int tt = tb + c * NCW;
#pragma unroll
            for (int w = 0; w < MAXW; w++) {
                const int d = lane + 32 * w;
                k[c][w] = (tt < t1 && d < hd) ? __ldcg(kb + (int64_t)tt * p.KVl + d) : 0.0f;
                v[c][w] = (tt < t1 && d < hd) ? __ldcg(vb + (int64_t)tt * p.KVl + d) : 0.0f;
            }
        }
#pragma unroll
        for (int c = 0; c < kAttnChunk; c++) {
            if (tb + c * NCW >= t1) break;
#pragma unroll
            for (int g = 0; g < GMAX; g++) {
                if (g < G) {
                    float sc = 0.0f;
#pragma unroll
                    for (int w = 0; w < MAXW; w++) sc = fmaf(k[c][w], q[g][w], sc);
                    sc = warp_sum(sc) * p.scale;
                    const float mn = fmaxf(m[g], sc);
                    const float corr = expf(m[g] - mn), e = expf(sc - mn);
                    l[g] = l[g] * corr + e;
#pragma unroll
                    for (int w = 0; w < MAXW; w++) o[g][w] = o[g][w] * corr + e * v[c][w];
                    m[g] = mn;
                }
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
    // this segment's (max, sum, acc) per query head -> global; the wo phase's prologue merges the
    // segments of each head while it quantizes the attention output (src/model.c:141-153)
    float *part = p.apart + ((int64_t)unit * p.maxseg + seg) * GMAX * ps;
#pragma unroll
    for (int g = 0; g < GMAX; g++) {
        if (g < G) {
            float *dst = part + g * ps;
            if (lane == 0) __stcg(dst, m[g]), __stcg(dst + 1, l[g]);
#pragma unroll
            for (int w = 0; w < MAXW; w++)
                if (lane + 32 * w < hd) __stcg(dst + kPartHead + lane + 32 * w, o[g][w]);
        }
    }
}

// ---------------------------------------------------------------- greedy argmax over the logits
__device__ void logits_argmax(const DecodeParams &p, uint8_t *sm, unsigned long long best) {
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
            const float x0 = __ldcg(p.logits);
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
    DecodePhase *dsm = (DecodePhase *)(sm + p.off_red + kRedDesc);
    desc_prefetch(p.ph, dsm);
    desc_wait();
    named_sync(kBarConsumers, NCT);
    for (int i = 0; i < p.nph; i++) {
        if (i > 0) {
            desc_wait();  // phase i's descriptor (copied during phase i - 1); the barrier publishes it
            if (!grid_sync(p, sm, (unsigned)i * gridDim.x, dead)) dead = true;
        }
        const DecodePhase &ph = dsm[i & 1];
        if (i + 1 < p.nph) desc_prefetch(p.ph + i + 1, dsm + ((i + 1) & 1));
        if (ph.kind == PH_ATTN) {
            attention(p, ph, sm, pos);
            continue;
        }
        prologue(p, ph, sm, token, pos);
        const bool two = ph.urows == 2;
        if (ph.dtype == QMC_Q8_0) {
            if (two) run_matvec<QMC_Q8_0, true>(p, ph, sm, full, empty, gk, dead, pos, best);
            else run_matvec<QMC_Q8_0, false>(p, ph, sm, full, empty, gk, dead, pos, best);
        } else {
            if (two) run_matvec<QMC_Q4_0, true>(p, ph, sm, full, empty, gk, dead, pos, best);
            else run_matvec<QMC_Q4_0, false>(p, ph, sm, full, empty, gk, dead, pos, best);
        }
        if (ph.kind == PH_OUT) logits_argmax(p, sm, best);
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
