// Persistent decode step: one cooperative launch of one CTA per SM runs the whole token step of
// src/model.c:158-191 -- embedding, L x {rmsnorm + QKV matvec + RoPE + KV store, attention, wo matvec +
// residual, rmsnorm + w1/w3 matvecs + SwiGLU, w2 matvec + residual}, final rmsnorm + output matvec +
// greedy argmax -- as a list of phases separated by grid barriers.
//
// Why one kernel: batch-1 decode streams every weight byte once and is bound by HBM, but a bulk copy
// takes ~3 us to land under load, so an SM needs ~130 KB in flight to draw its share of the bandwidth.
// Separate kernels per matvec cannot keep that: each boundary drains the pipeline, and co-residency
// with the next kernel caps the ring at half the shared memory.  Here one producer warp per CTA walks
// the weight stages of ALL phases in order through a ring of 33 (or 22, 11) slots in ~215 KB of shared
// memory and never waits on a grid barrier: while the consumers sit in a barrier, an activation
// prologue or the attention phase, the producer is already streaming the next matrices.
//
// Consumers: 11 warps, each its own stage group; global stage g goes to warp g % 11 and slot g % nslots
// (three slots per warp when the largest unit fits a third of the ring: a Llama-7B w2 row, 6.2 KB, does)
// (nslots is a multiple of 11, so a slot always serves one warp and the parity waits stay one phase
// apart).  A warp works alone on the units (rows, or the RoPE / SwiGLU row pairs) of its stages: lane l
// takes blocks l, l+32, ... of the row (the first four held in registers as Q8_0 activations for the
// whole phase), a warp sum forms the row dot and the epilogues (RoPE + K/V store, residual add, SwiGLU,
// logits + argmax key) run 32 units at a time across the lanes.  No CTA barrier runs inside the stream
// loop.  12 warps in all leave each thread 168 registers (at most 3 warps per SM sub-partition); with 13
// the cap is 128 and the kernel spills to local memory, whose reloads miss the small L1 left beside the
// ring and cost an L2 round trip each.
//
// Weights are in the split-row layout (decode.cuh): aligned 16-byte shared loads per block, no realignment.
// Per block the arithmetic is the reference's (src/kernels_scalar.c:12-34): integer block dot (dp4a; Q4_0
// as low nibbles x 1 + masked high nibbles x 16 against even/odd activations, minus 8 * sum x), then
// s += (float)acc * (dW * dX).  Activations are quantized per phase by every CTA (bit-exact Q8_0,
// src/quant.c:33-53) after the fused rmsnorm (src/ops.c:93-98).
//
// Attention (src/model.c:132-156): (KV head, position segment) units over the CTAs; the 11 warps of a
// CTA walk the segment's positions with an online softmax per query head and merge in shared memory;
// each segment's (max, sum, acc) partial goes to global memory and the wo phase's prologue merges the
// segments of a head while it quantizes the attention output (no extra barrier or ticket).
//
// Every wait is bounded (mbarrier waits, the grid barrier): on expiry a thread raises the error word and
// continues without waiting, so the launch always ends; the host then reports QMC_ETIMEOUT.
#include <algorithm>
#include <type_traits>

#include "actquant.cuh"
#include "decode.cuh"

namespace qmc {
namespace {

constexpr int NCW = kDecodeWarps;   // consumer warps (12 warps in all: at most 3 per SM sub-partition, so
                                    // each thread may hold 168 registers; with 13 warps the cap is 128 and
                                    // the whole-step kernel spills)
constexpr int NG = NCW, GW = 1;     // stage groups x warps per group: each warp consumes its own stages
constexpr int NT = (NCW + 1) * 32;  // + the producer warp
constexpr int NCT = NCW * 32;       // consumer threads
constexpr int QPR = NCT / 2;        // activation blocks per prologue round (2 threads per block)
constexpr int XW = 4;               // activation blocks per lane kept in registers (the rest from shared)
constexpr int GMAX = kDecodeHeadsPerUnit;  // query heads per attention unit (a larger GQA group spans units)
constexpr int MAXW = 4;             // head_dim / 32 (head_dim <= 128)
constexpr int kMinAttnPos = 32;     // an attention segment spans at least this many positions
constexpr int kAttnChunk = 4;       // positions per warp whose K/V rows are loaded together
constexpr int kPrefetchPos = 64;    // positions of a segment prefetched into L2 before the barrier
constexpr int kPartHead = kDecodePartHead;  // partial: (max, sum, 2 pad, acc[hd]), acc 16-byte aligned
constexpr int kFastSegs = kDecodeFastSegs;  // segment partials the wo prologue merges with all loads in flight
// named barriers: 0 = __syncthreads, kBarConsumers = all consumer warps (the producer warp never waits)
constexpr int kBarConsumers = 1;
// shared scratch at off_red: prologue partial sums, argmax keys, grid-barrier flag
constexpr int kRedDred = 0, kRedKeys = 128;
constexpr int kRedFlag = kRedKeys + (NCW * 8 + 15) / 16 * 16, kRedDesc = kRedFlag + 128;
constexpr int kRedBytes = kRedDesc + 2 * (int)sizeof(DecodePhase);  // + this and the next phase's descriptor
static_assert(sizeof(DecodePhase) % 16 == 0, "descriptors are copied in 16-byte chunks");
static_assert(kRedDesc % 16 == 0 && NCW * 8 <= kRedKeys, "shared scratch layout");
static_assert(NG <= 31, "one producer lane per stage group");

// ---------------------------------------------------------------- optional timing stamps
// Compiled in only with -DQMC_DECODE_TRACE (a profiling build of the library; the default build has no
// trace code): per phase and CTA, kTrSlots 64-bit words of globaltimer stamps (ns) and counters, written
// to the buffer given to qmc_decode_trace_set.
#ifdef QMC_DECODE_TRACE
__constant__ unsigned long long *g_dtrace;  // constant bank: read without a global round trip
#endif
enum : int {
    kTrStart = 0,  // consumers pass the phase's grid barrier (thread 0)
    kTrProEnd,     // activation prologue (or attention) done
    kTrMvEnd,      // last warp leaves the matvec (max over warps)
    kTrArrive,     // CTA arrives at the barrier that ends the phase
    kTrProdFirst,  // producer issues the phase's first stage
    kTrProdLast,   // ... and its last
    kTrProdWait,   // producer time waiting for free slots in the phase (SM cycles)
    kTrFullWait,   // consumer warps' time waiting for full stages (cycles, summed over warps)
    kTrUnits,      // units the CTA's warps computed
    kTrFlush,      // consumer warps' time in epilogue flushes (cycles, summed)
    kTrDot,        // consumer warps' time in row dots (cycles, summed)
    kTrProLoad,    // thread 0's first prologue loads (or attention's q) have landed
    kTrAttnKV,     // attention: thread 0's first K/V chunk has landed
    kTrAttnLoop,   // attention: warp 0 left its position loop
    kTrSlots = 16
};
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// a stamp taken only once x is computed (x is an input of the asm)
__device__ __forceinline__ unsigned long long gtime_after(float x) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t) : "f"(x));
    return t;
}
__device__ __forceinline__ unsigned long long *trace_slot(int ph, int k) {
#ifdef QMC_DECODE_TRACE
    return g_dtrace ? g_dtrace + ((size_t)ph * gridDim.x + blockIdx.x) * kTrSlots + k : nullptr;
#else
    (void)ph, (void)k;
    return nullptr;
#endif
}
// CTA 0 also records every stage g < kTrStages: [g][0] issued, [1] consumer saw it full, [2] released
#ifdef QMC_DECODE_TRACE
constexpr int kTrStages = 4096;
#endif
__device__ __forceinline__ unsigned long long *trace_stage(const DecodeParams &p, unsigned g, int k) {
#ifdef QMC_DECODE_TRACE
    return (g_dtrace && blockIdx.x == 0 && g < (unsigned)kTrStages)
               ? g_dtrace + (size_t)p.nph * gridDim.x * kTrSlots + (size_t)g * 4 + k
               : nullptr;
#else
    (void)p, (void)g, (void)k;
    return nullptr;
#endif
}
// the value expression is evaluated only in a trace build with a buffer set
#define DTRACE_SET(ph, k, v) do { if (unsigned long long *q_ = trace_slot(ph, k)) *q_ = (v); } while (0)
#define DTRACE_ADD(ph, k, v) do { if (unsigned long long *q_ = trace_slot(ph, k)) atomicAdd(q_, (unsigned long long)(v)); } while (0)
#define DTRACE_MAX(ph, k, v) do { if (unsigned long long *q_ = trace_slot(ph, k)) atomicMax(q_, (unsigned long long)(v)); } while (0)

__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// 32-bit arithmetic where blockIdx.x * units fits (a 64-bit division is a long software routine on the
// critical path of every phase)
__device__ __forceinline__ void split_units(int64_t units, int64_t &u0, int64_t &u1) {
    if (units <= 0xffffff) {
        const unsigned n = (unsigned)units, b = blockIdx.x;
        u0 = (int64_t)(b * n / gridDim.x);
        u1 = (int64_t)((b + 1) * n / gridDim.x);
    } else {
        u0 = (int64_t)blockIdx.x * units / gridDim.x;
        u1 = (int64_t)(blockIdx.x + 1) * units / gridDim.x;
    }
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
        DTRACE_SET((int)(target / gridDim.x) - 1, kTrArrive, gtime());
        red_release_add(p.gbar, 1u);
        if (!dead && !counter_wait(p.gbar, target)) {
            raise_error(p.err, kErrFlagTimeout);
            ok = 0;
        }
        *flag = ok;
    }
    named_sync(kBarConsumers, NCT);
    return *flag != 0;
}

// ---------------------------------------------------------------- cross-rank exchange (tensor parallelism)
// The wo / w2 row sums of a rank are partials over its column shard (src/model.c:178-186 split across the
// ranks).  Each goes to every rank as one 64-bit word (float bits, tag) with a relaxed system-scope store:
// single-copy atomic, so a reader that sees the tag sees the value, and no fence is needed -- a
// system-scope release costs 3-6 us per point on B200 over NVLink, the data's own tag about one NVLink
// latency.  After its own rows are done, each CTA polls the words of its rows (the same rows on every
// rank: same D, same grid), adds the ranks' partials in rank order to x -- the same bits on every rank --
// and stores x in place; the ordinary grid barrier that ends the phase then publishes x to the CTA's
// rank.  Tags never repeat: exchange e of the step with epoch ep carries ep * xph + e + 1 (0 = empty).
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_sys_add(unsigned *p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned *xch_word(const DecodeParams &p, int r, int off) {
    return (unsigned *)(p.peers.blk[r] + off);
}
__device__ __forceinline__ unsigned long long *xch_slot(const DecodeParams &p, int r, int xex) {
    return (unsigned long long *)(p.peers.blk[r] + kXchSync) + (int64_t)(xex & 1) * p.tp * p.D;
}
// this rank's partial of row `unit` into every rank's slot
__device__ __forceinline__ void xch_put(const DecodeParams &p, int xex, unsigned tag, int64_t unit, float a) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(a);
    for (int r = 0; r < p.tp; r++) st_relaxed_sys_u64(xch_slot(p, r, xex) + (int64_t)p.rank * p.D + unit, w);
}
// x += (p_0 + ... + p_{tp-1}) for this CTA's rows [u0, u1), the consumer threads one row each (bounded
// polls; on expiry the error word is raised and the row keeps what has arrived)
__device__ void xch_reduce(const DecodeParams &p, const DecodePhase &ph, unsigned tag) {
    int64_t u0, u1;
    split_units(ph.units, u0, u1);
    const unsigned long long *slot = xch_slot(p, p.rank, ph.xex);
    for (int64_t u = u0 + threadIdx.x; u < u1; u += NCT) {
        float s = 0.0f;
        for (int r = 0; r < p.tp; r++) {
            const unsigned long long *q = slot + (int64_t)r * p.D + u;
            unsigned long long w = ld_relaxed_sys_u64(q);
            if ((unsigned)(w >> 32) != tag) {
                const long long t0 = clock64();
                while ((unsigned)((w = ld_relaxed_sys_u64(q)) >> 32) != tag)
                    if (clock64() - t0 > kWaitCycles) {
                        raise_error(p.err, kErrFlagTimeout);
                        break;
                    }
            }
            s = r == 0 ? __uint_as_float((unsigned)w) : s + __uint_as_float((unsigned)w);
        }
        __stcg(ph.out + u, __ldcg(ph.out + u) + s);  // residual (src/model.c:179,186)
    }
}
__device__ __forceinline__ bool counter_wait_sys(const unsigned *ctr, unsigned target) {
    const long long t0 = clock64();
    while ((int)(ld_acquire_sys(ctr) - target) < 0)
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
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
// The producer warp walks this CTA's weight range of every matvec phase in stages of R units.  Global
// stage g belongs to consumer warp g % NG and goes to slot g % nslots; lane w < NG of the producer warp
// serves consumer warp w alone: it copies that warp's stages in order, each into its slot as soon as the
// warp released the slot's previous stage, so a slow warp never holds up another warp's refills.  The
// producer never waits on a grid barrier: while the consumers sit in a barrier, an activation prologue
// or attention, every warp's slots fill with its next stages, of the next phases too.
// byte range of stage k of the CTA's units [u0, u1) of a phase: R whole units, or (K-split) chunk
// k % C of unit u0 + k / C -- a unit's chunks are consecutive, each its rows' chunks back to back
__device__ __forceinline__ void stage_span(const DecodePhase &q, int64_t u0, int64_t u1, int k, int64_t &src,
                                           uint32_t &bytes) {
    if (q.C == 1) {
        const int64_t ua = u0 + (int64_t)k * q.R, ub = (int64_t)q.urows * q.rbytes;
        src = ua * ub;
        bytes = (uint32_t)(min((int64_t)q.R, u1 - ua) * ub);
        return;
    }
    const int64_t u = u0 + k / q.C;
    const int j = k % q.C, kbl = q.nb - (q.C - 1) * q.kb;
    const int64_t cb = chunk_row_bytes(q.dtype, q.kb), cbl = chunk_row_bytes(q.dtype, kbl);
    src = u * q.urows * ((q.C - 1) * cb + cbl) + (int64_t)q.urows * j * cb;
    bytes = (uint32_t)(q.urows * (j < q.C - 1 ? cb : cbl));
}

__device__ void producer(const DecodeParams &p, uint8_t *sm, uint64_t *full, uint64_t *empty) {
    const int w = threadIdx.x & 31;
    if (w >= NG) return;
    // cursor: phase i (a matvec phase or p.nph when done), stage k within it, G = global index of its
    // stage 0, this CTA's units [u0, u1) of it
    int i = -1, k = w;
    unsigned G = 0;
    int64_t u0 = 0, u1 = 0;
    int nst = 0;
    auto settle = [&]() {  // move the cursor onto the phase that holds stage G + k
        while (i < p.nph && (i < 0 || k >= nst)) {
            if (i >= 0) k -= nst, G += (unsigned)nst;
            while (++i < p.nph && p.ph[i].kind == PH_ATTN) {
            }
            if (i >= p.nph) break;
            const DecodePhase &q = p.ph[i];
            split_units(q.units, u0, u1);
            nst = q.C > 1 ? (int)((u1 - u0) * q.C) : (int)((u1 - u0 + q.R - 1) / q.R);
        }
    };
    settle();
    unsigned g_last = 0, nissued = 0;  // this lane's last issued stage and its count (for the drain)
    const uint64_t pol = l2_evict_first_policy();  // each weight byte is read once per step
    const long long t0 = clock64();
    while (true) {
        bool done = i >= p.nph, issued = false;
        if (!done) {
            const unsigned g = G + (unsigned)k;
            const int s = (int)(g % (unsigned)p.nslots);
            if (g < (unsigned)p.nslots || mbar_test(&empty[s], ((g / p.nslots) - 1) & 1u)) {
                const DecodePhase &q = p.ph[i];
                int64_t src;
                uint32_t bytes;
                stage_span(q, u0, u1, k, src, bytes);
                if (k == 0) DTRACE_SET(i, kTrProdFirst, gtime());
                if (k + NG >= nst) DTRACE_MAX(i, kTrProdLast, gtime());
                if (unsigned long long *q_ = trace_stage(p, g, 0)) *q_ = gtime();
                mbar_arrive_tx(&full[s], bytes);
                bulk_g2s_hint(sm + (size_t)s * p.slot_bytes, q.W + src, bytes, &full[s], pol);
                g_last = g, nissued++;
                k += NG;
                settle();
                issued = true;
            }
        }
        constexpr unsigned kLanes = (1u << NG) - 1u;  // lanes 0..NG-1 run this loop together
        if (!__any_sync(kLanes, !done)) break;
        if (!__any_sync(kLanes, issued)) {  // every lane waits on a slot: back off briefly
            __nanosleep(64);
            if (__any_sync(kLanes, clock64() - t0 > kWaitCycles)) {  // warp-uniform: all lanes leave together
                if (!done) raise_error(p.err, kErrMbarTimeout);
                break;
            }
        }
    }
    // drain: the CTA must not exit while a copy into its shared memory is in flight.  A slot is refilled
    // only after its consumer saw the previous copy land, so the copies that can still be in flight are
    // this lane's last one per slot (stages g_last, g_last - NG, ...); after a timeout nobody consumes
    // them, so wait for them here (bounded; in a normal step they landed long ago or land for the
    // consumers anyway)
    const long long td = clock64();
    const unsigned per_lane = (unsigned)(p.nslots / NG);
    for (unsigned j = 0; j < nissued && j < per_lane; j++) {
        const unsigned g = g_last - j * NG;
        if (!mbar_wait_since(&full[g % (unsigned)p.nslots], (g / p.nslots) & 1u, td)) {
            raise_error(p.err, kErrMbarTimeout);
            break;
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
        const int hq = (int)e0 / hd, d0 = (int)e0 % hd;  // e0 < K: 32-bit
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
#pragma unroll
    for (int i = 0; i < 16; i++) {  // generic: element by element (zero past K)
        const int64_t e = e0 + i;
        if (e >= K) {
            v[i] = 0.0f;
            continue;
        }
        const int hq = (int)e / hd, d = (int)e % hd;
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

// 16 elements e0..e0+15 of the token's embedding row (dequantized as src/quant.c:65-94, one rounding);
// zero past K
__device__ __forceinline__ void embed16(const DecodeParams &p, const uint8_t *erow, int64_t e0, int K,
                                        float (&v)[16]) {
    if (e0 >= K) {  // pairs past the last block (their block and its scale lie outside the row)
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = 0.0f;
        return;
    }
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
}

// 16 elements e0..e0+15 of a float vector, zero past K; CG: through L2 only (vectors other CTAs wrote
// during this step), else the default path (weights that stay fixed).  w is 16-byte aligned and its
// allocation extends past element K by at least 15 floats (every model buffer is its own cudaMalloc with
// 256 bytes of slack), e0 is a multiple of 16: four vector loads, then the tail past K masked to zero.
template <bool CG>
__device__ __forceinline__ void load16(const float *w, int64_t e0, int K, float (&v)[16]) {
    if (e0 >= K) {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = 0.0f;
        return;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 *q = (const float4 *)(w + e0) + i;
        const float4 a = CG ? __ldcg(q) : *q;
        v[4 * i] = a.x, v[4 * i + 1] = a.y, v[4 * i + 2] = a.z, v[4 * i + 3] = a.w;
    }
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = e0 + i < K ? v[i] : 0.0f;
}

// The phase input quantized into shared memory by the consumer threads, two per block: one loop over the
// rounds of QPR blocks, with one load site and one quantization site for every kind of phase, so the
// instruction footprint the SMs cycle through each layer stays small; the next round's input is loaded
// while the current one is quantized.
//  - rmsnorm phases (QKV, FFN, OUT): x * inv * w, inv = (float)(1 / sqrt(sum_double(x^2)/n + eps))
//    (src/ops.c:93-98), x the residual stream or, in the step's first phase, the token's embedding
//    (which CTA 0 also stores into x).  With one round, x and w are loaded together and x stays in
//    registers across the block sum; longer rows take a first pass for the sum;
//  - WO: the attention output, merged from the segment partials;
//  - W2: the SwiGLU output.
// Threads past the row's blocks load zeros and store nothing.
__device__ __forceinline__ void prologue_load(const DecodeParams &p, const DecodePhase &ph, const uint8_t *erow, int nseg,
                                              int64_t e0, float (&v)[16]) {
    if (erow) embed16(p, erow, e0, ph.K, v);
    else if (ph.kind == PH_WO) attn_out16(p, e0, ph.K, nseg, v);
    else load16<true>(ph.in, e0, ph.K, v);
}

__device__ void prologue(const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, int token, int pos, int phi) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, qd = t >> 1, j = t & 1;
    uint8_t *xq = sm + p.off_xq;
    int2 *xds = (int2 *)(sm + p.off_xds);
    const bool q4 = ph.dtype == QMC_Q4_0, norm = ph.norm_w != nullptr;
    const int K = ph.K, rounds = (ph.nb + QPR - 1) / QPR;
    const uint8_t *erow = ph.embed ? p.tok + (int64_t)token * row_bytes(p.dt_tok, K) : nullptr;
    const bool own_ss = norm;                    // the CTA sums the squares of its loads
    const bool two_pass = own_ss && rounds > 1;  // ... in a first pass when the row takes several rounds
    const bool keep_x = erow && blockIdx.x == 0;
    const int nseg = ph.kind == PH_WO ? attn_segments(p, pos) : 0;
    float inv = 1.0f;
    if (two_pass) {
        double ss = 0.0;
#pragma unroll 1
        for (int r = 0; r < rounds; r++) {
            float v[16];
            prologue_load(p, ph, erow, nseg, (int64_t)(r * QPR + qd) * 32 + 16 * j, v);
#pragma unroll
            for (int i = 0; i < 16; i++) ss = fma((double)v[i], (double)v[i], ss);
        }
        ss = warp_sum_d(ss);
        double *dred = (double *)(sm + p.off_red + kRedDred);
        if (lane == 0) dred[warp] = ss;
        named_sync(kBarConsumers, NCT);
        double tot = 0.0;
#pragma unroll
        for (int k = 0; k < NCW; k++) tot += dred[k];
        inv = (float)(1.0 / sqrt(tot / (double)K + (double)p.eps));
        named_sync(kBarConsumers, NCT);  // dred is free again
    }
    // w: the norm weights, or (phases without a norm) the next round's input, loaded while the current
    // round is quantized
    float v[16], w[16];
    prologue_load(p, ph, erow, nseg, (int64_t)qd * 32 + 16 * j, v);
    if (norm) load16<false>(ph.norm_w, (int64_t)qd * 32 + 16 * j, K, w);
    else if (rounds > 1) prologue_load(p, ph, erow, nseg, (int64_t)(QPR + qd) * 32 + 16 * j, w);
    if (t == 0) DTRACE_SET(phi, kTrProLoad, gtime_after(v[0] + w[0]));
#pragma unroll 1
    for (int r = 0; r < rounds; r++) {
        const int b = r * QPR + qd;
        const int64_t e0 = (int64_t)b * 32 + 16 * j;
        if (own_ss && !two_pass) {  // one round: the block sum of the registers' squares
            double ss = 0.0;
#pragma unroll
            for (int i = 0; i < 16; i++) ss = fma((double)v[i], (double)v[i], ss);
            ss = warp_sum_d(ss);
            double *dred = (double *)(sm + p.off_red + kRedDred);
            if (lane == 0) dred[warp] = ss;
            named_sync(kBarConsumers, NCT);
            float invl = 0.0f;
            if (lane == 0) {  // one lane per warp: double division and sqrt are slow
                double tot = 0.0;
#pragma unroll
                for (int k = 0; k < NCW; k++) tot += dred[k];
                invl = (float)(1.0 / sqrt(tot / (double)K + (double)p.eps));
            }
            inv = __shfl_sync(0xffffffffu, invl, 0);
        }
        if (keep_x) {
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (e0 + i < K) __stcg(p.x + e0 + i, v[i]);
        }

        if (norm) {
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = __fmul_rn(__fmul_rn(v[i], inv), w[i]);
        }
        quant_block(q4, xq, xds, b, j, b < ph.nb, v);
        if (r + 1 < rounds) {
            if (norm) {
                prologue_load(p, ph, erow, nseg, e0 + QPR * 32, v);
                load16<false>(ph.norm_w, e0 + QPR * 32, K, w);
            } else {  // round r + 1 is in w; round r + 2 goes in flight
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] = w[i];
                if (r + 2 < rounds) prologue_load(p, ph, erow, nseg, e0 + 2 * QPR * 32, w);
            }
        }
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
        if (vr < p.Dq + p.KVl) return p.rope[(int64_t)pos * (p.hd >> 1) + (((int)vr % p.hd) >> 1)];
        return make_float2(0.0f, 0.0f);
    }
    if (ph.kind == PH_WO || ph.kind == PH_W2) return make_float2(__ldcg(ph.out + unit), 0.0f);
    return make_float2(0.0f, 0.0f);
}

template <bool KV16>
__device__ __forceinline__ void epilogue(const DecodeParams &p, const DecodePhase &ph, int64_t unit, float a, float b,
                                         float2 opnd, int pos, unsigned long long &best, unsigned xtag) {
    switch (ph.kind) {
    case PH_QKV: {  // rows 2u, 2u+1: one RoPE pair of q or k, or two v values
        const int64_t vr = 2 * unit;
        float o0 = a, o1 = b;
        if constexpr (!KV16) {  // q, k and v are all fp32: one store pair through a selected pointer
            float *dst;
            if (vr < p.Dq + p.KVl) {
                rope_pair(a, b, opnd, o0, o1);
                dst = vr < p.Dq ? p.q + vr : (float *)ph.kc + (int64_t)pos * p.KVl + (vr - p.Dq);
            } else {
                dst = (float *)ph.vc + (int64_t)pos * p.KVl + (vr - p.Dq - p.KVl);
            }
            __stcg(dst, o0);
            __stcg(dst + 1, o1);
        } else {
            if (vr < p.Dq + p.KVl) rope_pair(a, b, opnd, o0, o1);
            if (vr < p.Dq) {
                __stcg(p.q + vr, o0);
                __stcg(p.q + vr + 1, o1);
            } else if (vr < p.Dq + p.KVl) {
                kv_st2(ph.kc, true, (int64_t)pos * p.KVl + (vr - p.Dq), o0, o1);
            } else {
                kv_st2(ph.vc, true, (int64_t)pos * p.KVl + (vr - p.Dq - p.KVl), o0, o1);
            }
        }
        break;
    }
    case PH_WO:
    case PH_W2:
        if (ph.xex < 0) __stcg(ph.out + unit, opnd.x + a);  // residual (src/model.c:179,186)
        else xch_put(p, ph.xex, xtag, unit, a);            // a partial: the residual follows in xch_reduce
        break;
    case PH_FFN: __stcg(ph.out + unit, __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), b)); break;  // src/ops.c:128-133
    default:  // PH_OUT
        if (p.tp == 1) {
            __stcg(ph.out + unit, a);
            if (a == a) best = max(best, argmax_key(a, (int)unit));
        } else {  // the vocabulary shard's logits into every rank's full logits
            const int64_t gu = (int64_t)p.rank * ph.units + unit;
            for (int r = 0; r < p.tp; r++) __stcg((float *)(p.peers.blk[r] + p.xlog_off) + gu, a);
            if (a == a) best = max(best, argmax_key(a, (int)gu));
        }
        break;
    }
}

// one unit (a row, or a row pair when two) of a stage: this lane's blocks lane, lane + 32, ... (the first
// XW from registers), summed over the warp
template <int DT>
__device__ __forceinline__ void unit_dot(bool two, const uint8_t *r0, int rbytes, int sbytes, int nb, const uint8_t *xq,
                                         const int2 *xds, const uint32_t (&xw)[XW][8], const float (&xd)[XW],
                                         const int (&xs)[XW], float &a0, float &a1) {
    const int lane = threadIdx.x & 31;
    const uint8_t *r1 = r0 + rbytes;
    a0 = 0.0f, a1 = 0.0f;
    if (nb >= 32 * XW) {  // every register block is in the row: no per-block test
#pragma unroll
        for (int c = 0; c < XW; c++) {
            a0 += dot_split<DT>(r0, sbytes, lane + 32 * c, xw[c], xd[c], xs[c]);
            if (two) a1 += dot_split<DT>(r1, sbytes, lane + 32 * c, xw[c], xd[c], xs[c]);
        }
        for (int b = lane + 32 * XW; b < nb; b += 32) {
            uint32_t xr[8];
            float rd;
            int rs;
            load_x(xq, xds, b, xr, rd, rs);
            a0 += dot_split<DT>(r0, sbytes, b, xr, rd, rs);
            if (two) a1 += dot_split<DT>(r1, sbytes, b, xr, rd, rs);
        }
    } else {
#pragma unroll
        for (int c = 0; c < XW; c++) {
            const int b = lane + 32 * c;
            if (b < nb) {
                a0 += dot_split<DT>(r0, sbytes, b, xw[c], xd[c], xs[c]);
                if (two) a1 += dot_split<DT>(r1, sbytes, b, xw[c], xd[c], xs[c]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        a0 += __shfl_xor_sync(0xffffffffu, a0, o);
        if (two) a1 += __shfl_xor_sync(0xffffffffu, a1, o);
    }
}

// One matvec phase on this CTA's units.  Group grp takes the stages g with g % NG == grp; within the
// group the units of its stages are dealt round-robin to its GW warps, so a warp works alone: its own
// row dots and warp sums, and one arrival on each of its group's stages.  Epilogues are deferred: lane
// k keeps the k-th pending unit's sums, and every 32 units (and at the end of the phase) all lanes run
// their epilogues at once, their operand loads (RoPE pairs, residual x) in flight together.
template <int DT, bool KV16>
__device__ void run_matvec(bool two, const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, uint64_t *full, uint64_t *empty,
                           unsigned &gk, bool &dead, int pos, unsigned long long &best, int phi, unsigned xtag) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, grp = warp / GW, wig = warp % GW;
    const uint8_t *xq = sm + p.off_xq;
    const int2 *xds = (const int2 *)(sm + p.off_xds);
    const int nb = ph.nb, sbytes = ph.sbytes, rbytes = ph.rbytes, R = ph.R;
    const int UR = two ? 2 : 1;
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
    unsigned long long twait = 0, tflush = 0, tdot = 0, nunits = 0;  // trace build only
    const int k0 = (int)((unsigned)(grp + NG) - gk % NG) % NG;  // this group's first stage of the phase
    // the first 32 units this warp will compute are known now: lane l loads unit l's epilogue operand
    // (RoPE pair, residual x) before the first stage, so the last flush does not wait on L2
    float2 opre = make_float2(0.0f, 0.0f);
    {
        const int64_t k = k0 + (int64_t)(lane / R) * NG, unit = u0 + k * R + lane % R;
        if (GW == 1 && k < nst && unit < u1) opre = epilogue_operand(p, ph, unit, pos);
    }
    bool first_batch = GW == 1;
    auto flush = [&]() {
        const unsigned long long tf = trace_slot(phi, kTrFlush) ? clock64() : 0;
        nunits += npend;
        if (lane < npend) {
            const float2 opnd = first_batch ? opre : epilogue_operand(p, ph, punit, pos);
            epilogue<KV16>(p, ph, punit, pa0, pa1, opnd, pos, best, xtag);
        }
        npend = 0;
        first_batch = false;
        if (trace_slot(phi, kTrFlush)) tflush += clock64() - tf;
    };
    for (int k = k0; k < nst; k += NG) {  // this group's stages
        const unsigned g = gk + (unsigned)k;
        const int s = (int)(g % (unsigned)p.nslots);
        const unsigned long long tw = trace_slot(phi, kTrFullWait) ? clock64() : 0;
        if (lane == 0)
            if (unsigned long long *q_ = trace_stage(p, g, 3))
                *q_ = gtime() | (mbar_test(&full[s], (g / p.nslots) & 1u) ? (1ull << 63) : 0ull);
        // warp-uniform verdict: a lane that timed out while another saw the copy land makes the whole warp
        // dead, so no lane computes on a stage that may still be filling and the shuffles stay full-warp
        if (!dead && __any_sync(0xffffffffu, !mbar_wait(&full[s], (g / p.nslots) & 1u))) {
            dead = true;
            if (lane == 0) raise_error(p.err, kErrMbarTimeout);
        }
        if (trace_slot(phi, kTrFullWait)) twait += clock64() - tw;
        if (lane == 0)
            if (unsigned long long *q_ = trace_stage(p, g, 1)) *q_ = gtime();
        const int64_t ua = u0 + (int64_t)k * R;
        const int n = (int)min((int64_t)R, u1 - ua);
        const uint8_t *stage = sm + (size_t)s * p.slot_bytes;
        if (!dead) {
            for (int i = (wig - uoff % GW + GW) % GW; i < n; i += GW) {
                float a0, a1;
                const unsigned long long td = trace_slot(phi, kTrDot) ? clock64() : 0;
                unit_dot<DT>(two, stage + (int64_t)i * UR * rbytes, rbytes, sbytes, nb, xq, xds, xw, xd, xs, a0, a1);
                if (trace_slot(phi, kTrDot)) tdot += clock64() - td;
                if (lane == npend) pa0 = a0, pa1 = a1, punit = ua + i;
                if (++npend == 32) flush();
            }
        }
        uoff += n;
        __syncwarp();
        if (lane == 0)
            if (unsigned long long *q_ = trace_stage(p, g, 2)) *q_ = gtime_after(pa0 + pa1);
        // a dead warp releases nothing: its slot may still be filling, and the producer must not refill it
        if (lane == 0 && !dead) mbar_arrive(&empty[s]);
    }
    if (!dead) flush();
    gk += (unsigned)nst;

    if (lane == 0) {
        DTRACE_ADD(phi, kTrFullWait, twait);
        DTRACE_ADD(phi, kTrFlush, tflush);
        DTRACE_ADD(phi, kTrDot, tdot);
        DTRACE_ADD(phi, kTrUnits, nunits);
        DTRACE_MAX(phi, kTrMvEnd, gtime());
    }
}

// A K-split matvec phase (rows too long for a ring slot): stage k of the CTA holds chunk j = k % C of its
// unit u0 + k / C; warp g % NG takes global stage g as in run_matvec.  A warp dots the chunk's blocks
// (activations from shared memory at block offset j * kb), sums over the warp and leaves the chunk's
// row sums in shared memory; once every warp is done, each consumer thread adds one unit's chunks in
// chunk order and runs its epilogue (operand loads of all units in flight together).
template <int DT, bool KV16>
__device__ void run_matvec_chunked(bool two, const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, uint64_t *full,
                                   uint64_t *empty, unsigned &gk, bool &dead, int pos, unsigned long long &best,
                                   unsigned xtag) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, grp = warp / GW;
    const uint8_t *xq = sm + p.off_xq;
    const int2 *xds = (const int2 *)(sm + p.off_xds);
    float *part = (float *)(sm + p.off_part);  // [unit][chunk][row]
    const int C = ph.C, kb = ph.kb, UR = two ? 2 : 1;
    int64_t u0, u1;
    split_units(ph.units, u0, u1);
    const int nunits = (int)(u1 - u0), nst = nunits * C;
    const int k0 = (int)((unsigned)(grp + NG) - gk % NG) % NG;
    for (int k = k0; k < nst; k += NG) {
        const unsigned g = gk + (unsigned)k;
        const int s = (int)(g % (unsigned)p.nslots);
        if (!dead && __any_sync(0xffffffffu, !mbar_wait(&full[s], (g / p.nslots) & 1u))) {
            dead = true;
            if (lane == 0) raise_error(p.err, kErrMbarTimeout);
        }
        const int lu = k / C, j = k % C, kbj = j < C - 1 ? kb : ph.nb - (C - 1) * kb;
        const int cbj = (int)chunk_row_bytes(DT, kbj), sbj = ((kbj * 2 + 15) / 16) * 16;
        const uint8_t *r0 = sm + (size_t)s * p.slot_bytes, *r1 = r0 + cbj;
        if (!dead) {
            float a0 = 0.0f, a1 = 0.0f;
            for (int b = lane; b < kbj; b += 32) {
                uint32_t xr[8];
                float rd;
                int rs;
                load_x(xq, xds, j * kb + b, xr, rd, rs);
                a0 += dot_split<DT>(r0, sbj, b, xr, rd, rs);
                if (two) a1 += dot_split<DT>(r1, sbj, b, xr, rd, rs);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                a0 += __shfl_xor_sync(0xffffffffu, a0, o);
                if (two) a1 += __shfl_xor_sync(0xffffffffu, a1, o);
            }
            if (lane == 0) {
                part[(lu * C + j) * UR] = a0;
                if (two) part[(lu * C + j) * UR + 1] = a1;
            }
        }
        __syncwarp();
        if (lane == 0 && !dead) mbar_arrive(&empty[s]);  // a dead warp releases nothing (see run_matvec)
    }
    gk += (unsigned)nst;
    named_sync(kBarConsumers, NCT);  // every chunk of the CTA's units is in part[]
    if (dead) return;
    for (int lu = t; lu < nunits; lu += NCT) {
        float a0 = 0.0f, a1 = 0.0f;
        for (int j = 0; j < C; j++) {
            a0 += part[(lu * C + j) * UR];
            if (two) a1 += part[(lu * C + j) * UR + 1];
        }
        const int64_t unit = u0 + lu;
        epilogue<KV16>(p, ph, unit, a0, a1, epilogue_operand(p, ph, unit, pos), pos, best, xtag);
    }
}

// ---------------------------------------------------------------- attention phase
// Lane l holds head dimensions dim(w), w < MAXW: fp32 cache, l + 32 w (each K/V element load is one
// coalesced 128-byte warp access); fp16 cache, the pairs 2 l + 64 i (+1), i < MAXW / 2, read as one
// half2 each, so a row takes half the load instructions and twice the positions fit the same registers.
template <bool F16>
__device__ __forceinline__ int att_dim(int lane, int w) {
    return F16 ? 64 * (w >> 1) + 2 * lane + (w & 1) : lane + 32 * w;
}

// The K and V rows this CTA's attention unit reads in the coming phase, brought into L2 (kept there in
// preference to the streamed weights) once the CTA's QKV work is done: their loads after the grid
// barrier then hit L2 instead of waiting on HBM.  Rows of earlier positions are fixed for the step; the
// row of `pos`, written during the QKV phase, is coherent in L2 either way (all cache reads are .cg).
template <typename KT>
__device__ void attn_prefetch(const DecodeParams &p, const DecodePhase &ph, int pos) {
    const int npos = pos + 1, nseg = attn_segments(p, pos);
    if ((int)blockIdx.x >= p.nkv * p.gsplit * nseg) return;
    const int unit = (int)blockIdx.x / nseg, seg = (int)blockIdx.x % nseg, kvh = unit / p.gsplit;
    // only the segment's first kPrefetchPos positions: the warps' first chunks wait on them, later chunks
    // follow in the loop, and a whole long segment (512 positions at the end of a 2048 window) kept
    // evict-last in L2 crowds out what the step reuses
    const int chunk = (npos + nseg - 1) / nseg, t0 = seg * chunk, t1 = min(npos, min(t0 + chunk, t0 + kPrefetchPos));
    const int rowb = p.hd * (int)sizeof(KT), lines = (rowb + 127) / 128 + 1;  // +1: the row's last byte
    const int total = max(0, t1 - t0) * 2 * lines;
    for (int e = threadIdx.x; e < total; e += NCT) {
        const int tt = t0 + e / (2 * lines), r = e % (2 * lines), kv = r / lines, ln = r % lines;
        const uint8_t *row = (const uint8_t *)((const KT *)(kv ? ph.vc : ph.kc) + (int64_t)tt * p.KVl + (int64_t)kvh * p.hd);
        prefetch_l2_keep(row + min(ln * 128, rowb - 1));
    }
}

template <typename KT>  // cache element: float or __half
__device__ void attention(const DecodeParams &p, const DecodePhase &ph, uint8_t *sm, int pos, int phi) {
    constexpr bool F16 = std::is_same<KT, __half>::value;
    constexpr int CH = F16 ? 2 * kAttnChunk : kAttnChunk;  // positions per warp loaded together
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int npos = pos + 1, nunit = p.nkv * p.gsplit;
    const int nseg = attn_segments(p, pos);
    const bool active = (int)blockIdx.x < nunit * nseg;
    const int unit = active ? (int)blockIdx.x / nseg : 0, seg = active ? (int)blockIdx.x % nseg : 0;
    const int kvh = unit / p.gsplit, gs = unit % p.gsplit, h0 = gs * GMAX, G = min(GMAX, p.group - h0);
    const int hd = p.hd, stride = hd + 2, ps = hd + kPartHead;
    const int chunk = (npos + nseg - 1) / nseg, t0 = seg * chunk, t1 = active ? min(npos, t0 + chunk) : 0;
    const int64_t hq = (int64_t)kvh * p.group + h0;  // first query head of this unit
    const KT *kb = (const KT *)ph.kc + (int64_t)kvh * hd, *vb = (const KT *)ph.vc + (int64_t)kvh * hd;

    float q[GMAX][MAXW], o[GMAX][MAXW], m[GMAX], l[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int w = 0; w < MAXW; w++) {
            const int d = att_dim<F16>(lane, w);
            q[g][w] = (active && g < G && d < hd) ? __ldcg(p.q + (hq + g) * hd + d) : 0.0f;
            o[g][w] = 0.0f;
        }
    }
    if (t == 0) DTRACE_SET(phi, kTrProLoad, gtime_after(q[0][0]));
    // positions t0 + warp, + NCW, ...: the K and V rows of up to CH of them are loaded at once
    bool first_chunk = true;
    for (int tb = t0 + warp; tb < t1; tb += CH * NCW) {
        float k[CH][MAXW], v[CH][MAXW];
        if constexpr (F16) {
            __half2 kh[CH][MAXW / 2], vh[CH][MAXW / 2];
#pragma unroll
            for (int c = 0; c < CH; c++) {
                const int tt = tb + c * NCW;
#pragma unroll
                for (int i = 0; i < MAXW / 2; i++) {
                    const int d = att_dim<true>(lane, 2 * i);  // even, and hd is even: the pair is in range
                    const bool ok = tt < t1 && d < hd;
                    kh[c][i] = ok ? __ldcg((const __half2 *)(kb + (int64_t)tt * p.KVl + d)) : __half2();
                    vh[c][i] = ok ? __ldcg((const __half2 *)(vb + (int64_t)tt * p.KVl + d)) : __half2();
                }
            }
#pragma unroll
            for (int c = 0; c < CH; c++)
#pragma unroll
                for (int i = 0; i < MAXW / 2; i++) {
                    const float2 kf = __half22float2(kh[c][i]), vf = __half22float2(vh[c][i]);
                    k[c][2 * i] = kf.x, k[c][2 * i + 1] = kf.y;
                    v[c][2 * i] = vf.x, v[c][2 * i + 1] = vf.y;
                }
        } else {
#pragma unroll
            for (int c = 0; c < CH; c++) {
                const int tt = tb + c * NCW;
#pragma unroll
                for (int w = 0; w < MAXW; w++) {
                    const int d = att_dim<false>(lane, w);
                    k[c][w] = (tt < t1 && d < hd) ? kv_ld(kb + (int64_t)tt * p.KVl + d) : 0.0f;
                    v[c][w] = (tt < t1 && d < hd) ? kv_ld(vb + (int64_t)tt * p.KVl + d) : 0.0f;
                }
            }
        }
        if (t == 0 && first_chunk) DTRACE_SET(phi, kTrAttnKV, gtime_after(k[0][0] + v[0][0]));
        first_chunk = false;
        if constexpr (!F16) {  // fp32 cache: one online softmax update per position
#pragma unroll
            for (int c = 0; c < CH; c++) {
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
            continue;
        }
        // fp16 cache (twice the positions per chunk): per query head the chunk's scores with their warp
        // reductions interleaved, then one online softmax update for the whole chunk
        const int nc = min(CH, (t1 - tb + NCW - 1) / NCW);  // valid positions of this chunk (>= 1)
#pragma unroll
        for (int g = 0; g < GMAX; g++) {
            if (g < G) {
                float sc[CH];
#pragma unroll
                for (int c = 0; c < CH; c++) {
                    sc[c] = 0.0f;
#pragma unroll
                    for (int w = 0; w < MAXW; w++) sc[c] = fmaf(k[c][w], q[g][w], sc[c]);
                }
#pragma unroll
                for (int off = 16; off; off >>= 1)
#pragma unroll
                    for (int c = 0; c < CH; c++) sc[c] += __shfl_xor_sync(0xffffffffu, sc[c], off);
                float mx = m[g];
#pragma unroll
                for (int c = 0; c < CH; c++) {
                    sc[c] *= p.scale;
                    if (c < nc) mx = fmaxf(mx, sc[c]);
                }
                const float corr = expf(m[g] - mx);
                l[g] *= corr;
#pragma unroll
                for (int w = 0; w < MAXW; w++) o[g][w] *= corr;
#pragma unroll
                for (int c = 0; c < CH; c++) {
                    if (c < nc) {
                        const float e = expf(sc[c] - mx);
                        l[g] += e;
#pragma unroll
                        for (int w = 0; w < MAXW; w++) o[g][w] = fmaf(e, v[c][w], o[g][w]);
                    }
                }
                m[g] = mx;
            }
        }
    }
    if (t == 0) DTRACE_SET(phi, kTrAttnLoop, gtime_after(l[0]));
    // merge the warps in one pass (the activation area is free during attention): every warp's (max, sum)
    // and acc per query head go to shared memory, then each consumer thread merges one (head, dimension)
    // over the NCW warps in warp order -- one CTA barrier instead of a tree of them -- and writes this
    // segment's (max, sum, acc) partial to global memory; the wo phase's prologue merges the segments of
    // each head while it quantizes the attention output (src/model.c:141-153)
    float *scr = (float *)(sm + p.off_xq);  // [NCW][G][hd + 2]
#pragma unroll
    for (int g = 0; g < GMAX; g++) {
        if (g < G) {
            float *dst = scr + (warp * G + g) * stride;
            if (lane == 0) dst[0] = m[g], dst[1] = l[g];
#pragma unroll
            for (int w = 0; w < MAXW; w++) {
                const int d = att_dim<F16>(lane, w);
                if (d < hd) dst[2 + d] = o[g][w];
            }
        }
    }
    named_sync(kBarConsumers, NCT);
    if (!active) return;  // the grid barrier that follows starts with a CTA barrier: the scratch stays
                          // untouched until every thread has read it
    float *part = p.apart + ((int64_t)unit * p.maxseg + seg) * GMAX * ps;
    for (int e = t; e < G * (hd + 1); e += NCT) {  // (head, dimension) pairs; dimension hd: (max, sum)
        const int g = e / (hd + 1), d = e % (hd + 1);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NCW; w++) {
            const float *src = scr + (w * G + g) * stride;
            if (src[1] > 0.0f) M = fmaxf(M, src[0]);
        }
        float den = 0.0f, acc = 0.0f;
#pragma unroll
        for (int w = 0; w < NCW; w++) {
            const float *src = scr + (w * G + g) * stride;
            const float lw = src[1], c = lw > 0.0f ? expf(src[0] - M) : 0.0f;
            den = fmaf(c, lw, den);
            if (d < hd) acc = fmaf(c, src[2 + d], acc);
        }
        float *dst = part + g * ps;
        if (d == hd) __stcg(dst, M), __stcg(dst + 1, den);
        else __stcg(dst + kPartHead + d, acc);
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
        if (p.tp > 1) __threadfence_system();  // the CTA's logits stores into the peers come first
        else __threadfence();
        if (atomicAdd(p.amax_ctr, 1) == (int)gridDim.x - 1) {
            __threadfence();
            unsigned long long gmax = atomicExch(p.amax_key, 0ull);
            if (p.tp > 1) {
                // the rank's key into every rank's table, then one system-scope arrival on every rank's
                // key counter; every rank then takes the same maximum (and so the same token)
                const unsigned ep = __ldcg(xch_word(p, p.rank, kXchEpoch));
                for (int r = 0; r < p.tp; r++)
                    __stcg((unsigned long long *)(p.peers.blk[r] + kXchKeys) + p.rank, gmax);
                for (int r = 0; r < p.tp; r++) red_release_sys_add(xch_word(p, r, kXchKeyCtr), 1u);
                if (!counter_wait_sys(xch_word(p, p.rank, kXchKeyCtr), (ep + 1) * (unsigned)p.tp))
                    raise_error(p.err, kErrFlagTimeout);
                for (int r = 0; r < p.tp; r++)
                    gmax = max(gmax, __ldcg((const unsigned long long *)(p.peers.blk[p.rank] + kXchKeys) + r));
                __stcg(xch_word(p, p.rank, kXchEpoch), ep + 1);  // the next step's cross-rank targets
            }
            int bi = argmax_index(gmax);
            const float x0 = __ldcg(p.logits);
            if (x0 != x0) bi = 0;  // a NaN in slot 0 is never replaced by the reference (src/sampler.c:27-32)
            advance_state(bi, p.state, p.forced, p.gen, p.gen_cap);
            *p.amax_ctr = 0;
            atomicExch(p.gbar, 0u);  // every CTA has passed the step's last grid barrier
        }
    }
}

template <bool KV16>  // the KV cache holds fp16 (else fp32): one kernel per cache type
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
        producer(p, sm, full, empty);
        return;
    }
    unsigned gk = 0;
    bool dead = false;
    // tags of this step's cross-rank exchanges count from epoch * xph (every rank runs the same steps)
    const unsigned xbase = p.tp > 1 ? __ldcg(xch_word(p, p.rank, kXchEpoch)) * (unsigned)p.xph : 0u;
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
        if (t == 0) DTRACE_SET(i, kTrStart, gtime());
        if (i + 1 < p.nph) desc_prefetch(p.ph + i + 1, dsm + ((i + 1) & 1));
        if (ph.kind == PH_ATTN) {
            if constexpr (KV16) attention<__half>(p, ph, sm, pos, i);
            else attention<float>(p, ph, sm, pos, i);
            if (t == 0) DTRACE_SET(i, kTrProEnd, gtime());
            continue;
        }
        prologue(p, ph, sm, token, pos, i);
        if (t == 0) DTRACE_SET(i, kTrProEnd, gtime());
        unsigned long long best = 0;  // this thread's argmax key (OUT phase)
        const bool two = ph.urows == 2;
        const unsigned xtag = ph.xex >= 0 ? xbase + (unsigned)ph.xex + 1u : 0u;
        if (ph.C > 1) {
            if (ph.dtype == QMC_Q8_0) run_matvec_chunked<QMC_Q8_0, KV16>(two, p, ph, sm, full, empty, gk, dead, pos, best, xtag);
            else run_matvec_chunked<QMC_Q4_0, KV16>(two, p, ph, sm, full, empty, gk, dead, pos, best, xtag);
        } else if (ph.dtype == QMC_Q8_0) {
            run_matvec<QMC_Q8_0, KV16>(two, p, ph, sm, full, empty, gk, dead, pos, best, i, xtag);
        } else {
            run_matvec<QMC_Q4_0, KV16>(two, p, ph, sm, full, empty, gk, dead, pos, best, i, xtag);
        }
        if (ph.xex >= 0 && !dead) {  // every warp's partials are out: add the ranks' partials of this CTA's rows
            named_sync(kBarConsumers, NCT);
            xch_reduce(p, ph, xtag);
        }
        if (ph.kind == PH_OUT) logits_argmax(p, sm, best);
        if (ph.kind == PH_QKV) {  // the attention phase that follows reads this layer's cache
            if constexpr (KV16) attn_prefetch<__half>(p, ph, pos);
            else attn_prefetch<float>(p, ph, pos);
        }
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

// one (row, block) per thread: the block's fp16 scale and quant bytes to their places in the K-split
// layout; the scale padding of each chunk row is zeroed by the thread of the chunk's last block
// where block b of global row gr lives in a K-split layout (chunks of kb blocks, units of urows rows, row
// gr at unit gr / per, position gr % per + pos0): its scale at *sc, its quants at *qu; zpad/zend: the
// scale padding of its chunk row, which the chunk's last block owns (empty for the others)
struct ChunkLayout {
    int dtype, urows, per, pos0;
    int64_t nb, kb, C, kbl, cb, cbl, ub;
    __device__ ChunkLayout(int dt, int64_t K, int kb_, int ur, int pr, int p0) : dtype(dt), urows(ur), per(pr), pos0(p0) {
        nb = nblocks(K);
        kb = kb_ < nb ? kb_ : nb;
        C = (nb + kb - 1) / kb;
        kbl = nb - (C - 1) * kb;
        cb = chunk_row_bytes(dt, kb);
        cbl = chunk_row_bytes(dt, kbl);
        ub = (int64_t)urows * ((C - 1) * cb + cbl);
    }
    __device__ void at(uint8_t *base, int64_t gr, int64_t b, uint8_t *&sc, uint8_t *&qu, uint8_t *&zpad, uint8_t *&zend) const {
        const int QB = dtype == QMC_Q8_0 ? 32 : 16;
        const int64_t u = gr / per, pos = gr % per + pos0, j = b / kb, bj = b % kb;
        const int64_t kbj = j < C - 1 ? kb : kbl, cbj = j < C - 1 ? cb : cbl, sbj = (kbj * 2 + 15) / 16 * 16;
        uint8_t *d = base + u * ub + (int64_t)urows * j * cb + pos * cbj;  // this row's chunk j
        sc = d + 2 * bj;
        qu = d + sbj + bj * QB;
        zpad = zend = d + sbj;
        if (bj == kbj - 1) zpad = d + 2 * kbj;
    }
};

// one (row, block) per thread: the block's fp16 scale and quant bytes from the file layout (AoS) to
// their places in the K-split layout
__global__ void repack_chunked_kernel(int dtype, const uint8_t *__restrict__ aos, int64_t row0, int64_t rows, int64_t K,
                                      int kb, int urows, int per, int pos0, uint8_t *__restrict__ dst) {
    const ChunkLayout L(dtype, K, kb, urows, per, pos0);
    const int BS = dtype == QMC_Q8_0 ? kQ8Bytes : kQ4Bytes, QB = BS - 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * L.nb; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / L.nb, b = i % L.nb;
        uint8_t *sc, *qu, *zp, *ze;
        L.at(dst, row0 + r, b, sc, qu, zp, ze);
        const uint8_t *s = aos + (r * L.nb + b) * BS;
        sc[0] = s[0];
        sc[1] = s[1];
        for (int k = 0; k < QB; k++) qu[k] = s[2 + k];
        for (uint8_t *z = zp; z < ze; z++) *z = 0;
    }
}

// the same matrix from one K-split layout to another (e.g. chunks -> whole rows), block by block
__global__ void relayout_chunked_kernel(int dtype, const uint8_t *__restrict__ src, int kb_src, uint8_t *__restrict__ dst,
                                        int kb_dst, int64_t rows, int64_t K, int urows, int per, int pos0) {
    const ChunkLayout Ls(dtype, K, kb_src, urows, per, pos0), Ld(dtype, K, kb_dst, urows, per, pos0);
    const int QB = dtype == QMC_Q8_0 ? 32 : 16;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * Ld.nb; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / Ld.nb, b = i % Ld.nb;
        uint8_t *ssc, *squ, *szp, *sze, *dsc, *dqu, *dzp, *dze;
        Ls.at(const_cast<uint8_t *>(src), r, b, ssc, squ, szp, sze);
        Ld.at(dst, r, b, dsc, dqu, dzp, dze);
        dsc[0] = ssc[0];
        dsc[1] = ssc[1];
        for (int k = 0; k < QB; k++) dqu[k] = squ[k];
        for (uint8_t *z = dzp; z < dze; z++) *z = 0;
    }
}

}  // namespace

int launch_repack_chunked(int dtype, const void *aos, int64_t row0, int64_t rows, int64_t K, int kb, int urows, int per,
                          int pos0, void *dst, cudaStream_t s) {
    if (dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "repack: dtype %d is not quantized", dtype);
    if (kb < 1 || urows < 1 || per < 1 || pos0 + per > urows || row0 < 0 || row0 % per)
        return set_error(QMC_EINVAL, "repack: bad chunk layout");
    if (rows <= 0) return QMC_OK;
    const int64_t work = rows * nblocks(K);
    const int grid = (int)std::min<int64_t>((work + 255) / 256, 65536);
    const int kbc = (int)std::min<int64_t>(kb, nblocks(K));
    repack_chunked_kernel<<<grid, 256, 0, s>>>(dtype, (const uint8_t *)aos, row0, rows, K, kbc, urows, per, pos0,
                                               (uint8_t *)dst);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_relayout_chunked(int dtype, const void *src, int kb_src, void *dst, int kb_dst, int64_t rows, int64_t K,
                            int urows, int per, int pos0, cudaStream_t s) {
    if (dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "relayout: dtype %d is not quantized", dtype);
    if (kb_src < 1 || kb_dst < 1 || urows < 1 || per < 1 || pos0 + per > urows) return set_error(QMC_EINVAL, "relayout: bad layout");
    if (rows <= 0) return QMC_OK;
    const int64_t work = rows * nblocks(K);
    const int grid = (int)std::min<int64_t>((work + 255) / 256, 65536);
    relayout_chunked_kernel<<<grid, 256, 0, s>>>(dtype, (const uint8_t *)src, kb_src, (uint8_t *)dst, kb_dst, rows, K, urows,
                                                 per, pos0);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

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

#ifdef QMC_DECODE_TRACE
// profiling build only: where the kernel writes its stamps ([phases][grid][kTrSlots] words; null: off)
extern "C" __attribute__((visibility("default"))) int qmc_decode_trace_set(void *dev_buf) {
    return (int)cudaMemcpyToSymbol(g_dtrace, &dev_buf, sizeof(dev_buf));
}
#endif

namespace {
int64_t r128(int64_t b) { return (b + 127) / 128 * 128; }
// shared memory besides the ring: activations (or the attention merge scratch), chunk partials, the
// reduction / descriptor area
int64_t plan_fixed(int nb_max, int hd, int group, int64_t part_bytes, int64_t *scratch_out) {
    const int64_t act = r128((int64_t)nb_max * 32) + r128((int64_t)nb_max * 8);
    // attention merge scratch: every warp's (max, sum, acc) per query head of a unit
    const int64_t tree = r128((int64_t)NCW * std::min(std::max(group, 1), GMAX) * (hd + 2) * 4);
    *scratch_out = std::max(act, tree);
    return *scratch_out + r128(part_bytes) + kRedBytes;
}
}  // namespace

// K-split chunks are cut to the slots of the 22-slot ring (two per consumer warp): fewer, larger stages
// than with 33 slots amortise each stage's wait / reduction / release (70B-shaped Q8_0: 62.8 against
// 60.2 tok/s)
int64_t decode_slot_bytes(int nb_max, int hd, int group, size_t smem_optin, int64_t part_bytes) {
    int64_t scratch;
    const int64_t fixed = plan_fixed(nb_max, hd, group, part_bytes, &scratch);
    const int ns = 2 * NG;
    return (((int64_t)smem_optin - r128((int64_t)ns * 2 * 8) - fixed) / ns) / 128 * 128;
}

bool plan_decode(int64_t max_unit_bytes, int nb_max, int hd, int group, size_t smem_optin, DecodePlan *out,
                 int64_t part_bytes) {
    if (hd > 32 * MAXW) return false;
    int64_t scratch;
    const int64_t fixed = plan_fixed(nb_max, hd, group, part_bytes, &scratch);
    const int64_t tree = r128((int64_t)NCW * std::min(std::max(group, 1), GMAX) * (hd + 2) * 4);
    for (int ns : {3 * NG, 2 * NG, NG}) {  // slots: a multiple of NG, so every slot belongs to one group
        const int64_t bars = r128((int64_t)ns * 2 * 8);  // full[ns], empty[ns]
        const int64_t avail = (int64_t)smem_optin - (bars + fixed);
        const int64_t slot = (avail / ns) / 128 * 128;
        if (slot < max_unit_bytes) continue;
        DecodePlan d;
        d.nslots = ns;
        d.groups = NG;
        d.slot_bytes = (int)slot;
        d.off_bars = (int)(ns * slot);
        d.off_xq = d.off_bars + (int)bars;
        d.off_xds = d.off_xq + (int)r128((int64_t)nb_max * 32);
        d.off_part = d.off_xq + (int)scratch;
        d.off_red = d.off_part + (int)r128(part_bytes);
        d.smem = (size_t)d.off_red + kRedBytes;
        if (d.off_xq < d.off_bars + ns * 16 || d.off_xds + (int64_t)nb_max * 8 > d.off_part ||
            d.off_xq + tree > d.off_part || (int64_t)d.smem > (int64_t)smem_optin)
            return false;  // regions overlap (cannot happen with the sizes above)
        *out = d;
        return true;
    }
    return false;
}

int launch_decode(const DecodeParams &p, const DecodePlan &plan, int grid, cudaStream_t s) {
    DevCtx *c = ctx();
    if (!c) return QMC_ECUDA;
    auto fn = p.kv16 ? decode_step_kernel<true> : decode_step_kernel<false>;
    static bool attr_done[64][2];
    if (!attr_done[c->device][p.kv16 != 0]) {
        QMC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->max_smem_optin));
        attr_done[c->device][p.kv16 != 0] = true;
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
    QMC_CUDA(cudaLaunchKernelEx(&cfg, fn, p));
    return QMC_OK;
}

}  // namespace qmc
