// Activation quantization shared by the decode kernel and the standalone matvec: a row of floats
// becomes Q8_0 blocks in shared memory, two or four threads per 32-element block, in the layout the dot
// loops read.
#pragma once

#include "common.cuh"

namespace qmc {

// activation block b is stored with its 16-byte halves swapped when bit 2 of b is set, so 8 threads
// loading consecutive blocks hit all 32 banks
__device__ __forceinline__ int xswz(int b) { return ((b >> 2) & 1) << 4; }

// x + kRound - kRound rounds |x| < 2^22 to the nearest integer, ties to even, in one round-to-nearest
// add; for |x| <= 127 the integer is also the low bits of x + kRound.  Used instead of rintf / floorf /
// float->int conversions, which issue at a fraction of the FMA pipe's rate.
constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
constexpr int kRoundBits = 0x4B400000;

// rint(RN(v / sc)) for an element whose product r = v * (1 / sc) lies within 1e-4 of a half-integer,
// without dividing (rare).  h = floor(r) + 0.5 is that half-integer; h * sc has at most 20 significant
// bits, so it and d = v - h * sc (Sterbenz: v and h * sc are within 0.1% of each other) are exact.
// RN(v / sc) equals h exactly when v / sc lies inside h's rounding interval, [h - u, h + u] with
// u = ulp(h) / 2 (the side towards zero is u / 2 when |h| = 0.5, a power of two), ties included since
// h's last mantissa bit is 0; rint then takes the even neighbour, else the side d points to.
__device__ __forceinline__ int quant_near_half(float v, float r, float sc) {
    const float fl = floorf(r), h = fl + 0.5f;
    const float d = fmaf(-h, sc, v);
    const float u = __int_as_float((__float_as_int(h) & 0x7f800000) - (24 << 23));  // ulp(h) / 2, |h| >= 0.5
    const bool toward0 = (d < 0.0f) == (h > 0.0f);
    const float lim = __fmul_rn((fabsf(h) == 0.5f && toward0) ? 0.5f * u : u, sc);
    const int f = __float_as_int(__fadd_rn(fl, kRound)) - kRoundBits;  // floor(r) as an integer
    const int q = fabsf(d) <= lim ? f + (f & 1) : (d > 0.0f ? f + 1 : f);
    return min(127, max(-127, q));
}

// The arithmetic of one Q8_0 block held by 32 / E lanes (part j: elements E j .. E j + E - 1; E = 16, a
// lane pair, or 8, a lane quad), bit-exact with src/quant.c:33-53: amax ignores NaN, IEEE division for
// the scale, fp16 RNE scale, then rint(v / scale) clamped to +-127 (NaN -> 0, as the float->int
// conversion gives).  All lanes call it (shuffles within the lane group).  Out: the lane's quants in
// element order (4 per word), the block's quant sum (every lane of the group) and its scale.
template <int E>
__device__ __forceinline__ void quant_group(const float (&v)[E], uint32_t (&w)[E / 4], int &sum, float &sc) {
    static_assert(E == 16 || E == 8, "a block is held by 2 or 4 lanes");
    constexpr int NWD = E / 4;  // quant words per lane
    uint32_t m[E / 2];
#pragma unroll
    for (int i = 0; i < E / 2; i++) {  // |v| bits order like floats; NaN -> 0
        const float a0 = fabsf(v[2 * i]), a1 = fabsf(v[2 * i + 1]);
        m[i] = max((a0 == a0) ? __float_as_uint(a0) : 0u, (a1 == a1) ? __float_as_uint(a1) : 0u);
    }
#pragma unroll
    for (int w = E / 4; w; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; i++) m[i] = max(m[i], m[i + w]);
    uint32_t ab = m[0];
#pragma unroll
    for (int o = 1; o < 32 / E; o <<= 1) ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, o));
    sc = h2f(f2h(__fdiv_rn(__uint_as_float(ab), 127.0f)));
    const float rs = __frcp_rn(sc);
    // q = rint(v / sc) clamped to +-127, as v * (1 / sc) + 1.5 * 2^23 (round to nearest even, no
    // float->int conversion).  |v / sc| < 256, so v * (1 / sc) lies within 4.6e-5 of the correctly
    // rounded quotient and rounds to the same integer unless it is within 1e-4 of a half-integer; those
    // elements take quant_near_half.  NaN gives 0.
#pragma unroll
    for (int i = 0; i < NWD; i++) w[i] = 0u;  // the lane's quants in element order, 4 per word
    sum = 0;
    bool near = false;
#pragma unroll
    for (int i = 0; i < E; i++) {
        const float r = __fmul_rn(v[i], rs);
        const float c = fminf(fmaxf(r, -127.0f), 127.0f);
        const float cr = __fadd_rn(c, kRound);
        const int q = (sc != 0.0f && r == r) ? __float_as_int(cr) - kRoundBits : 0;
        near |= fabsf(__fsub_rn(r, __fsub_rn(cr, kRound))) > 0.4999f;
        sum += q;
        w[i >> 2] |= (uint32_t)(q & 0xff) << (8 * (i & 3));
    }
    if (near) {  // rare: redo the lane's elements, the near-half ones exactly
        sum = 0;
#pragma unroll
        for (int i = 0; i < E; i++) {
            const float r = __fmul_rn(v[i], rs);
            const float c = fminf(fmaxf(r, -127.0f), 127.0f);
            const float cr = __fadd_rn(c, kRound);
            int q = (sc != 0.0f && r == r) ? __float_as_int(cr) - kRoundBits : 0;
            if (fabsf(__fsub_rn(r, __fsub_rn(cr, kRound))) > 0.4999f) q = quant_near_half(v[i], r, sc);
            sum += q;
            const uint32_t m = 0xffu << (8 * (i & 3));
            w[i >> 2] = (w[i >> 2] & ~m) | ((uint32_t)(q & 0xff) << (8 * (i & 3)));
        }
    }
#pragma unroll
    for (int o = 1; o < 32 / E; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
}

// Block b (quant_group) stored where the dot loops read it: int8 at xq + 32 b with the xswz swizzle, the
// (scale, quant sum) pair at xds[b].  All lanes call it; `active` lanes store.  Q4_0 weights take the
// block's even elements in bytes 0-15 and odd elements in bytes 16-31.  With `aos`, the active lanes
// also write the block in the .qlm Q8_0 layout at aos + 34 b.
template <int E = 16>
__device__ __forceinline__ void quant_block(bool q4, uint8_t *xq, int2 *xds, int b, int j, bool active,
                                            const float (&v)[E], uint8_t *aos = nullptr) {
    constexpr int NWD = E / 4;  // quant words per lane
    uint32_t w[NWD];
    int sum;
    float sc;
    quant_group<E>(v, w, sum, sc);
    if (!active) return;
    uint8_t *blk = xq + (int64_t)b * 32;
    const int sw = xswz(b);
    if (E == 16) {
        if (!q4) {
            *(uint4 *)(blk + ((16 * j) ^ sw)) = make_uint4(w[0], w[1], w[NWD - 2], w[NWD - 1]);
        } else {  // even elements (bytes 0, 2 of each word pair), then odd ones
            *(uint2 *)(blk + ((8 * j) ^ sw)) =
                make_uint2(__byte_perm(w[0], w[1], 0x6420), __byte_perm(w[NWD - 2], w[NWD - 1], 0x6420));
            *(uint2 *)(blk + ((16 + 8 * j) ^ sw)) =
                make_uint2(__byte_perm(w[0], w[1], 0x7531), __byte_perm(w[NWD - 2], w[NWD - 1], 0x7531));
        }
    } else {
        if (!q4) {
            *(uint2 *)(blk + ((8 * j) ^ sw)) = make_uint2(w[0], w[1]);
        } else {
            *(uint32_t *)(blk + ((4 * j) ^ sw)) = __byte_perm(w[0], w[1], 0x6420);
            *(uint32_t *)(blk + ((16 + 4 * j) ^ sw)) = __byte_perm(w[0], w[1], 0x7531);
        }
    }
    if (j == 0) xds[b] = make_int2(__float_as_int(sc), sum);
    if (aos) {  // the block in the file layout (fp16 scale, then the 32 quants in element order)
        uint8_t *o = aos + (int64_t)b * kQ8Bytes;
        if (j == 0) {
            const uint32_t h = f2h(sc);
            o[0] = (uint8_t)(h & 0xff), o[1] = (uint8_t)(h >> 8);
        }
#pragma unroll
        for (int i = 0; i < E; i++) o[2 + E * j + i] = (uint8_t)(w[i >> 2] >> (8 * (i & 3)));
    }
}

// 8 floats x[e0 .. e0 + 8), zero past n: two vector loads where the 8 are in range and 16-byte aligned
__device__ __forceinline__ void load8_any(const float *x, int64_t e0, int64_t n, float (&v)[8]) {
    if (e0 + 8 <= n && ((uintptr_t)(x + e0) & 15) == 0) {
        const float4 a = ((const float4 *)(x + e0))[0], c = ((const float4 *)(x + e0))[1];
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = c.x, v[5] = c.y, v[6] = c.z, v[7] = c.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = e0 + i < n ? x[e0 + i] : 0.0f;
    }
}

// Q8_0 of T rows of n floats by lane quads (quant_group<8>) into the row-major activation blocks of the
// prefill contractions: qs[t][nb][32] int8 in element order, d[t][nb] scales and, with dT, the scales
// again block-major at dT[b * ldT + t].  fetch(t, e0, v) gives elements e0 .. e0 + 7 of row t (zero past
// n).  A warp takes 8 consecutive blocks per step, so its lanes stay together for the quad shuffles.
template <class Fetch>
__device__ __forceinline__ void quant_rows_quads(int64_t T, int64_t n, Fetch &&fetch, int8_t *qs, float *d, float *dT,
                                                 int64_t ldT) {
    const int lane = threadIdx.x & 31, j = lane & 3;
    const int64_t nb = nblocks(n), total = T * nb;
    const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t base = w0 * 8; base < total; base += nw * 8) {
        const int64_t blk = base + (lane >> 2);
        const bool active = blk < total;
        const int64_t t = active ? blk / nb : 0, b = active ? blk % nb : 0;
        float v[8];
        if (active) {
            fetch(t, b * 32 + 8 * j, v);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = 0.0f;
        }
        uint32_t w[2];
        int sum;
        float sc;
        quant_group<8>(v, w, sum, sc);
        if (active) {
            *(uint2 *)(qs + (t * nb + b) * 32 + 8 * j) = make_uint2(w[0], w[1]);
            if (j == 0) {
                d[t * nb + b] = sc;
                if (dT) dT[b * ldT + t] = sc;
            }
        }
    }
}

}  // namespace qmc
