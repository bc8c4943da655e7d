// Shared device helpers for libquillm_cuda (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "quillm_cuda.h"

namespace qmc {

constexpr int kQ8Bytes = 34;  // {fp16 d; int8 qs[32]}
constexpr int kQ4Bytes = 18;  // {fp16 d; uint8 qs[16]}

__host__ __device__ inline int64_t nblocks(int64_t n) { return (n + 31) / 32; }
__host__ __device__ inline int64_t row_bytes(int dtype, int64_t n) {
    return dtype == QMC_F32 ? n * 4 : nblocks(n) * (dtype == QMC_Q8_0 ? kQ8Bytes : kQ4Bytes);
}

// ---------------------------------------------------------------- fp16 bits
// fp16 -> fp32 is exact (hardware cvt); fp32 -> fp16 is IEEE round-to-nearest-even (hardware cvt)
// with the reference's NaN rule (quiet, top 10 payload bits kept: src/fp16.c:40-41).
__device__ __forceinline__ float h2f(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }
__device__ __forceinline__ uint32_t f2h(float f) {
    uint32_t b = __float_as_uint(f);
    if ((b & 0x7fffffffu) > 0x7f800000u) return ((b >> 16) & 0x8000u) | 0x7e00u | ((b >> 13) & 0x3ffu);
    return __half_as_ushort(__float2half_rn(f));
}

// ---------------------------------------------------------------- KV cache elements
// The cache holds fp32 (the reference's layout, src/model.c:96) or, by choice, fp16: each K (after
// RoPE) and V value rounded to nearest-even once when stored, widened exactly when read.
__device__ __forceinline__ float kv_ld(const float *p) { return __ldcg(p); }
__device__ __forceinline__ float kv_ld(const __half *p) { return __half2float(__ldcg(p)); }
// stores the pair (a, b) at elements i, i + 1 (i even) of a cache of the given kind
__device__ __forceinline__ void kv_st2(void *base, bool f16, int64_t i, float a, float b) {
    if (f16) {
        __stcg((__half2 *)((__half *)base + i), __floats2half2_rn(a, b));
    } else {
        __stcg((float *)base + i, a);
        __stcg((float *)base + i + 1, b);
    }
}

// ---------------------------------------------------------------- warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// dequantized value of element c of a row (src/quant.c:65-94): fp32(d) * (float)q, one rounding
__device__ __forceinline__ float deq_elem(int dtype, const uint8_t *row, int64_t c) {
    if (dtype == QMC_F32) return ((const float *)row)[c];
    const int64_t b = c >> 5;
    const int k = (int)(c & 31);
    if (dtype == QMC_Q8_0) {
        const uint8_t *blk = row + b * kQ8Bytes;
        return h2f(blk[0] | (blk[1] << 8)) * (float)(int8_t)blk[2 + k];
    }
    const uint8_t *blk = row + b * kQ4Bytes;
    const int byte = blk[2 + (k >> 1)];
    const int q = (k & 1) ? (byte >> 4) : (byte & 15);
    return h2f(blk[0] | (blk[1] << 8)) * (float)(q - 8);
}

// ---------------------------------------------------------------- block quantization (warp per block)
// Lane i holds element i of a 32-element block (0 for the zero-padded tail).  Every lane returns
// its quantized value; *dd receives fp32(fp16(amax / qmax)) and *dh its fp16 bits.  Bit-exact with
// src/quant.c:33-53: amax ignores NaN (the reference's `a > amax` test), IEEE division, rintf
// (round half to even), clamp, q = 0 when the scale is 0.
__device__ __forceinline__ int quant_lane(float v, float qmax, int qmin, int qmaxi, float *dd, uint32_t *dh) {
    float a = fabsf(v);
    uint32_t ab = (a == a) ? __float_as_uint(a) : 0u;  // |v| bits order like floats; NaN -> 0
    uint32_t mb = __reduce_max_sync(0xffffffffu, ab);
    float d = __fdiv_rn(__uint_as_float(mb), qmax);
    uint32_t hb = f2h(d);
    float sc = h2f(hb);
    *dd = sc;
    *dh = hb;
    if (sc == 0.0f) return 0;
    float r = rintf(__fdiv_rn(v, sc));
    r = r < (float)qmin ? (float)qmin : r;
    r = r > (float)qmaxi ? (float)qmaxi : r;
    return (int)r;
}

// ---------------------------------------------------------------- error word
// Kernels whose spin-waits expire OR a code into *err and return; the host reads it with
// qmc_check_device_error().
enum : int { kErrMbarTimeout = 1, kErrFlagTimeout = 2, kErrBadState = 4 };
__device__ __forceinline__ void raise_error(int *err, int code) {
    if (err) atomicOr(err, code);
}
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// ---------------------------------------------------------------- mbarrier + bulk async copy (1-D TMA)
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, uint32_t tx) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(tx) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    // the suspend-time hint (ns) lets a waiting warp sleep in hardware until the phase completes instead
    // of re-issuing, so waiting consumers do not take issue slots from working ones
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}
// non-blocking test of a phase (no suspend): for a thread that has other work while it waits
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait: true when the phase completed, false after ~kWaitCycles
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}
// bounded wait against a deadline several waits share (t0 + kWaitCycles)
__device__ __forceinline__ bool mbar_wait_since(uint64_t *bar, uint32_t parity, long long t0) {
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// bounded poll of a counter other CTAs raise: true once *ctr reached `target` (modulo 2^32), false after
// ~kWaitCycles
__device__ __forceinline__ bool counter_wait(const unsigned *ctr, unsigned target) {
    const long long t0 = clock64();
    while ((int)(ld_acquire(ctr) - target) < 0)
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}
// L2 policy for data read once (streamed weights): evicted first, so activations, partials and the KV
// cache stay in L2 while gigabytes of weights pass through it
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// global -> shared bulk copy completing on `bar`, with an L2 cache policy; dst, src 16-byte aligned,
// bytes % 16 == 0
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
// bring the 128-byte line holding p into L2, kept there in preference to evict-first lines
__device__ __forceinline__ void prefetch_l2_keep(const void *p) {
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}
// global -> shared bulk copy completing on `bar`; dst, src 16-byte aligned, bytes % 16 == 0
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// ---------------------------------------------------------------- greedy token selection
// Order-preserving 64-bit key of (value, index): a larger value wins, equal values keep the lower
// index -- the reference's first-maximum rule (src/sampler.c:27-32).  -0.0 counts as +0.0; NaN never wins.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t u = v == 0.0f ? 0u : __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (uint32_t)(0xffffffffu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_index(unsigned long long key) {
    return key ? (int)(0xffffffffu - (uint32_t)(key & 0xffffffffu)) : 0;
}
// Device-resident generation state [token, pos, step, prompt length]: record the greedy token of step
// s (from the last prompt token on), feed the next prompt token while the prompt lasts, advance pos.
__device__ __forceinline__ void advance_state(int best, int *state, const int *forced, int *gen, int gen_cap) {
    const int s = state[2], forced_n = state[3];
    const int slot = s + 1 - forced_n;
    if (gen && slot >= 0 && slot < gen_cap) gen[slot] = best;
    state[0] = (s + 1 < forced_n) ? forced[s + 1] : best;
    state[1] += 1;
    state[2] = s + 1;
}

// ---------------------------------------------------------------- programmatic dependent launch
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

}  // namespace qmc

// ---------------------------------------------------------------- host side (qmc_* internals)
namespace qmc {
int set_error(int code, const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);
struct DevCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    int *err = nullptr;  // device error word
    int num_sms = 0;
    size_t max_smem_optin = 0;
};
DevCtx *ctx();  // context of the calling thread's current device (created on first use); nullptr on failure
inline cudaStream_t pick_stream(void *s) { return s ? (cudaStream_t)s : (ctx() ? ctx()->stream : nullptr); }
}  // namespace qmc

#define QMC_CUDA(call)                                                                                                 \
    do {                                                                                                               \
        cudaError_t e_ = (call);                                                                                       \
        if (e_ != cudaSuccess) return qmc::cuda_fail(e_, #call);                                                       \
    } while (0)
#define QMC_LAUNCH_CHECK() QMC_CUDA(cudaGetLastError())
