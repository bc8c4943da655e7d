// Quantized-weight prefill contraction on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// Row t of C is qm_matvec(W, A[t]) bit for bit (src/ops.c:57-61, src/kernels_scalar.c:12-34): for every
// 32-element block b the reference forms the exact int32 dot of the weight row's int8 values (Q4_0:
// nibble - 8) with the token's Q8_0 activation block, then accumulates s += (float)isum * (dw * dx) in
// block order, each operation rounded to float.  One tcgen05.mma of kind::i8 has K = 32, so it produces
// exactly those int32 block dots for a 128-row x NT-token tile, in tensor memory (TMEM).  The epilogue
// warps read each block's tile with tcgen05.ld and apply the scaled accumulation in the reference's
// order: the tensor cores do the 32 multiply-adds per (row, token, block), the CUDA cores the 4 float
// operations.
//
// CTA roles (9 warps): warp 0 allocates TMEM and one elected lane issues the MMAs; warps 1-4 are the
// epilogue (warp w may read TMEM lanes 32 (w % 4) .. + 31, i.e. weight rows of that quarter); warps 5-8
// produce the shared-memory operands of each stage of KS blocks: the weight blocks (split-row layout:
// 16-byte aligned payloads) as int8 and the activation blocks, both in the no-swizzle K-major core-matrix
// layout (a core matrix is 8 rows x 16 bytes; the two 16-byte halves of a block lie 128 bytes apart,
// 8-row groups 256 bytes apart), plus the blocks' scales.  A ring of NS stages (smem_full / smem_empty)
// and two TMEM buffers (tmem_full / tmem_empty) keep the three roles overlapped.  Every wait is bounded;
// after a timeout a role stops, raises the error word and falls through to the end, where the MMA lane
// first waits (bounded) for the MMAs it issued and warp 0 frees the TMEM it holds.
#include "matmul_tc.cuh"

namespace qmc {
namespace {

constexpr int MT = 128;  // weight rows per CTA (MMA M: TMEM lanes)
constexpr int NT = 32;   // tokens per CTA (MMA N)
constexpr int KS = 4;    // blocks per stage
constexpr int NS = 4;    // stages in the ring
constexpr int kWarps = 9, kThreads = 32 * kWarps;
constexpr int kTmemCols = 2 * KS * NT;  // two buffers of KS block tiles (power of 2, >= 32)
static_assert(kTmemCols == 256, "TMEM allocation size");

// stage layout (bytes)
constexpr int kWTile = MT * 32, kATile = NT * 32;  // one block's operand tiles
constexpr int kOffA = KS * kWTile, kOffDw = kOffA + KS * kATile, kOffDa = kOffDw + KS * MT * 4;
constexpr int kStage = kOffDa + KS * NT * 4;
constexpr int kOffBars = NS * kStage;  // smem_full[NS], smem_empty[NS], tmem_full[2], tmem_empty[2], tmem addr
constexpr int kSmem = kOffBars + (2 * NS + 4) * 8 + 16;
static_assert(kStage % 128 == 0, "stage alignment");

// no-swizzle K-major position of byte 16*h of row r inside a block tile
__device__ __forceinline__ int core_off(int r, int h) { return (r >> 3) * 256 + h * 128 + (r & 7) * 16; }

// shared-memory matrix descriptor: start, leading (K-direction) byte offset 128, stride (8-row group)
// byte offset 256, descriptor version 1, no swizzle
__device__ __forceinline__ uint64_t smem_desc(const void *p) {
    const uint64_t a = (smem_u32(p) >> 4) & 0x3fffu;
    return a | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) | (1ull << 46);
}
// instruction descriptor: s32 accumulator, s8 x s8, both K-major, N = NT, M = MT
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(MT >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(0)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct TcParams {
    const uint8_t *W;  // split rows: [rows][wstride]: scales (fp16, padded to 16 bytes) then quant payloads
    int64_t wstride, sbytes;
    const int8_t *aq;  // activation blocks [T][nb * 32]
    const float *ad;   // activation scales [T][nb]
    float *C, *C2;     // C[T][N]; with C2: weight row 2i -> C[t][i], 2i + 1 -> C2[t][i] (N / 2 columns each)
    int64_t T, N;
    int nb;
    int *err;
};

template <int DT>
__global__ void __launch_bounds__(kThreads, 1) matmul_q_tc_kernel(const TcParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *full = (uint64_t *)(sm + kOffBars), *empty = full + NS, *tfull = empty + NS, *tempty = tfull + 2;
    volatile uint32_t *tmem_slot = (volatile uint32_t *)(tempty + 2);
    volatile int *dead = (volatile int *)(tmem_slot + 1);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t n0 = (int64_t)blockIdx.x * MT, t0 = (int64_t)blockIdx.y * NT;
    const int nst = (p.nb + KS - 1) / KS;

    if (t == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 4);       // one arrival per producer warp
            mbar_init(&empty[s], 1 + 4);  // the MMA commit + one per epilogue warp (they read the scales)
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);   // MMA commit
            mbar_init(&tempty[b], 4);  // epilogue warps
        }
        *dead = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void *)tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 5) {  // ---------------------------------------------------------------- producers
        const int pt = t - 5 * 32;  // 0..127
        for (int g = 0; g < nst; g++) {
            const int s = g % NS;
            if (__any_sync(0xffffffffu, g >= NS && !mbar_wait(&empty[s], ((g / NS) - 1) & 1u))) {
                if (lane == 0) raise_error(p.err, kErrMbarTimeout);
                *dead = 1;
                break;
            }
            if (__any_sync(0xffffffffu, *dead != 0)) break;
            uint8_t *st = sm + s * kStage;
            const int b0 = g * KS;
            // weight payloads -> int8 core-matrix tiles
            if (DT == QMC_Q8_0) {
                for (int i = pt; i < MT * KS * 2; i += 128) {  // 16-byte chunks: row, block, half
                    const int r = i / (KS * 2), j = (i >> 1) % KS, h = i & 1;
                    uint4 v = make_uint4(0, 0, 0, 0);
                    if (n0 + r < p.N && b0 + j < p.nb)
                        v = __ldg((const uint4 *)(p.W + (n0 + r) * p.wstride + p.sbytes + (int64_t)(b0 + j) * 32 + h * 16));
                    *(uint4 *)(st + j * kWTile + core_off(r, h)) = v;
                }
            } else {
                for (int i = pt; i < MT * KS; i += 128) {  // one 16-byte nibble block: row, block
                    const int r = i / KS, j = i % KS;
                    uint4 v = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // -> 0
                    if (n0 + r < p.N && b0 + j < p.nb)
                        v = __ldg((const uint4 *)(p.W + (n0 + r) * p.wstride + p.sbytes + (int64_t)(b0 + j) * 16));
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                    uint32_t o[8];
#pragma unroll
                    for (int k = 0; k < 4; k++) {  // byte q holds element 2q (low nibble) and 2q + 1 (high)
                        const uint32_t lo = w[k] & 0x0f0f0f0fu, hi = (w[k] >> 4) & 0x0f0f0f0fu;
                        o[2 * k] = __vsub4(__byte_perm(lo, hi, 0x5140), 0x08080808u);
                        o[2 * k + 1] = __vsub4(__byte_perm(lo, hi, 0x7362), 0x08080808u);
                    }
                    *(uint4 *)(st + j * kWTile + core_off(r, 0)) = make_uint4(o[0], o[1], o[2], o[3]);
                    *(uint4 *)(st + j * kWTile + core_off(r, 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                }
            }
            {  // weight scales: row pt's KS fp16 scales are 8 aligned bytes
                float *dw = (float *)(st + kOffDw);
                uint2 v = make_uint2(0, 0);
                if (n0 + pt < p.N) v = __ldg((const uint2 *)(p.W + (n0 + pt) * p.wstride + 2 * b0));
                const uint32_t hw[4] = {v.x & 0xffffu, v.x >> 16, v.y & 0xffffu, v.y >> 16};
#pragma unroll
                for (int j = 0; j < KS; j++) dw[j * MT + pt] = b0 + j < p.nb ? h2f(hw[j]) : 0.0f;
            }
            for (int i = pt; i < NT * KS * 2; i += 128) {  // activation blocks
                const int r = i / (KS * 2), j = (i >> 1) % KS, h = i & 1;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (t0 + r < p.T && b0 + j < p.nb)
                    v = __ldg((const uint4 *)(p.aq + ((t0 + r) * p.nb + b0 + j) * 32 + h * 16));
                *(uint4 *)(st + kOffA + j * kATile + core_off(r, h)) = v;
            }
            if (pt < NT * KS) {  // activation scales
                const int r = pt / KS, j = pt % KS;
                float *da = (float *)(st + kOffDa);
                da[j * NT + r] = (t0 + r < p.T && b0 + j < p.nb) ? __ldg(p.ad + (t0 + r) * p.nb + b0 + j) : 0.0f;
            }
            fence_proxy_async();  // generic-proxy writes -> visible to the tensor core's reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
    } else if (warp == 0) {  // ---------------------------------------------------------------- MMA issuer
        int issued = 0;  // stages whose MMAs were committed
        if (lane == 0) {
            for (int g = 0; g < nst; g++) {
                const int s = g % NS, buf = g & 1;
                if (!mbar_wait(&full[s], (g / NS) & 1u) || (g >= 2 && !mbar_wait(&tempty[buf], ((g >> 1) - 1) & 1u))) {
                    raise_error(p.err, kErrMbarTimeout);
                    *dead = 1;
                    break;
                }
                if (*dead) break;
                tc_fence_after();
                const uint8_t *st = sm + s * kStage;
                const int nj = min(KS, p.nb - g * KS);
                for (int j = 0; j < nj; j++)
                    mma_i8(tmem + (uint32_t)((buf * KS + j) * NT), smem_desc(st + j * kWTile),
                           smem_desc(st + kOffA + j * kATile));
                mma_commit(&tfull[buf]);
                mma_commit(&empty[s]);
                issued = g + 1;
            }
            // the MMAs of the last committed stage must have completed before the TMEM is freed
            if (issued > 0) {
                const int g = issued - 1;
                if (!mbar_wait(&tfull[g & 1], (g >> 1) & 1u)) raise_error(p.err, kErrMbarTimeout);
            }
        }
        __syncwarp();
    } else {  // ---------------------------------------------------------------- epilogue (warps 1-4)
        const int q = warp & 3, row = 32 * q + lane;  // TMEM lane = weight row n0 + row
        float acc[NT];
#pragma unroll
        for (int c = 0; c < NT; c++) acc[c] = 0.0f;
        for (int g = 0; g < nst; g++) {
            const int s = g % NS, buf = g & 1;
            // warp-uniform verdicts: tcgen05.ld below is executed by the whole warp or not at all
            if (__any_sync(0xffffffffu, !mbar_wait(&tfull[buf], (g >> 1) & 1u))) {
                if (lane == 0) raise_error(p.err, kErrMbarTimeout);
                *dead = 1;
                break;
            }
            if (__any_sync(0xffffffffu, *dead != 0)) break;
            tc_fence_after();
            const uint8_t *st = sm + s * kStage;
            const float *dw = (const float *)(st + kOffDw), *da = (const float *)(st + kOffDa);
            const int nj = min(KS, p.nb - g * KS);
            for (int j = 0; j < nj; j++) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((buf * KS + j) * NT), r);
                const float wd = dw[j * MT + row];
#pragma unroll
                for (int c = 0; c < NT; c++)
                    acc[c] = __fadd_rn(acc[c], __fmul_rn((float)(int)r[c], __fmul_rn(wd, da[j * NT + c])));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tempty[buf]);
                mbar_arrive(&empty[s]);
            }
        }
        const int64_t n = n0 + row;
        if (!*dead && n < p.N) {
#pragma unroll
            for (int c = 0; c < NT; c++) {
                const int64_t tt = t0 + c;
                if (tt < p.T) {
                    if (p.C2) (n & 1 ? p.C2 : p.C)[tt * (p.N >> 1) + (n >> 1)] = acc[c];
                    else p.C[tt * p.N + n] = acc[c];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

}  // namespace

int launch_matmul_q_tc(int dtype, const void *Wsplit, int64_t wstride, const int8_t *aq, const float *ad, float *C,
                       float *C2, int64_t T, int64_t N, int64_t K, int *err, cudaStream_t s) {
    if (dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "matmul_q_tc: dtype must be Q8_0 or Q4_0");
    if (((uintptr_t)Wsplit & 15) || (wstride & 15) || ((uintptr_t)aq & 15))
        return set_error(QMC_EINVAL, "matmul_q_tc: operands must be 16-byte aligned");
    if (C2 && (N & 1)) return set_error(QMC_EINVAL, "matmul_q_tc: split output needs an even row count");
    if (T <= 0 || N <= 0) return QMC_OK;
    TcParams p;
    p.W = (const uint8_t *)Wsplit;
    p.wstride = wstride;
    p.sbytes = ((nblocks(K) * 2 + 15) / 16) * 16;
    p.aq = aq, p.ad = ad, p.C = C, p.C2 = C2, p.T = T, p.N = N, p.nb = (int)nblocks(K), p.err = err;
    auto fn = dtype == QMC_Q8_0 ? matmul_q_tc_kernel<QMC_Q8_0> : matmul_q_tc_kernel<QMC_Q4_0>;
    int dev = 0;
    QMC_CUDA(cudaGetDevice(&dev));
    static bool attr_done[64][2];
    if (dev < 0 || dev >= 64) return set_error(QMC_EINVAL, "matmul_q_tc: device %d out of range", dev);
    if (!attr_done[dev][dtype == QMC_Q4_0]) {
        QMC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
        attr_done[dev][dtype == QMC_Q4_0] = true;
    }
    dim3 grid((unsigned)((N + MT - 1) / MT), (unsigned)((T + NT - 1) / NT));
    fn<<<grid, kThreads, kSmem, s>>>(p);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

}  // namespace qmc
