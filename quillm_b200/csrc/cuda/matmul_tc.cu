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
// Operands reach shared memory by TMA (cp.async.bulk.tensor), issued by one producer lane up to NS
// stages ahead.  A stage holds KS = 4 blocks, i.e. 128 bytes of int8 per row: one TMA box per operand
// lands [rows][128 bytes] with the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r & 7)),
// which is the canonical K-major SWIZZLE_128B layout the MMA reads (8-row groups 1024 bytes apart); the
// MMA of block j starts 32 bytes into the rows.  Q4_0 payloads (16 bytes of nibbles per block) land raw
// ([rows][64 bytes]) and four converter warps expand them to int8 in the same swizzled layout.  The weight
// scales (the split row's leading fp16 array) and the block-major activation scales arrive by TMA too.
//
// CTA roles: warp 0 allocates TMEM and one lane issues the MMAs; warps 1-4 are the epilogue (warp w may
// read TMEM lanes 32 (w % 4) .. + 31, the weight rows of that quarter); warp 5 lane 0 issues the TMA
// copies; warps 6-9 (Q4_0 only) convert.  Barriers: tma_full (transaction bytes), full (Q4_0: converted),
// empty (MMA commit + epilogue warps), tmem_full / tmem_empty for two TMEM buffers.  Every wait is
// bounded; after a timeout a role stops, raises the error word and falls through to the end, where the
// producer waits (bounded) for its copies in flight, the MMA lane for the MMAs it issued, and warp 0 frees
// the TMEM it holds.
#include <cuda.h>

#include <mutex>

#include "matmul_tc.cuh"

namespace qmc {
namespace {

constexpr int MT = 128;  // weight rows per CTA (MMA M: TMEM lanes)
constexpr int NT = 32;   // tokens per CTA (MMA N)
constexpr int KS = 4;    // blocks per stage
// stages in the ring: 4 for Q8_0; 3 for Q4_0, whose stages also hold the raw nibbles, so that two CTAs
// still fit on an SM
template <int DT>
__host__ __device__ constexpr int ring() {
    return DT == QMC_Q4_0 ? 3 : 4;
}
constexpr int kTmemCols = 2 * KS * NT;  // two buffers of KS block tiles (power of 2, >= 32)
static_assert(kTmemCols == 256, "TMEM allocation size");

// stage layout (bytes, 1024-aligned tiles): int8 weight tile [MT][128] and activation tile [NT][128]
// (swizzled), weight scales [MT][16] (8 blocks' fp16 scales per row; this stage's 4 at byte 8 (g & 1)),
// activation scales [KS][NT] floats, then (Q4_0) the raw nibble payloads [MT][64]
constexpr int kRow = KS * 32;  // int8 bytes of a row per stage (the 128-byte swizzle span)
static_assert(kRow == 128, "one stage is one 128-byte swizzle atom wide");
constexpr int kOffA = MT * kRow, kOffDw = kOffA + NT * kRow, kOffDa = kOffDw + MT * 16;
constexpr int kOffRaw = kOffDa + KS * NT * 4;
template <int DT>
__host__ __device__ constexpr int stage_bytes() {
    return ((DT == QMC_Q4_0 ? kOffRaw + MT * KS * 16 : kOffRaw) + 1023) / 1024 * 1024;
}
template <int DT>
__host__ __device__ constexpr int warps() {
    return DT == QMC_Q4_0 ? 10 : 6;
}
template <int DT>
__host__ __device__ constexpr int smem_bytes() {
    return 1024 + ring<DT>() * stage_bytes<DT>() + (3 * ring<DT>() + 4) * 8 + 16;  // + slack to align the tiles
}
static_assert(kOffA % 1024 == 0 && kOffRaw % 128 == 0, "stage alignment");
// transaction bytes of one stage's TMA copies
template <int DT>
__host__ __device__ constexpr uint32_t stage_tx() {
    return (DT == QMC_Q4_0 ? MT * KS * 16 : MT * kRow) + NT * kRow + MT * 16 + KS * NT * 4;
}

// K-major SWIZZLE_128B descriptor: start (32 bytes further per block inside the atom), LBO 16 bytes
// (unused by the swizzled K-major form), SBO 1024 (8-row groups of 128-byte rows), version 1
__device__ __forceinline__ uint64_t smem_desc(const void *p) {
    const uint64_t a = (smem_u32(p) >> 4) & 0x3fffu;
    return a | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
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

// 2-D tiled TMA load of box (x, y) of the map into shared memory, completing on bar
__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 32 consecutive TMEM columns of this thread's lane
// The load and its wait are one asm statement: the registers it outputs exist only once the wait is
// done.  (With the wait as a separate statement nothing ties the registers to it, and the compiler may
// schedule arithmetic on them between the two -- reading registers the load has not yet written.)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

struct TcParams {
    int sbytes;     // bytes of a split row's scale array (the payload starts there)
    float *C, *C2;  // C[T][N]; with C2: weight row 2i -> C[t][i], 2i + 1 -> C2[t][i] (N / 2 columns each)
    int64_t T, N;
    int nb;
    int *err;
};

template <int DT>
__global__ void __launch_bounds__(32 * warps<DT>(), 2)
    matmul_q_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap dwmap,
                       const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap smap,
                       const TcParams p) {
    constexpr int SB = stage_bytes<DT>(), NS = ring<DT>();
    extern __shared__ __align__(128) uint8_t sm_raw[];
    uint8_t *sm = sm_raw + ((1024 - (smem_u32(sm_raw) & 1023)) & 1023);  // swizzled tiles: 1024-aligned
    uint64_t *tfull_s = (uint64_t *)(sm + NS * SB), *full = tfull_s + NS, *empty = full + NS, *tfull = empty + NS,
             *tempty = tfull + 2;
    volatile uint32_t *tmem_slot = (volatile uint32_t *)(tempty + 2);
    volatile int *dead = (volatile int *)(tmem_slot + 1);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int n0 = (int)blockIdx.x * MT, t0 = (int)blockIdx.y * NT;
    const int nst = (p.nb + KS - 1) / KS;

    if (t == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&tfull_s[s], 1);    // the producer's expect_tx arrival (+ the copies' bytes)
            mbar_init(&full[s], 4);       // Q4_0: one arrival per converter warp
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
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32((const void *)tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 5) {  // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            int issued = 0;
            for (int g = 0; g < nst; g++) {
                const int s = g % NS;
                if (g >= NS && !mbar_wait(&empty[s], ((g / NS) - 1) & 1u)) {
                    raise_error(p.err, kErrMbarTimeout);
                    *dead = 1;
                    break;
                }
                if (*dead) break;
                uint8_t *st = sm + s * SB;
                const int b0 = g * KS;
                mbar_arrive_tx(&tfull_s[s], stage_tx<DT>());
                if (DT == QMC_Q8_0) tma_2d(st, &wmap, p.sbytes + b0 * 32, n0, &tfull_s[s]);  // [MT][128], swizzled
                else tma_2d(st + kOffRaw, &wmap, p.sbytes + b0 * 16, n0, &tfull_s[s]);      // [MT][64] raw
                tma_2d(st + kOffA, &amap, b0 * 32, t0, &tfull_s[s]);            // [NT][128], swizzled
                tma_2d(st + kOffDw, &dwmap, 16 * (g >> 1), n0, &tfull_s[s]);  // 8 blocks' weight scales per row
                tma_2d(st + kOffDa, &smap, t0, b0, &tfull_s[s]);             // [KS blocks][NT tokens]
                issued = g + 1;
            }
            // no copy may still be landing when the CTA exits: wait (bounded) for the last stages issued
            const long long td = clock64();
            for (int g = issued - 1; g >= 0 && g >= issued - NS; g--)
                if (!mbar_wait_since(&tfull_s[g % NS], (g / NS) & 1u, td)) {
                    raise_error(p.err, kErrMbarTimeout);
                    break;
                }
        }
        __syncwarp();
    } else if (warp >= 6) {  // ---------------------------------------------------------------- Q4_0 converters
        const int r = t - 6 * 32;  // weight row of the tile, 0..127
        for (int g = 0; g < nst; g++) {
            const int s = g % NS;
            if (__any_sync(0xffffffffu, !mbar_wait(&tfull_s[s], (g / NS) & 1u))) {
                if (lane == 0) raise_error(p.err, kErrMbarTimeout);
                *dead = 1;
                break;
            }
            if (__any_sync(0xffffffffu, *dead != 0)) break;
            uint8_t *st = sm + s * SB;
#pragma unroll
            for (int j = 0; j < KS; j++) {
                const uint4 v = *(const uint4 *)(st + kOffRaw + r * (KS * 16) + j * 16);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                uint32_t o[8];
#pragma unroll
                for (int k = 0; k < 4; k++) {  // byte q holds element 2q (low nibble) and 2q + 1 (high)
                    const uint32_t lo = w[k] & 0x0f0f0f0fu, hi = (w[k] >> 4) & 0x0f0f0f0fu;
                    o[2 * k] = __vsub4(__byte_perm(lo, hi, 0x5140), 0x08080808u);
                    o[2 * k + 1] = __vsub4(__byte_perm(lo, hi, 0x7362), 0x08080808u);
                }
                // chunks 2j, 2j + 1 of row r, at their 128-byte-swizzle positions
                *(uint4 *)(st + r * kRow + (((2 * j) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                *(uint4 *)(st + r * kRow + (((2 * j + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
            }
            fence_proxy_async();  // generic-proxy writes -> visible to the tensor core's reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
    } else if (warp == 0) {  // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int issued = 0;  // stages whose MMAs were committed
            for (int g = 0; g < nst; g++) {
                const int s = g % NS, buf = g & 1;
                uint64_t *ready = DT == QMC_Q4_0 ? &full[s] : &tfull_s[s];
                if (!mbar_wait(ready, (g / NS) & 1u) || (g >= 2 && !mbar_wait(&tempty[buf], ((g >> 1) - 1) & 1u))) {
                    raise_error(p.err, kErrMbarTimeout);
                    *dead = 1;
                    break;
                }
                if (*dead) break;
                tc_fence_after();
                const uint8_t *st = sm + s * SB;
                const int nj = min(KS, p.nb - g * KS);
                for (int j = 0; j < nj; j++)
                    mma_i8(tmem + (uint32_t)((buf * KS + j) * NT), smem_desc(st + j * 32), smem_desc(st + kOffA + j * 32));
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
            const uint8_t *st = sm + s * SB;
            const uint2 wsc = *(const uint2 *)(st + kOffDw + row * 16 + 8 * (g & 1));  // this stage's 4 scales
            const uint32_t hw[4] = {wsc.x & 0xffffu, wsc.x >> 16, wsc.y & 0xffffu, wsc.y >> 16};
            const float *da = (const float *)(st + kOffDa);
            const int nj = min(KS, p.nb - g * KS);
#pragma unroll
            for (int j = 0; j < KS; j++) {
                if (j < nj) {
                    uint32_t r[32];
                    tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((buf * KS + j) * NT), r);
                    const float wd = h2f(hw[j]);
#pragma unroll
                    for (int c = 0; c < NT; c++)
                        acc[c] = __fadd_rn(acc[c], __fmul_rn((float)(int)r[c], __fmul_rn(wd, da[j * NT + c])));
                }
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

// ---------------------------------------------------------------- tensor maps (driver entry point)
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiled)f;
    });
    return fn;
}
// 2-D row-major map: `cols` elements per row, `rows` rows `pitch` bytes apart; boxes of box_cols x
// box_rows elements, optionally 128-byte swizzled; elements outside the matrix read as zero
int make_map(CUtensorMap *m, const void *base, CUtensorMapDataType type, int64_t cols, int64_t rows, int64_t pitch,
             int box_cols, int box_rows, bool swizzle = false) {
    EncodeTiled fn = encode_fn();
    if (!fn) return set_error(QMC_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows}, strides[1] = {(cuuint64_t)pitch};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows}, estr[2] = {1, 1};
    const CUresult r = fn(m, type, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(QMC_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QMC_OK;
}

template <int DT>
int launch_t(const CUtensorMap &wmap, const CUtensorMap &dwmap, const CUtensorMap &amap, const CUtensorMap &smap,
             const TcParams &p, cudaStream_t s) {
    int dev = 0;
    QMC_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(QMC_EINVAL, "matmul_q_tc: device %d out of range", dev);
    static bool attr_done[64];
    if (!attr_done[dev]) {
        QMC_CUDA(cudaFuncSetAttribute(matmul_q_tc_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes<DT>()));
        attr_done[dev] = true;
    }
    const dim3 grid((unsigned)((p.N + MT - 1) / MT), (unsigned)((p.T + NT - 1) / NT));
    matmul_q_tc_kernel<DT><<<grid, 32 * warps<DT>(), smem_bytes<DT>(), s>>>(wmap, dwmap, amap, smap, p);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

}  // namespace

int64_t matmul_tc_scale_ld(int64_t T) { return (T + 3) / 4 * 4; }

int launch_matmul_q_tc(int dtype, const void *Wsplit, int64_t wstride, const int8_t *aq, const float *adT, float *C,
                       float *C2, int64_t T, int64_t N, int64_t K, int *err, cudaStream_t s) {
    if (dtype != QMC_Q8_0 && dtype != QMC_Q4_0) return set_error(QMC_EINVAL, "matmul_q_tc: dtype must be Q8_0 or Q4_0");
    if (((uintptr_t)Wsplit & 15) || (wstride & 15) || ((uintptr_t)aq & 15) || ((uintptr_t)adT & 15))
        return set_error(QMC_EINVAL, "matmul_q_tc: operands must be 16-byte aligned");
    if (C2 && (N & 1)) return set_error(QMC_EINVAL, "matmul_q_tc: split output needs an even row count");
    if (T <= 0 || N <= 0) return QMC_OK;
    const int64_t nb = nblocks(K);
    if (wstride > INT32_MAX || N > INT32_MAX || T > INT32_MAX) return set_error(QMC_EINVAL, "matmul_q_tc: too large");
    TcParams p;
    p.sbytes = (int)(((nb * 2 + 15) / 16) * 16);
    p.C = C, p.C2 = C2, p.T = T, p.N = N, p.nb = (int)nb, p.err = err;
    CUtensorMap wmap, dwmap, amap, smap;
    const bool q8 = dtype == QMC_Q8_0;
    int rc;
    if ((rc = make_map(&wmap, Wsplit, CU_TENSOR_MAP_DATA_TYPE_UINT8, wstride, N, wstride, q8 ? 128 : KS * 16, MT, q8)) ||
        (rc = make_map(&dwmap, Wsplit, CU_TENSOR_MAP_DATA_TYPE_UINT8, wstride, N, wstride, 16, MT)) ||
        (rc = make_map(&amap, aq, CU_TENSOR_MAP_DATA_TYPE_UINT8, nb * 32, T, nb * 32, 128, NT, true)) ||
        (rc = make_map(&smap, adT, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, T, nb, matmul_tc_scale_ld(T) * 4, NT, KS)))
        return rc;
    return q8 ? launch_t<QMC_Q8_0>(wmap, dwmap, amap, smap, p, s) : launch_t<QMC_Q4_0>(wmap, dwmap, amap, smap, p, s);
}

}  // namespace qmc
