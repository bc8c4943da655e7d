// Prefill contractions: C[T,N] = A[T,K] . W[N,K]^T.
//
// matmul_q: quantized W (Q8_0/Q4_0).  Row t of C is defined as qm_matvec(W, A[t]) (A rows quantized to
// Q8_0), the semantics the reference gives a quantized matvec (src/ops.c:57-61).  64x64 output tiles,
// 256 threads x (4 rows x 4 tokens); K advances 4 blocks at a time through shared memory with W blocks
// decoded to int8 (Q4_0 nibbles become q - 8) and per-block scales beside them.  Each thread walks the
// blocks of its outputs in order and accumulates s += (float)acc * (dW * dX) with explicit rounding,
// the scalar kernel's exact sequence (src/kernels_scalar.c:12-34), so results equal the reference's
// scalar matvec bit for bit.
//
// gemm_f32: the f32 contract of qm_matmul_nt (src/ops.c:81-91), 64x64 tiles, 4x4 per thread.
#include "actquant.cuh"
#include "matmul.cuh"

namespace qmc {
namespace {

constexpr int TB = 64;     // tile edge (W rows and tokens)
constexpr int KB = 4;      // quant blocks per K step
constexpr int WS = KB * 8 + 1;  // padded row stride in 32-bit words

__global__ void quantize_act_kernel(const float *__restrict__ x, int64_t T, int64_t K, int8_t *__restrict__ qs,
                                    float *__restrict__ d, float *__restrict__ dT, int64_t ldT) {
    quant_rows_quads(
        T, K, [&](int64_t t, int64_t e0, float (&v)[8]) { load8_any(x + t * K, e0, K, v); }, qs, d, dT, ldT);
}

template <int DT>
__global__ void __launch_bounds__(256, 1) matmul_q_kernel(const uint8_t *__restrict__ W, const int8_t *__restrict__ aq,
                                                       const float *__restrict__ ad, float *__restrict__ C, int64_t T,
                                                       int64_t N, int64_t K) {
    __shared__ uint32_t ws[TB * WS], as[TB * WS];
    __shared__ float wd[TB][KB], adv[TB][KB];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t n0 = (int64_t)blockIdx.x * TB, t0 = (int64_t)blockIdx.y * TB;
    const int64_t nb = nblocks(K), rb = row_bytes(DT, K);
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

    for (int64_t b0 = 0; b0 < nb; b0 += KB) {
        {  // one (row, block) of W and one (token, block) of A per thread
            const int r = tid >> 2, kb = tid & 3;
            const int64_t n = n0 + r, b = b0 + kb;
            uint32_t words[8];
            float dw = 0.0f;
            if (n < N && b < nb) {
                const uint16_t *blk = (const uint16_t *)(W + n * rb + b * (DT == QMC_Q8_0 ? kQ8Bytes : kQ4Bytes));
                dw = h2f(blk[0]);
                if (DT == QMC_Q8_0) {
#pragma unroll
                    for (int i = 0; i < 8; i++) words[i] = (uint32_t)blk[1 + 2 * i] | ((uint32_t)blk[2 + 2 * i] << 16);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) {  // 4 packed bytes -> 8 elements (q - 8) as two int8x4 words
                        const uint32_t pk = (uint32_t)blk[1 + 2 * i] | ((uint32_t)blk[2 + 2 * i] << 16);
                        const uint32_t lo = pk & 0x0f0f0f0fu, hi = (pk >> 4) & 0x0f0f0f0fu;
                        // interleave: element 2j = lo byte j, 2j+1 = hi byte j
                        const uint32_t e0 = __byte_perm(lo, hi, 0x5140), e1 = __byte_perm(lo, hi, 0x7362);
                        words[2 * i] = __vsub4(e0, 0x08080808u);
                        words[2 * i + 1] = __vsub4(e1, 0x08080808u);
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) words[i] = 0u;
            }
#pragma unroll
            for (int i = 0; i < 8; i++) ws[r * WS + kb * 8 + i] = words[i];
            wd[r][kb] = dw;
            const int64_t t = t0 + r;
            float da = 0.0f;
            if (t < T && b < nb) {
                const uint32_t *src = (const uint32_t *)(aq + (t * nb + b) * 32);
#pragma unroll
                for (int i = 0; i < 8; i++) words[i] = src[i];
                da = ad[t * nb + b];
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) words[i] = 0u;
            }
#pragma unroll
            for (int i = 0; i < 8; i++) as[r * WS + kb * 8 + i] = words[i];
            adv[r][kb] = da;
        }
        __syncthreads();
        const int kmax = (int)(nb - b0 < KB ? nb - b0 : KB);
        for (int kb = 0; kb < kmax; kb++) {
            int ia[4][4];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) ia[i][j] = 0;
#pragma unroll
            for (int w = 0; w < 8; w++) {
                int wv[4], av[4];
#pragma unroll
                for (int i = 0; i < 4; i++) wv[i] = (int)ws[(ty + 16 * i) * WS + kb * 8 + w];
#pragma unroll
                for (int j = 0; j < 4; j++) av[j] = (int)as[(tx + 16 * j) * WS + kb * 8 + w];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) ia[i][j] = __dp4a(wv[i], av[j], ia[i][j]);
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn((float)ia[i][j],
                                                               __fmul_rn(wd[ty + 16 * i][kb], adv[tx + 16 * j][kb])));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int64_t n = n0 + ty + 16 * i, t = t0 + tx + 16 * j;
            if (n < N && t < T) C[t * N + n] = acc[i][j];
        }
}

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                       float *__restrict__ C, int64_t M, int64_t N, int64_t K) {
    __shared__ float as[16][TB + 1], bs[16][TB + 1];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * TB, n0 = (int64_t)blockIdx.x * TB;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += 16) {
        for (int e = tid; e < 16 * TB; e += 256) {
            const int kk = e & 15, r = e >> 4;
            as[kk][r] = (m0 + r < M && k0 + kk < K) ? A[(m0 + r) * K + k0 + kk] : 0.0f;
            bs[kk][r] = (n0 + r < N && k0 + kk < K) ? B[(n0 + r) * K + k0 + kk] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = as[kk][ty + 16 * i], b[i] = bs[kk][tx + 16 * i];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int64_t m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
            if (m < M && n < N) C[m * N + n] = acc[i][j];
        }
}

}  // namespace

int launch_quantize_act(const float *x, int64_t T, int64_t K, int8_t *qs, float *d, cudaStream_t s, float *dT,
                        int64_t ldT) {
    const int64_t grid = (T * nblocks(K) * 4 + 255) / 256;  // a thread per 8 elements (the loop covers the rest)
    quantize_act_kernel<<<(int)(grid < 65535 ? grid : 65535), 256, 0, s>>>(x, T, K, qs, d, dT, ldT);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_matmul_q(int dtype, const void *W, const int8_t *aq, const float *ad, float *C, int64_t T, int64_t N,
                    int64_t K, cudaStream_t s) {
    dim3 grid((unsigned)((N + TB - 1) / TB), (unsigned)((T + TB - 1) / TB));
    if (dtype == QMC_Q8_0) matmul_q_kernel<QMC_Q8_0><<<grid, 256, 0, s>>>((const uint8_t *)W, aq, ad, C, T, N, K);
    else if (dtype == QMC_Q4_0) matmul_q_kernel<QMC_Q4_0><<<grid, 256, 0, s>>>((const uint8_t *)W, aq, ad, C, T, N, K);
    else return set_error(QMC_EINVAL, "matmul_q: dtype must be Q8_0 or Q4_0");
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

int launch_gemm_f32(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, cudaStream_t s) {
    dim3 grid((unsigned)((N + TB - 1) / TB), (unsigned)((M + TB - 1) / TB));
    gemm_f32_kernel<<<grid, 256, 0, s>>>(A, B, C, M, N, K);
    QMC_LAUNCH_CHECK();
    return QMC_OK;
}

}  // namespace qmc
