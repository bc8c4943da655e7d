/* quillm-b200 dispatch surface (src/kernels.h:7-34): one descriptor, QM_ISA_CUDA.  Its entries take
 * host pointers like the reference's per-ISA kernels and compute on the GPU. */
#include "kernels.h"
#include "ops.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "hostgpu.h"

static float gpu_dot(int dt, const void *w, size_t wb, const void *x, size_t xb, int64_t n, const char *op) {
    float r = NAN;
    if (qh_begin() != 0) return r;
    void *dw = qh_put(0, w, wb), *dx = qh_put(1, x, xb), *dr = qh_slot(2, 4);
    if (!(dw && dx && dr && qmc_dot(dt, dw, dx, n, dr, NULL) == QMC_OK && !qh_get(&r, dr, 4) && !qh_finish())) {
        qh_fail(op);
        r = NAN;
    }
    qh_end();
    return r;
}

static float dot_f32_cuda(const float *a, const float *b, int64_t n) {
    if (n <= 0) return 0.0f;
    return gpu_dot(QM_F32, a, (size_t)n * 4, b, (size_t)n * 4, n, "dot_f32");
}

static float dot_q8_cuda(const qm_block_q8 *w, const qm_block_q8 *x, int64_t nb) {
    if (nb <= 0) return 0.0f;
    return gpu_dot(QM_Q8_0, w, (size_t)nb * 34, x, (size_t)nb * 34, nb * 32, "dot_q8");
}

static float dot_q4_cuda(const qm_block_q4 *w, const qm_block_q8 *x, int64_t nb) {
    if (nb <= 0) return 0.0f;
    return gpu_dot(QM_Q4_0, w, (size_t)nb * 18, x, (size_t)nb * 34, nb * 32, "dot_q4");
}

/* C[M,N] = A[M,K] B[N,K]^T with leading dimensions; strided operands are packed on the host first */
static void gemm_nt_cuda(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, int64_t lda,
                         int64_t ldb, int64_t ldc) {
    if (M <= 0 || N <= 0) return;
    float *a = (float *)A, *b = (float *)B, *c = malloc(sizeof(float) * (size_t)(M * N));
    if (lda != K) {
        a = malloc(sizeof(float) * (size_t)(M * K));
        for (int64_t i = 0; i < M; i++) memcpy(a + i * K, A + i * lda, (size_t)K * 4);
    }
    if (ldb != K) {
        b = malloc(sizeof(float) * (size_t)(N * K));
        for (int64_t j = 0; j < N; j++) memcpy(b + j * K, B + j * ldb, (size_t)K * 4);
    }
    qm_matmul_nt(NULL, a, b, c, M, N, K);
    for (int64_t i = 0; i < M; i++) memcpy(C + i * ldc, c + i * N, (size_t)N * 4);
    if (a != A) free(a);
    if (b != B) free(b);
    free(c);
}

const qm_kernels qm_kernels_cuda = {QM_ISA_CUDA, dot_f32_cuda, dot_q8_cuda, dot_q4_cuda, gemm_nt_cuda};

const qm_kernels *qm_kernels_for(qm_isa isa) { return (isa == QM_ISA_CUDA && qm_cpu_supports(isa)) ? &qm_kernels_cuda : NULL; }

int qm_kernels_select(qm_isa isa) { return qm_kernels_for(isa) ? 0 : -1; }

const qm_kernels *qm_kernels_active(void) { return &qm_kernels_cuda; }
