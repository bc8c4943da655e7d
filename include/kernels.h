/* quillm-b200 kernel dispatch surface: drop-in for the reference's src/kernels.h:7-38.
 * The only descriptor is the CUDA one (isa QM_ISA_CUDA).  Its entries take host pointers like the
 * reference's and run on the GPU; per-row dots are correct but pay a host<->device round trip each, the
 * whole-matrix ops in ops.h are the fast path. */
#ifndef QM_KERNELS_H
#define QM_KERNELS_H

#include "qm_base.h"

#pragma GCC visibility push(default)

typedef struct {
    qm_isa isa;
    float (*dot_f32)(const float *a, const float *b, int64_t n);
    float (*dot_q8)(const qm_block_q8 *w, const qm_block_q8 *x, int64_t nb);
    float (*dot_q4)(const qm_block_q4 *w, const qm_block_q8 *x, int64_t nb);
    void (*gemm_nt)(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, int64_t lda,
                    int64_t ldb, int64_t ldc);
} qm_kernels;

extern const qm_kernels qm_kernels_cuda;

/* the CUDA descriptor for QM_ISA_CUDA on a machine with a CUDA device, else NULL */
const qm_kernels *qm_kernels_for(qm_isa isa);
/* the CUDA descriptor (env QUILLM_ISA accepts only "cuda") */
const qm_kernels *qm_kernels_active(void);
/* 0 for QM_ISA_CUDA with a device present, -1 otherwise */
int qm_kernels_select(qm_isa isa);

/* kept for source compatibility (the reference's CPU GEMM blocking, src/kernels.h:37-38) */
#define QM_GEMM_NB 64
#define QM_GEMM_KC 256

#pragma GCC visibility pop
#endif
