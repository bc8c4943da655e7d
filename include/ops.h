/* quillm-b200 tensor type and ops.  Drop-in for the reference's src/ops.h:1-36: same qm_tensor layout
 * and op signatures, with host pointers in and out; each op runs on the GPU (libquillm_cuda). */
#ifndef QM_OPS_H
#define QM_OPS_H

#include "kernels.h"
#include "threadpool.h"

#pragma GCC visibility push(default)

/* row-major tensor; ne[0] is the outermost dimension (src/ops.h:9-15) */
typedef struct {
    char name[64];
    qm_dtype type;
    int ndim;
    int64_t ne[4];
    const void *data;
} qm_tensor;

int64_t qm_tensor_nelem(const qm_tensor *t);
int64_t qm_tensor_rows(const qm_tensor *t);
int64_t qm_tensor_cols(const qm_tensor *t);
size_t qm_tensor_bytes(const qm_tensor *t);
const void *qm_tensor_row(const qm_tensor *t, int64_t r);

/* y[rows] = W . x (src/ops.h:23-25).  Quantized W: x is quantized to Q8_0 on the GPU and the blocks
 * are written to xq (qm_nblocks(cols) blocks), as in the reference.  A W made resident with
 * qm_tensor_upload is read from HBM; otherwise its bytes are copied to the device for this call. */
void qm_matvec(qm_pool *p, const qm_tensor *W, const float *x, float *y, qm_block_q8 *xq);
/* C[M,N] = A[M,K] . B[N,K]^T, f32 (src/ops.h:26-27) */
void qm_matmul_nt(qm_pool *p, const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K);
/* prefill with a quantized (or f32) W: row t of C[T, rows(W)] equals qm_matvec(W, A[t]) */
void qm_matmul_nt_q(qm_pool *p, const qm_tensor *W, const float *A, float *C, int64_t T);

void qm_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps);
void qm_softmax(float *x, int64_t n);
void qm_rope(float *v, int64_t n_heads, int64_t head_dim, int64_t pos, float theta);
void qm_swiglu(float *gate, const float *up, int64_t n);

/* keep W's bytes resident in HBM (keyed by W->data) until qm_tensor_release; 0 on success */
int qm_tensor_upload(const qm_tensor *W);
void qm_tensor_release(const qm_tensor *W);

#pragma GCC visibility pop
#endif
