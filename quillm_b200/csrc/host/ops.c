/* quillm-b200 host ops: the reference's qm_* operator API (src/ops.h:9-34) over libquillm_cuda.
 * Host buffers in and out; the arithmetic runs on the GPU.  Tensors made resident with
 * qm_tensor_upload are read from HBM; other weights are copied to the device for the call. */
#include "ops.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "hostgpu.h"

/* ------------------------------------------------------------------ tensor helpers (src/ops.c:5-24) */
int64_t qm_tensor_nelem(const qm_tensor *t) {
    int64_t n = 1;
    for (int i = 0; i < t->ndim; i++) n *= t->ne[i];
    return n;
}

int64_t qm_tensor_cols(const qm_tensor *t) { return t->ndim > 0 ? t->ne[t->ndim - 1] : 1; }

int64_t qm_tensor_rows(const qm_tensor *t) {
    int64_t r = 1;
    for (int i = 0; i + 1 < t->ndim; i++) r *= t->ne[i];
    return r;
}

size_t qm_tensor_bytes(const qm_tensor *t) { return (size_t)qm_tensor_rows(t) * qm_row_bytes(t->type, qm_tensor_cols(t)); }

const void *qm_tensor_row(const qm_tensor *t, int64_t r) {
    return (const uint8_t *)t->data + (size_t)r * qm_row_bytes(t->type, qm_tensor_cols(t));
}

/* ------------------------------------------------------------------ resident tensors */
typedef struct {
    const void *host;
    size_t bytes;
    void *dev;
} resident;

#define MAX_RESIDENT 16384
static resident g_res[MAX_RESIDENT];
static int g_nres;
static pthread_mutex_t g_res_mu = PTHREAD_MUTEX_INITIALIZER;

const void *qh_resident(const void *host, size_t bytes) {
    const void *d = NULL;
    pthread_mutex_lock(&g_res_mu);
    for (int i = 0; i < g_nres; i++)
        if (g_res[i].host == host && g_res[i].bytes == bytes) {
            d = g_res[i].dev;
            break;
        }
    pthread_mutex_unlock(&g_res_mu);
    return d;
}

int qm_tensor_upload(const qm_tensor *W) {
    const size_t bytes = qm_tensor_bytes(W);
    if (qh_resident(W->data, bytes)) return 0;
    if (qh_begin() != 0) return -1;
    void *d = NULL;
    int rc = -1;
    if (qmc_malloc(&d, bytes + 256) == QMC_OK && qmc_memcpy_h2d(d, W->data, bytes, NULL) == QMC_OK && !qh_finish()) {
        pthread_mutex_lock(&g_res_mu);
        if (g_nres < MAX_RESIDENT) {
            g_res[g_nres++] = (resident){W->data, bytes, d};
            rc = 0;
        } else {
            qh_set_error("too many resident tensors");
        }
        pthread_mutex_unlock(&g_res_mu);
    } else {
        qh_fail("tensor upload");
    }
    if (rc && d) qmc_free(d);
    qh_end();
    return rc;
}

void qm_tensor_release(const qm_tensor *W) {
    const size_t bytes = qm_tensor_bytes(W);
    void *d = NULL;
    pthread_mutex_lock(&g_res_mu);
    for (int i = 0; i < g_nres; i++)
        if (g_res[i].host == W->data && g_res[i].bytes == bytes) {
            d = g_res[i].dev;
            g_res[i] = g_res[--g_nres];
            break;
        }
    pthread_mutex_unlock(&g_res_mu);
    if (d && qh_begin() == 0) {
        qmc_sync();
        qmc_free(d);
        qh_end();
    }
}

/* device view of a weight: the resident copy, else staged into `slot` */
static const void *weights_on_device(const qm_tensor *W, int slot) {
    const size_t bytes = qm_tensor_bytes(W);
    const void *d = qh_resident(W->data, bytes);
    return d ? d : qh_put(slot, W->data, bytes);
}

/* ------------------------------------------------------------------ matvec / matmul */
void qm_matvec(qm_pool *p, const qm_tensor *W, const float *x, float *y, qm_block_q8 *xq) {
    (void)p;
    const int64_t rows = qm_tensor_rows(W), cols = qm_tensor_cols(W);
    if (rows <= 0) return;
    if (qh_begin() != 0) {
        qh_fill_nan(y, (size_t)rows);
        return;
    }
    const int quant = W->type != QM_F32;
    const size_t xqb = (size_t)qm_nblocks(cols) * sizeof(qm_block_q8);
    const void *dw = weights_on_device(W, 0);
    void *dx = qh_put(1, x, (size_t)cols * 4), *dy = qh_slot(2, (size_t)rows * 4);
    void *dq = quant ? qh_slot(3, xqb) : NULL;
    int ok = dw && dx && dy && (!quant || dq) &&
             qmc_matvec((int)W->type, dw, rows, cols, dx, dy, dq, NULL) == QMC_OK && !qh_get(y, dy, (size_t)rows * 4) &&
             (!quant || !xq || !qh_get(xq, dq, xqb)) && !qh_finish();
    if (!ok) {
        qh_fail("qm_matvec");
        qh_fill_nan(y, (size_t)rows);
    }
    qh_end();
}

void qm_matmul_nt(qm_pool *p, const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K) {
    (void)p;
    if (M <= 0 || N <= 0) return;
    if (qh_begin() != 0) {
        qh_fill_nan(C, (size_t)(M * N));
        return;
    }
    const void *dB = qh_resident(B, (size_t)(N * K) * 4);
    if (!dB) dB = qh_put(1, B, (size_t)(N * K) * 4);
    void *dA = qh_put(0, A, (size_t)(M * K) * 4), *dC = qh_slot(2, (size_t)(M * N) * 4);
    int ok = dA && dB && dC && qmc_matmul_nt(dA, dB, dC, M, N, K, NULL) == QMC_OK &&
             !qh_get(C, dC, (size_t)(M * N) * 4) && !qh_finish();
    if (!ok) {
        qh_fail("qm_matmul_nt");
        qh_fill_nan(C, (size_t)(M * N));
    }
    qh_end();
}

void qm_matmul_nt_q(qm_pool *p, const qm_tensor *W, const float *A, float *C, int64_t T) {
    (void)p;
    const int64_t N = qm_tensor_rows(W), K = qm_tensor_cols(W);
    if (T <= 0 || N <= 0) return;
    if (qh_begin() != 0) {
        qh_fill_nan(C, (size_t)(T * N));
        return;
    }
    const void *dw = weights_on_device(W, 0);
    void *dA = qh_put(1, A, (size_t)(T * K) * 4), *dC = qh_slot(2, (size_t)(T * N) * 4);
    int ok = dw && dA && dC && qmc_matmul_nt_q((int)W->type, dw, dA, dC, T, N, K, NULL) == QMC_OK &&
             !qh_get(C, dC, (size_t)(T * N) * 4) && !qh_finish();
    if (!ok) {
        qh_fail("qm_matmul_nt_q");
        qh_fill_nan(C, (size_t)(T * N));
    }
    qh_end();
}

/* ------------------------------------------------------------------ elementwise (src/ops.c:93-133) */
void qm_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps) {
    if (n <= 0 || qh_begin() != 0) return;
    void *dx = qh_put(0, x, (size_t)n * 4), *dw = qh_put(1, w, (size_t)n * 4), *dy = qh_slot(2, (size_t)n * 4);
    if (!(dx && dw && dy && qmc_rmsnorm(dy, dx, dw, n, eps, NULL) == QMC_OK && !qh_get(out, dy, (size_t)n * 4) &&
          !qh_finish())) {
        qh_fail("qm_rmsnorm");
        qh_fill_nan(out, (size_t)n);
    }
    qh_end();
}

void qm_softmax(float *x, int64_t n) {
    if (n <= 0 || qh_begin() != 0) return;
    void *dx = qh_put(0, x, (size_t)n * 4);
    if (!(dx && qmc_softmax(dx, n, NULL) == QMC_OK && !qh_get(x, dx, (size_t)n * 4) && !qh_finish())) {
        qh_fail("qm_softmax");
        qh_fill_nan(x, (size_t)n);
    }
    qh_end();
}

void qm_rope(float *v, int64_t n_heads, int64_t head_dim, int64_t pos, float theta) {
    const size_t bytes = (size_t)(n_heads * head_dim) * 4;
    if (!bytes || qh_begin() != 0) return;
    void *dv = qh_put(0, v, bytes);
    if (!(dv && qmc_rope(dv, n_heads, head_dim, pos, theta, NULL) == QMC_OK && !qh_get(v, dv, bytes) && !qh_finish())) {
        qh_fail("qm_rope");
        qh_fill_nan(v, bytes / 4);
    }
    qh_end();
}

void qm_swiglu(float *gate, const float *up, int64_t n) {
    if (n <= 0 || qh_begin() != 0) return;
    void *dg = qh_put(0, gate, (size_t)n * 4), *du = qh_put(1, up, (size_t)n * 4);
    if (!(dg && du && qmc_swiglu(dg, du, n, NULL) == QMC_OK && !qh_get(gate, dg, (size_t)n * 4) && !qh_finish())) {
        qh_fail("qm_swiglu");
        qh_fill_nan(gate, (size_t)n);
    }
    qh_end();
}

/* ------------------------------------------------------------------ qm_pool (inline) */
struct qm_pool {
    int n;
};

qm_pool *qm_pool_create(int n_threads) {
    qm_pool *p = calloc(1, sizeof *p);
    if (p) p->n = n_threads < 1 ? 1 : n_threads;
    return p;
}

void qm_pool_destroy(qm_pool *p) { free(p); }

int qm_pool_size(const qm_pool *p) { return p ? p->n : 1; }

void qm_pool_run(qm_pool *p, int64_t n, int64_t grain, qm_task_fn fn, void *ctx) {
    (void)p;
    (void)grain;
    if (n > 0) fn(ctx, 0, n, 0);
}
