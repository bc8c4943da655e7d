/* quillm-b200 oracle harness -- TEST / BASELINE INFRASTRUCTURE ONLY.
 *
 * Compiled together with the UNMODIFIED reference sources (read in place by oracle/Makefile) into
 * oracle/_ref/libquillm_ref.so, so tests and bench.py's reference leg can drive the reference's own
 * public API (src/model.h:33-36, src/ops.h:23-34, src/kernels.h:30-34) from Python through ctypes.
 * The functions here only marshal arguments: every number they return is computed by reference code.
 */
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "model.h"
#include "sampler.h"

static double now_s(void) { /* CLOCK_MONOTONIC like src/main.c:10-14 */
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + (double)ts.tv_nsec * 1e-9;
}

int ref_isa_supported(int isa) { return qm_kernels_for((qm_isa)isa) != NULL; }
int ref_isa_select(int isa) { return qm_kernels_select((qm_isa)isa); }
int ref_isa_active(void) { return (int)qm_kernels_active()->isa; }
int ref_isa_best(void) { return (int)qm_cpu_best(); }

float ref_fp16_to_fp32(uint16_t h) { return qm_fp16_to_fp32(h); }
uint16_t ref_fp32_to_fp16(float f) { return qm_fp32_to_fp16(f); }

void ref_quantize_row(int dtype, const float *x, void *out, int64_t n) {
    if (dtype == QM_Q8_0) qm_quantize_row_q8(x, out, n);
    else qm_quantize_row_q4(x, out, n);
}

float ref_dot(int isa, int dtype, const void *w, const void *xq, const float *x, int64_t n) {
    const qm_kernels *k = qm_kernels_for((qm_isa)isa);
    if (!k) return 0.0f;
    if (dtype == QM_F32) return k->dot_f32(w, x, n);
    if (dtype == QM_Q8_0) return k->dot_q8(w, xq, qm_nblocks(n));
    return k->dot_q4(w, xq, qm_nblocks(n));
}

/* one pool per thread count, created on first use */
static qm_pool *pool_for(int n_threads) {
    static qm_pool *pools[257];
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (!pools[n_threads]) pools[n_threads] = qm_pool_create(n_threads);
    return pools[n_threads];
}

void ref_matvec(int dtype, const void *W, int64_t rows, int64_t cols, const float *x, float *y, void *xq,
                int n_threads) {
    qm_tensor t;
    memset(&t, 0, sizeof t);
    t.type = (qm_dtype)dtype;
    t.ndim = 2;
    t.ne[0] = rows;
    t.ne[1] = cols;
    t.data = W;
    qm_matvec(pool_for(n_threads), &t, x, y, xq);
}

/* the reference bench's timing method (bench/bench.c:25-38): best of 3 runs of >= min_time seconds */
double ref_matvec_time(int dtype, const void *W, int64_t rows, int64_t cols, const float *x, float *y, void *xq,
                       int n_threads, double min_time) {
    double best = 1e30;
    for (int r = 0; r < 3; r++) {
        int iters = 0;
        double t0 = now_s(), t;
        do {
            ref_matvec(dtype, W, rows, cols, x, y, xq, n_threads);
            iters++;
            t = now_s() - t0;
        } while (t < min_time);
        if (t / iters < best) best = t / iters;
    }
    return best;
}

void ref_matmul_nt(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, int n_threads) {
    qm_matmul_nt(pool_for(n_threads), A, B, C, M, N, K);
}

void *ref_model_load(const char *path, int n_threads, int max_seq, char *err, size_t errlen) {
    qm_model *m = malloc(sizeof *m);
    if (!m) return NULL;
    if (qm_model_load(m, path, n_threads, max_seq, err, errlen) != 0) {
        free(m);
        return NULL;
    }
    return m;
}

void ref_model_free(void *m) {
    if (!m) return;
    qm_model_free(m);
    free(m);
}

void ref_model_config(void *vm, int32_t cfg[7]) {
    qm_model *m = vm;
    int32_t c[7] = {m->cfg.dim, m->cfg.hidden_dim, m->cfg.n_layers, m->cfg.n_heads,
                    m->cfg.n_kv_heads, m->cfg.vocab_size, m->cfg.max_seq};
    memcpy(cfg, c, sizeof c);
}

const float *ref_model_forward(void *m, int32_t token, int32_t pos) { return qm_model_forward(m, token, pos); }

/* prompt fed one token at a time, then greedy decode (src/main.c:127-146 with temp 0 -> qm_argmax).
 * out_tokens receives n_gen generated ids; prompt/decode wall times in seconds. Returns 0 or -1. */
int ref_greedy_run(void *vm, const int32_t *prompt, int n_prompt, int n_gen, int32_t *out_tokens, double *prompt_s,
                   double *gen_s) {
    qm_model *m = vm;
    int V = m->cfg.vocab_size, pos = 0;
    float *lg = NULL;
    double t0 = now_s();
    for (int i = 0; i < n_prompt; i++, pos++)
        if (!(lg = qm_model_forward(m, prompt[i], pos))) return -1;
    double t1 = now_s();
    for (int i = 0; i < n_gen; i++, pos++) {
        int32_t tok = qm_argmax(lg, V);
        out_tokens[i] = tok;
        if (i + 1 < n_gen && !(lg = qm_model_forward(m, tok, pos))) return -1;
    }
    double t2 = now_s();
    if (prompt_s) *prompt_s = t1 - t0;
    if (gen_s) *gen_s = t2 - t1;
    return 0;
}

/* time n_steps decode forwards starting at pos0, each fed the previous greedy token (bench/bench.c:139-147) */
double ref_decode_time(void *vm, int32_t token, int32_t pos0, int n_steps, int32_t *last_token) {
    qm_model *m = vm;
    double t0 = now_s();
    for (int i = 0; i < n_steps; i++) {
        float *lg = qm_model_forward(m, token, pos0 + i);
        if (!lg) return -1.0;
        token = qm_argmax(lg, m->cfg.vocab_size);
    }
    double t = now_s() - t0;
    if (last_token) *last_token = token;
    return t;
}
