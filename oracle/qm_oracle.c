/* quillm-b200 CPU ORACLE -- TEST INFRASTRUCTURE ONLY (see qm_oracle.h).
 *
 * Each function restates one reference algorithm; the reference location is cited beside it
 * (paths relative to the reference project root).  Compiled with -ffp-contract=off so that every
 * float expression rounds exactly like the reference's -O2 x86-64 build (no FMA contraction).
 */
#include "qm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ fp16 (src/fp16.c:6-56) */
float orc_fp16_to_fp32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u, out;
    if (e == 31u) {
        out = s | 0x7f800000u | (m << 13); /* inf / NaN, payload kept */
    } else if (e != 0u) {
        out = s | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0u) {
        out = s;
    } else { /* subnormal half: value m * 2^-24, normalise */
        int k = 0;
        while (!(m & 1024u)) {
            m <<= 1;
            k++;
        }
        out = s | ((uint32_t)(113 - k) << 23) | ((m & 1023u) << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

uint16_t orc_fp32_to_fp16(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    uint16_t s = (uint16_t)((b >> 16) & 0x8000u);
    uint32_t a = b & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(s | 0x7e00u | ((a >> 13) & 0x3ffu)); /* quiet NaN, top payload */
    if (a >= 0x477ff000u) return (uint16_t)(s | 0x7c00u);                     /* rounds to +-inf */
    if (a >= 0x38800000u) {                                                    /* normal half */
        uint32_t lsb = (a >> 13) & 1u;
        return (uint16_t)(s | ((a + 0xfffu + lsb - 0x38000000u) >> 13));
    }
    uint32_t e = a >> 23;
    if (e < 102u) return s; /* below half of the smallest subnormal */
    uint32_t m = (a & 0x7fffffu) | 0x800000u, sh = 126u - e;
    uint32_t q = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(s | q);
}

/* ------------------------------------------------------------------ quantizers (src/quant.c:7-102) */
size_t orc_row_bytes(int dtype, int64_t n) {
    int64_t nb = (n + 31) / 32;
    return dtype == ORC_F32 ? (size_t)n * 4 : (size_t)nb * (dtype == ORC_Q8_0 ? 34u : 18u);
}

/* block scale: fp32 amax / qmax, stored as fp16, used as fp32(fp16) (quant.c:33-45) */
static float scale_of(const float v[32], float qmax, uint16_t *dh) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
        float a = fabsf(v[i]);
        if (a > amax) amax = a;
    }
    *dh = orc_fp32_to_fp16(amax / qmax);
    return orc_fp16_to_fp32(*dh);
}

/* q = clamp(rint(v / dd)) (quant.c:47-53) */
static int q_of(float v, float dd, int lo, int hi) {
    if (dd == 0.0f) return 0;
    float r = rintf(v / dd);
    if (r < (float)lo) r = (float)lo;
    if (r > (float)hi) r = (float)hi;
    return (int)r;
}

static void put_u16(uint8_t *p, uint16_t v) {
    p[0] = (uint8_t)(v & 0xff);
    p[1] = (uint8_t)(v >> 8);
}
static uint16_t get_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

void orc_quantize_row(int dtype, const float *x, void *out, int64_t n) {
    uint8_t *o = out;
    if (dtype == ORC_F32) {
        memcpy(o, x, (size_t)n * 4);
        return;
    }
    int64_t nb = (n + 31) / 32;
    for (int64_t b = 0; b < nb; b++) {
        float v[32];
        for (int i = 0; i < 32; i++) v[i] = (b * 32 + i < n) ? x[b * 32 + i] : 0.0f; /* zero tail (quant.c:28-31) */
        uint16_t dh;
        if (dtype == ORC_Q8_0) { /* quant.c:55-63 */
            uint8_t *blk = o + b * 34;
            float dd = scale_of(v, 127.0f, &dh);
            put_u16(blk, dh);
            for (int i = 0; i < 32; i++) blk[2 + i] = (uint8_t)(int8_t)q_of(v[i], dd, -127, 127);
        } else { /* quant.c:72-84 */
            uint8_t *blk = o + b * 18;
            float dd = scale_of(v, 7.0f, &dh);
            put_u16(blk, dh);
            for (int j = 0; j < 16; j++) {
                int lo = q_of(v[2 * j], dd, -8, 7) + 8, hi = q_of(v[2 * j + 1], dd, -8, 7) + 8;
                blk[2 + j] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

void orc_quantize_rows(int dtype, const float *x, void *out, int64_t rows, int64_t cols) {
    size_t rb = orc_row_bytes(dtype, cols);
    for (int64_t r = 0; r < rows; r++) orc_quantize_row(dtype, x + r * cols, (uint8_t *)out + (size_t)r * rb, cols);
}

/* quant.c:65-70, 86-94 */
void orc_dequantize_row(int dtype, const void *in, float *y, int64_t n) {
    const uint8_t *p = in;
    if (dtype == ORC_F32) {
        memcpy(y, p, (size_t)n * 4);
        return;
    }
    for (int64_t i = 0; i < n; i++) {
        int64_t b = i / 32;
        int k = (int)(i % 32);
        if (dtype == ORC_Q8_0) {
            const uint8_t *blk = p + b * 34;
            y[i] = orc_fp16_to_fp32(get_u16(blk)) * (float)(int8_t)blk[2 + k];
        } else {
            const uint8_t *blk = p + b * 18;
            int q = (k & 1) ? (blk[2 + k / 2] >> 4) : (blk[2 + k / 2] & 15);
            y[i] = orc_fp16_to_fp32(get_u16(blk)) * (float)(q - 8);
        }
    }
}

/* ------------------------------------------------------------------ scalar dots (src/kernels_scalar.c:6-34) */
float orc_dot_f32(const float *a, const float *b, int64_t n) {
    float s = 0.0f;
    for (int64_t i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

float orc_dot_q8(const void *w, const void *xq, int64_t nb) {
    const uint8_t *W = w, *X = xq;
    float s = 0.0f;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *wb = W + b * 34, *xb = X + b * 34;
        int32_t acc = 0;
        for (int i = 0; i < 32; i++) acc += (int32_t)(int8_t)wb[2 + i] * (int32_t)(int8_t)xb[2 + i];
        s += (float)acc * (orc_fp16_to_fp32(get_u16(wb)) * orc_fp16_to_fp32(get_u16(xb)));
    }
    return s;
}

float orc_dot_q4(const void *w, const void *xq, int64_t nb) {
    const uint8_t *W = w, *X = xq;
    float s = 0.0f;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *wb = W + b * 18, *xb = X + b * 34;
        int32_t acc = 0;
        for (int j = 0; j < 16; j++) {
            int lo = (wb[2 + j] & 15) - 8, hi = (wb[2 + j] >> 4) - 8;
            acc += lo * (int8_t)xb[2 + 2 * j] + hi * (int8_t)xb[2 + 2 * j + 1];
        }
        s += (float)acc * (orc_fp16_to_fp32(get_u16(wb)) * orc_fp16_to_fp32(get_u16(xb)));
    }
    return s;
}

/* ------------------------------------------------------------------ matvec (src/ops.c:36-61) */
void orc_matvec(int dtype, const void *W, int64_t rows, int64_t cols, const float *x, float *y, void *xq) {
    size_t rb = orc_row_bytes(dtype, cols);
    int64_t nb = (cols + 31) / 32;
    if (dtype != ORC_F32) orc_quantize_row(ORC_Q8_0, x, xq, cols);
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t *row = (const uint8_t *)W + (size_t)r * rb;
        if (dtype == ORC_F32) y[r] = orc_dot_f32((const float *)row, x, cols);
        else if (dtype == ORC_Q8_0) y[r] = orc_dot_q8(row, xq, nb);
        else y[r] = orc_dot_q4(row, xq, nb);
    }
}

/* float64 truth: integer block dots scaled in double (tests/test_kernels.c:205-220); f32 rows use the
 * double product sum (tests/test_kernels.c:178-182). */
void orc_matvec_exact(int dtype, const void *W, int64_t rows, int64_t cols, const float *x, const void *xq,
                      double *ref, double *abs_sum) {
    size_t rb = orc_row_bytes(dtype, cols);
    int64_t nb = (cols + 31) / 32;
    const uint8_t *X = xq;
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t *row = (const uint8_t *)W + (size_t)r * rb;
        double s = 0.0, a = 0.0;
        if (dtype == ORC_F32) {
            const float *w = (const float *)row;
            for (int64_t i = 0; i < cols; i++) {
                double t = (double)w[i] * (double)x[i];
                s += t;
                a += fabs(t);
            }
        } else {
            for (int64_t b = 0; b < nb; b++) {
                const uint8_t *xb = X + b * 34;
                long acc = 0;
                double dw;
                if (dtype == ORC_Q8_0) {
                    const uint8_t *wb = row + b * 34;
                    for (int i = 0; i < 32; i++) acc += (long)(int8_t)wb[2 + i] * (int8_t)xb[2 + i];
                    dw = orc_fp16_to_fp32(get_u16(wb));
                } else {
                    const uint8_t *wb = row + b * 18;
                    for (int i = 0; i < 32; i++) {
                        int q = ((wb[2 + i / 2] >> ((i & 1) * 4)) & 15) - 8;
                        acc += (long)q * (int8_t)xb[2 + i];
                    }
                    dw = orc_fp16_to_fp32(get_u16(wb));
                }
                double t = (double)acc * dw * (double)orc_fp16_to_fp32(get_u16(xb));
                s += t;
                a += fabs(t);
            }
        }
        ref[r] = s;
        abs_sum[r] = a;
    }
}

/* tests/test_kernels.c:13 (quantized dots are checked with n = nb * 8, tests/test_kernels.c:222-223) */
double orc_accum_tol(int64_t n, double abs_sum) { return 4.0 * (double)(n + 16) * 6e-8 * abs_sum + 1e-30; }

/* tests/test_kernels.c:246-253 */
void orc_gemm_exact(const float *A, const float *B, double *C, double *abs_sum, int64_t M, int64_t N, int64_t K) {
    for (int64_t i = 0; i < M; i++)
        for (int64_t j = 0; j < N; j++) {
            double s = 0.0, a = 0.0;
            for (int64_t k = 0; k < K; k++) {
                double t = (double)A[i * K + k] * (double)B[j * K + k];
                s += t;
                a += fabs(t);
            }
            C[i * N + j] = s;
            abs_sum[i * N + j] = a;
        }
}

void orc_matmul_q(int dtype, const void *W, int64_t N, int64_t K, const float *A, int64_t T, float *C) {
    uint8_t *xq = malloc(orc_row_bytes(ORC_Q8_0, K) + 64);
    for (int64_t t = 0; t < T; t++) orc_matvec(dtype, W, N, K, A + t * K, C + t * N, xq);
    free(xq);
}

/* ------------------------------------------------------------------ elementwise (src/ops.c:93-133) */
void orc_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps) {
    double ss = 0.0;
    for (int64_t i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
    for (int64_t i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

void orc_softmax(float *x, int64_t n) {
    if (n <= 0) return;
    float mx = x[0];
    for (int64_t i = 1; i < n; i++) mx = x[i] > mx ? x[i] : mx;
    double sum = 0.0;
    for (int64_t i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    float inv = (float)(1.0 / sum);
    for (int64_t i = 0; i < n; i++) x[i] *= inv;
}

void orc_rope(float *v, int64_t n_heads, int64_t head_dim, int64_t pos, float theta) {
    for (int64_t i = 0; i < head_dim / 2; i++) {
        double ang = (double)pos * pow((double)theta, -2.0 * (double)i / (double)head_dim);
        float c = (float)cos(ang), s = (float)sin(ang);
        for (int64_t h = 0; h < n_heads; h++) {
            float *p = v + h * head_dim + 2 * i;
            float a = p[0], b = p[1];
            p[0] = a * c - b * s;
            p[1] = a * s + b * c;
        }
    }
}

void orc_swiglu(float *gate, const float *up, int64_t n) {
    for (int64_t i = 0; i < n; i++) gate[i] = gate[i] / (1.0f + expf(-gate[i])) * up[i];
}

/* src/sampler.c:27-32: first maximum wins */
int32_t orc_argmax(const float *x, int32_t n) {
    int32_t best = 0;
    for (int32_t i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return best;
}

/* ------------------------------------------------------------------ .qlm reading (src/qlm_file.h:1-9) */
typedef struct {
    char name[64];
    int dtype, ndim;
    int64_t ne[4];
    const uint8_t *data;
} orc_tensor;

struct orc_model {
    uint8_t *file;
    size_t size;
    int32_t cfg[7]; /* dim hidden layers heads kv_heads vocab max_seq */
    float theta, eps;
    int n_t;
    orc_tensor *t;
    const orc_tensor *tok, *norm, *out;
    const orc_tensor **lay; /* [L][9]: attn_norm wq wk wv wo ffn_norm w1 w2 w3 */
    float *x, *xb, *xb2, *q, *hb, *hb2, *att, *logits, *kc, *vc;
    uint8_t *xq;
    int kv_f16;
};

static uint32_t rd32(const uint8_t *p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
static uint64_t rd64(const uint8_t *p) { return (uint64_t)rd32(p) | (uint64_t)rd32(p + 4) << 32; }

static const orc_tensor *find_t(const orc_model *m, const char *name, int64_t d0, int64_t d1) {
    for (int i = 0; i < m->n_t; i++)
        if (!strcmp(m->t[i].name, name)) {
            const orc_tensor *t = &m->t[i];
            if (d1 == 0 ? (t->ndim == 1 && t->ne[0] == d0 && t->dtype == ORC_F32)
                        : (t->ndim == 2 && t->ne[0] == d0 && t->ne[1] == d1))
                return t;
            return NULL;
        }
    return NULL;
}

#define OFAIL(...)                                                                                                     \
    do {                                                                                                               \
        snprintf(err, errlen, __VA_ARGS__);                                                                            \
        orc_model_close(m);                                                                                            \
        return NULL;                                                                                                   \
    } while (0)

orc_model *orc_model_open(const char *path, int max_seq, char *err, size_t errlen) {
    orc_model *m = calloc(1, sizeof *m);
    FILE *f = fopen(path, "rb");
    if (!f) OFAIL("cannot open %s", path);
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    m->size = (size_t)sz;
    m->file = malloc(m->size ? m->size : 1);
    size_t got = fread(m->file, 1, m->size, f);
    fclose(f);
    if (got != m->size || m->size < 24 || memcmp(m->file, "QLMF", 4) || rd32(m->file + 4) != 1) OFAIL("bad file");
    const uint8_t *p = m->file + 8, *end = m->file + m->size;
    uint32_t n_kv = rd32(p), n_t = rd32(p + 4);
    uint64_t data_off = rd64(p + 8);
    p += 16;
    m->theta = 10000.0f;
    m->eps = 1e-5f;
    static const char *keys[7] = {"llama.dim", "llama.hidden_dim", "llama.n_layers", "llama.n_heads",
                                  "llama.n_kv_heads", "llama.vocab_size", "llama.max_seq"};
    for (uint32_t i = 0; i < n_kv; i++) {
        if (p + 8 > end) OFAIL("truncated kv");
        uint32_t kl = rd32(p);
        char key[64] = {0};
        if (kl >= 64 || p + 4 + kl + 4 > end) OFAIL("bad key");
        memcpy(key, p + 4, kl);
        p += 4 + kl;
        uint32_t ty = rd32(p);
        p += 4;
        if (ty == 0 || ty == 1) {
            uint32_t v = rd32(p);
            for (int k = 0; k < 7; k++)
                if (ty == 0 && !strcmp(key, keys[k])) m->cfg[k] = (int32_t)v;
            if (ty == 1 && !strcmp(key, "llama.rope_theta")) memcpy(&m->theta, &v, 4);
            if (ty == 1 && !strcmp(key, "llama.norm_eps")) memcpy(&m->eps, &v, 4);
            p += 4;
        } else if (ty == 2) {
            p += 4 + rd32(p);
        } else if (ty == 3) {
            p += 4 + 4 * (size_t)rd32(p);
        } else {
            OFAIL("bad kv type");
        }
    }
    m->n_t = (int)n_t;
    m->t = calloc(n_t ? n_t : 1, sizeof(orc_tensor));
    for (uint32_t i = 0; i < n_t; i++) {
        orc_tensor *t = &m->t[i];
        uint32_t nl = rd32(p);
        if (nl >= 64) OFAIL("bad name");
        memcpy(t->name, p + 4, nl);
        p += 4 + nl;
        t->dtype = (int)rd32(p);
        t->ndim = (int)rd32(p + 4);
        p += 8;
        for (int d = 0; d < t->ndim && d < 4; d++, p += 8) t->ne[d] = (int64_t)rd64(p);
        t->data = m->file + data_off + rd64(p);
        p += 8;
    }
    int32_t *c = m->cfg;
    for (int k = 0; k < 7; k++)
        if (c[k] <= 0) OFAIL("missing %s", keys[k]);
    if (max_seq > 0 && max_seq < c[6]) c[6] = max_seq;
    int64_t D = c[0], H = c[1], L = c[2], hd = D / c[3], KV = hd * c[4], V = c[5], S = c[6];
    if (!(m->tok = find_t(m, "tok_embd", V, D)) || !(m->norm = find_t(m, "norm", D, 0)) ||
        !(m->out = find_t(m, "output", V, D)))
        OFAIL("missing top-level tensor");
    m->lay = calloc((size_t)L * 9, sizeof(*m->lay));
    static const char *nm[9] = {"attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w1", "w2", "w3"};
    int64_t sh[9][2] = {{D, 0}, {D, D}, {KV, D}, {KV, D}, {D, D}, {D, 0}, {H, D}, {D, H}, {H, D}};
    for (int64_t l = 0; l < L; l++)
        for (int k = 0; k < 9; k++) {
            char name[64];
            snprintf(name, sizeof name, "layers.%d.%s", (int)l, nm[k]);
            if (!(m->lay[l * 9 + k] = find_t(m, name, sh[k][0], sh[k][1]))) OFAIL("missing %s", name);
        }
    int64_t mx = D > H ? D : H;
    m->x = calloc((size_t)D, 4);
    m->xb = calloc((size_t)D, 4);
    m->xb2 = calloc((size_t)D, 4);
    m->q = calloc((size_t)D, 4);
    m->hb = calloc((size_t)H, 4);
    m->hb2 = calloc((size_t)H, 4);
    m->att = calloc((size_t)S, 4);
    m->logits = calloc((size_t)V, 4);
    m->kc = calloc((size_t)(L * S * KV), 4);
    m->vc = calloc((size_t)(L * S * KV), 4);
    m->xq = calloc((size_t)orc_row_bytes(ORC_Q8_0, mx) + 64, 1);
    if (!m->kc || !m->vc) OFAIL("out of memory");
    return m;
}

void orc_model_close(orc_model *m) {
    if (!m) return;
    free(m->file);
    free(m->t);
    free(m->lay);
    free(m->x), free(m->xb), free(m->xb2), free(m->q), free(m->hb), free(m->hb2), free(m->att);
    free(m->logits), free(m->kc), free(m->vc), free(m->xq);
    free(m);
}

void orc_model_set_kv_f16(orc_model *m, int on) { m->kv_f16 = on != 0; }

void orc_model_config(const orc_model *m, int32_t cfg[7], float fcfg[2]) {
    memcpy(cfg, m->cfg, sizeof m->cfg);
    fcfg[0] = m->theta;
    fcfg[1] = m->eps;
}

static void mv(orc_model *m, const orc_tensor *W, const float *x, float *y) {
    orc_matvec(W->dtype, W->data, W->ne[0], W->ne[1], x, y, m->xq);
}

/* src/model.c:158-191 with the attention of src/model.c:132-156 */
const float *orc_model_forward(orc_model *m, int32_t token, int32_t pos) {
    int32_t *c = m->cfg;
    if (token < 0 || token >= c[5] || pos < 0 || pos >= c[6]) return NULL;
    int64_t D = c[0], H = c[1], hd = D / c[3], KV = hd * c[4], S = c[6], grp = c[3] / c[4];
    orc_dequantize_row(m->tok->dtype, m->tok->data + (size_t)token * orc_row_bytes(m->tok->dtype, D), m->x, D);
    float scale = 1.0f / sqrtf((float)hd);
    for (int64_t l = 0; l < c[2]; l++) {
        const orc_tensor **L = m->lay + l * 9;
        float *kslot = m->kc + ((size_t)l * S + pos) * KV, *vslot = m->vc + ((size_t)l * S + pos) * KV;
        orc_rmsnorm(m->xb, m->x, (const float *)L[0]->data, D, m->eps);
        mv(m, L[1], m->xb, m->q);
        mv(m, L[2], m->xb, kslot);
        mv(m, L[3], m->xb, vslot);
        orc_rope(m->q, c[3], hd, pos, m->theta);
        orc_rope(kslot, c[4], hd, pos, m->theta);
        if (m->kv_f16)
            for (int64_t i = 0; i < KV; i++) {
                kslot[i] = orc_fp16_to_fp32(orc_fp32_to_fp16(kslot[i]));
                vslot[i] = orc_fp16_to_fp32(orc_fp32_to_fp16(vslot[i]));
            }
        const float *kl = m->kc + (size_t)l * S * KV, *vl = m->vc + (size_t)l * S * KV;
        for (int64_t h = 0; h < c[3]; h++) {
            int64_t g = h / grp;
            for (int32_t t = 0; t <= pos; t++) m->att[t] = orc_dot_f32(m->q + h * hd, kl + (size_t)t * KV + g * hd, hd) * scale;
            orc_softmax(m->att, pos + 1);
            float *o = m->xb + h * hd;
            for (int64_t i = 0; i < hd; i++) o[i] = 0.0f;
            for (int32_t t = 0; t <= pos; t++)
                for (int64_t i = 0; i < hd; i++) o[i] += m->att[t] * vl[(size_t)t * KV + g * hd + i];
        }
        mv(m, L[4], m->xb, m->xb2);
        for (int64_t i = 0; i < D; i++) m->x[i] += m->xb2[i];
        orc_rmsnorm(m->xb, m->x, (const float *)L[5]->data, D, m->eps);
        mv(m, L[6], m->xb, m->hb);
        mv(m, L[8], m->xb, m->hb2);
        orc_swiglu(m->hb, m->hb2, H);
        mv(m, L[7], m->hb, m->xb);
        for (int64_t i = 0; i < D; i++) m->x[i] += m->xb[i];
    }
    orc_rmsnorm(m->x, m->x, (const float *)m->norm->data, D, m->eps);
    mv(m, m->out, m->x, m->logits);
    return m->logits;
}

/* ------------------------------------------------------------------ synthetic models
 * The generator is this project's own definition (the reference ships none for N(0, std) weights).
 * Only +, -, *, / and sqrt appear, in a fixed order, so a device implementation that performs the
 * same IEEE double operations (no FMA contraction) produces identical bits. */
static uint64_t syn_fmix(uint64_t z) { /* splitmix64 finaliser (Steele, Lea, Flood 2014) */
    z ^= z >> 30;
    z *= 0xbf58476d1ce4e5b9ULL;
    z ^= z >> 27;
    z *= 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

/* natural log for x in (0, 1]: x = m * 2^e, m in [sqrt(1/2), sqrt(2)), log m = 2 atanh((m-1)/(m+1)) */
static double syn_log(double x) {
    uint64_t b;
    memcpy(&b, &x, 8);
    int e = (int)((b >> 52) & 0x7ff) - 1023;
    b = (b & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL;
    double m;
    memcpy(&m, &b, 8);
    if (m > 1.4142135623730951) {
        m = m * 0.5;
        e += 1;
    }
    double s = (m - 1.0) / (m + 1.0), s2 = s * s, p = 1.0 / 25.0;
    for (int k = 11; k >= 0; k--) p = 1.0 / (double)(2 * k + 1) + s2 * p;
    return (double)e * 0.6931471805599453 + 2.0 * s * p;
}

/* Acklam's rational approximation of the inverse standard normal CDF (relative error < 1.2e-9) */
static double syn_probit(double u) {
    static const double a[6] = {-3.969683028665376e+01, 2.209460984245205e+02, -2.759285104469687e+02,
                                1.383577518672690e+02, -3.066479806614716e+01, 2.506628277459239e+00};
    static const double b[5] = {-5.447609879822406e+01, 1.615858368580409e+02, -1.556989798598866e+02,
                                6.680131188771972e+01, -1.328068155288572e+01};
    static const double c[6] = {-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e+00,
                                -2.549732539343734e+00, 4.374664141464968e+00, 2.938163982698783e+00};
    static const double d[4] = {7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e+00,
                                3.754408661907416e+00};
    if (u < 0.02425 || u > 0.97575) {
        double t = sqrt(-2.0 * syn_log(u < 0.5 ? u : 1.0 - u));
        double num = ((((c[0] * t + c[1]) * t + c[2]) * t + c[3]) * t + c[4]) * t + c[5];
        double den = (((d[0] * t + d[1]) * t + d[2]) * t + d[3]) * t + 1.0;
        return u < 0.5 ? num / den : -(num / den);
    }
    double q = u - 0.5, r = q * q;
    double num = (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q;
    double den = ((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1.0;
    return num / den;
}

double orc_synth_normal(uint64_t seed, uint64_t tid, uint64_t idx) {
    uint64_t key = syn_fmix(seed ^ syn_fmix(tid + 0x632be59bd9b4e019ULL));
    uint64_t h = syn_fmix(key + idx * 0x9e3779b97f4a7c15ULL);
    double u = ((double)(h >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    return syn_probit(u);
}

void orc_synth_rows(uint64_t seed, uint64_t tid, int64_t r0, int64_t nrows, int64_t cols, double std, float *out) {
    for (int64_t r = 0; r < nrows; r++)
        for (int64_t c = 0; c < cols; c++)
            out[r * cols + c] = (float)(std * orc_synth_normal(seed, tid, (uint64_t)((r0 + r) * cols + c)));
}

typedef struct {
    uint64_t seed, tid;
    int64_t r0, r1, cols;
    int dtype;
    double std;
    uint8_t *dst;
} syn_job;

static void *syn_worker(void *arg) {
    syn_job *j = arg;
    size_t rb = orc_row_bytes(j->dtype, j->cols);
    float *row = malloc((size_t)j->cols * 4);
    for (int64_t r = j->r0; r < j->r1; r++) {
        orc_synth_rows(j->seed, j->tid, r, 1, j->cols, j->std, row);
        orc_quantize_row(j->dtype, row, j->dst + (size_t)(r - j->r0) * rb, j->cols);
    }
    free(row);
    return NULL;
}

static void w32(FILE *f, uint32_t v) {
    uint8_t b[4] = {(uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24)};
    fwrite(b, 1, 4, f);
}
static void w64(FILE *f, uint64_t v) {
    w32(f, (uint32_t)v);
    w32(f, (uint32_t)(v >> 32));
}
static void wstr(FILE *f, const char *s) {
    w32(f, (uint32_t)strlen(s));
    fwrite(s, 1, strlen(s), f);
}

/* layout written exactly as tools/qlm.py:94-132 (write_qlm) with the kvs of tools/qlm.py:246-251 */
int orc_synth_write(const char *path, const int32_t cfg[7], float rope_theta, float norm_eps, int dtype, uint64_t seed,
                    double std, int n_threads) {
    int64_t D = cfg[0], H = cfg[1], L = cfg[2], KV = cfg[0] / cfg[3] * cfg[4], V = cfg[5];
    int64_t nt = 3 + 9 * L;
    char (*names)[64] = calloc((size_t)nt, 64);
    int64_t(*shape)[2] = calloc((size_t)nt, sizeof(*shape));
    int k = 0;
    snprintf(names[k], 64, "tok_embd"), shape[k][0] = V, shape[k][1] = D, k++;
    static const char *nm[9] = {"attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w1", "w2", "w3"};
    int64_t sh[9][2] = {{D, 0}, {D, D}, {KV, D}, {KV, D}, {D, D}, {D, 0}, {H, D}, {D, H}, {H, D}};
    for (int64_t l = 0; l < L; l++)
        for (int j = 0; j < 9; j++, k++) {
            snprintf(names[k], 64, "layers.%d.%s", (int)l, nm[j]);
            shape[k][0] = sh[j][0];
            shape[k][1] = sh[j][1];
        }
    snprintf(names[k], 64, "norm"), shape[k][0] = D, shape[k][1] = 0, k++;
    snprintf(names[k], 64, "output"), shape[k][0] = V, shape[k][1] = D, k++;

    FILE *f = fopen(path, "wb");
    if (!f) {
        free(names), free(shape);
        return -1;
    }
    /* header body first, to know data_off */
    char *hb = NULL;
    size_t hlen = 0;
    FILE *h = open_memstream(&hb, &hlen);
    wstr(h, "general.name"), w32(h, 2), wstr(h, "quillm-synth");
    static const char *ck[7] = {"llama.dim", "llama.hidden_dim", "llama.n_layers", "llama.n_heads",
                                "llama.n_kv_heads", "llama.vocab_size", "llama.max_seq"};
    for (int j = 0; j < 7; j++) wstr(h, ck[j]), w32(h, 0), w32(h, (uint32_t)cfg[j]);
    uint32_t tb, eb;
    memcpy(&tb, &rope_theta, 4);
    memcpy(&eb, &norm_eps, 4);
    wstr(h, "llama.rope_theta"), w32(h, 1), w32(h, tb);
    wstr(h, "llama.norm_eps"), w32(h, 1), w32(h, eb);
    uint64_t off = 0;
    uint64_t *offs = calloc((size_t)nt, 8);
    for (int64_t t = 0; t < nt; t++) {
        int two = shape[t][1] != 0;
        int dt = two ? dtype : ORC_F32;
        uint64_t bytes = two ? (uint64_t)shape[t][0] * orc_row_bytes(dt, shape[t][1]) : (uint64_t)shape[t][0] * 4;
        offs[t] = off;
        off += (bytes + 63) / 64 * 64;
        wstr(h, names[t]);
        w32(h, (uint32_t)dt), w32(h, two ? 2u : 1u);
        w64(h, (uint64_t)shape[t][0]);
        if (two) w64(h, (uint64_t)shape[t][1]);
        w64(h, offs[t]);
    }
    fclose(h);
    uint64_t data_off = (24 + hlen + 63) / 64 * 64;
    fwrite("QLMF", 1, 4, f), w32(f, 1), w32(f, 10), w32(f, (uint32_t)nt), w64(f, data_off);
    fwrite(hb, 1, hlen, f);
    for (uint64_t i = 24 + hlen; i < data_off; i++) fputc(0, f);
    free(hb);

    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    const int64_t chunk_rows_max = 1 << 14;
    int rc = 0;
    for (int64_t t = 0; t < nt && !rc; t++) {
        int64_t rows = shape[t][0], cols = shape[t][1];
        if (cols == 0) { /* norm weights: 1.0 */
            float one = 1.0f;
            for (int64_t i = 0; i < rows; i++) fwrite(&one, 4, 1, f);
            uint64_t pad = (uint64_t)(rows * 4 + 63) / 64 * 64 - (uint64_t)rows * 4;
            for (uint64_t i = 0; i < pad; i++) fputc(0, f);
            continue;
        }
        size_t rb = orc_row_bytes(dtype, cols);
        int64_t chunk = chunk_rows_max < rows ? chunk_rows_max : rows;
        uint8_t *buf = malloc(rb * (size_t)chunk);
        for (int64_t r0 = 0; r0 < rows; r0 += chunk) {
            int64_t n = rows - r0 < chunk ? rows - r0 : chunk;
            pthread_t th[256];
            syn_job jobs[256];
            int used = 0;
            for (int w = 0; w < n_threads; w++) {
                int64_t a = r0 + n * w / n_threads, b = r0 + n * (w + 1) / n_threads;
                if (a >= b) continue;
                jobs[used] = (syn_job){seed, (uint64_t)t, a, b, cols, dtype, std, buf + (size_t)(a - r0) * rb};
                pthread_create(&th[used], NULL, syn_worker, &jobs[used]);
                used++;
            }
            for (int w = 0; w < used; w++) pthread_join(th[w], NULL);
            if (fwrite(buf, rb, (size_t)n, f) != (size_t)n) rc = -1;
        }
        uint64_t bytes = (uint64_t)rows * rb, pad = (bytes + 63) / 64 * 64 - bytes;
        for (uint64_t i = 0; i < pad; i++) fputc(0, f);
        free(buf);
    }
    if (fclose(f) != 0) rc = -1;
    free(offs), free(names), free(shape);
    return rc;
}
