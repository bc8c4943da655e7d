/* quillm-b200 host layer: scalar fp16 helpers, dtype metadata, GPU-backed row quantizers, arena, ISA
 * names and the device staging used by every host-pointer op (hostgpu.h). */
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "hostgpu.h"
#include "qm_base.h"

/* ------------------------------------------------------------------ errors */
static _Thread_local char g_err[512];

const char *qm_last_error(void) { return g_err; }

void qh_set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

void qh_fail(const char *op) {
    qh_set_error("%s: %s", op, qmc_last_error());
    fprintf(stderr, "quillm-b200: %s\n", g_err);
}

void qh_fill_nan(float *p, size_t n) {
    for (size_t i = 0; i < n; i++) p[i] = NAN;
}

/* ------------------------------------------------------------------ staging */
#define QH_MAX_DEV 64
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static void *g_buf[QH_MAX_DEV][QH_SLOTS];
static size_t g_cap[QH_MAX_DEV][QH_SLOTS];
static int g_dev = 0;

int qh_begin(void) {
    pthread_mutex_lock(&g_mu);
    int n = 0;
    if (qmc_device_count(&n) != QMC_OK || n <= 0) {
        qh_set_error("no CUDA device: the quillm-b200 ops run only on the GPU");
        fprintf(stderr, "quillm-b200: %s\n", g_err);
        pthread_mutex_unlock(&g_mu);
        return -1;
    }
    if (qmc_get_device(&g_dev) != QMC_OK || g_dev < 0 || g_dev >= QH_MAX_DEV || qmc_set_device(g_dev) != QMC_OK) {
        qh_fail("device setup");
        pthread_mutex_unlock(&g_mu);
        return -1;
    }
    return 0;
}

void qh_end(void) { pthread_mutex_unlock(&g_mu); }

void *qh_slot(int slot, size_t bytes) {
    if (bytes == 0) bytes = 16;
    bytes = (bytes + 255) & ~(size_t)255;
    if (g_cap[g_dev][slot] < bytes) {
        if (g_buf[g_dev][slot]) {
            qmc_sync();
            qmc_free(g_buf[g_dev][slot]);
            g_buf[g_dev][slot] = NULL;
            g_cap[g_dev][slot] = 0;
        }
        if (qmc_malloc(&g_buf[g_dev][slot], bytes + 256) != QMC_OK) {
            qh_fail("staging allocation");
            return NULL;
        }
        g_cap[g_dev][slot] = bytes;
    }
    return g_buf[g_dev][slot];
}

void *qh_put(int slot, const void *host, size_t bytes) {
    void *d = qh_slot(slot, bytes);
    if (!d) return NULL;
    if (bytes && qmc_memcpy_h2d(d, host, bytes, NULL) != QMC_OK) {
        qh_fail("host-to-device copy");
        return NULL;
    }
    return d;
}

int qh_get(void *host, const void *dev, size_t bytes) {
    if (bytes && qmc_memcpy_d2h(host, dev, bytes, NULL) != QMC_OK) {
        qh_fail("device-to-host copy");
        return -1;
    }
    return 0;
}

int qh_finish(void) {
    if (qmc_sync() != QMC_OK) {
        qh_fail("synchronize");
        return -1;
    }
    return 0;
}

/* ------------------------------------------------------------------ fp16 (IEEE binary16, RNE) */
float qm_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu, bits;
    if (ex == 0x1fu) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (ex) {
        bits = sign | ((ex - 15u + 127u) << 23) | (man << 13);
    } else if (!man) {
        bits = sign;
    } else { /* subnormal: shift the leading one into the implicit position */
        uint32_t e = 127u - 15u + 1u;
        while (!(man & 0x400u)) {
            man <<= 1;
            e--;
        }
        bits = sign | (e << 23) | ((man & 0x3ffu) << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

uint16_t qm_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t mag = x & 0x7fffffffu;
    if (mag > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((mag >> 13) & 0x3ffu)); /* NaN: quiet, keep payload */
    if (mag >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);                       /* overflow to infinity */
    if (mag >= 0x38800000u) {                                                        /* normal result */
        const uint32_t r = mag + 0x0fffu + ((mag >> 13) & 1u);
        return (uint16_t)(sign | ((r - ((uint32_t)(127 - 15) << 23)) >> 13));
    }
    const uint32_t e = mag >> 23;
    if (e < 127u - 25u) return sign; /* below half the smallest subnormal */
    const uint32_t man = (mag & 0x7fffffu) | 0x800000u, sh = 126u - e;
    uint32_t q = man >> sh;
    const uint32_t rest = man & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    if (rest > half || (rest == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/* ------------------------------------------------------------------ dtype metadata */
size_t qm_row_bytes(qm_dtype t, int64_t n) {
    switch (t) {
    case QM_F32: return (size_t)n * 4;
    case QM_Q8_0: return (size_t)qm_nblocks(n) * sizeof(qm_block_q8);
    case QM_Q4_0: return (size_t)qm_nblocks(n) * sizeof(qm_block_q4);
    }
    return 0;
}

const char *qm_dtype_name(qm_dtype t) {
    return t == QM_F32 ? "f32" : t == QM_Q8_0 ? "q8_0" : t == QM_Q4_0 ? "q4_0" : "?";
}

int qm_dtype_valid(uint32_t t) { return t == QM_F32 || t == QM_Q8_0 || t == QM_Q4_0; }

/* ------------------------------------------------------------------ row quantizers (GPU) */
static void quant_row(int dt, const float *x, void *y, int64_t n, const char *op) {
    if (n <= 0) return;
    const size_t ob = qm_row_bytes((qm_dtype)dt, n);
    if (qh_begin() != 0) {
        memset(y, 0xff, ob);
        return;
    }
    void *dx = qh_put(0, x, (size_t)n * 4), *dy = qh_slot(1, ob);
    if (!dx || !dy || qmc_quantize_rows(dt, dx, dy, 1, n, NULL) != QMC_OK || qh_get(y, dy, ob) || qh_finish()) {
        qh_fail(op);
        memset(y, 0xff, ob);
    }
    qh_end();
}

static void dequant_row(int dt, const void *x, float *y, int64_t n, const char *op) {
    if (n <= 0) return;
    if (qh_begin() != 0) {
        qh_fill_nan(y, (size_t)n);
        return;
    }
    void *dx = qh_put(0, x, qm_row_bytes((qm_dtype)dt, n)), *dy = qh_slot(1, (size_t)n * 4);
    if (!dx || !dy || qmc_dequantize_rows(dt, dx, dy, 1, n, NULL) != QMC_OK || qh_get(y, dy, (size_t)n * 4) ||
        qh_finish()) {
        qh_fail(op);
        qh_fill_nan(y, (size_t)n);
    }
    qh_end();
}

void qm_quantize_row_q8(const float *x, qm_block_q8 *y, int64_t n) { quant_row(QM_Q8_0, x, y, n, "quantize_row_q8"); }
void qm_quantize_row_q4(const float *x, qm_block_q4 *y, int64_t n) { quant_row(QM_Q4_0, x, y, n, "quantize_row_q4"); }
void qm_dequantize_row_q8(const qm_block_q8 *x, float *y, int64_t n) { dequant_row(QM_Q8_0, x, y, n, "dequantize_row_q8"); }
void qm_dequantize_row_q4(const qm_block_q4 *x, float *y, int64_t n) { dequant_row(QM_Q4_0, x, y, n, "dequantize_row_q4"); }
void qm_row_to_f32(qm_dtype t, const void *row, float *y, int64_t n) {
    if (t == QM_F32) memcpy(y, row, (size_t)n * 4);
    else dequant_row(t, row, y, n, "row_to_f32");
}

/* ------------------------------------------------------------------ arena */
int qm_arena_init(qm_arena *a, size_t cap) {
    cap = (cap + QM_ALIGN - 1) & ~(size_t)(QM_ALIGN - 1);
    if (!cap) cap = QM_ALIGN;
    a->base = aligned_alloc(QM_ALIGN, cap);
    if (!a->base) return -1;
    memset(a->base, 0, cap);
    a->cap = cap;
    a->used = a->peak = 0;
    return 0;
}

void *qm_arena_alloc(qm_arena *a, size_t n) {
    const size_t sz = (n + QM_ALIGN - 1) & ~(size_t)(QM_ALIGN - 1);
    if (sz < n || sz > a->cap - a->used) return NULL;
    void *p = a->base + a->used;
    a->used += sz;
    if (a->used > a->peak) a->peak = a->used;
    return p;
}

void qm_arena_reset(qm_arena *a) {
    memset(a->base, 0, a->used);
    a->used = 0;
}

void qm_arena_free(qm_arena *a) {
    free(a->base);
    a->base = NULL;
    a->cap = a->used = 0;
}

/* ------------------------------------------------------------------ ISA levels */
static const char *g_isa_names[QM_ISA_COUNT] = {"scalar", "avx2", "avx512", "neon", "cuda"};

int qm_cpu_supports(qm_isa isa) {
    if (isa != QM_ISA_CUDA) return 0;
    int n = 0;
    return qmc_device_count(&n) == QMC_OK && n > 0;
}

qm_isa qm_cpu_best(void) { return QM_ISA_CUDA; }

const char *qm_isa_name(qm_isa isa) { return (isa >= 0 && isa < QM_ISA_COUNT) ? g_isa_names[isa] : "?"; }

int qm_isa_from_name(const char *s) {
    for (int i = 0; i < QM_ISA_COUNT; i++)
        if (s && strcmp(s, g_isa_names[i]) == 0) return i;
    return -1;
}
