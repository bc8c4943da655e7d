/* quillm-b200 core types: dtypes, quantization blocks, fp16, arena, ISA levels.
 * Drop-in for the reference's src/qm_base.h:1-66 (same names, values, block layouts and signatures);
 * in this build every compute entry point runs on the GPU through libquillm_cuda. */
#ifndef QM_BASE_H
#define QM_BASE_H

#include <stddef.h>
#include <stdint.h>

#pragma GCC visibility push(default)

#define QM_ALIGN 64
#define QM_BLOCK 32 /* elements per quantization block */

typedef enum {
    QM_F32 = 0,
    QM_Q8_0 = 2, /* 32 int8 + fp16 scale: 34 bytes */
    QM_Q4_0 = 3, /* 32 nibbles (offset 8) + fp16 scale: 18 bytes */
} qm_dtype;

/* the .qlm block layouts (src/qm_base.h:17-29): value = d * qs[i] / d * (nibble - 8) */
typedef struct {
    uint16_t d;
    int8_t qs[32];
} qm_block_q8;

typedef struct {
    uint16_t d;
    uint8_t qs[16]; /* byte j: element 2j in the low nibble, element 2j+1 in the high nibble */
} qm_block_q4;

_Static_assert(sizeof(qm_block_q8) == 34, "Q8_0 block is 34 bytes");
_Static_assert(sizeof(qm_block_q4) == 18, "Q4_0 block is 18 bytes");

/* scalar fp16 <-> fp32 (IEEE binary16, round to nearest even): host format helpers (src/fp16.c) */
float qm_fp16_to_fp32(uint16_t h);
uint16_t qm_fp32_to_fp16(float f);

static inline int64_t qm_nblocks(int64_t n) { return (n + QM_BLOCK - 1) / QM_BLOCK; }
size_t qm_row_bytes(qm_dtype t, int64_t n);
const char *qm_dtype_name(qm_dtype t);
int qm_dtype_valid(uint32_t t);
/* quantize / dequantize one row (src/quant.c:55-102); run on the GPU, bit-exact with the reference */
void qm_quantize_row_q8(const float *x, qm_block_q8 *y, int64_t n);
void qm_dequantize_row_q8(const qm_block_q8 *x, float *y, int64_t n);
void qm_quantize_row_q4(const float *x, qm_block_q4 *y, int64_t n);
void qm_dequantize_row_q4(const qm_block_q4 *x, float *y, int64_t n);
void qm_row_to_f32(qm_dtype t, const void *row, float *y, int64_t n);

/* 64-byte aligned, zeroed bump allocator for host-side buffers (src/arena.c) */
typedef struct {
    uint8_t *base;
    size_t cap, used, peak;
} qm_arena;

int qm_arena_init(qm_arena *a, size_t cap);
void *qm_arena_alloc(qm_arena *a, size_t n);
void qm_arena_reset(qm_arena *a);
void qm_arena_free(qm_arena *a);

/* ISA levels (src/qm_base.h:60).  This build adds QM_ISA_CUDA and implements only it: the CPU levels
 * report "unsupported", so qm_kernels_for() returns NULL for them and there is no CPU fallback. */
typedef enum { QM_ISA_SCALAR = 0, QM_ISA_AVX2 = 1, QM_ISA_AVX512 = 2, QM_ISA_NEON = 3, QM_ISA_CUDA = 4, QM_ISA_COUNT } qm_isa;
int qm_cpu_supports(qm_isa isa);
qm_isa qm_cpu_best(void);
const char *qm_isa_name(qm_isa isa);
int qm_isa_from_name(const char *s);

/* text of the calling thread's last GPU-side error ("" if none); the reference has no error channel on
 * ops, so void ops report failures here and leave their outputs as NaN */
const char *qm_last_error(void);

#pragma GCC visibility pop
#endif
