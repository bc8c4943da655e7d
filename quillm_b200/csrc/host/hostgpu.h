/* Internal to libquillm.so: device staging for the host-pointer qm_* ops.
 * Every qm_* op that takes host pointers runs under qh_begin()/qh_end() (one op at a time per process),
 * copies its inputs into per-device staging buffers, launches through libquillm_cuda on the library
 * stream, copies the outputs back and synchronises. */
#ifndef QM_HOSTGPU_H
#define QM_HOSTGPU_H

#include <stddef.h>

#include "quillm_cuda.h"

enum { QH_SLOTS = 6 };

int qh_begin(void); /* locks; 0 when a CUDA device is usable */
void qh_end(void);
void *qh_slot(int slot, size_t bytes);                        /* device buffer of >= bytes (grows) */
void *qh_put(int slot, const void *host, size_t bytes);       /* H2D into slot; device pointer or NULL */
int qh_get(void *host, const void *dev, size_t bytes);        /* D2H (async on the library stream) */
int qh_finish(void);                                          /* synchronise + device error check */
void qh_fail(const char *op);                                 /* record + report the last qmc error */
void qh_set_error(const char *fmt, ...);
void qh_fill_nan(float *p, size_t n);

/* resident-tensor registry (ops.c): device copy of a host tensor's bytes, or NULL */
const void *qh_resident(const void *host, size_t bytes);

#endif
