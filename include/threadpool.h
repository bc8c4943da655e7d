/* quillm-b200 qm_pool: kept for source compatibility with the reference's src/threadpool.h:9-16.
 * The GPU build has no worker threads (the parallelism of every op is on the device): a pool only
 * records its size, and qm_pool_run executes fn(ctx, 0, n, 0) on the calling thread. */
#ifndef QM_THREADPOOL_H
#define QM_THREADPOOL_H

#include <stdint.h>

#pragma GCC visibility push(default)

typedef struct qm_pool qm_pool;
typedef void (*qm_task_fn)(void *ctx, int64_t start, int64_t end, int tid);

qm_pool *qm_pool_create(int n_threads);
void qm_pool_destroy(qm_pool *p);
int qm_pool_size(const qm_pool *p);
void qm_pool_run(qm_pool *p, int64_t n, int64_t grain, qm_task_fn fn, void *ctx);

#pragma GCC visibility pop
#endif
