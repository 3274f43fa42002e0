/*
 * Minimal stand-in for the subset of the pthreadpool C API that the reference
 * uses through include/mruntime/pthreadpool_raii.h:23-77 (google/pthreadpool
 * @ 0e6ca137, pinned in the reference's CMakeLists.txt:43-47 and not vendored).
 * The declarations keep that library's published names and argument meaning
 * so the reference's headers compile unchanged; the implementation in
 * pthreadpool.c is this repository's own persistent pool.
 *
 * TEST INFRASTRUCTURE ONLY: it exists to build the reference's CPU gemm as the
 * oracle and CPU baseline.
 */
#ifndef MRT_ORACLE_PTHREADPOOL_SHIM_H
#define MRT_ORACLE_PTHREADPOOL_SHIM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct pthreadpool* pthreadpool_t;
typedef void (*pthreadpool_task_1d_t)(void* context, size_t index);

/* threads_count == 0 means one thread per online CPU. */
pthreadpool_t pthreadpool_create(size_t threads_count);
size_t pthreadpool_get_threads_count(pthreadpool_t pool);
size_t pthreadpool_set_threads_count(pthreadpool_t pool, size_t threads_count);
/* Calls function(context, i) for every i in [0, range); returns when all are
 * done.  A NULL pool runs the loop on the calling thread. */
void pthreadpool_parallelize_1d(pthreadpool_t pool, pthreadpool_task_1d_t function,
                                void* context, size_t range, uint32_t flags);
void pthreadpool_destroy(pthreadpool_t pool);

#ifdef __cplusplus
}
#endif
#endif
