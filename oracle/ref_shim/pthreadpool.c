/*
 * Persistent worker pool behind the pthreadpool API subset declared in
 * pthreadpool.h.  Workers sleep on a condition variable between jobs, so the
 * reference's CpuBackend (which calls parallelize_1d once per gemm,
 * src/core/cpu_backend.cpp:168) is timed without per-call thread creation.
 * Work items are handed out one at a time from an atomic counter; the calling
 * thread takes part.
 *
 * TEST INFRASTRUCTURE ONLY.
 */
#include "pthreadpool.h"

#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <unistd.h>

struct pthreadpool {
    size_t threads;      /* worker threads + the caller */
    size_t active;       /* threads that take part (set_threads_count) */
    pthread_t* workers;
    pthread_mutex_t mu;
    pthread_cond_t wake;
    pthread_cond_t done;
    unsigned long generation;
    int stop;
    pthreadpool_task_1d_t fn;
    void* ctx;
    size_t range;
    atomic_size_t next;
    size_t pending; /* workers still inside the current job */
};

struct worker_arg {
    struct pthreadpool* pool;
    size_t id;
};

static void run_items(struct pthreadpool* p) {
    for (;;) {
        const size_t i = atomic_fetch_add_explicit(&p->next, 1, memory_order_relaxed);
        if (i >= p->range) break;
        p->fn(p->ctx, i);
    }
}

static void* worker_main(void* raw) {
    struct worker_arg* a = (struct worker_arg*)raw;
    struct pthreadpool* p = a->pool;
    const size_t id = a->id;
    free(a);
    unsigned long seen = 0;
    pthread_mutex_lock(&p->mu);
    for (;;) {
        while (!p->stop && p->generation == seen) pthread_cond_wait(&p->wake, &p->mu);
        if (p->stop) break;
        seen = p->generation;
        const int take_part = id < p->active;
        pthread_mutex_unlock(&p->mu);
        if (take_part) run_items(p);
        pthread_mutex_lock(&p->mu);
        if (--p->pending == 0) pthread_cond_signal(&p->done);
    }
    pthread_mutex_unlock(&p->mu);
    return NULL;
}

pthreadpool_t pthreadpool_create(size_t threads_count) {
    if (threads_count == 0) {
        long n = sysconf(_SC_NPROCESSORS_ONLN);
        threads_count = n > 0 ? (size_t)n : 1;
    }
    struct pthreadpool* p = (struct pthreadpool*)calloc(1, sizeof(*p));
    if (!p) return NULL;
    p->threads = threads_count;
    p->active = threads_count;
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->wake, NULL);
    pthread_cond_init(&p->done, NULL);
    atomic_init(&p->next, 0);
    if (threads_count > 1) {
        p->workers = (pthread_t*)calloc(threads_count - 1, sizeof(pthread_t));
        for (size_t i = 0; i + 1 < threads_count; ++i) {
            struct worker_arg* a = (struct worker_arg*)malloc(sizeof(*a));
            a->pool = p;
            a->id = i + 1; /* the caller is thread 0 */
            pthread_create(&p->workers[i], NULL, worker_main, a);
        }
    }
    return p;
}

size_t pthreadpool_get_threads_count(pthreadpool_t p) { return p ? p->threads : 1; }

size_t pthreadpool_set_threads_count(pthreadpool_t p, size_t threads_count) {
    if (!p) return 1;
    if (threads_count == 0 || threads_count > p->threads) threads_count = p->threads;
    pthread_mutex_lock(&p->mu);
    p->active = threads_count;
    pthread_mutex_unlock(&p->mu);
    return threads_count;
}

void pthreadpool_parallelize_1d(pthreadpool_t p, pthreadpool_task_1d_t fn, void* ctx,
                                size_t range, uint32_t flags) {
    (void)flags;
    if (!p || p->threads <= 1 || range <= 1) {
        for (size_t i = 0; i < range; ++i) fn(ctx, i);
        return;
    }
    pthread_mutex_lock(&p->mu);
    p->fn = fn;
    p->ctx = ctx;
    p->range = range;
    atomic_store_explicit(&p->next, 0, memory_order_relaxed);
    p->pending = p->threads - 1;
    ++p->generation;
    pthread_cond_broadcast(&p->wake);
    pthread_mutex_unlock(&p->mu);
    run_items(p);
    pthread_mutex_lock(&p->mu);
    while (p->pending != 0) pthread_cond_wait(&p->done, &p->mu);
    pthread_mutex_unlock(&p->mu);
}

void pthreadpool_destroy(pthreadpool_t p) {
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    p->stop = 1;
    pthread_cond_broadcast(&p->wake);
    pthread_mutex_unlock(&p->mu);
    for (size_t i = 0; i + 1 < p->threads; ++i) pthread_join(p->workers[i], NULL);
    free(p->workers);
    pthread_mutex_destroy(&p->mu);
    pthread_cond_destroy(&p->wake);
    pthread_cond_destroy(&p->done);
    free(p);
}
