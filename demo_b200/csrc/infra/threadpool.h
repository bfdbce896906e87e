/*
 * Fixed-size worker pool with a FIFO task queue, plus a countdown latch.
 *
 * Replaces threadpool_create/threadpool_submit/threadpool_destroy and the
 * sema_* helpers of CrossCache's absent infrastructure submodule (call sites
 * src/cache/cache.c:447,491,583-585,776-777 and the batch semaphore
 * :202-217,536-592).  Workers run host-side copies for the CPU backend and
 * asynchronous cache operations whose CUDA work they drive through streams
 * and events.
 */
#ifndef CC_THREADPOOL_H
#define CC_THREADPOOL_H

#include <pthread.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct threadpool threadpool_t;

threadpool_t *threadpool_create(const char *name, int nthreads);
/* runs every queued task, then joins the workers */
void threadpool_destroy(threadpool_t *tp);
int threadpool_submit(threadpool_t *tp, void *arg, void (*fn)(void *));
int threadpool_size(const threadpool_t *tp);

/* countdown latch: the batch-completion barrier (first negative ret wins) */
typedef struct {
    pthread_mutex_t mu;
    pthread_cond_t cv;
    int64_t pending;
    int ret;
} cc_latch_t;

void cc_latch_init(cc_latch_t *l, int64_t count);
void cc_latch_done(cc_latch_t *l, int ret);
int cc_latch_wait(cc_latch_t *l);
void cc_latch_fini(cc_latch_t *l);

#ifdef __cplusplus
}
#endif

#endif
