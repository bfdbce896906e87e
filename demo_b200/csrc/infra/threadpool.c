#include "threadpool.h"

#include <stdlib.h>
#include <string.h>

struct task {
    void (*fn)(void *);
    void *arg;
    struct task *next;
};

struct threadpool {
    pthread_mutex_t mu;
    pthread_cond_t cv;
    struct task *head, *tail;
    int stop;
    int nthreads;
    pthread_t *threads;
};

static void *worker(void *p)
{
    threadpool_t *tp = p;

    for (;;) {
        struct task *t;
        pthread_mutex_lock(&tp->mu);
        while (!tp->head && !tp->stop)
            pthread_cond_wait(&tp->cv, &tp->mu);
        if (!tp->head && tp->stop) {
            pthread_mutex_unlock(&tp->mu);
            return NULL;
        }
        t = tp->head;
        tp->head = t->next;
        if (!tp->head)
            tp->tail = NULL;
        pthread_mutex_unlock(&tp->mu);
        t->fn(t->arg);
        free(t);
    }
}

threadpool_t *threadpool_create(const char *name, int nthreads)
{
    threadpool_t *tp;
    int i;

    (void)name;
    if (nthreads <= 0)
        return NULL;
    tp = calloc(1, sizeof(*tp));
    if (!tp)
        return NULL;
    tp->threads = calloc((size_t)nthreads, sizeof(pthread_t));
    if (!tp->threads) {
        free(tp);
        return NULL;
    }
    pthread_mutex_init(&tp->mu, NULL);
    pthread_cond_init(&tp->cv, NULL);
    for (i = 0; i < nthreads; i++) {
        if (pthread_create(&tp->threads[i], NULL, worker, tp)) {
            tp->nthreads = i;
            threadpool_destroy(tp);
            return NULL;
        }
    }
    tp->nthreads = nthreads;
    return tp;
}

void threadpool_destroy(threadpool_t *tp)
{
    int i;

    if (!tp)
        return;
    pthread_mutex_lock(&tp->mu);
    tp->stop = 1;
    pthread_cond_broadcast(&tp->cv);
    pthread_mutex_unlock(&tp->mu);
    for (i = 0; i < tp->nthreads; i++)
        pthread_join(tp->threads[i], NULL);
    pthread_mutex_destroy(&tp->mu);
    pthread_cond_destroy(&tp->cv);
    free(tp->threads);
    free(tp);
}

int threadpool_submit(threadpool_t *tp, void *arg, void (*fn)(void *))
{
    struct task *t = malloc(sizeof(*t));

    if (!t)
        return -1;
    t->fn = fn;
    t->arg = arg;
    t->next = NULL;
    pthread_mutex_lock(&tp->mu);
    if (tp->tail)
        tp->tail->next = t;
    else
        tp->head = t;
    tp->tail = t;
    pthread_cond_signal(&tp->cv);
    pthread_mutex_unlock(&tp->mu);
    return 0;
}

int threadpool_size(const threadpool_t *tp) { return tp->nthreads; }

void cc_latch_init(cc_latch_t *l, int64_t count)
{
    pthread_mutex_init(&l->mu, NULL);
    pthread_cond_init(&l->cv, NULL);
    l->pending = count;
    l->ret = 0;
}

void cc_latch_done(cc_latch_t *l, int ret)
{
    pthread_mutex_lock(&l->mu);
    if (ret < 0 && l->ret == 0)
        l->ret = ret;
    if (--l->pending <= 0)
        pthread_cond_broadcast(&l->cv);
    pthread_mutex_unlock(&l->mu);
}

int cc_latch_wait(cc_latch_t *l)
{
    int ret;
    pthread_mutex_lock(&l->mu);
    while (l->pending > 0)
        pthread_cond_wait(&l->cv, &l->mu);
    ret = l->ret;
    pthread_mutex_unlock(&l->mu);
    return ret;
}

void cc_latch_fini(cc_latch_t *l)
{
    pthread_mutex_destroy(&l->mu);
    pthread_cond_destroy(&l->cv);
}
