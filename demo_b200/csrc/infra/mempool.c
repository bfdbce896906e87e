#include "mempool.h"

#include <stdlib.h>

struct mempool {
    uint8_t *base;
    uint64_t objsize;
    uint64_t count;
    uint64_t nfree;
    int64_t *stack;    /* free slab indices; top = stack[nfree - 1] */
    uint8_t *in_use;   /* double-free guard */
};

mempool_t *mempool_create(uint64_t objsize, uint64_t count, void *base)
{
    mempool_t *p;
    uint64_t i;

    if (!objsize || !count || !base)
        return NULL;
    p = calloc(1, sizeof(*p));
    if (!p)
        return NULL;
    p->stack = malloc(count * sizeof(int64_t));
    p->in_use = calloc(count, 1);
    if (!p->stack || !p->in_use) {
        free(p->stack);
        free(p->in_use);
        free(p);
        return NULL;
    }
    p->base = base;
    p->objsize = objsize;
    p->count = count;
    /* lowest index on top so a fresh pool hands out slabs in address order */
    for (i = 0; i < count; i++)
        p->stack[i] = (int64_t)(count - 1 - i);
    p->nfree = count;
    return p;
}

void mempool_destroy(mempool_t *p)
{
    if (!p)
        return;
    free(p->stack);
    free(p->in_use);
    free(p);
}

int64_t mempool_alloc_index(mempool_t *p)
{
    int64_t idx;

    if (!p->nfree)
        return -1;
    idx = p->stack[--p->nfree];
    p->in_use[idx] = 1;
    return idx;
}

void mempool_free_index(mempool_t *p, int64_t idx)
{
    if (idx < 0 || (uint64_t)idx >= p->count || !p->in_use[idx])
        return;
    p->in_use[idx] = 0;
    p->stack[p->nfree++] = idx;
}

void *mempool_alloc(mempool_t *p)
{
    int64_t idx = mempool_alloc_index(p);
    return idx < 0 ? NULL : mempool_addr(p, idx);
}

void mempool_free(mempool_t *p, void *addr)
{
    mempool_free_index(p, mempool_index(p, addr));
}

void *mempool_addr(const mempool_t *p, int64_t idx)
{
    return p->base + (uint64_t)idx * p->objsize;
}

int64_t mempool_index(const mempool_t *p, const void *addr)
{
    const uint8_t *a = addr;
    uint64_t off;

    if (a < p->base)
        return -1;
    off = (uint64_t)(a - p->base);
    if (off % p->objsize || off / p->objsize >= p->count)
        return -1;
    return (int64_t)(off / p->objsize);
}

uint64_t mempool_count(const mempool_t *p) { return p->count; }
uint64_t mempool_free_count(const mempool_t *p) { return p->nfree; }
uint64_t mempool_objsize(const mempool_t *p) { return p->objsize; }
