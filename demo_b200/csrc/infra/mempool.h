/*
 * Fixed-size slab pool over one contiguous (pinned) region.
 *
 * Replaces mempool_create/mempool_alloc/mempool_free of CrossCache's absent
 * infrastructure submodule (call sites src/cache/cache.c:287,330,658,699):
 * `count` records of `objsize` bytes carved from `base`.  Slabs are handed
 * out by index so that the key map can address records without pointers.
 * Not internally locked: the owner serialises calls.
 */
#ifndef CC_MEMPOOL_H
#define CC_MEMPOOL_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mempool mempool_t;

mempool_t *mempool_create(uint64_t objsize, uint64_t count, void *base);
void mempool_destroy(mempool_t *pool);

/* index of a free slab, or -1 when the pool is exhausted */
int64_t mempool_alloc_index(mempool_t *pool);
void mempool_free_index(mempool_t *pool, int64_t idx);

/* address forms (reference call shape): NULL when exhausted */
void *mempool_alloc(mempool_t *pool);
void mempool_free(mempool_t *pool, void *addr);

void *mempool_addr(const mempool_t *pool, int64_t idx);
int64_t mempool_index(const mempool_t *pool, const void *addr);
uint64_t mempool_count(const mempool_t *pool);
uint64_t mempool_free_count(const mempool_t *pool);
uint64_t mempool_objsize(const mempool_t *pool);

#ifdef __cplusplus
}
#endif

#endif
