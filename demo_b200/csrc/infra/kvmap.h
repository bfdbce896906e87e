/*
 * Key -> record map with LRU order for the record pool.
 *
 * Replaces the chained hashmap of CrossCache's absent infrastructure
 * submodule as used by src/cache/cache.c (hashmap_search with the
 * key_access timestamp refresh :155-159,559,735; hashmap_insert with
 * EEXIST dedupe :480-486,498-504; hashmap_eviction :306-317).
 *
 * Keys are 32-byte block hashes compared with memcmp (reference key_cmp,
 * cache.c:139-145).  Each map entry is identified by the index of the pool
 * record it owns, so the map holds at most `capacity` entries.  Entries are
 *   KVMAP_PENDING  key reserved, record data still in flight (not visible to
 *                  lookups; a second store of the key sees it and skips)
 *   KVMAP_READY    record data valid; member of the LRU list
 * Eviction is deterministic least-recently-used over READY entries whose pin
 * count is zero (the reference evicts entries idle for > 3 s and may spin
 * forever when none is, cache.c:291-343).
 *
 * Not internally locked: the owner serialises calls; the batched entry points
 * exist so that one lock acquisition covers a whole request batch.
 */
#ifndef CC_KVMAP_H
#define CC_KVMAP_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVMAP_KEY_LEN 32

enum kvmap_state { KVMAP_FREE = 0, KVMAP_PENDING = 1, KVMAP_READY = 2 };

typedef struct kvmap kvmap_t;

kvmap_t *kvmap_create(uint32_t capacity);
void kvmap_destroy(kvmap_t *map);

/* record index owning `key`, or -1 */
int64_t kvmap_find(const kvmap_t *map, const uint8_t *key);

/* bind record `idx` (currently FREE) to `key` (not present) in `state` */
int kvmap_insert(kvmap_t *map, int64_t idx, const uint8_t *key, int state);

/* PENDING -> READY, entering the LRU list at the most-recent end */
void kvmap_publish(kvmap_t *map, int64_t idx);

/* unbind record idx (any state) */
void kvmap_remove(kvmap_t *map, int64_t idx);

int kvmap_state(const kvmap_t *map, int64_t idx);
void kvmap_touch(kvmap_t *map, int64_t idx);   /* READY: move to MRU end */
void kvmap_pin(kvmap_t *map, int64_t idx);
void kvmap_unpin(kvmap_t *map, int64_t idx);
int32_t kvmap_pins(const kvmap_t *map, int64_t idx);

/* least-recently-used READY, unpinned entry: removed from the map and its
 * index returned; -1 when every entry is pending or pinned */
int64_t kvmap_evict_lru(kvmap_t *map);

/* batched lookup: out_idx[i] = kvmap_find(keys + i * key_stride) if that
 * entry is READY, else -1.  When touch != 0 the hits move to the MRU end in
 * key order.  Returns the number of hits. */
uint32_t kvmap_find_batch(kvmap_t *map, const uint8_t *keys, uint32_t n,
                          uint32_t key_stride, int touch, int64_t *out_idx);

uint32_t kvmap_size(const kvmap_t *map);
uint32_t kvmap_capacity(const kvmap_t *map);

/* LRU order, least recent first, into out[0..max) ; returns count */
uint32_t kvmap_lru_order(const kvmap_t *map, int64_t *out, uint32_t max);

#ifdef __cplusplus
}
#endif

#endif
