#include "kvmap.h"

#include <stdlib.h>
#include <string.h>

struct kvrec {
    uint8_t key[KVMAP_KEY_LEN];
    uint32_t prev, next;   /* LRU links (indices; `nil` = capacity) */
    int32_t pins;
    uint8_t state;
};

struct kvmap {
    uint32_t capacity;
    uint32_t size;
    uint64_t mask;         /* table size - 1 (power of two >= 2 * capacity) */
    uint32_t *table;       /* record index + 1, 0 = empty */
    struct kvrec *recs;    /* [capacity + 1], the last one is the LRU sentinel */
};

static inline uint64_t key_bucket(const uint8_t *key)
{
    /* keys are SHA-256 digests: any 8 bytes are uniformly distributed */
    uint64_t h;
    memcpy(&h, key + 8, sizeof(h));
    return h * 0x9E3779B97F4A7C15ull;
}

kvmap_t *kvmap_create(uint32_t capacity)
{
    kvmap_t *m;
    uint64_t tsize = 16;
    uint32_t i;

    if (!capacity)
        return NULL;
    while (tsize < 2ull * capacity)
        tsize <<= 1;
    m = calloc(1, sizeof(*m));
    if (!m)
        return NULL;
    m->table = calloc(tsize, sizeof(uint32_t));
    m->recs = calloc((uint64_t)capacity + 1, sizeof(struct kvrec));
    if (!m->table || !m->recs) {
        free(m->table);
        free(m->recs);
        free(m);
        return NULL;
    }
    m->capacity = capacity;
    m->mask = tsize - 1;
    for (i = 0; i <= capacity; i++)
        m->recs[i].prev = m->recs[i].next = capacity;
    return m;
}

void kvmap_destroy(kvmap_t *m)
{
    if (!m)
        return;
    free(m->table);
    free(m->recs);
    free(m);
}

static uint64_t probe_slot(const kvmap_t *m, const uint8_t *key, int *found)
{
    uint64_t h = key_bucket(key) & m->mask;

    for (;;) {
        uint32_t v = m->table[h];
        if (!v) {
            *found = 0;
            return h;
        }
        if (!memcmp(m->recs[v - 1].key, key, KVMAP_KEY_LEN)) {
            *found = 1;
            return h;
        }
        h = (h + 1) & m->mask;
    }
}

int64_t kvmap_find(const kvmap_t *m, const uint8_t *key)
{
    int found;
    uint64_t h = probe_slot(m, key, &found);
    return found ? (int64_t)m->table[h] - 1 : -1;
}

static void lru_unlink(kvmap_t *m, uint32_t i)
{
    struct kvrec *r = &m->recs[i];
    m->recs[r->prev].next = r->next;
    m->recs[r->next].prev = r->prev;
    r->prev = r->next = m->capacity;
}

static void lru_push_mru(kvmap_t *m, uint32_t i)
{
    uint32_t nil = m->capacity;
    struct kvrec *s = &m->recs[nil];
    struct kvrec *r = &m->recs[i];

    /* sentinel.next = most recent, sentinel.prev = least recent */
    r->next = s->next;
    r->prev = nil;
    m->recs[s->next].prev = i;
    s->next = i;
}

static int lru_linked(const kvmap_t *m, uint32_t i)
{
    const struct kvrec *r = &m->recs[i];
    uint32_t nil = m->capacity;
    return r->prev != nil || r->next != nil || m->recs[nil].next == i;
}

int kvmap_insert(kvmap_t *m, int64_t idx, const uint8_t *key, int state)
{
    int found;
    uint64_t h;
    struct kvrec *r;

    if (idx < 0 || (uint64_t)idx >= m->capacity)
        return -1;
    r = &m->recs[idx];
    if (r->state != KVMAP_FREE)
        return -1;
    h = probe_slot(m, key, &found);
    if (found)
        return -1;
    memcpy(r->key, key, KVMAP_KEY_LEN);
    r->state = (uint8_t)state;
    r->pins = 0;
    m->table[h] = (uint32_t)idx + 1;
    m->size++;
    if (state == KVMAP_READY)
        lru_push_mru(m, (uint32_t)idx);
    return 0;
}

void kvmap_publish(kvmap_t *m, int64_t idx)
{
    struct kvrec *r = &m->recs[idx];
    if (r->state != KVMAP_PENDING)
        return;
    r->state = KVMAP_READY;
    lru_push_mru(m, (uint32_t)idx);
}

void kvmap_remove(kvmap_t *m, int64_t idx)
{
    struct kvrec *r = &m->recs[idx];
    int found;
    uint64_t h, j;

    if (r->state == KVMAP_FREE)
        return;
    if (lru_linked(m, (uint32_t)idx))
        lru_unlink(m, (uint32_t)idx);
    h = probe_slot(m, r->key, &found);
    r->state = KVMAP_FREE;
    r->pins = 0;
    m->size--;
    if (!found)
        return;
    /* backward-shift deletion keeps linear probing tombstone-free */
    m->table[h] = 0;
    j = h;
    for (;;) {
        uint32_t v;
        uint64_t home;
        j = (j + 1) & m->mask;
        v = m->table[j];
        if (!v)
            break;
        home = key_bucket(m->recs[v - 1].key) & m->mask;
        /* move v back to h if h lies cyclically in [home, j) */
        if (((j - home) & m->mask) >= ((j - h) & m->mask)) {
            m->table[h] = v;
            m->table[j] = 0;
            h = j;
        }
    }
}

int kvmap_state(const kvmap_t *m, int64_t idx) { return m->recs[idx].state; }

void kvmap_touch(kvmap_t *m, int64_t idx)
{
    if (m->recs[idx].state != KVMAP_READY)
        return;
    lru_unlink(m, (uint32_t)idx);
    lru_push_mru(m, (uint32_t)idx);
}

void kvmap_pin(kvmap_t *m, int64_t idx) { m->recs[idx].pins++; }

void kvmap_unpin(kvmap_t *m, int64_t idx)
{
    if (m->recs[idx].pins > 0)
        m->recs[idx].pins--;
}

int32_t kvmap_pins(const kvmap_t *m, int64_t idx) { return m->recs[idx].pins; }

int64_t kvmap_evict_lru(kvmap_t *m)
{
    uint32_t nil = m->capacity;
    uint32_t i = m->recs[nil].prev;
    uint32_t steps = 0;

    while (i != nil && steps++ <= m->capacity) {
        if (m->recs[i].state == KVMAP_READY && m->recs[i].pins == 0) {
            kvmap_remove(m, i);
            return i;
        }
        i = m->recs[i].prev;
    }
    return -1;
}

uint32_t kvmap_find_batch(kvmap_t *m, const uint8_t *keys, uint32_t n,
                          uint32_t key_stride, int touch, int64_t *out_idx)
{
    uint32_t i, hits = 0;

    for (i = 0; i < n; i++) {
        int64_t idx = kvmap_find(m, keys + (uint64_t)i * key_stride);
        if (idx >= 0 && m->recs[idx].state == KVMAP_READY) {
            out_idx[i] = idx;
            hits++;
            if (touch)
                kvmap_touch(m, idx);
        } else {
            out_idx[i] = -1;
        }
    }
    return hits;
}

uint32_t kvmap_size(const kvmap_t *m) { return m->size; }
uint32_t kvmap_capacity(const kvmap_t *m) { return m->capacity; }

uint32_t kvmap_lru_order(const kvmap_t *m, int64_t *out, uint32_t max)
{
    uint32_t nil = m->capacity, i = m->recs[nil].prev, n = 0;
    while (i != nil && n < max) {
        out[n++] = i;
        i = m->recs[i].prev;
    }
    return n;
}
