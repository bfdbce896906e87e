/*
 * Cache manager: per-(model, tp_size, tp_rank) record pools, key maps and the
 * store / load / lookup operations of include/cache.h.
 *
 * Behaviour follows CrossCache src/cache/cache.c:
 *   - one runtime entry per (model tag, tp size, tp rank)        :54-58,598-684
 *   - a store or load of bnum blocks is split into
 *     bnum / (chunk_size / block_size) records, record i covering blocks
 *     [i * bpc, (i + 1) * bpc) and keyed by the i-th key             :513-593
 *   - a store of a key that is already cached keeps the existing record
 *     (reference: EEXIST on insert frees the new copy)      :480-486,498-504
 *   - a key becomes visible to lookups only after its data landed  :495-504
 *   - lookup walks keys in order, stops at the first miss and returns the
 *     byte offset i * key_len                                       :712-745
 *   - load/lookup hits refresh the record's recency (key_access)   :155-159
 * Differences, by design:
 *   - all records of one call move in one batched adaptor transfer
 *     (transfer_kvcache_batch) instead of one pipeline task per record;
 *   - eviction is deterministic LRU over unpinned records and fails with
 *     -ENOMEM instead of spinning when everything is in flight (:319-343);
 *   - records being loaded are pinned so eviction cannot recycle them;
 *   - the disk tier (:222-278) is not part of this build: a load of a key
 *     that is not in memory fails with -ENOENT.
 */
#include "cache.h"
#include "device.h"

#include "../infra/kvmap.h"
#include "../infra/log.h"
#include "../infra/mempool.h"

#include <errno.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define KV_H_TO_D false
#define KV_D_TO_H true

struct rt_entry {
    char *model_tag;
    uint8_t tp_size;
    uint8_t tp_id;
    int32_t ref;

    uint32_t num_blocks;
    uint32_t block_size;
    uint8_t element_size;
    uint16_t num_layers;
    uint32_t hidden_dim_size;
    uint32_t per_token_size;
    uint64_t objsize;

    void *host_base;
    void *dev_base;
    uint64_t pool_bytes;
    mempool_t *pool;
    kvmap_t *map;
    struct cache_stats stats;
    pthread_mutex_t mu;

    struct rt_entry *next;
};

struct cache_manager {
    int initialised;
    uint32_t chunk_size;
    uint64_t pool_size;
    int backend;
    char *local_dir;
    adaptor_t *adaptor;
    pthread_mutex_t mu;        /* guards the entry list */
    struct rt_entry *entries;
};

static struct cache_manager g_mgr = {.mu = PTHREAD_MUTEX_INITIALIZER};

static struct rt_entry *find_entry_locked(const char *tag, uint8_t tp_size,
                                          uint8_t tp_id)
{
    struct rt_entry *e;
    for (e = g_mgr.entries; e; e = e->next)
        if (!strcmp(e->model_tag, tag) && e->tp_size == tp_size &&
            e->tp_id == tp_id)
            return e;
    return NULL;
}

static struct rt_entry *get_entry(struct worker_context *wctx)
{
    struct rt_entry *e;
    if (!g_mgr.initialised || !wctx || !wctx->model.model_name)
        return NULL;
    pthread_mutex_lock(&g_mgr.mu);
    e = find_entry_locked(wctx->model.model_name, wctx->world_size,
                          wctx->rank_id);
    pthread_mutex_unlock(&g_mgr.mu);
    return e;
}

static void destroy_entry(struct rt_entry *e)
{
    kvmap_destroy(e->map);
    mempool_destroy(e->pool);
    if (e->host_base)
        free_pinned_ptr(g_mgr.adaptor, e->host_base, e->pool_bytes);
    pthread_mutex_destroy(&e->mu);
    free(e->model_tag);
    free(e);
}

/* ------------------------------------------------------------------ */

int cache_init_backend(uint32_t chunk_size, uint64_t pool_size,
                       const char *root_dir, int backend)
{
    adaptor_t *ad;

    /* transfer_params.num_tokens is 16-bit (reference device.h:25) */
    if (!chunk_size || chunk_size > UINT16_MAX)
        return -EINVAL;
    pthread_mutex_lock(&g_mgr.mu);
    if (g_mgr.initialised) {
        pthread_mutex_unlock(&g_mgr.mu);
        return -EBUSY;
    }
    if (backend == CACHE_BACKEND_CUDA)
        ad = cuda_adaptor_create();
    else if (backend == CACHE_BACKEND_MEM)
        ad = mem_adaptor_create();
    else
        ad = NULL;
    if (!ad) {
        pthread_mutex_unlock(&g_mgr.mu);
        log_error("cache_init: no adaptor for backend %d", backend);
        return -ENODEV;
    }
    g_mgr.adaptor = ad;
    g_mgr.backend = backend;
    g_mgr.chunk_size = chunk_size;
    g_mgr.pool_size = pool_size;
    g_mgr.local_dir = root_dir ? strdup(root_dir) : NULL;
    g_mgr.entries = NULL;
    g_mgr.initialised = 1;
    pthread_mutex_unlock(&g_mgr.mu);
    log_info("cache_init chunk_size:%u pool_size:%lu backend:%d", chunk_size,
             (unsigned long)pool_size, backend);
    return 0;
}

int cache_init(uint32_t chunk_size, uint64_t pool_size, const char *root_dir)
{
    return cache_init_backend(chunk_size, pool_size, root_dir,
                              CACHE_BACKEND_CUDA);
}

void cache_exit()
{
    struct rt_entry *e, *n;

    pthread_mutex_lock(&g_mgr.mu);
    if (!g_mgr.initialised) {
        pthread_mutex_unlock(&g_mgr.mu);
        return;
    }
    for (e = g_mgr.entries; e; e = n) {
        n = e->next;
        destroy_entry(e);
    }
    g_mgr.entries = NULL;
    if (g_mgr.backend == CACHE_BACKEND_CUDA)
        cuda_adaptor_destroy(g_mgr.adaptor);
    else
        mem_adaptor_destroy(g_mgr.adaptor);
    g_mgr.adaptor = NULL;
    free(g_mgr.local_dir);
    g_mgr.local_dir = NULL;
    g_mgr.initialised = 0;
    pthread_mutex_unlock(&g_mgr.mu);
}

int cache_register(struct worker_context *wctx)
{
    struct rt_entry *e;
    void *dptrs, *haddr = NULL, *daddr = NULL;
    uint64_t chunk_bytes, m_count, unit;
    int kv, ret;

    if (!g_mgr.initialised)
        return -ENODEV;
    if (!wctx || !wctx->model.model_name || !wctx->k_raw_ptrs ||
        !wctx->model.num_layers || !wctx->block_size ||
        g_mgr.chunk_size % wctx->block_size)
        return -EINVAL;
    kv = wctx->v_raw_ptrs ? 2 : 1;
    unit = (uint64_t)wctx->model.hidden_dim_size * wctx->model.element_size;
    if (!unit || wctx->per_token_size != kv * wctx->model.num_layers * unit) {
        log_error("register: per_token_size %u != %d * %u layers * %lu",
                  wctx->per_token_size, kv, wctx->model.num_layers,
                  (unsigned long)unit);
        return -EINVAL;
    }
    chunk_bytes = (uint64_t)wctx->per_token_size * g_mgr.chunk_size;
    /* reference asserts 4 KiB alignment of a record (cache.c:621-622) */
    if (chunk_bytes % 4096)
        return -EINVAL;

    wctx->k_ptrs = wctx->v_ptrs = NULL;
    dptrs = open_ipc_keys(g_mgr.adaptor, wctx->node_id, wctx->per_len,
                          wctx->model.num_layers, wctx->k_raw_ptrs);
    if (!dptrs)
        return -ENOMEM;
    wctx->k_ptrs = dptrs;
    if (wctx->v_raw_ptrs) {
        dptrs = open_ipc_keys(g_mgr.adaptor, wctx->node_id, wctx->per_len,
                              wctx->model.num_layers, wctx->v_raw_ptrs);
        if (!dptrs) {
            ret = -ENOMEM;
            goto unpin_k;
        }
        wctx->v_ptrs = dptrs;
    }

    pthread_mutex_lock(&g_mgr.mu);
    e = find_entry_locked(wctx->model.model_name, wctx->world_size,
                          wctx->rank_id);
    if (e) {
        /* another worker of the same (model, tp) shares the pool */
        if (e->objsize != chunk_bytes || e->block_size != wctx->block_size ||
            e->num_layers != wctx->model.num_layers) {
            pthread_mutex_unlock(&g_mgr.mu);
            ret = -EINVAL;
            goto unpin_v;
        }
        e->ref++;
        pthread_mutex_unlock(&g_mgr.mu);
        return 0;
    }

    ret = -ENOMEM;
    m_count = g_mgr.pool_size / chunk_bytes;
    if (!m_count || m_count > UINT32_MAX - 1) {
        pthread_mutex_unlock(&g_mgr.mu);
        goto unpin_v;
    }
    e = calloc(1, sizeof(*e));
    if (!e) {
        pthread_mutex_unlock(&g_mgr.mu);
        goto unpin_v;
    }
    pthread_mutex_init(&e->mu, NULL);
    e->model_tag = strdup(wctx->model.model_name);
    e->tp_size = wctx->world_size;
    e->tp_id = wctx->rank_id;
    e->ref = 1;
    e->num_blocks = wctx->num_blocks;
    e->block_size = wctx->block_size;
    e->element_size = wctx->model.element_size;
    e->num_layers = wctx->model.num_layers;
    e->hidden_dim_size = wctx->model.hidden_dim_size;
    e->per_token_size = wctx->per_token_size;
    e->objsize = chunk_bytes;
    e->pool_bytes = m_count * chunk_bytes;
    if (e->model_tag)
        haddr = alloc_pinned_ptr(g_mgr.adaptor, wctx->node_id, e->pool_bytes,
                                 0, &daddr);
    if (!haddr) {
        e->host_base = NULL;
        destroy_entry(e);
        pthread_mutex_unlock(&g_mgr.mu);
        goto unpin_v;
    }
    e->host_base = haddr;
    e->dev_base = daddr;
    e->pool = mempool_create(chunk_bytes, m_count, haddr);
    e->map = kvmap_create((uint32_t)m_count);
    if (!e->pool || !e->map) {
        destroy_entry(e);
        pthread_mutex_unlock(&g_mgr.mu);
        goto unpin_v;
    }
    e->stats.records_total = m_count;
    e->next = g_mgr.entries;
    g_mgr.entries = e;
    pthread_mutex_unlock(&g_mgr.mu);
    log_debug("register [%s,%u,%u] records:%lu x %lu B", e->model_tag,
              e->tp_size, e->tp_id, (unsigned long)m_count,
              (unsigned long)chunk_bytes);
    return 0;

unpin_v:
    if (wctx->v_ptrs)
        close_ipc_keys(g_mgr.adaptor, wctx->v_ptrs);
    wctx->v_ptrs = NULL;
unpin_k:
    close_ipc_keys(g_mgr.adaptor, wctx->k_ptrs);
    wctx->k_ptrs = NULL;
    return ret;
}

void cache_unregister(struct worker_context *wctx)
{
    struct rt_entry *e, **pp;
    uint8_t nid;

    if (!g_mgr.initialised || !wctx || !wctx->model.model_name)
        return;
    nid = wctx->node_id;
    pthread_mutex_lock(&g_mgr.mu);
    for (pp = &g_mgr.entries; (e = *pp); pp = &e->next)
        if (!strcmp(e->model_tag, wctx->model.model_name) &&
            e->tp_size == wctx->world_size && e->tp_id == wctx->rank_id)
            break;
    if (!e) {
        pthread_mutex_unlock(&g_mgr.mu);
        return;
    }
    if (--e->ref <= 0) {
        *pp = e->next;
        destroy_entry(e);
    }
    pthread_mutex_unlock(&g_mgr.mu);
    if (wctx->k_ptrs)
        close_ipc_keys(g_mgr.adaptor, wctx->k_ptrs);
    if (wctx->v_ptrs)
        close_ipc_keys(g_mgr.adaptor, wctx->v_ptrs);
    wctx->k_ptrs = wctx->v_ptrs = NULL;
    /* CUDA backend: drains and releases this process's streams and staging
     * buffers on the device; it never resets a (shared) GPU. */
    reset_device(g_mgr.adaptor, nid);
}

/* ------------------------------------------------------------------ */

static int run_transfer(struct rt_entry *e, struct worker_context *wctx,
                        bool direction, const int64_t *idx,
                        const uint64_t *bids, uint32_t n)
{
    struct transfer_batch tb;
    void **recs;
    uint32_t i;
    int ret;

    if (!n)
        return 0;
    recs = malloc(n * sizeof(void *));
    if (!recs)
        return -ENOMEM;
    for (i = 0; i < n; i++)
        recs[i] = mempool_addr(e->pool, idx[i]);
    memset(&tb, 0, sizeof(tb));
    tb.keys_ptrs = wctx->k_ptrs;
    tb.value_ptrs = wctx->v_ptrs;
    tb.page_buffer_size = (uint64_t)wctx->num_blocks * wctx->block_size;
    tb.records = recs;
    tb.block_ids = bids;
    tb.num_records = n;
    tb.block_size = wctx->block_size;
    tb.hidden_dim_size = wctx->model.hidden_dim_size;
    tb.num_layers = wctx->model.num_layers;
    tb.num_tokens = (uint16_t)g_mgr.chunk_size;
    tb.devid = wctx->node_id;
    tb.caches_element_size = wctx->model.element_size;
    tb.record_on_device = 0;
    tb.direction = direction;
    ret = transfer_kvcache_batch(g_mgr.adaptor, &tb);
    free(recs);
    return ret;
}

static int cache_op(struct worker_context *wctx, uint8_t *keys,
                    uint32_t key_len, uint64_t *bids, uint32_t bnum,
                    bool store)
{
    struct rt_entry *e;
    uint32_t bpc, key_num, i, n = 0;
    int64_t *idx = NULL;
    uint64_t *tbids = NULL;
    int ret = 0, xret;

    e = get_entry(wctx);
    if (!e)
        return -ENOENT;
    if (!keys || key_len < KVMAP_KEY_LEN || (bnum && !bids))
        return -EINVAL;
    if (!wctx->k_ptrs)
        return -EINVAL;
    bpc = g_mgr.chunk_size / wctx->block_size;
    key_num = bnum / bpc;
    if (!key_num)
        return 0;
    idx = malloc(key_num * sizeof(int64_t));
    tbids = malloc((uint64_t)key_num * bpc * sizeof(uint64_t));
    if (!idx || !tbids) {
        free(idx);
        free(tbids);
        return -ENOMEM;
    }

    pthread_mutex_lock(&e->mu);
    for (i = 0; i < key_num; i++) {
        const uint8_t *key = keys + (uint64_t)i * key_len;
        int64_t r = kvmap_find(e->map, key);
        if (store) {
            if (r >= 0) {               /* cached or in flight: keep it */
                e->stats.store_dedup++;
                continue;
            }
            r = mempool_alloc_index(e->pool);
            if (r < 0) {
                r = kvmap_evict_lru(e->map);
                if (r >= 0)
                    e->stats.evictions++;
            }
            if (r < 0) {
                log_warn("store: pool exhausted (all records pinned/in flight)");
                ret = -ENOMEM;
                break;
            }
            kvmap_insert(e->map, r, key, KVMAP_PENDING);
        } else {
            if (r < 0 || kvmap_state(e->map, r) != KVMAP_READY) {
                e->stats.load_misses++;
                ret = -ENOENT;
                continue;
            }
            kvmap_touch(e->map, r);
            kvmap_pin(e->map, r);
        }
        idx[n] = r;
        memcpy(tbids + (uint64_t)n * bpc, bids + (uint64_t)i * bpc,
               bpc * sizeof(uint64_t));
        n++;
    }
    pthread_mutex_unlock(&e->mu);

    xret = run_transfer(e, wctx, store ? KV_D_TO_H : KV_H_TO_D, idx, tbids, n);
    if (xret < 0 && ret == 0)
        ret = xret;

    pthread_mutex_lock(&e->mu);
    for (i = 0; i < n; i++) {
        if (store) {
            if (xret == 0) {
                kvmap_publish(e->map, idx[i]);
                e->stats.stored++;
                e->stats.bytes_saved += e->objsize;
            } else {
                kvmap_remove(e->map, idx[i]);
                mempool_free_index(e->pool, idx[i]);
            }
        } else {
            kvmap_unpin(e->map, idx[i]);
            if (xret == 0) {
                e->stats.loaded++;
                e->stats.bytes_loaded += e->objsize;
            }
        }
    }
    pthread_mutex_unlock(&e->mu);
    free(idx);
    free(tbids);
    return ret;
}

int cache_store(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                uint64_t *bids, uint32_t bnum)
{
    return cache_op(wctx, keys, key_len, bids, bnum, true);
}

int cache_load(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
               uint64_t *bids, uint32_t bnum)
{
    return cache_op(wctx, keys, key_len, bids, bnum, false);
}

static uint32_t prefix_hits_locked(struct rt_entry *e, const uint8_t *keys,
                                   uint32_t key_num, uint32_t key_len)
{
    uint32_t i;
    for (i = 0; i < key_num; i++) {
        int64_t r = kvmap_find(e->map, keys + (uint64_t)i * key_len);
        e->stats.lookups++;
        if (r < 0 || kvmap_state(e->map, r) != KVMAP_READY)
            break;
        e->stats.lookup_hits++;
        kvmap_touch(e->map, r);
    }
    return i;
}

int cache_lookup(struct worker_context *wctx, uint8_t *keys, uint32_t key_num,
                 uint32_t key_len)
{
    struct rt_entry *e = get_entry(wctx);
    uint32_t hits;

    if (!e || !keys || key_len < KVMAP_KEY_LEN)
        return 0;
    pthread_mutex_lock(&e->mu);
    hits = prefix_hits_locked(e, keys, key_num, key_len);
    pthread_mutex_unlock(&e->mu);
    return (int)(hits * key_len);
}

int cache_lookup_batch(struct worker_context *wctx, const uint8_t *keys,
                       const uint32_t *key_nums, uint32_t num_req,
                       uint32_t key_len, uint32_t *hit_keys)
{
    struct rt_entry *e = get_entry(wctx);
    uint64_t off = 0;
    uint32_t r;

    if (!hit_keys || (num_req && !key_nums))
        return -EINVAL;
    if (!e) {
        for (r = 0; r < num_req; r++)
            hit_keys[r] = 0;
        return -ENOENT;
    }
    if (key_len < KVMAP_KEY_LEN || (num_req && !keys))
        return -EINVAL;
    pthread_mutex_lock(&e->mu);
    for (r = 0; r < num_req; r++) {
        hit_keys[r] = prefix_hits_locked(e, keys + off, key_nums[r], key_len);
        off += (uint64_t)key_nums[r] * key_len;
    }
    pthread_mutex_unlock(&e->mu);
    return 0;
}

int cache_get_stats(struct worker_context *wctx, struct cache_stats *out)
{
    struct rt_entry *e = get_entry(wctx);
    if (!e || !out)
        return -ENOENT;
    pthread_mutex_lock(&e->mu);
    *out = e->stats;
    out->records_used = kvmap_size(e->map);
    pthread_mutex_unlock(&e->mu);
    return 0;
}

int cache_clear(struct worker_context *wctx)
{
    struct rt_entry *e = get_entry(wctx);
    uint64_t i;

    if (!e)
        return -ENOENT;
    pthread_mutex_lock(&e->mu);
    for (i = 0; i < e->stats.records_total; i++) {
        if (kvmap_state(e->map, (int64_t)i) == KVMAP_READY &&
            kvmap_pins(e->map, (int64_t)i) == 0) {
            kvmap_remove(e->map, (int64_t)i);
            mempool_free_index(e->pool, (int64_t)i);
        }
    }
    pthread_mutex_unlock(&e->mu);
    return 0;
}
