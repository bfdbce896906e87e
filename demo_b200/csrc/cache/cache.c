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
 *   - records being loaded are pinned so eviction cannot recycle them.
 *
 * Disk tier (enabled when cache_init gets a directory; cache.c:222-278,
 * 471-504, 739-742, 759-787):
 *   - every stored record is also written to a file (write-through, as the
 *     reference's pipeline_io does), but behind the call: the store returns
 *     once the record is in host memory and a pool of IO threads writes it
 *     out, the record pinned until its file is complete.  cache_flush waits
 *     for those writes;
 *   - a lookup that misses in memory asks the disk (stat) and keeps walking
 *     on a hit (reference lookup_file);
 *   - a load reads the records missing from memory from their files in
 *     parallel into pool records, then moves them in the same batched
 *     host-to-device transfer as the memory hits; the read records stay
 *     cached in memory (reference pipeline_io PIPELINE_START branch).
 *   File naming and layout are in disk.h.
 */
#include "cache.h"
#include "device.h"
#include "disk.h"

#include "../infra/kvmap.h"
#include "../infra/log.h"
#include "../infra/mempool.h"
#include "../infra/threadpool.h"

#include <errno.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

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
    pthread_cond_t cv;         /* signalled when a disk write completes */

    uint32_t async_live;       /* async handles begun and not yet finished */
    int32_t busy;              /* API calls using the entry (g_mgr.mu) */
    int dfd;                   /* namespace directory, -1 without disk tier */
    uint32_t disk_pending;     /* write-behind jobs not yet finished */
    int disk_err;              /* first write error since the last flush */

    struct rt_entry *next;
};

/* paged geometry of a worker registered with cache_register_paged (workers
 * of plain cache_register have none: dense token-major planes) */
struct paged_geom {
    const void *k_ptrs;        /* the worker's imported K layer table */
    uint64_t block_stride;
    uint32_t head_bytes;
    struct paged_geom *next;
};

struct cache_manager {
    int initialised;
    uint32_t chunk_size;
    uint64_t pool_size;
    int backend;
    char *local_dir;
    int dirfd;                 /* root of the disk tier, -1 when disabled */
    threadpool_t *io_write;    /* write-behind of stored records */
    threadpool_t *io_read;     /* record reads of loads */
    adaptor_t *adaptor;
    pthread_mutex_t mu;        /* guards the entry list, dev_workers, busy */
    pthread_cond_t idle_cv;    /* an entry's busy count reached 0 */
    struct rt_entry *entries;
    uint32_t dev_workers[256]; /* registered workers per device (node_id) */
    pthread_mutex_t geom_mu;   /* leaf lock of geoms */
    struct paged_geom *geoms;
};

static struct cache_manager g_mgr = {.mu = PTHREAD_MUTEX_INITIALIZER,
                                     .idle_cv = PTHREAD_COND_INITIALIZER,
                                     .dirfd = -1,
                                     .geom_mu = PTHREAD_MUTEX_INITIALIZER};

/* the paged geometry of the worker whose K layer table is k_ptrs */
static void geom_of(const void *k_ptrs, uint64_t *block_stride, uint32_t *head_bytes)
{
    struct paged_geom *g;

    *block_stride = 0;
    *head_bytes = 0;
    pthread_mutex_lock(&g_mgr.geom_mu);
    for (g = g_mgr.geoms; g; g = g->next)
        if (g->k_ptrs == k_ptrs) {
            *block_stride = g->block_stride;
            *head_bytes = g->head_bytes;
            break;
        }
    pthread_mutex_unlock(&g_mgr.geom_mu);
}

static void geom_drop(const void *k_ptrs)
{
    struct paged_geom *g, **pp;

    pthread_mutex_lock(&g_mgr.geom_mu);
    for (pp = &g_mgr.geoms; (g = *pp); pp = &g->next)
        if (g->k_ptrs == k_ptrs) {
            *pp = g->next;
            free(g);
            break;
        }
    pthread_mutex_unlock(&g_mgr.geom_mu);
}

/* a store waits at most this long for write-behind to release pool records */
#define DISK_WAIT_SEC 30

struct disk_job {
    struct rt_entry *e;
    int64_t idx;
    uint8_t key[KVMAP_KEY_LEN];
    int ret;
    cc_latch_t *latch;         /* reads: the load's completion latch */
};

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

/* The entry of wctx's (model, world size, rank), held busy until
 * put_entry: the last cache_unregister unlinks an entry and waits for its
 * busy calls before freeing it (a lookup needs no registration of its own,
 * so it can race with the last worker leaving). */
static struct rt_entry *get_entry(struct worker_context *wctx)
{
    struct rt_entry *e;
    if (!g_mgr.initialised || !wctx || !wctx->model.model_name)
        return NULL;
    pthread_mutex_lock(&g_mgr.mu);
    e = find_entry_locked(wctx->model.model_name, wctx->world_size,
                          wctx->rank_id);
    if (e)
        e->busy++;
    pthread_mutex_unlock(&g_mgr.mu);
    return e;
}

static void put_entry(struct rt_entry *e)
{
    pthread_mutex_lock(&g_mgr.mu);
    if (--e->busy == 0)
        pthread_cond_broadcast(&g_mgr.idle_cv);
    pthread_mutex_unlock(&g_mgr.mu);
}

/* whether wctx's entry is registered (for error codes only) */
static int get_entry_exists(struct worker_context *wctx)
{
    struct rt_entry *e = get_entry(wctx);
    if (e)
        put_entry(e);
    return e != NULL;
}

/* with g_mgr.mu held: wait until no API call uses e (they all end) */
static void wait_idle_locked(struct rt_entry *e)
{
    while (e->busy)
        pthread_cond_wait(&g_mgr.idle_cv, &g_mgr.mu);
}

/* wait until every write-behind job of e finished; returns the first write
 * error since the last cache_flush, clearing it when `consume` is set */
static int drain_writes(struct rt_entry *e, int consume)
{
    int ret;

    pthread_mutex_lock(&e->mu);
    while (e->disk_pending)
        pthread_cond_wait(&e->cv, &e->mu);
    ret = e->disk_err;
    if (consume)
        e->disk_err = 0;
    pthread_mutex_unlock(&e->mu);
    return ret;
}

static void destroy_entry(struct rt_entry *e)
{
    drain_writes(e, 1);
    kvmap_destroy(e->map);
    mempool_destroy(e->pool);
    if (e->host_base && e->async_live) {
        /* copies of unfinished async handles may still reach the pool: keep
         * it mapped (and leak it) rather than let the device touch freed
         * memory */
        log_error("[%s] %u async transfers were never finished; their pinned pool is kept",
                  e->model_tag, e->async_live);
    } else if (e->host_base) {
        free_pinned_ptr(g_mgr.adaptor, e->host_base, e->pool_bytes);
    }
    if (e->dfd >= 0)
        close(e->dfd);
    pthread_cond_destroy(&e->cv);
    pthread_mutex_destroy(&e->mu);
    free(e->model_tag);
    free(e);
}

static int io_threads(void)
{
    const char *s = getenv("CROSSCACHE_IO_THREADS");
    int n = s ? atoi(s) : 4;     /* reference: threadpool_create("CaIO", 4) */
    return n < 1 ? 1 : (n > 64 ? 64 : n);
}

/* ------------------------------------------------------------------ */

int cache_init_backend(uint32_t chunk_size, uint64_t pool_size,
                       const char *root_dir, int backend)
{
    adaptor_t *ad;
    int ret = 0;

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
    g_mgr.dirfd = -1;
    g_mgr.io_write = g_mgr.io_read = NULL;
    g_mgr.local_dir = NULL;
    if (root_dir && *root_dir) {
        ret = disk_open_root(root_dir);
        if (ret < 0) {
            log_error("cache_init: cache dir %s: %d", root_dir, ret);
            goto fail;
        }
        g_mgr.dirfd = ret;
        ret = 0;
        g_mgr.local_dir = strdup(root_dir);
        g_mgr.io_write = threadpool_create("CaIOw", io_threads());
        g_mgr.io_read = threadpool_create("CaIOr", io_threads());
        if (!g_mgr.local_dir || !g_mgr.io_write || !g_mgr.io_read) {
            ret = -ENOMEM;
            goto fail;
        }
    }
    g_mgr.adaptor = ad;
    g_mgr.backend = backend;
    memset(g_mgr.dev_workers, 0, sizeof(g_mgr.dev_workers));
    g_mgr.chunk_size = chunk_size;
    g_mgr.pool_size = pool_size;
    g_mgr.entries = NULL;
    g_mgr.initialised = 1;
    pthread_mutex_unlock(&g_mgr.mu);
    log_info("cache_init chunk_size:%u pool_size:%lu backend:%d dir:%s",
             chunk_size, (unsigned long)pool_size, backend,
             g_mgr.local_dir ? g_mgr.local_dir : "(none)");
    return 0;

fail:
    threadpool_destroy(g_mgr.io_write);
    threadpool_destroy(g_mgr.io_read);
    g_mgr.io_write = g_mgr.io_read = NULL;
    if (g_mgr.dirfd >= 0)
        close(g_mgr.dirfd);
    g_mgr.dirfd = -1;
    free(g_mgr.local_dir);
    g_mgr.local_dir = NULL;
    if (backend == CACHE_BACKEND_CUDA)
        cuda_adaptor_destroy(ad);
    else
        mem_adaptor_destroy(ad);
    pthread_mutex_unlock(&g_mgr.mu);
    return ret;
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
    /* finishes every queued write before the pools go away */
    threadpool_destroy(g_mgr.io_write);
    threadpool_destroy(g_mgr.io_read);
    g_mgr.io_write = g_mgr.io_read = NULL;
    for (e = g_mgr.entries; e; e = n) {
        n = e->next;
        wait_idle_locked(e);
        destroy_entry(e);
    }
    g_mgr.entries = NULL;
    pthread_mutex_lock(&g_mgr.geom_mu);
    while (g_mgr.geoms) {
        struct paged_geom *g = g_mgr.geoms;
        g_mgr.geoms = g->next;
        free(g);
    }
    pthread_mutex_unlock(&g_mgr.geom_mu);
    if (g_mgr.backend == CACHE_BACKEND_CUDA)
        cuda_adaptor_destroy(g_mgr.adaptor);
    else
        mem_adaptor_destroy(g_mgr.adaptor);
    g_mgr.adaptor = NULL;
    if (g_mgr.dirfd >= 0)
        close(g_mgr.dirfd);
    g_mgr.dirfd = -1;
    free(g_mgr.local_dir);
    g_mgr.local_dir = NULL;
    g_mgr.initialised = 0;
    pthread_mutex_unlock(&g_mgr.mu);
}

int cache_register(struct worker_context *wctx)
{
    return cache_register_paged(wctx, 0, 0);
}

static int register_worker(struct worker_context *wctx);

int cache_register_paged(struct worker_context *wctx, uint64_t block_stride,
                         uint32_t head_bytes)
{
    struct paged_geom *g = NULL;
    uint64_t unit;
    int ret;

    if (!wctx || !wctx->block_size)
        return -EINVAL;
    unit = (uint64_t)wctx->model.hidden_dim_size * wctx->model.element_size;
    if ((block_stride && block_stride < (uint64_t)wctx->block_size * unit) ||
        (head_bytes && (!unit || unit % head_bytes)))
        return -EINVAL;
    if (block_stride || head_bytes) {
        g = calloc(1, sizeof(*g));
        if (!g)
            return -ENOMEM;
    }
    ret = register_worker(wctx);
    if (ret || !g) {
        free(g);
        return ret;
    }
    g->k_ptrs = wctx->k_ptrs;
    g->block_stride = block_stride;
    g->head_bytes = head_bytes;
    pthread_mutex_lock(&g_mgr.geom_mu);
    g->next = g_mgr.geoms;
    g_mgr.geoms = g;
    pthread_mutex_unlock(&g_mgr.geom_mu);
    return 0;
}

static int register_worker(struct worker_context *wctx)
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
        g_mgr.dev_workers[wctx->node_id]++;
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
    pthread_cond_init(&e->cv, NULL);
    e->dfd = -1;
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
    if (g_mgr.dirfd >= 0) {
        e->dfd = disk_open_ns(g_mgr.dirfd, e->model_tag, e->tp_size, e->tp_id);
        if (e->dfd < 0) {
            log_error("register: disk namespace of %s: %d", e->model_tag,
                      e->dfd);
            ret = e->dfd;
            e->dfd = -1;
            destroy_entry(e);
            pthread_mutex_unlock(&g_mgr.mu);
            goto unpin_v;
        }
    }
    e->stats.records_total = m_count;
    e->next = g_mgr.entries;
    g_mgr.entries = e;
    g_mgr.dev_workers[wctx->node_id]++;
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
    int last;

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
        *pp = e->next;          /* no new call finds it ... */
        wait_idle_locked(e);    /* ... and the running ones end first */
        destroy_entry(e);
    }
    pthread_mutex_unlock(&g_mgr.mu);
    if (wctx->k_ptrs) {
        geom_drop(wctx->k_ptrs);
        close_ipc_keys(g_mgr.adaptor, wctx->k_ptrs);
    }
    if (wctx->v_ptrs)
        close_ipc_keys(g_mgr.adaptor, wctx->v_ptrs);
    wctx->k_ptrs = wctx->v_ptrs = NULL;
    /* CUDA backend: releases this process's idle streams and staging
     * buffers on the device once its last registered worker has left
     * (another worker's transfers may be running); it never resets a
     * (shared) GPU. */
    pthread_mutex_lock(&g_mgr.mu);
    last = g_mgr.dev_workers[nid] > 0 && --g_mgr.dev_workers[nid] == 0;
    pthread_mutex_unlock(&g_mgr.mu);
    if (last)
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
    geom_of(wctx->k_ptrs, &tb.block_stride, &tb.head_bytes);
    ret = transfer_kvcache_batch(g_mgr.adaptor, &tb);
    free(recs);
    return ret;
}

/* ---- disk jobs ------------------------------------------------------ */

static void write_job(void *p)
{
    struct disk_job *j = p;
    struct rt_entry *e = j->e;
    int ret = disk_write(e->dfd, j->key, mempool_addr(e->pool, j->idx),
                         e->objsize);

    pthread_mutex_lock(&e->mu);
    kvmap_unpin(e->map, j->idx);
    if (ret == 0) {
        e->stats.disk_writes++;
        e->stats.bytes_written_disk += e->objsize;
    } else if (ret == 1) {
        e->stats.disk_write_skips++;
    } else {
        e->stats.disk_write_errors++;
        if (!e->disk_err)
            e->disk_err = ret;
    }
    e->disk_pending--;
    pthread_cond_broadcast(&e->cv);
    pthread_mutex_unlock(&e->mu);
    free(j);
}

static void read_job(void *p)
{
    struct disk_job *j = p;
    struct rt_entry *e = j->e;

    j->ret = disk_read(e->dfd, j->key, mempool_addr(e->pool, j->idx),
                       e->objsize);
    cc_latch_done(j->latch, 0);
}

/* queue the write-behind of records idx[0..n) (already pinned and counted
 * in disk_pending by the caller) */
static void submit_writes(struct rt_entry *e, const int64_t *idx,
                          const uint8_t *const *keys, uint32_t n)
{
    uint32_t i;

    for (i = 0; i < n; i++) {
        struct disk_job *j = calloc(1, sizeof(*j));
        if (j) {
            j->e = e;
            j->idx = idx[i];
            memcpy(j->key, keys[i], KVMAP_KEY_LEN);
            if (threadpool_submit(g_mgr.io_write, j, write_job) == 0)
                continue;
            write_job(j);          /* no queue slot: write inline */
            continue;
        }
        pthread_mutex_lock(&e->mu);
        kvmap_unpin(e->map, idx[i]);
        e->stats.disk_write_errors++;
        if (!e->disk_err)
            e->disk_err = -ENOMEM;
        e->disk_pending--;
        pthread_cond_broadcast(&e->cv);
        pthread_mutex_unlock(&e->mu);
    }
}

/* a free or evicted record index; with write-behind in flight, waits for
 * writes to release records.  Called and returns with e->mu held; may drop
 * it while waiting (then *waited is set and the caller re-checks its key). */
static int64_t alloc_record_locked(struct rt_entry *e, int *waited)
{
    struct timespec ts;
    int64_t r;

    *waited = 0;
    r = mempool_alloc_index(e->pool);
    if (r >= 0)
        return r;
    r = kvmap_evict_lru(e->map);
    if (r >= 0) {
        e->stats.evictions++;
        return r;
    }
    if (!e->disk_pending)
        return -1;
    clock_gettime(CLOCK_REALTIME, &ts);
    ts.tv_sec += DISK_WAIT_SEC;
    if (pthread_cond_timedwait(&e->cv, &e->mu, &ts))
        return -1;
    *waited = 1;
    return -1;
}

/* ---- store / load --------------------------------------------------- */

struct op_args {
    struct rt_entry *e;
    struct worker_context *wctx;
    const uint8_t *keys;
    uint32_t key_len;
    const uint64_t *bids;
    uint32_t key_num;
    uint32_t bpc;
    int64_t *idx;              /* [key_num] record per transferred key */
    uint64_t *tbids;           /* [key_num * bpc] their block ids */
    uint32_t *kpos;            /* [key_num] key index of each transfer */
    uint8_t *from_disk;        /* [key_num] load: record read from a file */
    int32_t *kstat;            /* [key_num] per-key result, or NULL */
};

/* the first failure of key i, for the batch entry points */
static void key_fail(struct op_args *a, uint32_t i, int ret)
{
    if (a->kstat && !a->kstat[i])
        a->kstat[i] = ret;
}

static void add_transfer(struct op_args *a, uint32_t *n, uint32_t i,
                         int64_t r, int from_disk)
{
    a->idx[*n] = r;
    a->kpos[*n] = i;
    a->from_disk[*n] = (uint8_t)from_disk;
    memcpy(a->tbids + (uint64_t)*n * a->bpc, a->bids + (uint64_t)i * a->bpc,
           a->bpc * sizeof(uint64_t));
    (*n)++;
}

static int do_store(struct op_args *a)
{
    struct rt_entry *e = a->e;
    const uint8_t **wkeys = NULL;
    uint32_t i, n = 0;
    int ret = 0, xret, waited;

    pthread_mutex_lock(&e->mu);
    for (i = 0; i < a->key_num; i++) {
        const uint8_t *key = a->keys + (uint64_t)i * a->key_len;
        int64_t r;
    again:
        r = kvmap_find(e->map, key);
        if (r >= 0) {                   /* cached or in flight: keep it */
            e->stats.store_dedup++;
            continue;
        }
        r = alloc_record_locked(e, &waited);
        if (waited)
            goto again;
        if (r < 0) {
            log_warn("store: pool exhausted (all records pinned/in flight)");
            ret = -ENOMEM;
            for (; i < a->key_num; i++)
                key_fail(a, i, -ENOMEM);
            break;
        }
        kvmap_insert(e->map, r, key, KVMAP_PENDING);
        add_transfer(a, &n, i, r, 0);
    }
    pthread_mutex_unlock(&e->mu);

    xret = n ? run_transfer(e, a->wctx, KV_D_TO_H, a->idx, a->tbids, n) : 0;
    if (xret < 0 && ret == 0)
        ret = xret;
    for (i = 0; xret && i < n; i++)
        key_fail(a, a->kpos[i], xret);

    if (xret == 0 && n && e->dfd >= 0)
        wkeys = malloc(n * sizeof(*wkeys));
    pthread_mutex_lock(&e->mu);
    for (i = 0; i < n; i++) {
        if (xret == 0) {
            kvmap_publish(e->map, a->idx[i]);
            e->stats.stored++;
            e->stats.bytes_saved += e->objsize;
            if (wkeys) {
                kvmap_pin(e->map, a->idx[i]);   /* until its file is written */
                e->disk_pending++;
                wkeys[i] = a->keys + (uint64_t)a->kpos[i] * a->key_len;
            }
        } else {
            kvmap_remove(e->map, a->idx[i]);
            mempool_free_index(e->pool, a->idx[i]);
        }
    }
    if (xret == 0 && n && e->dfd >= 0 && !wkeys) {
        e->stats.disk_write_errors += n;
        if (!e->disk_err)
            e->disk_err = -ENOMEM;
    }
    pthread_mutex_unlock(&e->mu);
    if (wkeys) {
        submit_writes(e, a->idx, wkeys, n);
        free(wkeys);
    }
    return ret;
}

static int do_load(struct op_args *a)
{
    struct rt_entry *e = a->e;
    uint32_t i, n = 0, nc = 0, nd = 0, ok;
    uint32_t *cand = NULL;
    struct disk_job *jobs = NULL;
    cc_latch_t latch;
    int ret = 0, xret, waited;

    if (e->dfd >= 0) {
        cand = malloc(a->key_num * sizeof(*cand));
        if (!cand)
            return -ENOMEM;
    }
    /* 1. memory hits are pinned; absent keys become disk candidates */
    pthread_mutex_lock(&e->mu);
    for (i = 0; i < a->key_num; i++) {
        const uint8_t *key = a->keys + (uint64_t)i * a->key_len;
        int64_t r = kvmap_find(e->map, key);
        if (r >= 0 && kvmap_state(e->map, r) == KVMAP_READY) {
            kvmap_touch(e->map, r);
            kvmap_pin(e->map, r);
            add_transfer(a, &n, i, r, 0);
        } else if (r < 0 && cand) {
            cand[nc++] = i;
        } else {
            e->stats.load_misses++;
            key_fail(a, i, -ENOENT);
            ret = -ENOENT;
        }
    }
    pthread_mutex_unlock(&e->mu);

    /* 2. which candidates have a file (no lock held) */
    for (i = 0; i < nc; i++) {
        if (disk_stat(e->dfd, a->keys + (uint64_t)cand[i] * a->key_len,
                      e->objsize) == 0)
            cand[nd++] = cand[i];
        else
            key_fail(a, cand[i], -ENOENT);
    }

    /* 3. a PENDING record per file; a key another thread cached meanwhile
     *    is a memory hit after all */
    pthread_mutex_lock(&e->mu);
    if (nd < nc) {
        e->stats.load_misses += nc - nd;
        ret = -ENOENT;
    }
    for (i = 0; i < nd; i++) {
        const uint8_t *key = a->keys + (uint64_t)cand[i] * a->key_len;
        int64_t r;
    again:
        r = kvmap_find(e->map, key);
        if (r >= 0) {
            if (kvmap_state(e->map, r) == KVMAP_READY) {
                kvmap_touch(e->map, r);
                kvmap_pin(e->map, r);
                add_transfer(a, &n, cand[i], r, 0);
            } else {
                e->stats.load_misses++;
                key_fail(a, cand[i], -ENOENT);
                ret = -ENOENT;
            }
            continue;
        }
        r = alloc_record_locked(e, &waited);
        if (waited)
            goto again;
        if (r < 0) {
            log_warn("load: no pool record free for a disk read");
            e->stats.load_misses++;
            key_fail(a, cand[i], -ENOMEM);
            ret = -ENOMEM;
            continue;
        }
        kvmap_insert(e->map, r, key, KVMAP_PENDING);
        add_transfer(a, &n, cand[i], r, 1);
    }
    pthread_mutex_unlock(&e->mu);
    free(cand);

    /* 4. read the files in parallel */
    for (i = 0, nd = 0; i < n; i++)
        nd += a->from_disk[i];
    if (nd) {
        jobs = calloc(n, sizeof(*jobs));
        if (jobs) {
            cc_latch_init(&latch, nd);
            for (i = 0; i < n; i++) {
                struct disk_job *j = &jobs[i];
                if (!a->from_disk[i])
                    continue;
                j->e = e;
                j->idx = a->idx[i];
                memcpy(j->key, a->keys + (uint64_t)a->kpos[i] * a->key_len,
                       KVMAP_KEY_LEN);
                j->latch = &latch;
                if (threadpool_submit(g_mgr.io_read, j, read_job))
                    read_job(j);
            }
            cc_latch_wait(&latch);
            cc_latch_fini(&latch);
        }
    }
    /* drop failed reads from the transfer list */
    for (i = 0, ok = 0; i < n; i++) {
        int rr = !a->from_disk[i] ? 0 : (jobs ? jobs[i].ret : -ENOMEM);
        if (rr == 0) {
            if (ok != i) {
                a->idx[ok] = a->idx[i];
                a->kpos[ok] = a->kpos[i];
                a->from_disk[ok] = a->from_disk[i];
                memcpy(a->tbids + (uint64_t)ok * a->bpc,
                       a->tbids + (uint64_t)i * a->bpc,
                       a->bpc * sizeof(uint64_t));
            }
            ok++;
            continue;
        }
        pthread_mutex_lock(&e->mu);
        kvmap_remove(e->map, a->idx[i]);
        mempool_free_index(e->pool, a->idx[i]);
        e->stats.disk_read_errors++;
        e->stats.load_misses++;
        pthread_mutex_unlock(&e->mu);
        key_fail(a, a->kpos[i], rr == -ENOENT ? -ENOENT : -EIO);
        if (ret == 0)
            ret = rr == -ENOENT ? -ENOENT : -EIO;
    }
    free(jobs);
    n = ok;

    /* 5. one batched host-to-device transfer for memory and disk records */
    xret = n ? run_transfer(e, a->wctx, KV_H_TO_D, a->idx, a->tbids, n) : 0;
    if (xret < 0 && ret == 0)
        ret = xret;
    for (i = 0; xret && i < n; i++)
        key_fail(a, a->kpos[i], xret);

    /* 6. records read from disk join the memory tier (their host copy is
     *    valid even when the device transfer failed) */
    pthread_mutex_lock(&e->mu);
    for (i = 0; i < n; i++) {
        if (a->from_disk[i]) {
            kvmap_publish(e->map, a->idx[i]);
            e->stats.disk_reads++;
            e->stats.bytes_read_disk += e->objsize;
        } else {
            kvmap_unpin(e->map, a->idx[i]);
        }
        if (xret == 0) {
            e->stats.loaded++;
            e->stats.bytes_loaded += e->objsize;
        }
    }
    pthread_mutex_unlock(&e->mu);
    return ret;
}

static int cache_op(struct worker_context *wctx, uint8_t *keys,
                    uint32_t key_len, uint64_t *bids, uint32_t bnum,
                    bool store, int32_t *kstat)
{
    struct op_args a;
    int ret;

    memset(&a, 0, sizeof(a));
    a.kstat = kstat;
    if (!keys || key_len < KVMAP_KEY_LEN || (bnum && !bids))
        return get_entry_exists(wctx) ? -EINVAL : -ENOENT;
    a.e = get_entry(wctx);
    if (!a.e)
        return -ENOENT;
    if (!wctx->k_ptrs) {
        put_entry(a.e);
        return -EINVAL;
    }
    a.wctx = wctx;
    a.keys = keys;
    a.key_len = key_len;
    a.bids = bids;
    a.bpc = g_mgr.chunk_size / wctx->block_size;
    a.key_num = bnum / a.bpc;
    if (!a.key_num) {
        put_entry(a.e);
        return 0;
    }
    a.idx = malloc(a.key_num * sizeof(int64_t));
    a.kpos = malloc(a.key_num * sizeof(uint32_t));
    a.from_disk = malloc(a.key_num);
    a.tbids = malloc((uint64_t)a.key_num * a.bpc * sizeof(uint64_t));
    if (!a.idx || !a.kpos || !a.from_disk || !a.tbids)
        ret = -ENOMEM;
    else
        ret = store ? do_store(&a) : do_load(&a);
    free(a.idx);
    free(a.kpos);
    free(a.from_disk);
    free(a.tbids);
    put_entry(a.e);
    return ret;
}

int cache_store(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                uint64_t *bids, uint32_t bnum)
{
    return cache_op(wctx, keys, key_len, bids, bnum, true, NULL);
}

int cache_load(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
               uint64_t *bids, uint32_t bnum)
{
    return cache_op(wctx, keys, key_len, bids, bnum, false, NULL);
}

/* several requests in one batched transfer, with a result per request */
static int batch_op(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                    const uint32_t *key_nums, uint32_t num_req, uint64_t *bids,
                    int32_t *req_status, bool store)
{
    uint64_t total = 0, off = 0;
    uint32_t r, k, bpc;
    int32_t *kstat;
    int ret;

    if (!req_status || (num_req && !key_nums))
        return -EINVAL;
    if (!get_entry_exists(wctx)) {
        for (r = 0; r < num_req; r++)
            req_status[r] = -ENOENT;
        return -ENOENT;
    }
    bpc = g_mgr.chunk_size / wctx->block_size;
    for (r = 0; r < num_req; r++)
        total += key_nums[r];
    if (total * bpc > UINT32_MAX)
        return -E2BIG;
    kstat = calloc(total ? total : 1, sizeof(*kstat));
    if (!kstat)
        return -ENOMEM;
    ret = cache_op(wctx, keys, key_len, bids, (uint32_t)(total * bpc), store, kstat);
    for (r = 0; r < num_req; r++) {
        req_status[r] = 0;
        for (k = 0; k < key_nums[r]; k++)
            if (kstat[off + k] && !req_status[r])
                req_status[r] = kstat[off + k];
        off += key_nums[r];
    }
    free(kstat);
    return ret;
}

int cache_store_batch(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                      const uint32_t *key_nums, uint32_t num_req, uint64_t *bids,
                      int32_t *req_status)
{
    return batch_op(wctx, keys, key_len, key_nums, num_req, bids, req_status, true);
}

int cache_load_batch(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                     const uint32_t *key_nums, uint32_t num_req, uint64_t *bids,
                     int32_t *req_status)
{
    return batch_op(wctx, keys, key_len, key_nums, num_req, bids, req_status, false);
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

/* leading hits of one request: memory first; past the first memory miss,
 * keys are asked of the disk tier one by one (reference cache.c:733-742),
 * with the entry lock dropped around each stat */
static uint32_t prefix_hits(struct rt_entry *e, const uint8_t *keys,
                            uint32_t key_num, uint32_t key_len)
{
    uint32_t i = 0;

    pthread_mutex_lock(&e->mu);
    for (;;) {
        i += prefix_hits_locked(e, keys + (uint64_t)i * key_len, key_num - i,
                                key_len);
        if (i >= key_num || e->dfd < 0)
            break;
        pthread_mutex_unlock(&e->mu);
        if (disk_stat(e->dfd, keys + (uint64_t)i * key_len, e->objsize)) {
            pthread_mutex_lock(&e->mu);
            break;
        }
        pthread_mutex_lock(&e->mu);
        e->stats.lookup_hits++;
        e->stats.disk_lookup_hits++;
        i++;
    }
    pthread_mutex_unlock(&e->mu);
    return i;
}

int cache_lookup(struct worker_context *wctx, uint8_t *keys, uint32_t key_num,
                 uint32_t key_len)
{
    struct rt_entry *e;
    int ret;

    if (!keys || key_len < KVMAP_KEY_LEN)
        return 0;
    e = get_entry(wctx);
    if (!e)
        return 0;
    ret = (int)(prefix_hits(e, keys, key_num, key_len) * key_len);
    put_entry(e);
    return ret;
}

int cache_lookup_batch(struct worker_context *wctx, const uint8_t *keys,
                       const uint32_t *key_nums, uint32_t num_req,
                       uint32_t key_len, uint32_t *hit_keys)
{
    struct rt_entry *e;
    uint64_t off = 0;
    uint32_t r;

    if (!hit_keys || (num_req && !key_nums))
        return -EINVAL;
    e = get_entry(wctx);
    if (!e) {
        for (r = 0; r < num_req; r++)
            hit_keys[r] = 0;
        return -ENOENT;
    }
    if (key_len < KVMAP_KEY_LEN || (num_req && !keys)) {
        put_entry(e);
        return -EINVAL;
    }
    if (e->dfd >= 0) {
        for (r = 0; r < num_req; r++) {
            hit_keys[r] = prefix_hits(e, keys + off, key_nums[r], key_len);
            off += (uint64_t)key_nums[r] * key_len;
        }
    } else {
        /* memory only: one lock acquisition for the whole batch */
        pthread_mutex_lock(&e->mu);
        for (r = 0; r < num_req; r++) {
            hit_keys[r] = prefix_hits_locked(e, keys + off, key_nums[r], key_len);
            off += (uint64_t)key_nums[r] * key_len;
        }
        pthread_mutex_unlock(&e->mu);
    }
    put_entry(e);
    return 0;
}

int cache_flush(struct worker_context *wctx)
{
    struct rt_entry *e = get_entry(wctx);
    int ret;

    if (!e)
        return -ENOENT;
    ret = drain_writes(e, 1);
    put_entry(e);
    return ret;
}

int cache_get_stats(struct worker_context *wctx, struct cache_stats *out)
{
    struct rt_entry *e;
    if (!out)
        return -ENOENT;
    e = get_entry(wctx);
    if (!e)
        return -ENOENT;
    pthread_mutex_lock(&e->mu);
    *out = e->stats;
    out->records_used = kvmap_size(e->map);
    pthread_mutex_unlock(&e->mu);
    put_entry(e);
    return 0;
}

int cache_clear(struct worker_context *wctx)
{
    struct rt_entry *e = get_entry(wctx);
    uint64_t i;

    if (!e)
        return -ENOENT;
    drain_writes(e, 0);     /* write-behind pins its records until done */
    pthread_mutex_lock(&e->mu);
    for (i = 0; i < e->stats.records_total; i++) {
        if (kvmap_state(e->map, (int64_t)i) == KVMAP_READY &&
            kvmap_pins(e->map, (int64_t)i) == 0) {
            kvmap_remove(e->map, (int64_t)i);
            mempool_free_index(e->pool, (int64_t)i);
        }
    }
    pthread_mutex_unlock(&e->mu);
    put_entry(e);
    return 0;
}

/* ---- asynchronous, layer-ordered store / load ------------------------ */

struct cache_async {
    struct rt_entry *e;
    struct transfer_async *x;
    int store;
    uint32_t n;                /* records covered */
    int64_t *idx;
    uint8_t *keys;             /* store: KVMAP_KEY_LEN bytes per record */
    uint8_t *layer_done;       /* store: one flag per layer */
    uint32_t num_layers;
    int status;                /* first device failure while enqueuing */
};

static void async_free(struct cache_async *h)
{
    free(h->idx);
    free(h->keys);
    free(h->layer_done);
    free(h);
}

static int async_begin_entry(struct rt_entry *e, struct worker_context *wctx, uint8_t *keys,
                             uint32_t key_len, uint64_t *bids, uint32_t bnum, int store,
                             cache_async_t **out);

static int async_begin(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                       uint64_t *bids, uint32_t bnum, int store, cache_async_t **out)
{
    struct rt_entry *e;
    int ret;

    if (!out)
        return -EINVAL;
    *out = NULL;
    if (!wctx)
        return -ENOENT;
    if (!keys || key_len < KVMAP_KEY_LEN || (bnum && !bids) || !wctx->k_ptrs)
        return get_entry_exists(wctx) ? -EINVAL : -ENOENT;
    e = get_entry(wctx);
    if (!e)
        return -ENOENT;
    ret = async_begin_entry(e, wctx, keys, key_len, bids, bnum, store, out);
    put_entry(e);
    return ret;
}

/* async_begin with e held busy by the caller */
static int async_begin_entry(struct rt_entry *e, struct worker_context *wctx, uint8_t *keys,
                             uint32_t key_len, uint64_t *bids, uint32_t bnum, int store,
                             cache_async_t **out)
{
    struct cache_async *h;
    struct transfer_batch tb;
    uint64_t *tbids = NULL;
    void **recs = NULL;
    uint32_t bpc, key_num, i, misses = 0;
    int ret = 0, err = 0, waited;

    bpc = g_mgr.chunk_size / wctx->block_size;
    key_num = bnum / bpc;
    h = calloc(1, sizeof(*h));
    if (!h)
        return -ENOMEM;
    h->e = e;
    h->store = store;
    h->num_layers = wctx->model.num_layers;
    h->idx = malloc((key_num ? key_num : 1) * sizeof(int64_t));
    h->keys = store ? malloc((key_num ? key_num : 1) * (size_t)KVMAP_KEY_LEN) : NULL;
    h->layer_done = store ? calloc(h->num_layers, 1) : NULL;
    tbids = malloc(((uint64_t)key_num * bpc + 1) * sizeof(uint64_t));
    recs = malloc((key_num ? key_num : 1) * sizeof(void *));
    if (!h->idx || (store && (!h->keys || !h->layer_done)) || !tbids || !recs) {
        free(tbids);
        free(recs);
        async_free(h);
        return -ENOMEM;
    }

    pthread_mutex_lock(&e->mu);
    for (i = 0; i < key_num; i++) {
        const uint8_t *key = keys + (uint64_t)i * key_len;
        int64_t r;
    again:
        r = kvmap_find(e->map, key);
        if (store) {
            if (r >= 0) {
                e->stats.store_dedup++;
                continue;
            }
            r = alloc_record_locked(e, &waited);
            if (waited)
                goto again;
            if (r < 0) {
                ret = -ENOMEM;
                break;
            }
            kvmap_insert(e->map, r, key, KVMAP_PENDING);
            memcpy(h->keys + (uint64_t)h->n * KVMAP_KEY_LEN, key, KVMAP_KEY_LEN);
        } else {
            if (r < 0 || kvmap_state(e->map, r) != KVMAP_READY) {
                e->stats.load_misses++;
                misses++;
                continue;
            }
            kvmap_touch(e->map, r);
            kvmap_pin(e->map, r);
        }
        h->idx[h->n] = r;
        recs[h->n] = mempool_addr(e->pool, r);
        memcpy(tbids + (uint64_t)h->n * bpc, bids + (uint64_t)i * bpc, bpc * sizeof(uint64_t));
        h->n++;
    }
    pthread_mutex_unlock(&e->mu);

    memset(&tb, 0, sizeof(tb));
    tb.keys_ptrs = wctx->k_ptrs;
    tb.value_ptrs = wctx->v_ptrs;
    tb.page_buffer_size = (uint64_t)wctx->num_blocks * wctx->block_size;
    tb.records = recs;
    tb.block_ids = tbids;
    tb.num_records = h->n;
    tb.block_size = wctx->block_size;
    tb.hidden_dim_size = wctx->model.hidden_dim_size;
    tb.num_layers = wctx->model.num_layers;
    tb.num_tokens = (uint16_t)g_mgr.chunk_size;
    tb.devid = wctx->node_id;
    tb.caches_element_size = wctx->model.element_size;
    tb.direction = store ? KV_D_TO_H : KV_H_TO_D;
    geom_of(wctx->k_ptrs, &tb.block_stride, &tb.head_bytes);
    h->x = ret ? NULL : transfer_async_begin(g_mgr.adaptor, &tb, &err);
    free(tbids);
    free(recs);
    if (h->x) {
        pthread_mutex_lock(&e->mu);
        e->async_live++;
        pthread_mutex_unlock(&e->mu);
    }
    if (!h->x) {
        if (!ret)
            ret = err ? err : -EIO;
        pthread_mutex_lock(&e->mu);
        for (i = 0; i < h->n; i++) {
            if (store) {
                kvmap_remove(e->map, h->idx[i]);
                mempool_free_index(e->pool, h->idx[i]);
            } else {
                kvmap_unpin(e->map, h->idx[i]);
            }
        }
        pthread_mutex_unlock(&e->mu);
        async_free(h);
        return ret;
    }
    *out = h;
    return misses ? -ENOENT : 0;
}

int cache_load_async(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                     uint64_t *bids, uint32_t bnum, cache_async_t **out)
{
    return async_begin(wctx, keys, key_len, bids, bnum, 0, out);
}

int cache_store_async(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                      uint64_t *bids, uint32_t bnum, cache_async_t **out)
{
    return async_begin(wctx, keys, key_len, bids, bnum, 1, out);
}

int cache_async_layers(cache_async_t *h, uint32_t layer_begin, uint32_t layer_end,
                       void *stream, void *wait_event)
{
    uint32_t l;
    int ret;

    if (!h || layer_begin >= layer_end || layer_end > h->num_layers)
        return -EINVAL;
    ret = transfer_async_layers(g_mgr.adaptor, h->x, layer_begin, layer_end, stream, wait_event);
    if (ret) {
        /* a rejected request (-EINVAL) enqueued nothing; a device failure
         * fails the whole handle (a store missing layers fails anyway) */
        if (ret != -EINVAL && !h->status)
            h->status = ret;
        return ret;
    }
    if (h->store)
        for (l = layer_begin; l < layer_end; l++)
            h->layer_done[l] = 1;
    return 0;
}

int cache_async_stream_wait(cache_async_t *h, uint32_t layer, void *stream)
{
    if (!h)
        return -EINVAL;
    return transfer_async_stream_wait(g_mgr.adaptor, h->x, layer, stream);
}

int cache_async_query(cache_async_t *h)
{
    if (!h)
        return -EINVAL;
    return transfer_async_query(g_mgr.adaptor, h->x);
}

uint32_t cache_async_records(const cache_async_t *h)
{
    return h ? h->n : 0;
}

int cache_async_finish(cache_async_t *h)
{
    struct rt_entry *e;
    const uint8_t **wkeys = NULL;
    uint32_t i, l, nw = 0;
    int64_t *widx = NULL;
    int ret, complete = 1;

    if (!h)
        return -EINVAL;
    e = h->e;
    ret = transfer_async_end(g_mgr.adaptor, h->x);
    if (ret == -ETIMEDOUT) {
        /* the device may still touch these records: keep them pinned /
         * pending, and the handle counted so the pool is never freed */
        log_error("async %s of %u records timed out; records stay reserved",
                  h->store ? "store" : "load", h->n);
        async_free(h);
        return ret;
    }
    if (!ret && h->status)
        ret = h->status;
    if (h->store) {
        for (l = 0; l < h->num_layers; l++)
            complete = complete && h->layer_done[l];
        if (!ret && !complete && h->n)
            ret = -EINVAL;             /* a record needs every layer */
        if (!ret && h->n && e->dfd >= 0) {
            wkeys = malloc(h->n * sizeof(*wkeys));
            widx = malloc(h->n * sizeof(*widx));
        }
    }
    pthread_mutex_lock(&e->mu);
    e->async_live--;
    for (i = 0; i < h->n; i++) {
        if (!h->store) {
            kvmap_unpin(e->map, h->idx[i]);
            if (!ret) {
                e->stats.loaded++;
                e->stats.bytes_loaded += e->objsize;
            }
        } else if (!ret) {
            kvmap_publish(e->map, h->idx[i]);
            e->stats.stored++;
            e->stats.bytes_saved += e->objsize;
            if (wkeys && widx) {
                kvmap_pin(e->map, h->idx[i]);
                e->disk_pending++;
                wkeys[nw] = h->keys + (uint64_t)i * KVMAP_KEY_LEN;
                widx[nw++] = h->idx[i];
            }
        } else {
            kvmap_remove(e->map, h->idx[i]);
            mempool_free_index(e->pool, h->idx[i]);
        }
    }
    pthread_mutex_unlock(&e->mu);
    if (nw)
        submit_writes(e, widx, wkeys, nw);
    free(wkeys);
    free(widx);
    async_free(h);
    return ret;
}
