/*
 * Cache-manager C API.
 *
 * The seven reference entry points keep the names, arguments, return
 * conventions and semantics of CrossCache's include/cache/cache.h:8-23
 * (implemented there in src/cache/cache.c:598-802):
 *
 *   cache_init        chunk_size tokens per record, pool_size bytes of pinned
 *                     host memory per registered (model, tp_size, tp_rank),
 *                     root_dir for the disk tier (NULL or "": memory only;
 *                     created if missing, one level).  CUDA backend.
 *   cache_register    import the worker's per-layer KV handles, allocate and
 *                     pin the record pool.  0 or -ENOMEM/-EINVAL.
 *   cache_lookup      walk keys in order and stop at the first key that is
 *                     not cached; returns the BYTE OFFSET i * key_len of the
 *                     first miss (reference cache.c:712-745).
 *   cache_store       save bnum blocks as bnum / (chunk_size / block_size)
 *                     records, one 32-byte key per record (cache.c:513-593).
 *   cache_load        restore records for the keys into the given blocks.
 *
 * With a disk tier every stored record is also written to
 * <root_dir>/<model tag>.tp<tp_size>.<tp_rank>/<64 hex digits of its key>
 * by IO threads after cache_store returns; lookups and loads fall back to
 * those files for keys that are not in memory, across restarts too.
 *
 * Additions (new, no reference counterpart) are listed after them.
 */
#ifndef __CACHE_H__
#define __CACHE_H__

#include "inner.h"

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int cache_register(struct worker_context *wctx);

void cache_unregister(struct worker_context *wctx);

int cache_lookup(struct worker_context *wctx, uint8_t *keys,
                 uint32_t key_num, uint32_t key_len);

int cache_store(struct worker_context *wctx, uint8_t *keys,
                uint32_t key_len, uint64_t *bids, uint32_t bnum);

int cache_load(struct worker_context *wctx, uint8_t *keys,
               uint32_t key_len, uint64_t *bids, uint32_t bnum);

int cache_init(uint32_t chunk_size, uint64_t pool_size, const char *root_dir);

void cache_exit();

/* ---- new -------------------------------------------------------------- */

#define CACHE_BACKEND_CUDA 0   /* sm_100a kernels + copy engines (default) */
#define CACHE_BACKEND_MEM  1   /* host memcpy; paged cache in host memory   */

/* cache_init with an explicit device backend.  cache_init() is
 * cache_init_backend(..., CACHE_BACKEND_CUDA). */
int cache_init_backend(uint32_t chunk_size, uint64_t pool_size,
                       const char *root_dir, int backend);

/* cache_register for a worker whose layer planes are not dense token-major
 * (the reference supports only vLLM FlashAttention's
 * [2][num_blocks][block_size][heads][head_dim]).  block_stride = bytes
 * between consecutive blocks of a plane (0: block_size * unit); head_bytes
 * > 0 marks head-major blocks [unit / head_bytes][block_size][head_bytes]
 * (kv_copy_desc in kvcopy.h).  vLLM FlashInfer on sm_100 registers K
 * planes at each layer tensor, V planes half a block later, block_stride =
 * 2 * block_size * unit and head_bytes = head_dim * element size.  Records
 * stay token-major, so workers of different geometries share records.
 * cache_register(w) is cache_register_paged(w, 0, 0).  -EINVAL for a
 * block_stride below block_size * unit or a head_bytes not dividing the
 * unit; otherwise as cache_register. */
int cache_register_paged(struct worker_context *wctx, uint64_t block_stride,
                         uint32_t head_bytes);

/* Batched prefix lookup over num_req requests.  Request r owns key_nums[r]
 * consecutive keys of key_len bytes (requests are packed back to back in
 * keys).  hit_keys[r] receives the number of leading keys of request r that
 * are cached -- the value cache_lookup would return divided by key_len.
 * Hits refresh the LRU position of their records.  Returns 0 or -ENOENT when
 * the worker is not registered (then every hit_keys[r] is 0). */
int cache_lookup_batch(struct worker_context *wctx, const uint8_t *keys,
                       const uint32_t *key_nums, uint32_t num_req,
                       uint32_t key_len, uint32_t *hit_keys);

/* cache_store / cache_load of num_req requests in one batched transfer.
 * Request r owns key_nums[r] consecutive keys (key_len bytes each) and the
 * key_nums[r] * (chunk_size / block_size) consecutive block ids that go with
 * them.  req_status[r] receives request r's own result: 0, or the first
 * error among its keys (-ENOENT for a key that is not cached, -ENOMEM, a
 * transfer error), so a miss of one request does not fail the others.
 * Returns 0 when every request succeeded, else the first error (the
 * cache_store / cache_load convention), or -EINVAL / -ENOENT (unregistered
 * worker: every req_status is -ENOENT). */
int cache_store_batch(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                      const uint32_t *key_nums, uint32_t num_req, uint64_t *bids,
                      int32_t *req_status);
int cache_load_batch(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                     const uint32_t *key_nums, uint32_t num_req, uint64_t *bids,
                     int32_t *req_status);

struct cache_stats {
    uint64_t records_total;     /* records the pinned pool holds          */
    uint64_t records_used;      /* records currently mapped to a key      */
    uint64_t lookups;           /* keys examined by lookups               */
    uint64_t lookup_hits;       /* ... of which cached                    */
    uint64_t stored;            /* records written by cache_store         */
    uint64_t store_dedup;       /* store keys already cached (no copy)    */
    uint64_t loaded;            /* records restored by cache_load         */
    uint64_t load_misses;       /* load keys that were not cached         */
    uint64_t evictions;         /* records reclaimed by LRU eviction      */
    uint64_t bytes_saved;
    uint64_t bytes_loaded;
    /* disk tier */
    uint64_t disk_writes;       /* record files written                   */
    uint64_t disk_write_skips;  /* ... already on disk, not rewritten      */
    uint64_t disk_write_errors;
    uint64_t disk_reads;        /* records a load read from files         */
    uint64_t disk_read_errors;  /* files that vanished or failed to read   */
    uint64_t disk_lookup_hits;  /* lookup keys found on disk only          */
    uint64_t bytes_written_disk;
    uint64_t bytes_read_disk;
};

/* Counters of the (model, world_size, rank_id) entry of wctx.  0 or -ENOENT. */
int cache_get_stats(struct worker_context *wctx, struct cache_stats *out);

/* Drop every cached record of wctx's entry from memory (the pool stays
 * pinned; record files of the disk tier stay).  Waits for pending disk
 * writes first.  0 or -ENOENT. */
int cache_clear(struct worker_context *wctx);

/* Wait until every record stored so far through wctx's entry is written to
 * its file.  Returns 0, the first write error (-errno) since the previous
 * cache_flush, or -ENOENT when the worker is not registered.  Without a
 * disk tier it returns 0 at once. */
int cache_flush(struct worker_context *wctx);

/* ---- asynchronous, layer-ordered store / load (new) -------------------
 * For a caller that overlaps the transfer with its own kernels layer by
 * layer (vLLM's wait_for_layer_load / save_kv_layer).  The kernels move the
 * records straight between the paged cache and the pinned host pool (no
 * staging), each launch capped to a few CTAs (CROSSCACHE_ASYNC_CTAS, 32).
 *
 *   cache_load_async    pins the cached records of the keys (keys that are
 *                       not cached are skipped: -ENOENT, with a valid handle
 *                       for the others) and returns a handle; nothing moves
 *                       yet.  Memory tier only.
 *   cache_store_async   reserves a record per new key (keys already cached
 *                       are skipped, as cache_store does); nothing moves yet.
 *   cache_async_layers  enqueue the copy of layers [layer_begin, layer_end)
 *                       on `stream` (cudaStream_t of the worker's device)
 *                       after `wait_event` (cudaEvent_t or NULL).  The CPU
 *                       backend copies at once and takes NULL for both.
 *   cache_async_stream_wait
 *                       make `stream` wait (on the GPU) for the enqueued
 *                       copy covering `layer`; -ENOENT if none was enqueued.
 *   cache_async_query   1 when all enqueued copies finished, 0 if not.
 *   cache_async_finish  wait for them (deadline CROSSCACHE_TIMEOUT_MS) and
 *                       release the handle.  A load unpins its records; a
 *                       store publishes its records when every layer was
 *                       enqueued and the kernels succeeded (then the disk
 *                       tier writes them), else drops them.  0, -EINVAL
 *                       (bad block id, or a store missing layers),
 *                       -ETIMEDOUT (records stay reserved).
 *   cache_async_records number of records the handle moves.
 * Finish every handle before cache_unregister / cache_exit (a handle must
 * not be used after them).  If one is left unfinished, teardown still keeps
 * the device safe: the entry keeps its pinned pool mapped (leaked) and
 * cache_exit waits for the device's queued copies before unmapping memory. */
typedef struct cache_async cache_async_t;

int cache_load_async(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                     uint64_t *bids, uint32_t bnum, cache_async_t **out);
int cache_store_async(struct worker_context *wctx, uint8_t *keys, uint32_t key_len,
                      uint64_t *bids, uint32_t bnum, cache_async_t **out);
int cache_async_layers(cache_async_t *h, uint32_t layer_begin, uint32_t layer_end,
                       void *stream, void *wait_event);
int cache_async_stream_wait(cache_async_t *h, uint32_t layer, void *stream);
int cache_async_query(cache_async_t *h);
int cache_async_finish(cache_async_t *h);
uint32_t cache_async_records(const cache_async_t *h);

#ifdef __cplusplus
}
#endif

#endif
