/*
 * ORACLE -- test infrastructure only.  Plain-C restatement of CrossCache's CPU
 * KV transfer path, used by tests/ and by bench.py's cpu_baseline leg as the
 * checker and CPU baseline; never linked into or called by the product
 * library.
 *
 *   oracle_slot_mapping   src/cache/cache.c:345-398 (create_slot_mapping +
 *                         get_slot_mapping): slot[i*bs + j] = bids[i]*bs + j
 *   oracle_transfer       src/device/mem/mem.cpp:114-173 (TransferKVCache)
 *                         without the per-token log string: for each layer
 *                         and token, memcpy `unit` bytes between
 *                         record[(l*C + t)*unit] (+ L*C*unit for V) and
 *                         layer[slot[t]*unit]
 *   oracle_cache_op       src/cache/cache.c:513-593 (cache_op chunking):
 *                         record i covers blocks [i*bpc, (i+1)*bpc), run on
 *                         `nthreads` workers like the CaCopy pool (:777)
 */
#include <pthread.h>
#include <stdbool.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

void oracle_slot_mapping(const uint64_t *bids, uint32_t bnum, uint32_t block_size,
                         int64_t *out_slots)
{
    for (uint32_t i = 0; i < bnum; i++)
        for (uint32_t j = 0; j < block_size; j++)
            out_slots[(uint64_t)i * block_size + j] = (int64_t)(bids[i] * block_size + j);
}

int oracle_transfer(uint8_t *caches, const uint64_t *key_ptrs, const uint64_t *val_ptrs,
                    const int64_t *slots, uint16_t num_layers, uint16_t num_tokens,
                    uint32_t hidden_dim_size, uint8_t element_size, bool direction)
{
    uint64_t copy_len = (uint64_t)element_size * hidden_dim_size;

    for (uint32_t l = 0; l < num_layers; l++) {
        for (uint32_t t = 0; t < num_tokens; t++) {
            uint64_t cpos = ((uint64_t)l * num_tokens + t) * copy_len;
            uint64_t ppos = (uint64_t)slots[t] * copy_len;
            uint8_t *k = (uint8_t *)(uintptr_t)key_ptrs[l];
            if (direction)
                memcpy(caches + cpos, k + ppos, copy_len);
            else
                memcpy(k + ppos, caches + cpos, copy_len);
            if (val_ptrs) {
                uint8_t *v = (uint8_t *)(uintptr_t)val_ptrs[l];
                cpos += (uint64_t)num_layers * num_tokens * copy_len;
                if (direction)
                    memcpy(caches + cpos, v + ppos, copy_len);
                else
                    memcpy(v + ppos, caches + cpos, copy_len);
            }
        }
    }
    return 0;
}

struct op_ctx {
    uint8_t **records;
    const uint64_t *key_ptrs, *val_ptrs, *bids;
    uint32_t key_num, bpc, block_size, chunk_size, hidden;
    uint16_t num_layers;
    uint8_t elt;
    bool direction;
    uint32_t next;
    pthread_mutex_t mu;
};

static void *op_worker(void *arg)
{
    struct op_ctx *c = arg;
    int64_t *slots = malloc((uint64_t)c->chunk_size * sizeof(int64_t));

    if (!slots)
        return NULL;
    for (;;) {
        uint32_t i;
        pthread_mutex_lock(&c->mu);
        i = c->next++;
        pthread_mutex_unlock(&c->mu);
        if (i >= c->key_num)
            break;
        oracle_slot_mapping(c->bids + (uint64_t)i * c->bpc, c->bpc, c->block_size, slots);
        oracle_transfer(c->records[i], c->key_ptrs, c->val_ptrs, slots, c->num_layers,
                        (uint16_t)c->chunk_size, c->hidden, c->elt, c->direction);
    }
    free(slots);
    return NULL;
}

int oracle_cache_op(uint8_t **records, const uint64_t *key_ptrs, const uint64_t *val_ptrs,
                    const uint64_t *bids, uint32_t bnum, uint32_t chunk_size,
                    uint32_t block_size, uint16_t num_layers, uint32_t hidden_dim_size,
                    uint8_t element_size, bool direction, int nthreads)
{
    struct op_ctx c;
    pthread_t th[256];
    int n = nthreads < 1 ? 1 : (nthreads > 256 ? 256 : nthreads);

    if (!block_size || chunk_size % block_size)
        return -1;
    memset(&c, 0, sizeof(c));
    c.records = records;
    c.key_ptrs = key_ptrs;
    c.val_ptrs = val_ptrs;
    c.bids = bids;
    c.bpc = chunk_size / block_size;
    c.key_num = bnum / c.bpc;
    c.block_size = block_size;
    c.chunk_size = chunk_size;
    c.hidden = hidden_dim_size;
    c.num_layers = num_layers;
    c.elt = element_size;
    c.direction = direction;
    pthread_mutex_init(&c.mu, NULL);
    for (int i = 0; i < n; i++)
        pthread_create(&th[i], NULL, op_worker, &c);
    for (int i = 0; i < n; i++)
        pthread_join(th[i], NULL);
    pthread_mutex_destroy(&c.mu);
    return 0;
}
