/*
 * Worker context shared by the cache manager and its callers.
 *
 * Field order, types and meaning are kept identical to CrossCache's
 * include/inner_h/inner.h:6-30 so that a server or client compiled against
 * the reference header passes the same struct to this library.
 *
 *   model            model identity and KV shape per token
 *   node_id          worker slot == CUDA device ordinal of the paged cache
 *   world_size/rank  tensor-parallel size and this worker's TP rank
 *   per_token_size   bytes of KV one token occupies across all layers
 *                    (kv * num_layers * hidden_dim_size * element_size)
 *   num_blocks       vLLM paged blocks per layer
 *   block_size       tokens per vLLM block
 *   per_len          bytes of one per-layer handle in k_raw_ptrs/v_raw_ptrs:
 *                      8  -> raw device pointer of this process (uint64)
 *                      64 -> cudaIpcMemHandle_t of the layer's allocation
 *                      72 -> cudaIpcMemHandle_t followed by a uint64 byte
 *                            offset of the layer inside that allocation
 *   k_raw_ptrs       num_layers handles for K (host memory)
 *   v_raw_ptrs       num_layers handles for V, or NULL for K-only (MLA)
 *   k_ptrs/v_ptrs    OUT: device arrays of num_layers uint64 layer bases
 */
#ifndef __INNER_H__
#define __INNER_H__

#include <stdint.h>

struct model_info {
    char *model_name;
    uint8_t element_size;
    uint8_t num_layers;
    uint32_t hidden_dim_size;
};

struct worker_context {
    struct model_info model;
    uint8_t node_id;
    uint8_t world_size;
    uint8_t rank_id;
    uint32_t per_token_size;
    uint32_t num_blocks;
    uint32_t block_size;

    uint16_t per_len;

    void *k_raw_ptrs;
    void *v_raw_ptrs;

    void *k_ptrs;
    void *v_ptrs;
};

#endif
