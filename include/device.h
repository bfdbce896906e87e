/*
 * Device adaptor C ABI.
 *
 * struct transfer_params and the eight adaptor entry points keep the layout,
 * names and semantics of CrossCache's include/inner_h/device.h:13-50, so the
 * cache manager (or any caller written against the reference header) links
 * against this library unchanged.  The reference selects the NPU, NPU-SDK or
 * CPU-memcpy backend at compile time (device.h:32-41); this build adds the
 * CUDA backend (cuda_adaptor_create) and keeps a CPU memcpy backend
 * (mem_adaptor_create) for host-only operation.
 *
 * Additions beyond the reference ABI (marked "new" below) sit beside the
 * reference entry points and never change them.
 */
#ifndef __DEVICE_H__
#define __DEVICE_H__

#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DEV_PTR

/* One record (chunk) transfer; reference device.h:13-28.
 *   caches            device-usable address of the record (pinned host alias
 *                     from alloc_pinned_ptr, or device memory)
 *   caches_h          host address of the same record
 *   keys_ptrs         device array of num_layers uint64 K layer bases
 *   value_ptrs        same for V, or NULL for a K-only (MLA) cache
 *   page_buffer_size  slots per layer (num_blocks * block_size)
 *   slot_mapping      device array of num_tokens int64 slots
 *   direction         true: paged cache -> record (save, D->H);
 *                     false: record -> paged cache (load, H->D)
 * Record layout: K part [num_layers][num_tokens][unit] followed by the V part
 * with the same shape, unit = hidden_dim_size * caches_element_size bytes
 * (reference mem.cpp:141-157). */
struct transfer_params {
    void *caches, *caches_h;

    void DEV_PTR *keys_ptrs;
    void DEV_PTR *value_ptrs;
    uint64_t page_buffer_size;
    void DEV_PTR *slot_mapping;

    uint8_t devid;
    uint8_t caches_element_size;

    uint16_t num_layers;
    uint16_t num_tokens;
    uint32_t hidden_dim_size;
    bool direction;
};

typedef struct Adaptor adaptor_t;

/* CUDA backend (sm_100a kernels, copy engines, pinned host pool).
 * Replaces npu_adaptor_create/npu_adaptor_destroy (reference device.h:32-35,
 * src/device/npu/npu.cpp:259-275). */
adaptor_t *cuda_adaptor_create(void);
void cuda_adaptor_destroy(adaptor_t *adaptor);

/* CPU memcpy backend (reference device.h:39-40, src/device/mem/mem.cpp:175-191):
 * only used when the caller asks for it explicitly (cache_init_backend with
 * CACHE_BACKEND_MEM); pointers in open_ipc_keys must then be host addresses. */
adaptor_t *mem_adaptor_create(void);
void mem_adaptor_destroy(adaptor_t *adaptor);

/* Reference device.h:43-50 (semantics of src/device/npu/npu.cpp:49-257). */
void *alloc_pinned_ptr(adaptor_t *adaptor, uint8_t nid, uint64_t size, unsigned int flags, void **daddr);
void free_pinned_ptr(adaptor_t *adaptor, void *addr, uint64_t size);
void *wrapper_ptr(adaptor_t *adaptor, uint8_t nid, void *addr, uint64_t size);
void unwrapper_ptr(adaptor_t *adaptor, void *daddr);
void *open_ipc_keys(adaptor_t *adaptor, uint8_t nid, uint16_t per_len, uint16_t num, void *data);
void close_ipc_keys(adaptor_t *adaptor, void *daddr);
int transfer_kvcache(adaptor_t *adaptor, struct transfer_params *params);
void reset_device(adaptor_t *adaptor, uint8_t nid);

/* ---- new: batched transfer of many records in one call ----------------
 * Moves num_records records between the paged cache and records[] with one
 * metadata upload and a pipelined sequence of kernels and copy-engine
 * transfers.  Record r holds the blocks
 *   block_ids[r * (num_tokens / block_size) ... + (num_tokens / block_size) - 1]
 * in the record layout of struct transfer_params.  records[] are host
 * addresses inside a pool returned by alloc_pinned_ptr (record_on_device = 0)
 * or device addresses (record_on_device = 1).  Synchronous: returns 0 after
 * every byte has landed, a negative errno otherwise (-EINVAL for a block id
 * outside the paged cache, -ETIMEDOUT when the device did not finish within
 * the adaptor's deadline).  Thread-safe. */
struct transfer_batch {
    void DEV_PTR *keys_ptrs;
    void DEV_PTR *value_ptrs;
    uint64_t page_buffer_size;
    void **records;
    const uint64_t *block_ids;
    uint32_t num_records;
    uint32_t block_size;
    uint32_t hidden_dim_size;
    uint16_t num_layers;
    uint16_t num_tokens;
    uint8_t devid;
    uint8_t caches_element_size;
    uint8_t record_on_device;
    bool direction;
    /* paged geometry of the layer planes (kv_copy_desc block_stride /
     * head_bytes in kvcopy.h); both 0 = dense token-major */
    uint64_t block_stride;
    uint32_t head_bytes;
};

int transfer_kvcache_batch(adaptor_t *adaptor, struct transfer_batch *batch);

/* new: asynchronous, layer-ranged transfers of a batch (no reference
 * counterpart; the reference moves whole records synchronously).  The
 * kernels read or write the records where they are -- mapped pinned host
 * memory, or HBM when record_on_device -- with no staging, so layers can
 * move while the caller's kernels run.
 *   transfer_async_begin   validate the batch and copy its block ids and
 *                          record addresses aside; nothing runs yet.  NULL
 *                          and *err = -errno on failure.
 *   transfer_async_layers  on `stream` (a cudaStream_t of the batch's
 *                          device), after `wait_event` (a cudaEvent_t, or
 *                          NULL), copy record layers [layer_begin, layer_end)
 *                          of every record; the launch is capped to a few
 *                          CTAs (CROSSCACHE_ASYNC_CTAS, default 32).
 *   transfer_async_stream_wait
 *                          make `stream` wait for the copy that covered
 *                          `layer` (-ENOENT if none has been enqueued).
 *   transfer_async_query   1 when everything enqueued has finished, 0 if not.
 *   transfer_async_end     wait (deadline CROSSCACHE_TIMEOUT_MS) for it,
 *                          read the kernels' error bits and release the
 *                          handle: 0, -EINVAL (bad block id), -ETIMEDOUT.
 * The CPU (MEM) backend copies inside transfer_async_layers and takes NULL
 * streams and events only. */
struct transfer_async;

struct transfer_async *transfer_async_begin(adaptor_t *adaptor, const struct transfer_batch *batch,
                                            int *err);
int transfer_async_layers(adaptor_t *adaptor, struct transfer_async *h, uint32_t layer_begin,
                          uint32_t layer_end, void *stream, void *wait_event);
int transfer_async_stream_wait(adaptor_t *adaptor, struct transfer_async *h, uint32_t layer,
                               void *stream);
int transfer_async_query(adaptor_t *adaptor, struct transfer_async *h);
int transfer_async_end(adaptor_t *adaptor, struct transfer_async *h);

/* new: CUDA counterpart of CrossCache's ipckey_from_tensor
 * (python/ipckey_utils.cpp:19-33, aclrtIpcMemGetExportKey, 64 bytes).
 * Writes the 72-byte key of device address dptr into key_out: the
 * cudaIpcMemHandle_t of the cudaMalloc allocation that contains dptr,
 * followed by the uint64 byte offset of dptr inside that allocation -- the
 * per_len 72 form open_ipc_keys accepts.  0, -EINVAL (not device memory from
 * cudaMalloc) or -ENOSYS. */
int ipc_export_key(const void *dptr, uint8_t *key_out);

/* new: number of device kernels this library has launched since load
 * (every backend; the CPU backend never launches any). */
uint64_t crosscache_kernel_launches(void);

#ifdef __cplusplus
}
#endif

#endif
