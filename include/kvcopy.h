/*
 * Kernel-level C ABI of the paged-KV record gather (save) and scatter (load)
 * kernels for sm_100a.
 *
 * This is the device half of CrossCache's TransferKVCache
 * (src/device/npu/npu.cpp:188-251 launching
 * src/device/npu/kernels/multi_layer_memcpy_kernel.cpp:165-198), with the byte
 * mapping of the reference CPU path src/device/mem/mem.cpp:136-167:
 *
 *   for record r, kv in {K, V}, layer l, token t < num_tokens:
 *     record_r[((kv * num_layers + l) * num_tokens + t) * unit ...+unit)
 *       <-> layer_{kv}[l][slot(r, t) * unit ...+unit)
 *
 *   slot(r, t) = slots[r * num_tokens + t]                   (slots != NULL)
 *              = block_ids[r * (num_tokens / block_size) + t / block_size]
 *                * block_size + t % block_size                 (slots == NULL)
 *
 * The second form is the reference's slot mapping (src/cache/cache.c:345-398)
 * generated on the device from block ids instead of uploading 8 bytes per
 * token.  All pointers below are device-accessible (device memory, or a
 * mapped alias of pinned host memory for records).
 */
#ifndef __KVCOPY_H__
#define __KVCOPY_H__

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* error bits the kernels OR into *error */
#define KVCOPY_ERR_SLOT_RANGE   0x1   /* slot < 0 or slot >= page_buffer_size */
#define KVCOPY_ERR_NULL_LAYER   0x2   /* a layer base pointer is 0            */

struct kv_copy_desc {
    const uint64_t *layer_k;     /* [num_layers] K layer base addresses      */
    const uint64_t *layer_v;     /* [num_layers] V layer bases, or NULL      */
    const uint64_t *records;     /* [num_records] record base addresses      */
    const int64_t *slots;        /* [num_records * num_tokens] or NULL       */
    const uint64_t *block_ids;   /* [num_records * num_tokens / block_size]  */
    int32_t *error;              /* device int32 error bits, or NULL         */
    uint64_t page_buffer_size;   /* slots per layer                          */
    uint32_t unit_bytes;         /* bytes per token per layer per K/V        */
    uint32_t num_tokens;         /* tokens per record                        */
    uint32_t block_size;         /* tokens per paged block                   */
    uint32_t num_layers;
    uint32_t num_records;
    int32_t direction;           /* 1: paged -> record, 0: record -> paged   */
};

/* Launch the gather/scatter on `stream` (a cudaStream_t, NULL = legacy
 * default stream).  Asynchronous; returns 0, or -EINVAL for a malformed
 * descriptor, or -EIO when the launch failed. */
int kv_copy_launch(const struct kv_copy_desc *desc, void *stream);

/* Algorithmic payload of one launch: kv * num_layers * num_tokens * unit_bytes
 * * num_records (each byte is read once and written once). */
uint64_t kv_copy_payload_bytes(const struct kv_copy_desc *desc);

#ifdef __cplusplus
}
#endif

#endif
