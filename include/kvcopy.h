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
#define KVCOPY_ERR_TIMEOUT      0x4   /* a bulk copy did not complete in time */
#define KVCOPY_ERR_ALIGN        0x8   /* bulk path given a misaligned base    */

/* kv_copy_desc.flags */
#define KVCOPY_FLAG_BULK        0x1   /* the caller guarantees that records and
                                       * layers are device memory (HBM) and that
                                       * every layer base and record address is
                                       * 16-byte aligned: block-id transfers
                                       * whose block run (block_size * unit) is a
                                       * multiple of 16 bytes from 8 to 32 KiB
                                       * then use TMA bulk copies
                                       * (cp.async.bulk) staged in shared memory
                                       * (head-major blocks with head_bytes a
                                       * multiple of 16: transposed there too) */
#define KVCOPY_FLAG_TEST_STALL  0x100 /* fault-detection tests only, bulk path:
                                       * CTA 0 arms its first stage's mbarrier
                                       * for 16 bytes it never copies, so that
                                       * wait runs out after a few ms (no copy
                                       * is in flight on that stage); the
                                       * kernel sets KVCOPY_ERR_TIMEOUT, drains
                                       * its other loads and returns.  The
                                       * other CTAs copy their tiles. */

/* kv_copy_path() results: the kernel a descriptor selects */
#define KVCOPY_PATH_REGISTER    1     /* kv_copy_kernel: 16-byte register copies */
#define KVCOPY_PATH_BULK        2     /* kv_copy_bulk_kernel: cp.async.bulk via shared memory */
#define KVCOPY_PATH_BULK_HND    3     /* kv_copy_bulk_hnd_kernel: bulk + head-major transpose */

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
    uint32_t flags;              /* KVCOPY_FLAG_*                            */
    /* layer sub-range (new): copy record layers [layer_begin, layer_begin +
     * num_layers) of records holding record_layers layers (0: num_layers);
     * layer_k / layer_v still list every layer of the cache */
    uint32_t layer_begin;
    uint32_t record_layers;
    uint32_t max_ctas;           /* cap on the launch's CTAs, 0 = fill the GPU */
    /* paged geometry (new): where a slot lives inside a layer plane.  With
     * both fields 0 the plane is dense and token-major, slot s at byte
     * s * unit (the reference's only layout: vLLM FlashAttention,
     * [2][num_blocks][block_size][heads][head_dim]).  Otherwise slot s sits
     * in block b = s / block_size at token j = s % block_size, block b
     * starting at byte b * block_stride of the plane (0: block_size * unit);
     *   head_bytes == 0: token j at + j * unit                        (NHD)
     *   head_bytes  > 0: the block holds unit / head_bytes heads, each
     *                    [block_size][head_bytes]; byte o of token j's
     *                    unit at + (o / head_bytes) * block_size *
     *                    head_bytes + j * head_bytes + o % head_bytes (HND)
     * vLLM FlashInfer keeps K and V of a block side by side
     * ([num_blocks][2][...]): its K plane starts at the layer tensor, its V
     * plane one half-block later, block_stride = 2 * block_size * unit, and
     * on sm_100 the block is HND.  Records stay token-major whatever the
     * paged geometry, so every geometry reads and writes the same record
     * bytes. */
    uint64_t block_stride;
    uint32_t head_bytes;
};

/* Launch the gather/scatter on `stream` (a cudaStream_t, NULL = legacy
 * default stream).  Asynchronous; returns 0, or -EINVAL for a malformed
 * descriptor (including a block_stride below block_size * unit, a unit
 * that head_bytes does not divide, or a non-dense geometry with
 * page_buffer_size >= 2^32 in slot mode), or -EIO when the launch failed. */
int kv_copy_launch(const struct kv_copy_desc *desc, void *stream);

/* The kernel kv_copy_launch would run for `desc` (KVCOPY_PATH_*), or -EINVAL
 * for a descriptor it would reject (including unknown flag bits).  Launches
 * nothing: lets a caller label its measurements with the path taken (the
 * bulk path needs KVCOPY_FLAG_BULK, block ids, block runs of 8-32 KiB and
 * 16-byte multiples; everything else takes the register path). */
int kv_copy_path(const struct kv_copy_desc *desc);

/* Algorithmic payload of one launch: kv * num_layers * num_tokens * unit_bytes
 * * num_records (each byte is read once and written once). */
uint64_t kv_copy_payload_bytes(const struct kv_copy_desc *desc);

/* ---- no-allocation variant -------------------------------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory -- an engine that has handed all free HBM to its paged KV cache and
 * caching allocator, or an embedder whose allocator owns every device byte --
 * this entry point runs the same gather (direction 1) / scatter (0) without
 * calling cudaMalloc, cudaFree or any allocating library routine.  Its scratch
 * (layer bases, record addresses, block ids, error word) is one static device
 * array of about 548 KiB that every GPU it was set up on holds until exit;
 * requests beyond the limits below return -E2BIG.
 *   layer_k / layer_v  HOST arrays of num_layers layer base addresses
 *                      (layer_v NULL for a K-only cache)
 *   records            HOST array of num_records device-accessible record
 *                      addresses (HBM, or mapped pinned host memory)
 *   block_ids          HOST array, num_tokens / block_size ids per record
 *   flags              0 or KVCOPY_FLAG_BULK (same meaning as in
 *                      kv_copy_desc: records and layers in HBM, 16-byte
 *                      aligned; the TMA bulk kernels then run where the
 *                      block run allows); other bits are -EINVAL
 * Synchronous on `stream`: returns 0 once the kernel finished, -EINVAL for a
 * bad argument or a block id outside the paged cache, -E2BIG, -ETIMEDOUT
 * (deadline CROSSCACHE_TIMEOUT_MS, or a bulk copy that did not complete) or
 * -EIO.
 * Set-up: the first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and loads every kv_copy kernel onto the device.
 * CUDA loads modules lazily by default, so that is the moment the driver
 * places the array and the kernels' code in device memory; a call with
 * num_records == 0 (the pointer arguments may then be NULL) does only this
 * set-up.  Make it at start-up, before the engine hands its free HBM to the
 * KV cache, and before any stream capture.  A failed set-up is retried by the
 * next call.
 * Every call shares the array, which keeps the last call's contents (the
 * error word is cleared per call); calls that overlap on the GPU race --
 * calls through this entry point in one process are serialised, but one that
 * returned -ETIMEDOUT may still be running. */
#define KVCOPY_NOALLOC_MAX_LAYERS  256
#define KVCOPY_NOALLOC_MAX_RECORDS 4096
#define KVCOPY_NOALLOC_MAX_BLOCKS  65536

int kv_copy_noalloc(int device, const uint64_t *layer_k, const uint64_t *layer_v,
                    const uint64_t *records, const uint64_t *block_ids,
                    uint32_t num_records, uint64_t page_buffer_size, uint32_t unit_bytes,
                    uint32_t num_tokens, uint32_t block_size, uint32_t num_layers,
                    int32_t direction, uint32_t flags, void *stream);

#ifdef __cplusplus
}
#endif

#endif
