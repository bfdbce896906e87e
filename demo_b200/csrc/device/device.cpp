/*
 * extern "C" thunks of the device ABI onto the Adaptor virtuals
 * (same forwarding as CrossCache src/device/device.cpp:3-41).
 */
#include "adaptor.h"

#include <cerrno>

std::atomic<uint64_t> g_cc_kernel_launches{0};

void *alloc_pinned_ptr(adaptor_t *adaptor, uint8_t nid, uint64_t size, unsigned int flags, void **daddr)
{
    return adaptor ? adaptor->AllocPinnedPtr(nid, size, flags, daddr) : nullptr;
}

void free_pinned_ptr(adaptor_t *adaptor, void *addr, uint64_t size)
{
    if (adaptor)
        adaptor->FreePinnedPtr(addr, size);
}

void *wrapper_ptr(adaptor_t *adaptor, uint8_t nid, void *addr, uint64_t size)
{
    return adaptor ? adaptor->WrapperPtr(nid, addr, size) : nullptr;
}

void unwrapper_ptr(adaptor_t *adaptor, void *daddr)
{
    if (adaptor)
        adaptor->UnWrapperPtr(daddr);
}

void *open_ipc_keys(adaptor_t *adaptor, uint8_t nid, uint16_t per_len, uint16_t num, void *data)
{
    return adaptor ? adaptor->OpenIPCKeys(nid, per_len, num, data) : nullptr;
}

void close_ipc_keys(adaptor_t *adaptor, void *daddr)
{
    if (adaptor)
        adaptor->CloseIPCKeys(daddr);
}

int transfer_kvcache(adaptor_t *adaptor, struct transfer_params *params)
{
    return (adaptor && params) ? adaptor->TransferKVCache(params) : -EINVAL;
}

int transfer_kvcache_batch(adaptor_t *adaptor, struct transfer_batch *batch)
{
    return (adaptor && batch) ? adaptor->TransferKVCacheBatch(batch) : -EINVAL;
}

struct transfer_async *transfer_async_begin(adaptor_t *adaptor, const struct transfer_batch *batch, int *err)
{
    if (!adaptor || !batch) {
        if (err)
            *err = -EINVAL;
        return nullptr;
    }
    return adaptor->AsyncBegin(batch, err);
}

int transfer_async_layers(adaptor_t *adaptor, struct transfer_async *h, uint32_t layer_begin,
                          uint32_t layer_end, void *stream, void *wait_event)
{
    return (adaptor && h) ? adaptor->AsyncLayers(h, layer_begin, layer_end, stream, wait_event) : -EINVAL;
}

int transfer_async_stream_wait(adaptor_t *adaptor, struct transfer_async *h, uint32_t layer, void *stream)
{
    return (adaptor && h) ? adaptor->AsyncStreamWait(h, layer, stream) : -EINVAL;
}

int transfer_async_query(adaptor_t *adaptor, struct transfer_async *h)
{
    return (adaptor && h) ? adaptor->AsyncQuery(h) : -EINVAL;
}

int transfer_async_end(adaptor_t *adaptor, struct transfer_async *h)
{
    return (adaptor && h) ? adaptor->AsyncEnd(h) : -EINVAL;
}

void reset_device(adaptor_t *adaptor, uint8_t nid)
{
    if (adaptor)
        adaptor->Reset(nid);
}

uint64_t crosscache_kernel_launches(void)
{
    return g_cc_kernel_launches.load(std::memory_order_relaxed);
}
