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

void reset_device(adaptor_t *adaptor, uint8_t nid)
{
    if (adaptor)
        adaptor->Reset(nid);
}

uint64_t crosscache_kernel_launches(void)
{
    return g_cc_kernel_launches.load(std::memory_order_relaxed);
}
