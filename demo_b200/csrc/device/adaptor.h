/*
 * Backend interface behind the device C ABI (include/device.h).
 * Same virtual set as CrossCache src/device/adaptor.h:7-35, plus the batched
 * transfer used by this build's cache manager.
 */
#ifndef CC_ADAPTOR_H
#define CC_ADAPTOR_H

#include "device.h"

#include <atomic>
#include <cstdint>

class Adaptor
{
public:
    virtual ~Adaptor() {}

    virtual void *AllocPinnedPtr(uint8_t nid, uint64_t size, unsigned int flags, void **daddr) = 0;
    virtual void FreePinnedPtr(void *addr, uint64_t size) = 0;
    virtual void *WrapperPtr(uint8_t nid, void *addr, uint64_t size) = 0;
    virtual void UnWrapperPtr(void *daddr) = 0;
    virtual void *OpenIPCKeys(uint8_t nid, uint16_t per_len, uint16_t num, void *data) = 0;
    virtual void CloseIPCKeys(void *daddr) = 0;
    virtual int TransferKVCache(struct transfer_params *params) = 0;
    virtual int TransferKVCacheBatch(struct transfer_batch *batch) = 0;
    virtual void Reset(uint8_t nid) = 0;

    /* asynchronous layer-ranged transfers (include/device.h) */
    virtual struct transfer_async *AsyncBegin(const struct transfer_batch *batch, int *err) = 0;
    virtual int AsyncLayers(struct transfer_async *h, uint32_t l0, uint32_t l1, void *stream,
                            void *wait_event) = 0;
    virtual int AsyncStreamWait(struct transfer_async *h, uint32_t layer, void *stream) = 0;
    virtual int AsyncQuery(struct transfer_async *h) = 0;
    virtual int AsyncEnd(struct transfer_async *h) = 0;
};

/* launches of this library's kernels (all devices) */
extern std::atomic<uint64_t> g_cc_kernel_launches;

/* Load the code of every kv_copy kernel onto the current device (modules load
 * lazily by default, so a kernel's first launch would otherwise be the moment
 * the driver places it in device memory); 0 or -EIO.  kv_copy.cu. */
int kv_copy_preload(void);

#endif
