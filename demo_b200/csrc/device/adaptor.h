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
};

/* launches of this library's kernels (all devices) */
extern std::atomic<uint64_t> g_cc_kernel_launches;

#endif
