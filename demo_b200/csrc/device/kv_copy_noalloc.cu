/*
 * kv_copy_noalloc: the paged-KV record gather/scatter for callers that cannot
 * allocate device memory.
 *
 * Who needs it: a serving engine that has already handed (almost) all free
 * HBM to its paged KV cache and its caching allocator -- vLLM sizes the KV
 * cache to fill the memory left after profiling -- cannot count on a fresh
 * cudaMalloc succeeding while it serves, and an embedder whose allocator owns
 * every byte of the device may forbid other libraries from calling
 * cudaMalloc at all.  The batched transfer of the CUDA adaptor allocates its
 * metadata buffers, error word and staging ring on first use; this entry
 * point needs none of that.
 *
 * How: the per-call metadata the kernel reads (layer bases, record addresses,
 * block ids) and its error word live in one file-scope
 * `static __device__ __align__(256)` array of fixed size (about 548 KiB,
 * limits below), which every GPU that sets the entry point up holds until
 * the process exits.  Host code cannot use the array's name as a device
 * address (it is a host-side stand-in: a kernel given it faults or, where the
 * GPU can reach host memory, silently uses the wrong memory), so the set-up
 * looks up the array's device address with cudaGetSymbolAddress, with that
 * device current, and keeps it.  CUDA loads modules lazily by default: the
 * driver places the array, and each kernel's code, in device memory when
 * they are first used.  The set-up therefore also loads every kv_copy kernel
 * (cudaFuncGetAttributes), so that after it no call of this entry point
 * makes the driver allocate either.  The set-up runs on the first call on a
 * device; a call with num_records == 0 does only the set-up.  Make that call
 * at start-up -- before the engine hands its free HBM to the KV cache, and
 * before any stream capture.  A set-up that failed (for instance for lack
 * of device memory) is not remembered: the next call tries again.  Records
 * must already be device-accessible (HBM, or the mapped alias of pinned host
 * memory): no staging is used.
 *
 * Every call shares the array, which keeps the last call's contents; each
 * call clears the error word before its launch.  Calls that overlap on the
 * GPU race on the array.  Calls made through this entry point in one process
 * are serialised by a per-device mutex and each returns only after its
 * kernel finished, so they cannot overlap -- except after a call that
 * returned -ETIMEDOUT, whose kernel may still be running: a later call then
 * races with it.
 *
 * No cudaMalloc, cudaFree or allocating library routine is called: the
 * uploads are cudaMemcpyAsync into the array, the wait is a cudaStreamQuery
 * poll with a deadline (CROSSCACHE_TIMEOUT_MS, default 120000).
 */
#include "kvcopy.h"
#include "adaptor.h"

extern "C" {
#include "../infra/log.h"
}

#include <cuda_runtime.h>

#include <cerrno>
#include <chrono>
#include <cstdlib>
#include <mutex>
#include <thread>

namespace {

constexpr uint32_t kLayersMax = KVCOPY_NOALLOC_MAX_LAYERS;
constexpr uint32_t kRecordsMax = KVCOPY_NOALLOC_MAX_RECORDS;
constexpr uint32_t kBlocksMax = KVCOPY_NOALLOC_MAX_BLOCKS;

/* word layout: K bases | V bases | record addresses | block ids | error word */
constexpr size_t kOffK = 0;
constexpr size_t kOffV = kOffK + kLayersMax;
constexpr size_t kOffRec = kOffV + kLayersMax;
constexpr size_t kOffBids = kOffRec + kRecordsMax;
constexpr size_t kOffErr = kOffBids + kBlocksMax;
constexpr size_t kWords = kOffErr + 1;

static __device__ __align__(256) uint64_t g_noalloc_scratch[kWords];

struct DeviceScratch {
    std::mutex mu;       /* serialises calls on the device (they share the array) */
    uint64_t *ptr = nullptr;
    bool ready = false;
};

DeviceScratch g_scratch[64];

/* the set-up of `dev` (which must be current), under s.mu: the array's
 * device address, and every kv_copy kernel loaded onto the device */
uint64_t *setup_locked(int dev)
{
    DeviceScratch &s = g_scratch[dev];
    if (s.ready)
        return s.ptr;
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
        log_error("kv_copy_noalloc: cudaGetSymbolAddress on device %d failed: %s", dev, cudaGetErrorString(e));
        return nullptr;
    }
    if (kv_copy_preload() != 0) {
        log_error("kv_copy_noalloc: loading the kv_copy kernels on device %d failed: %s", dev,
                  cudaGetErrorString(cudaGetLastError()));
        return nullptr;
    }
    s.ptr = static_cast<uint64_t *>(p);
    s.ready = true;
    return s.ptr;
}

int run(int device, const uint64_t *layer_k, const uint64_t *layer_v, const uint64_t *records,
        const uint64_t *block_ids, uint32_t num_records, uint64_t page_buffer_size,
        uint32_t unit_bytes, uint32_t num_tokens, uint32_t block_size, uint32_t num_layers,
        int32_t direction, uint32_t flags, cudaStream_t stream)
{
    std::lock_guard<std::mutex> lk(g_scratch[device].mu);
    uint64_t *scr = setup_locked(device);
    if (!scr)
        return -EIO;
    if (!num_records)
        return 0;                                   /* set-up only */
    const uint64_t nblk = (uint64_t)num_records * (num_tokens / block_size);
    if (cudaMemcpyAsync(scr + kOffK, layer_k, num_layers * 8ull, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        (layer_v && cudaMemcpyAsync(scr + kOffV, layer_v, num_layers * 8ull, cudaMemcpyHostToDevice, stream) != cudaSuccess) ||
        cudaMemcpyAsync(scr + kOffRec, records, num_records * 8ull, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync(scr + kOffBids, block_ids, nblk * 8, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaMemsetAsync(scr + kOffErr, 0, 8, stream) != cudaSuccess)
        return -EIO;

    kv_copy_desc d{};
    d.layer_k = scr + kOffK;
    d.layer_v = layer_v ? scr + kOffV : nullptr;
    d.records = scr + kOffRec;
    d.slots = nullptr;
    d.block_ids = scr + kOffBids;
    d.error = reinterpret_cast<int32_t *>(scr + kOffErr);
    d.page_buffer_size = page_buffer_size;
    d.unit_bytes = unit_bytes;
    d.num_tokens = num_tokens;
    d.block_size = block_size;
    d.num_layers = num_layers;
    d.num_records = num_records;
    d.direction = direction;
    d.flags = flags;
    int ret = kv_copy_launch(&d, stream);
    if (ret)
        return ret;

    const char *t = getenv("CROSSCACHE_TIMEOUT_MS");
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(t ? atoi(t) : 120000);
    int spins = 0;
    for (;;) {
        cudaError_t e = cudaStreamQuery(stream);
        if (e == cudaSuccess)
            break;
        if (e != cudaErrorNotReady)
            return -EIO;
        if (std::chrono::steady_clock::now() > deadline) {
            log_error("kv_copy_noalloc: device %d did not finish before the deadline", device);
            return -ETIMEDOUT;
        }
        if (++spins > 64)
            std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    int32_t err = 0;
    /* pageable destination: returns once the copy is done (the stream is idle) */
    if (cudaMemcpyAsync(&err, scr + kOffErr, sizeof(err), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
        cudaStreamQuery(stream) != cudaSuccess)
        return -EIO;
    if (err) {
        log_error("kv_copy_noalloc: kernel reported error bits 0x%x", err);
        return (err & KVCOPY_ERR_TIMEOUT) ? -ETIMEDOUT : -EINVAL;
    }
    return 0;
}

}  // namespace

extern "C" int kv_copy_noalloc(int device, const uint64_t *layer_k, const uint64_t *layer_v,
                               const uint64_t *records, const uint64_t *block_ids,
                               uint32_t num_records, uint64_t page_buffer_size,
                               uint32_t unit_bytes, uint32_t num_tokens, uint32_t block_size,
                               uint32_t num_layers, int32_t direction, uint32_t flags, void *stream)
{
    if (device < 0 || device >= 64)
        return -EINVAL;
    if (num_records && (!layer_k || !records || !block_ids || !unit_bytes || !num_tokens || !block_size ||
                        num_tokens % block_size || !num_layers || (flags & ~(uint32_t)KVCOPY_FLAG_BULK)))
        return -EINVAL;
    if (num_records) {
        const uint64_t nblk = (uint64_t)num_records * (num_tokens / block_size);
        if (num_layers > kLayersMax || num_records > kRecordsMax || nblk > kBlocksMax) {
            log_error("kv_copy_noalloc: request exceeds the static scratch (layers %u > %u, records %u > %u "
                      "or blocks %lu > %u)", num_layers, kLayersMax, num_records, kRecordsMax,
                      (unsigned long)nblk, kBlocksMax);
            return -E2BIG;
        }
    }
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess)
        return -EIO;
    int ret = run(device, layer_k, layer_v, records, block_ids, num_records, page_buffer_size,
                  unit_bytes, num_tokens, block_size, num_layers, direction, flags,
                  static_cast<cudaStream_t>(stream));
    cudaSetDevice(prev);
    return ret;
}
