/*
 * CUDA backend of the device adaptor ABI (include/device.h).
 *
 * Replaces CrossCache's Ascend adaptor src/device/npu/npu.cpp:
 *   AllocPinnedPtr  mmap + cudaHostRegister(MAPPED|PORTABLE)   (npu.cpp:49-90)
 *   WrapperPtr      device copy of a host buffer               (npu.cpp:100-123)
 *   OpenIPCKeys     per-layer handle -> device pointer array   (npu.cpp:131-180)
 *                   per_len 8: raw pointers of this process; 64: a
 *                   cudaIpcMemHandle_t; 72: handle + uint64 byte offset
 *   TransferKVCache one record, synchronous                    (npu.cpp:188-251)
 *   Reset           drains and frees this process's streams and staging
 *                   buffers on the device.  It does NOT reset the GPU (the
 *                   reference calls aclrtResetDeviceForce, npu.cpp:253-257).
 *
 * Transfers run on "lanes": per device a small pool of (kernel stream, copy
 * stream, staging ring of NSUB sub-slots in HBM, events, metadata buffers),
 * created once and reused, so no call allocates device memory or creates a
 * stream (the reference creates a stream and allocates the slot map per
 * chunk, npu.cpp:100-123,205).  A save gathers a group of records into a
 * staging sub-slot with the kv_copy kernel, then a copy engine moves it to
 * the pinned host records while the next group is gathered; a load is the
 * mirror image.  Waits are host-side cudaEventQuery polls with a deadline
 * (CROSSCACHE_TIMEOUT_MS, default 120000) that end in -ETIMEDOUT; no kernel
 * spins on anything.
 *
 * CROSSCACHE_XFER_MODE=direct makes the kernels read/write the mapped pinned
 * records over the host link instead (no staging, no copy engine).
 */
#include "adaptor.h"
#include "kvcopy.h"

extern "C" {
#include "../infra/log.h"
}

#include <cuda_runtime.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <deque>
#include <cstring>
#include <map>
#include <string>
#include <memory>
#include <mutex>
#include <new>
#include <sys/mman.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

constexpr int kNumSub = 3;                       /* staging ring depth per lane */
constexpr uint64_t kGroupTarget = 32ull << 20;   /* staging sub-slot target size */
constexpr uint64_t kAsyncRingMax = 768ull << 20; /* HBM ring of one staged async transfer */

#define CU_OK(expr)                                                              \
    ([&]() -> bool {                                                             \
        cudaError_t _e = (expr);                                                 \
        if (_e != cudaSuccess) {                                                 \
            log_error("%s failed: %s", #expr, cudaGetErrorString(_e));           \
            return false;                                                        \
        }                                                                        \
        return true;                                                             \
    }())

int env_int(const char *name, int dflt)
{
    const char *s = getenv(name);
    return s ? atoi(s) : dflt;
}

/* Fault a fresh anonymous mapping in from several threads (one write per
 * 4 KiB page; with transparent huge pages the first write of each 2 MiB
 * faults the whole page) before cudaHostRegister pins it, which otherwise
 * faults and zeroes every page on the calling thread.  The reference
 * prefaults its pool too (npu.cpp:49-90), on one thread.  Threads:
 * CROSSCACHE_PREFAULT_THREADS, default min(16, host threads). */
void prefault(void *addr, uint64_t size)
{
    const uint64_t page = 4096, chunk = 2ull << 20;
    unsigned n = std::thread::hardware_concurrency();
    n = n ? std::min(16u, n) : 1u;
    if (const char *e = getenv("CROSSCACHE_PREFAULT_THREADS"))
        n = (unsigned)std::max(1, atoi(e));
    const uint64_t chunks = (size + chunk - 1) / chunk;
    if (chunks < 64 || n == 1)
        n = 1;
    auto touch = [addr, size, page](uint64_t b, uint64_t e) {
        volatile uint8_t *p = static_cast<volatile uint8_t *>(addr);
        for (uint64_t o = b; o < e && o < size; o += page)
            p[o] = 0;
    };
    if (n == 1) {
        touch(0, size);
        return;
    }
    std::vector<std::thread> th;
    const uint64_t per = (chunks + n - 1) / n * chunk;
    for (unsigned i = 0; i < n; i++)
        th.emplace_back(touch, (uint64_t)i * per, (uint64_t)(i + 1) * per);
    for (auto &t : th)
        t.join();
}

/* poll an event until it completes or the deadline passes */
int wait_event(cudaEvent_t ev, std::chrono::steady_clock::time_point deadline)
{
    int spins = 0;
    for (;;) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess)
            return 0;
        if (e != cudaErrorNotReady) {
            log_error("event wait: %s", cudaGetErrorString(e));
            return -EIO;
        }
        if (std::chrono::steady_clock::now() > deadline)
            return -ETIMEDOUT;
        if (++spins > 64)
            std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

struct Lane {
    int dev = -1;
    int dir = 0;                 /* 1: saves (D2H), 0: loads (H2D) -- a lane serves one direction */
    cudaStream_t ks = nullptr;   /* kernels */
    cudaStream_t cs = nullptr;   /* copy engine */
    cudaEvent_t kdone[kNumSub] = {};
    cudaEvent_t cdone[kNumSub] = {};
    cudaEvent_t fin = nullptr;
    cudaEvent_t mready = nullptr;  /* metadata uploaded (on cs) before the first kernel */
    uint8_t *staging = nullptr;  /* kNumSub sub-slots of sub_bytes */
    uint64_t sub_bytes = 0;
    uint64_t *d_subrec = nullptr;  /* kNumSub x max_group record pointers */
    uint32_t max_group = 0;
    uint64_t cur_rec_bytes = 0;    /* record size d_subrec was built for */
    uint64_t *d_meta = nullptr;    /* device metadata (block ids / records) */
    uint64_t *h_meta = nullptr;    /* pinned host mirror */
    uint64_t meta_cap = 0;         /* uint64 words */
    int32_t *d_err = nullptr;
    int32_t *h_err = nullptr;
    bool poisoned = false;

    bool init(int device)
    {
        dev = device;
        if (!CU_OK(cudaStreamCreateWithFlags(&ks, cudaStreamNonBlocking)) ||
            !CU_OK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking)))
            return false;
        for (int i = 0; i < kNumSub; i++)
            if (!CU_OK(cudaEventCreateWithFlags(&kdone[i], cudaEventDisableTiming)) ||
                !CU_OK(cudaEventCreateWithFlags(&cdone[i], cudaEventDisableTiming)))
                return false;
        if (!CU_OK(cudaEventCreateWithFlags(&fin, cudaEventDisableTiming)) ||
            !CU_OK(cudaEventCreateWithFlags(&mready, cudaEventDisableTiming)) ||
            !CU_OK(cudaMalloc(&d_err, sizeof(int32_t))) ||
            !CU_OK(cudaHostAlloc(&h_err, sizeof(int32_t), cudaHostAllocDefault)))
            return false;
        return ensure_meta(1 << 16);
    }

    bool ensure_meta(uint64_t words)
    {
        if (words <= meta_cap)
            return true;
        uint64_t cap = std::max<uint64_t>(words, meta_cap * 2);
        if (d_meta)
            cudaFree(d_meta);
        if (h_meta)
            cudaFreeHost(h_meta);
        d_meta = nullptr;
        h_meta = nullptr;
        meta_cap = 0;
        if (!CU_OK(cudaMalloc(&d_meta, cap * 8)) ||
            !CU_OK(cudaHostAlloc(&h_meta, cap * 8, cudaHostAllocDefault)))
            return false;
        meta_cap = cap;
        return true;
    }

    /* staging sub-slots able to hold `group` records of rec_bytes each */
    bool ensure_staging(uint64_t rec_bytes, uint32_t *group)
    {
        uint64_t want = std::max(kGroupTarget, rec_bytes);
        if (want > sub_bytes) {
            if (staging)
                cudaFree(staging);
            if (d_subrec)
                cudaFree(d_subrec);
            staging = nullptr;
            d_subrec = nullptr;
            sub_bytes = 0;
            max_group = 0;
            cur_rec_bytes = 0;
            if (!CU_OK(cudaMalloc(&staging, want * kNumSub)))
                return false;
            sub_bytes = want;
        }
        uint32_t g = (uint32_t)std::max<uint64_t>(1, sub_bytes / rec_bytes);
        if (g > max_group) {
            if (d_subrec)
                cudaFree(d_subrec);
            d_subrec = nullptr;
            max_group = 0;
            cur_rec_bytes = 0;
            if (!CU_OK(cudaMalloc(&d_subrec, (uint64_t)kNumSub * g * 8)))
                return false;
            max_group = g;
        }
        *group = g;
        if (rec_bytes == cur_rec_bytes)
            return true;
        /* record pointers of each sub-slot for this record size (tiny upload) */
        std::vector<uint64_t> ptrs((size_t)kNumSub * max_group);
        for (int s = 0; s < kNumSub; s++)
            for (uint32_t j = 0; j < max_group; j++)
                ptrs[(size_t)s * max_group + j] =
                    (uint64_t)(uintptr_t)(staging + s * sub_bytes + (uint64_t)j * rec_bytes);
        if (!CU_OK(cudaMemcpyAsync(d_subrec, ptrs.data(), ptrs.size() * 8,
                                   cudaMemcpyHostToDevice, ks)) ||
            !CU_OK(cudaStreamSynchronize(ks)))
            return false;
        cur_rec_bytes = rec_bytes;
        return true;
    }

    void release()
    {
        if (dev < 0)
            return;
        cudaSetDevice(dev);
        if (ks)
            cudaStreamSynchronize(ks);
        if (cs)
            cudaStreamSynchronize(cs);
        for (int i = 0; i < kNumSub; i++) {
            if (kdone[i])
                cudaEventDestroy(kdone[i]);
            if (cdone[i])
                cudaEventDestroy(cdone[i]);
        }
        if (fin)
            cudaEventDestroy(fin);
        if (mready)
            cudaEventDestroy(mready);
        if (staging)
            cudaFree(staging);
        if (d_subrec)
            cudaFree(d_subrec);
        if (d_meta)
            cudaFree(d_meta);
        if (h_meta)
            cudaFreeHost(h_meta);
        if (d_err)
            cudaFree(d_err);
        if (h_err)
            cudaFreeHost(h_err);
        if (ks)
            cudaStreamDestroy(ks);
        if (cs)
            cudaStreamDestroy(cs);
        *this = Lane();
    }
};

/* one asynchronous layer-ranged transfer (transfer_async_*): its metadata
 * (block ids, record addresses), error word and one event per enqueued
 * layer range.  Reused through a per-device free list. */
struct AsyncOp {
    struct Mark {
        uint32_t l0, l1;
        cudaEvent_t ev;
    };
    int dev = -1;
    cudaStream_t own = nullptr;      /* error readback only */
    cudaEvent_t uploaded = nullptr;
    cudaStream_t upload_stream = nullptr;
    bool is_uploaded = false;
    uint64_t *d_meta = nullptr;
    uint64_t *h_meta = nullptr;
    uint64_t meta_cap = 0;
    uint64_t meta_words = 0;
    int32_t *d_err = nullptr;
    int32_t *h_err = nullptr;
    std::vector<Mark> marks;
    std::vector<cudaEvent_t> spare;
    kv_copy_desc base{};
    uint32_t total_layers = 0;
    bool poisoned = false;

    /* staged mode (host records): each layer's slices cross the host link on
     * a copy engine into an HBM ring slot, and the kernel moves them between
     * the slot and the paged cache -- the SMs never wait on the link */
    static constexpr int kRing = 3;
    bool staged = false;
    cudaStream_t cs = nullptr;
    uint8_t *ring = nullptr;
    uint64_t ring_cap = 0;
    uint64_t slot_bytes = 0;      /* records * kv * layer_bytes */
    uint64_t layer_bytes = 0;     /* num_tokens * unit: one layer of one K/V part */
    uint32_t nkv = 1;
    uint32_t nrec = 0;
    uint32_t rec_words = 0;       /* block id words before the slot record tables */
    uint32_t next_slot = 0;
    bool slot_used[kRing] = {};
    cudaEvent_t slot_ready[kRing] = {};
    cudaEvent_t slot_free[kRing] = {};
    std::vector<uint8_t *> host_recs;
    /* records in host-address order, grouped into runs of consecutive
     * records (stride = record bytes): one copy command per run and K/V part
     * instead of one per record -- a command costs ~4 us of copy-engine time,
     * as much as 220 KB of transfer */
    struct Run {
        uint8_t *host;      /* first record of the run */
        uint32_t pos;       /* its place in a ring slot, in records */
        uint32_t count;
    };
    std::vector<Run> runs;
    uint64_t rec_bytes = 0;

    /* the caller's thread queues jobs, the device's async worker thread
     * enqueues them: marks, counters and spare events are shared */
    std::mutex mu;
    std::condition_variable cv;
    uint32_t jobs_submitted = 0;
    uint32_t jobs_done = 0;
    int enqueue_err = 0;
    std::vector<std::pair<uint32_t, uint32_t>> requested;
    cudaStream_t gate = nullptr;   /* turns a caller's event into one of ours */

    bool init(int device)
    {
        dev = device;
        if (!CU_OK(cudaStreamCreateWithFlags(&own, cudaStreamNonBlocking)) ||
            !CU_OK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking)) ||
            !CU_OK(cudaStreamCreateWithFlags(&gate, cudaStreamNonBlocking)) ||
            !CU_OK(cudaEventCreateWithFlags(&uploaded, cudaEventDisableTiming)) ||
            !CU_OK(cudaMalloc(&d_err, sizeof(int32_t))) ||
            !CU_OK(cudaHostAlloc(&h_err, sizeof(int32_t), cudaHostAllocDefault)))
            return false;
        for (int i = 0; i < kRing; i++)
            if (!CU_OK(cudaEventCreateWithFlags(&slot_ready[i], cudaEventDisableTiming)) ||
                !CU_OK(cudaEventCreateWithFlags(&slot_free[i], cudaEventDisableTiming)))
                return false;
        return true;
    }

    bool ensure_ring(uint64_t bytes)
    {
        if (bytes <= ring_cap)
            return true;
        if (ring)
            cudaFree(ring);
        ring = nullptr;
        ring_cap = 0;
        if (!CU_OK(cudaMalloc(&ring, bytes)))
            return false;
        ring_cap = bytes;
        return true;
    }

    bool ensure_meta(uint64_t words)
    {
        if (words <= meta_cap)
            return true;
        uint64_t cap = std::max<uint64_t>(words, std::max<uint64_t>(1024, meta_cap * 2));
        if (d_meta)
            cudaFree(d_meta);
        if (h_meta)
            cudaFreeHost(h_meta);
        d_meta = nullptr;
        h_meta = nullptr;
        meta_cap = 0;
        if (!CU_OK(cudaMalloc(&d_meta, cap * 8)) || !CU_OK(cudaHostAlloc(&h_meta, cap * 8, cudaHostAllocDefault)))
            return false;
        meta_cap = cap;
        return true;
    }

    cudaEvent_t take_event()
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!spare.empty()) {
            cudaEvent_t e = spare.back();
            spare.pop_back();
            return e;
        }
        cudaEvent_t e = nullptr;
        return CU_OK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming)) ? e : nullptr;
    }

    void reset_for_reuse()
    {
        for (auto &m : marks)
            spare.push_back(m.ev);
        marks.clear();
        is_uploaded = false;
        upload_stream = nullptr;
        meta_words = 0;
        base = kv_copy_desc{};
        total_layers = 0;
        staged = false;
        next_slot = 0;
        for (int i = 0; i < kRing; i++)
            slot_used[i] = false;
        host_recs.clear();
        runs.clear();
        jobs_submitted = jobs_done = 0;
        enqueue_err = 0;
        requested.clear();
    }

    void release()
    {
        if (dev < 0)
            return;
        cudaSetDevice(dev);
        if (own)
            cudaStreamSynchronize(own);
        reset_for_reuse();
        for (cudaEvent_t e : spare)
            cudaEventDestroy(e);
        spare.clear();
        if (uploaded)
            cudaEventDestroy(uploaded);
        if (cs)
            cudaStreamSynchronize(cs);
        for (int i = 0; i < kRing; i++) {
            if (slot_ready[i])
                cudaEventDestroy(slot_ready[i]);
            if (slot_free[i])
                cudaEventDestroy(slot_free[i]);
        }
        if (ring)
            cudaFree(ring);
        if (cs)
            cudaStreamDestroy(cs);
        if (gate) {
            cudaStreamSynchronize(gate);
            cudaStreamDestroy(gate);
        }
        if (d_meta)
            cudaFree(d_meta);
        if (h_meta)
            cudaFreeHost(h_meta);
        if (d_err)
            cudaFree(d_err);
        if (h_err)
            cudaFreeHost(h_err);
        if (own)
            cudaStreamDestroy(own);
        dev = -1;
    }
};

struct AsyncJob {
    AsyncOp *op;
    uint32_t l0, l1;
    cudaStream_t s;
    cudaEvent_t gate;     /* completes after the caller's wait event, or null */
};

/* Layer l of every record between the host records and ring slot `slot`
 * (slot layout: record at position p holds K then V of the layer, nkv *
 * layer_bytes each), on the op's copy stream. */
bool copy_runs(AsyncOp *op, uint8_t *slot, uint32_t l, cudaMemcpyKind kind)
{
    const uint64_t lb = op->layer_bytes;
    const uint64_t hp = (uint64_t)op->total_layers * lb;   /* K part -> V part in a host record */
    const uint64_t sp = (uint64_t)op->nkv * lb;            /* record stride in the slot */
    const bool h2d = kind == cudaMemcpyHostToDevice;
    for (const AsyncOp::Run &rn : op->runs) {
        uint8_t *dev = slot + (uint64_t)rn.pos * sp;
        uint8_t *host = rn.host + (uint64_t)l * lb;
        if (rn.count == 1) {
            /* K and V slices of one record: two rows of the record's pitch */
            if (!CU_OK(h2d ? cudaMemcpy2DAsync(dev, lb, host, hp, lb, op->nkv, kind, op->cs)
                           : cudaMemcpy2DAsync(host, hp, dev, lb, lb, op->nkv, kind, op->cs)))
                return false;
            continue;
        }
        /* a run of records: one row per record, for the K part then the V part */
        for (uint32_t kv = 0; kv < op->nkv; kv++) {
            uint8_t *d = dev + kv * lb;
            uint8_t *h = host + kv * hp;
            if (!CU_OK(h2d ? cudaMemcpy2DAsync(d, sp, h, op->rec_bytes, lb, rn.count, kind, op->cs)
                           : cudaMemcpy2DAsync(h, op->rec_bytes, d, sp, lb, rn.count, kind, op->cs)))
                return false;
        }
    }
    return true;
}

/* Enqueue one job's copies on the GPU (the device's async worker thread).
 * Appends one mark per layer range it covered to `out`. */
int async_enqueue(AsyncOp *op, const AsyncJob &j, std::vector<AsyncOp::Mark> &out)
{
    cudaStream_t s = j.s;
    if (j.gate && !CU_OK(cudaStreamWaitEvent(s, j.gate, 0)))
        return -EIO;
    if (!op->is_uploaded) {
        if (!CU_OK(cudaMemsetAsync(op->d_err, 0, sizeof(int32_t), s)) ||
            !CU_OK(cudaMemcpyAsync(op->d_meta, op->h_meta, op->meta_words * 8, cudaMemcpyHostToDevice, s)) ||
            !CU_OK(cudaEventRecord(op->uploaded, s)))
            return -EIO;
        op->is_uploaded = true;
        op->upload_stream = s;
    } else if (s != op->upload_stream && !CU_OK(cudaStreamWaitEvent(s, op->uploaded, 0))) {
        return -EIO;
    }
    auto mark = [&](uint32_t l0, uint32_t l1, cudaStream_t on) -> int {
        cudaEvent_t ev = op->take_event();
        if (!ev || !CU_OK(cudaEventRecord(ev, on)))
            return -EIO;
        out.push_back(AsyncOp::Mark{l0, l1, ev});
        return 0;
    };
    if (!op->staged) {
        if (op->base.num_records) {
            kv_copy_desc d = op->base;
            d.layer_begin = j.l0;
            d.num_layers = j.l1 - j.l0;
            int ret = kv_copy_launch(&d, s);
            if (ret)
                return ret;
        }
        return mark(j.l0, j.l1, s);
    }
    const bool load = op->base.direction == 0;
    for (uint32_t l = j.l0; l < j.l1; l++) {
        const int sl = (int)(op->next_slot++ % AsyncOp::kRing);
        uint8_t *slot = op->ring + (uint64_t)sl * op->slot_bytes;
        kv_copy_desc d = op->base;
        d.records = op->d_meta + op->rec_words + (uint64_t)sl * op->nrec;
        d.layer_k = op->base.layer_k + l;
        d.layer_v = op->base.layer_v ? op->base.layer_v + l : nullptr;
        d.num_layers = 1;
        d.layer_begin = 0;
        d.record_layers = 1;
        if (load) {
            if (op->slot_used[sl] && !CU_OK(cudaStreamWaitEvent(op->cs, op->slot_free[sl], 0)))
                return -EIO;
            if (!copy_runs(op, slot, l, cudaMemcpyHostToDevice))
                return -EIO;
            if (!CU_OK(cudaEventRecord(op->slot_ready[sl], op->cs)) ||
                !CU_OK(cudaStreamWaitEvent(s, op->slot_ready[sl], 0)))
                return -EIO;
            int ret = kv_copy_launch(&d, s);
            if (ret)
                return ret;
            if (!CU_OK(cudaEventRecord(op->slot_free[sl], s)))
                return -EIO;
            op->slot_used[sl] = true;
            if ((ret = mark(l, l + 1, s)))
                return ret;
        } else {
            if (op->slot_used[sl] && !CU_OK(cudaStreamWaitEvent(s, op->slot_free[sl], 0)))
                return -EIO;
            int ret = kv_copy_launch(&d, s);
            if (ret)
                return ret;
            if (!CU_OK(cudaEventRecord(op->slot_ready[sl], s)) ||
                !CU_OK(cudaStreamWaitEvent(op->cs, op->slot_ready[sl], 0)))
                return -EIO;
            if (!copy_runs(op, slot, l, cudaMemcpyDeviceToHost))
                return -EIO;
            if (!CU_OK(cudaEventRecord(op->slot_free[sl], op->cs)))
                return -EIO;
            op->slot_used[sl] = true;
            if ((ret = mark(l, l + 1, op->cs)))
                return ret;
        }
    }
    return 0;
}

struct DeviceCtx {
    int dev;
    std::mutex mu;
    std::condition_variable cv;
    std::vector<Lane *> all;
    std::vector<Lane *> idle[2];         /* per direction: [0] loads, [1] saves */
    int nlanes[2] = {0, 0};
    std::vector<AsyncOp *> async_idle;   /* finished async ops, reusable */
    int max_lanes;                       /* per direction */
    int host_ptr_ok = 0;   /* registered host memory usable at its host address */

    /* async worker: enqueues the jobs of every async op of this device in
     * submission order, off the callers' threads */
    std::mutex jmu;
    std::condition_variable jcv;
    std::deque<AsyncJob> jobs;
    bool jstop = false;
    std::thread worker;

    void submit(const AsyncJob &j)
    {
        std::lock_guard<std::mutex> lk(jmu);
        if (!worker.joinable())
            worker = std::thread([this] { run_jobs(); });
        jobs.push_back(j);
        jcv.notify_one();
    }

    void run_jobs()
    {
        cudaSetDevice(dev);
        for (;;) {
            AsyncJob j;
            {
                std::unique_lock<std::mutex> lk(jmu);
                jcv.wait(lk, [&] { return jstop || !jobs.empty(); });
                if (jobs.empty())
                    return;
                j = jobs.front();
                jobs.pop_front();
            }
            std::vector<AsyncOp::Mark> marks;
            int ret = j.op->poisoned ? -EIO : async_enqueue(j.op, j, marks);
            std::lock_guard<std::mutex> lk(j.op->mu);
            for (auto &m : marks)
                j.op->marks.push_back(m);
            if (j.gate)
                j.op->spare.push_back(j.gate);   /* its wait is already enqueued */
            if (ret && !j.op->enqueue_err)
                j.op->enqueue_err = ret;
            j.op->jobs_done++;
            j.op->cv.notify_all();
        }
    }

    /* enqueue what is queued, then end the worker */
    void stop_worker()
    {
        {
            std::lock_guard<std::mutex> lk(jmu);
            jstop = true;
            jcv.notify_all();
        }
        if (worker.joinable())
            worker.join();
    }

    ~DeviceCtx() { stop_worker(); }
};

struct IpcSet {
    int dev;
    std::vector<std::string> opened;  /* handles this set holds a reference on */
    std::vector<uint64_t> host_ptrs;  /* layer bases (host mirror) */
};

/* one mapping per (device, handle): PyTorch sub-allocates several layer
 * tensors from one cudaMalloc block, so several keys can name the same
 * handle; it is opened once and reference counted */
struct IpcMapping {
    void *base;
    int refs;
};

struct PinnedRegion {
    uint64_t size;
};

class CudaAdaptor : public Adaptor
{
public:
    CudaAdaptor()
    {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
            log_error("cuda adaptor: no CUDA device visible");
            throw std::bad_alloc();
        }
        num_devices_ = n;
        timeout_ms_ = env_int("CROSSCACHE_TIMEOUT_MS", 120000);
        lanes_per_dev_ = std::max(1, env_int("CROSSCACHE_LANES", 2));   /* per direction */
        const char *m = getenv("CROSSCACHE_XFER_MODE");
        direct_ = m && !strcmp(m, "direct");
        async_ctas_ = (uint32_t)std::max(1, env_int("CROSSCACHE_ASYNC_CTAS", 32));
    }

    ~CudaAdaptor() override
    {
        std::lock_guard<std::mutex> g(reg_mu_);
        /* copies of async transfers a caller never finished may still be
         * queued: let them run out before the memory they touch goes away */
        for (auto &kv : devs_) {
            kv.second->stop_worker();
            if (cudaSetDevice(kv.first) == cudaSuccess)
                cudaDeviceSynchronize();
        }
        for (auto &kv : devs_)
            drain(kv.second.get());
        for (auto &kv : ipc_) {
            cudaSetDevice(kv.second.dev);
            release_handles_locked(kv.second);
            cudaFree(kv.first);
        }
        for (auto &kv : pinned_) {
            cudaHostUnregister(kv.first);
            munmap(kv.first, kv.second.size);
        }
    }

    void *AllocPinnedPtr(uint8_t nid, uint64_t size, unsigned int, void **daddr) override
    {
        if (!size || size % 4096) {
            log_error("device(%u) pinned size %lu is not 4 KiB aligned", nid, (unsigned long)size);
            return nullptr;
        }
        if (nid >= num_devices_ || !CU_OK(cudaSetDevice(nid)))
            return nullptr;
        void *addr = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
        if (addr == MAP_FAILED) {
            log_error("device(%u) mmap(%lu) failed errno %d", nid, (unsigned long)size, errno);
            return nullptr;
        }
        madvise(addr, size, MADV_HUGEPAGE);
        prefault(addr, size);
        if (!CU_OK(cudaHostRegister(addr, size, cudaHostRegisterMapped | cudaHostRegisterPortable))) {
            munmap(addr, size);
            return nullptr;
        }
        void *dptr = nullptr;
        if (!CU_OK(cudaHostGetDevicePointer(&dptr, addr, 0))) {
            cudaHostUnregister(addr);
            munmap(addr, size);
            return nullptr;
        }
        {
            std::lock_guard<std::mutex> g(reg_mu_);
            pinned_[addr] = PinnedRegion{size};
        }
        if (daddr)
            *daddr = dptr;
        log_debug("device(%u) pinned %lu B host %p dev %p", nid, (unsigned long)size, addr, dptr);
        return addr;
    }

    void FreePinnedPtr(void *addr, uint64_t size) override
    {
        {
            std::lock_guard<std::mutex> g(reg_mu_);
            pinned_.erase(addr);
        }
        cudaHostUnregister(addr);
        munmap(addr, size);
    }

    void *WrapperPtr(uint8_t nid, void *addr, uint64_t size) override
    {
        void *d = nullptr;
        if (nid >= num_devices_ || !CU_OK(cudaSetDevice(nid)) || !CU_OK(cudaMalloc(&d, size)))
            return nullptr;
        if (!CU_OK(cudaMemcpy(d, addr, size, cudaMemcpyHostToDevice))) {
            cudaFree(d);
            return nullptr;
        }
        return d;
    }

    void UnWrapperPtr(void *daddr) override
    {
        if (daddr)
            cudaFree(daddr);
    }

    void *OpenIPCKeys(uint8_t nid, uint16_t per_len, uint16_t num, void *data) override
    {
        if (!num || !data || nid >= num_devices_ || !CU_OK(cudaSetDevice(nid)))
            return nullptr;
        if (per_len != 8 && per_len != sizeof(cudaIpcMemHandle_t) &&
            per_len != sizeof(cudaIpcMemHandle_t) + 8) {
            log_error("open_ipc_keys: unsupported per_len %u (8, 64 or 72)", per_len);
            return nullptr;
        }
        IpcSet set;
        set.dev = nid;
        const uint8_t *p = static_cast<const uint8_t *>(data);
        std::unique_lock<std::mutex> lk(reg_mu_);
        for (uint16_t i = 0; i < num; i++, p += per_len) {
            uint64_t ptr = 0;
            if (per_len == 8) {
                memcpy(&ptr, p, 8);
            } else {
                cudaIpcMemHandle_t h;
                uint64_t off = 0;
                memcpy(&h, p, sizeof(h));
                if (per_len > sizeof(h))
                    memcpy(&off, p + sizeof(h), 8);
                std::string key(reinterpret_cast<const char *>(p), sizeof(h));
                key.push_back((char)nid);
                auto it = ipc_maps_.find(key);
                void *base = nullptr;
                if (it != ipc_maps_.end()) {
                    it->second.refs++;
                    base = it->second.base;
                } else {
                    if (!CU_OK(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess))) {
                        release_handles_locked(set);
                        return nullptr;
                    }
                    ipc_maps_[key] = IpcMapping{base, 1};
                }
                set.opened.push_back(key);
                ptr = (uint64_t)(uintptr_t)base + off;
            }
            set.host_ptrs.push_back(ptr);
        }
        void *d = nullptr;
        if (!CU_OK(cudaMalloc(&d, (size_t)num * 8)) ||
            !CU_OK(cudaMemcpy(d, set.host_ptrs.data(), (size_t)num * 8, cudaMemcpyHostToDevice))) {
            if (d)
                cudaFree(d);
            release_handles_locked(set);
            return nullptr;
        }
        ipc_[d] = std::move(set);
        return d;
    }

    void CloseIPCKeys(void *daddr) override
    {
        std::lock_guard<std::mutex> g(reg_mu_);
        auto it = ipc_.find(daddr);
        if (it == ipc_.end())
            return;
        cudaSetDevice(it->second.dev);
        release_handles_locked(it->second);
        ipc_.erase(it);
        cudaFree(daddr);
    }

    int TransferKVCache(struct transfer_params *p) override;
    int TransferKVCacheBatch(struct transfer_batch *b) override;
    struct transfer_async *AsyncBegin(const struct transfer_batch *b, int *err) override;
    int AsyncLayers(struct transfer_async *h, uint32_t l0, uint32_t l1, void *stream,
                    void *wait_event) override;
    int AsyncStreamWait(struct transfer_async *h, uint32_t layer, void *stream) override;
    int AsyncQuery(struct transfer_async *h) override;
    int AsyncEnd(struct transfer_async *h) override;

    /* Release this process's idle transfer resources on the device (lanes:
     * streams, staging rings, metadata; finished async ops).  Lanes and ops
     * in use by other threads stay, and so does the device context, which
     * transfers in flight still point to; the GPU itself is never reset. */
    void Reset(uint8_t nid) override
    {
        DeviceCtx *ctx;
        {
            std::lock_guard<std::mutex> g(reg_mu_);
            auto it = devs_.find(nid);
            if (it == devs_.end())
                return;
            ctx = it->second.get();
        }
        std::lock_guard<std::mutex> lk(ctx->mu);
        for (int d = 0; d < 2; d++) {
            for (Lane *l : ctx->idle[d]) {
                ctx->all.erase(std::remove(ctx->all.begin(), ctx->all.end(), l), ctx->all.end());
                ctx->nlanes[d]--;
                l->release();
                delete l;
            }
            ctx->idle[d].clear();
        }
        for (AsyncOp *op : ctx->async_idle) {
            op->release();
            delete op;
        }
        ctx->async_idle.clear();
    }

private:
    DeviceCtx *device(int dev)
    {
        std::lock_guard<std::mutex> g(reg_mu_);
        auto &slot = devs_[dev];
        if (!slot) {
            slot.reset(new DeviceCtx());
            slot->dev = dev;
            slot->max_lanes = lanes_per_dev_;
            int ok = 0;
            cudaDeviceGetAttribute(&ok, cudaDevAttrCanUseHostPointerForRegisteredMem, dev);
            slot->host_ptr_ok = ok;
        }
        return slot.get();
    }

    /* A lane of direction `dir` (1: saves, 0: loads), created on first need
     * up to max_lanes per direction.  Saves and loads never share a lane,
     * like the reference's separate Store and Load thread pools
     * (src/main.c:394-410): a burst of saves cannot hold every lane while a
     * load waits for one, or the other way round. */
    Lane *acquire(DeviceCtx *ctx, int dir)
    {
        std::unique_lock<std::mutex> lk(ctx->mu);
        for (;;) {
            std::vector<Lane *> &idle = ctx->idle[dir];
            if (!idle.empty()) {
                Lane *l = idle.back();
                idle.pop_back();
                return l;
            }
            if (ctx->nlanes[dir] < ctx->max_lanes) {
                Lane *l = new (std::nothrow) Lane();
                if (!l || !l->init(ctx->dev)) {
                    if (l) {
                        l->release();
                        delete l;
                    }
                    return nullptr;
                }
                l->dir = dir;
                ctx->all.push_back(l);
                ctx->nlanes[dir]++;
                return l;
            }
            if (ctx->cv.wait_for(lk, std::chrono::milliseconds(timeout_ms_)) == std::cv_status::timeout &&
                ctx->idle[dir].empty())
                return nullptr;
        }
    }

    void give_back(DeviceCtx *ctx, Lane *l)
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        if (l->poisoned)
            return;   /* device work may still be in flight: never reuse */
        ctx->idle[l->dir].push_back(l);
        ctx->cv.notify_all();
    }

    void drain(DeviceCtx *ctx)
    {
        if (!ctx)
            return;
        std::lock_guard<std::mutex> lk(ctx->mu);
        for (Lane *l : ctx->all) {
            if (!l->poisoned) {
                l->release();
                delete l;
            }
        }
        ctx->all.clear();
        ctx->idle[0].clear();
        ctx->idle[1].clear();
        ctx->nlanes[0] = ctx->nlanes[1] = 0;
        /* async ops still held by callers stay theirs; the idle ones go */
        for (AsyncOp *op : ctx->async_idle) {
            op->release();
            delete op;
        }
        ctx->async_idle.clear();
    }

    std::chrono::steady_clock::time_point deadline() const
    {
        return std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms_);
    }

    void release_handles_locked(IpcSet &set)
    {
        for (const std::string &key : set.opened) {
            auto it = ipc_maps_.find(key);
            if (it == ipc_maps_.end())
                continue;
            if (--it->second.refs == 0) {
                cudaIpcCloseMemHandle(it->second.base);
                ipc_maps_.erase(it);
            }
        }
        set.opened.clear();
    }

    /* true when every layer base registered under this device array is 16-byte aligned */
    bool layers_aligned(const void *dptrs)
    {
        if (!dptrs)
            return true;
        std::lock_guard<std::mutex> g(reg_mu_);
        auto it = ipc_.find(const_cast<void *>(dptrs));
        if (it == ipc_.end())
            return false;
        for (uint64_t p : it->second.host_ptrs)
            if (p % 16)
                return false;
        return true;
    }

    int run_batch(Lane *l, DeviceCtx *ctx, const struct transfer_batch *b);
    int finish(Lane *l, cudaStream_t last, int ret);

    int num_devices_ = 0;
    uint32_t async_ctas_ = 32;
    int timeout_ms_ = 120000;
    int lanes_per_dev_ = 2;
    bool direct_ = false;
    std::mutex reg_mu_;
    std::map<int, std::unique_ptr<DeviceCtx>> devs_;
    std::map<void *, IpcSet> ipc_;
    std::map<std::string, IpcMapping> ipc_maps_;
    std::map<void *, PinnedRegion> pinned_;
};

/* read back the error word after everything queued on `last`, then wait.
 * The read-back goes through the lane's copy stream: every copy command a
 * lane issues (metadata up, records, error word down) is on cs and the
 * kernel stream carries only kernels.  A tiny copy on the kernel stream can
 * be given a copy engine that the other lane is keeping busy with 32 MiB
 * record copies, and then waits behind them -- measured on B200 with one
 * lane saving while another loads: H2D fell to half the rate the link gives
 * plain copies in both directions at once. */
int CudaAdaptor::finish(Lane *l, cudaStream_t last, int ret)
{
    if (ret == 0 && last != l->cs &&
        (!CU_OK(cudaEventRecord(l->fin, last)) || !CU_OK(cudaStreamWaitEvent(l->cs, l->fin, 0))))
        ret = -EIO;
    if (ret == 0 && (!CU_OK(cudaMemcpyAsync(l->h_err, l->d_err, 4, cudaMemcpyDeviceToHost, l->cs)) ||
                     !CU_OK(cudaEventRecord(l->fin, l->cs))))
        ret = -EIO;
    if (ret == 0 || ret == -EIO) {
        int w = wait_event(l->fin, deadline());
        if (w == -ETIMEDOUT) {
            log_error("device(%d) transfer timed out after %d ms", l->dev, timeout_ms_);
            l->poisoned = true;
            return -ETIMEDOUT;
        }
        if (w)
            ret = w;
    }
    if (ret == 0 && *l->h_err) {
        log_error("device(%d) kv copy reported error bits 0x%x", l->dev, *l->h_err);
        ret = -EINVAL;
    }
    return ret;
}

int CudaAdaptor::run_batch(Lane *l, DeviceCtx *ctx, const struct transfer_batch *b)
{
    const uint32_t R = b->num_records;
    const uint32_t bpr = b->num_tokens / b->block_size;
    const uint64_t unit = (uint64_t)b->hidden_dim_size * b->caches_element_size;
    const uint64_t rec_bytes = (uint64_t)(b->value_ptrs ? 2 : 1) * b->num_layers * b->num_tokens * unit;
    const bool save = b->direction;
    const bool device_recs = b->record_on_device != 0;
    const bool direct = device_recs || direct_;

    /* metadata: block ids, then (direct modes) record addresses */
    uint64_t words = (uint64_t)R * bpr + (direct ? R : 0);
    if (!l->ensure_meta(words))
        return -ENOMEM;
    memcpy(l->h_meta, b->block_ids, (uint64_t)R * bpr * 8);
    if (direct) {
        for (uint32_t r = 0; r < R; r++) {
            void *p = b->records[r];
            if (!device_recs && !ctx->host_ptr_ok) {
                void *dp = nullptr;
                if (!CU_OK(cudaHostGetDevicePointer(&dp, p, 0)))
                    return -EINVAL;
                p = dp;
            }
            l->h_meta[(uint64_t)R * bpr + r] = (uint64_t)(uintptr_t)p;
        }
    }
    /* metadata up through the copy stream (see finish); kernels wait for it */
    if (!CU_OK(cudaMemsetAsync(l->d_err, 0, 4, l->cs)) ||
        !CU_OK(cudaMemcpyAsync(l->d_meta, l->h_meta, words * 8, cudaMemcpyHostToDevice, l->cs)) ||
        !CU_OK(cudaEventRecord(l->mready, l->cs)) || !CU_OK(cudaStreamWaitEvent(l->ks, l->mready, 0)))
        return -EIO;

    kv_copy_desc d{};
    d.layer_k = static_cast<const uint64_t *>(b->keys_ptrs);
    d.layer_v = static_cast<const uint64_t *>(b->value_ptrs);
    d.error = l->d_err;
    d.page_buffer_size = b->page_buffer_size;
    d.unit_bytes = (uint32_t)unit;
    d.num_tokens = b->num_tokens;
    d.block_size = b->block_size;
    d.num_layers = b->num_layers;
    d.direction = save ? 1 : 0;
    d.block_stride = b->block_stride;
    d.head_bytes = b->head_bytes;
    /* TMA bulk copies need HBM records (staging or device records) and
     * 16-byte aligned bases; mapped host records keep the register path */
    bool recs_aligned = true;
    if (device_recs)
        for (uint32_t r = 0; r < R; r++)
            recs_aligned = recs_aligned && ((uintptr_t)b->records[r] % 16 == 0);
    if ((device_recs || !direct) && recs_aligned && layers_aligned(b->keys_ptrs) &&
        layers_aligned(b->value_ptrs))
        d.flags = KVCOPY_FLAG_BULK;

    if (direct) {
        d.block_ids = l->d_meta;
        d.records = l->d_meta + (uint64_t)R * bpr;
        d.num_records = R;
        int ret = kv_copy_launch(&d, l->ks);
        if (ret)
            return ret;
        return finish(l, l->ks, 0);
    }

    uint32_t G = 1;
    if (!l->ensure_staging(rec_bytes, &G))
        return -ENOMEM;
    const uint32_t ngroups = (R + G - 1) / G;
    for (uint32_t gi = 0; gi < ngroups; gi++) {
        const int s = gi % kNumSub;
        const uint32_t r0 = gi * G;
        const uint32_t n = std::min(G, R - r0);
        uint8_t *sub = l->staging + s * l->sub_bytes;
        d.block_ids = l->d_meta + (uint64_t)r0 * bpr;
        d.records = l->d_subrec + (uint64_t)s * l->max_group;
        d.num_records = n;
        if (save) {
            if (gi >= (uint32_t)kNumSub && !CU_OK(cudaStreamWaitEvent(l->ks, l->cdone[s], 0)))
                return -EIO;
            if (kv_copy_launch(&d, l->ks))
                return -EIO;
            if (!CU_OK(cudaEventRecord(l->kdone[s], l->ks)) ||
                !CU_OK(cudaStreamWaitEvent(l->cs, l->kdone[s], 0)))
                return -EIO;
            for (uint32_t j = 0; j < n; j++)
                if (!CU_OK(cudaMemcpyAsync(b->records[r0 + j], sub + j * rec_bytes, rec_bytes,
                                           cudaMemcpyDeviceToHost, l->cs)))
                    return -EIO;
            if (!CU_OK(cudaEventRecord(l->cdone[s], l->cs)))
                return -EIO;
        } else {
            if (gi >= (uint32_t)kNumSub && !CU_OK(cudaStreamWaitEvent(l->cs, l->kdone[s], 0)))
                return -EIO;
            for (uint32_t j = 0; j < n; j++)
                if (!CU_OK(cudaMemcpyAsync(sub + j * rec_bytes, b->records[r0 + j], rec_bytes,
                                           cudaMemcpyHostToDevice, l->cs)))
                    return -EIO;
            if (!CU_OK(cudaEventRecord(l->cdone[s], l->cs)) ||
                !CU_OK(cudaStreamWaitEvent(l->ks, l->cdone[s], 0)))
                return -EIO;
            if (kv_copy_launch(&d, l->ks))
                return -EIO;
            if (!CU_OK(cudaEventRecord(l->kdone[s], l->ks)))
                return -EIO;
        }
    }
    /* save: the last copies are on cs; load: the last kernel is on ks */
    return finish(l, save ? l->cs : l->ks, 0);
}

/* paged geometry a kernel can address: blocks that do not overlap, heads
 * that tile the token's unit */
static bool geometry_ok(const struct transfer_batch *b)
{
    const uint64_t unit = (uint64_t)b->hidden_dim_size * b->caches_element_size;
    return (!b->block_stride || b->block_stride >= (uint64_t)b->block_size * unit) &&
           (!b->head_bytes || unit % b->head_bytes == 0);
}

int CudaAdaptor::TransferKVCacheBatch(struct transfer_batch *b)
{
    if (!b->num_records)
        return 0;
    if (!b->keys_ptrs || !b->records || !b->block_ids || !b->block_size || !b->num_layers ||
        !b->num_tokens || b->num_tokens % b->block_size || !b->hidden_dim_size ||
        !b->caches_element_size || b->devid >= num_devices_ || !geometry_ok(b))
        return -EINVAL;
    if (!CU_OK(cudaSetDevice(b->devid)))
        return -EIO;
    DeviceCtx *ctx = device(b->devid);
    Lane *l = acquire(ctx, b->direction ? 1 : 0);
    if (!l)
        return -EBUSY;
    int ret = run_batch(l, ctx, b);
    if (ret && ret != -ETIMEDOUT && !l->poisoned) {
        /* drain whatever was queued before the failure */
        cudaStreamSynchronize(l->ks);
        cudaStreamSynchronize(l->cs);
    }
    give_back(ctx, l);
    return ret;
}

/* ---- asynchronous layer-ranged transfers -------------------------------- */

struct transfer_async *CudaAdaptor::AsyncBegin(const struct transfer_batch *b, int *err)
{
    auto fail = [&](int e) -> struct transfer_async * {
        if (err)
            *err = e;
        return nullptr;
    };
    if (!b->keys_ptrs || (b->num_records && (!b->records || !b->block_ids)) || !b->block_size ||
        !b->num_layers || !b->num_tokens || b->num_tokens % b->block_size || !b->hidden_dim_size ||
        !b->caches_element_size || b->devid >= num_devices_ || !geometry_ok(b))
        return fail(-EINVAL);
    if (!CU_OK(cudaSetDevice(b->devid)))
        return fail(-EIO);
    DeviceCtx *ctx = device(b->devid);
    AsyncOp *op = nullptr;
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        if (!ctx->async_idle.empty()) {
            op = ctx->async_idle.back();
            ctx->async_idle.pop_back();
        }
    }
    if (!op) {
        op = new (std::nothrow) AsyncOp();
        if (!op)
            return fail(-ENOMEM);
        if (!op->init(b->devid)) {
            op->release();
            delete op;
            return fail(-EIO);
        }
    }
    auto give_back = [&]() {
        op->reset_for_reuse();
        std::lock_guard<std::mutex> lk(ctx->mu);
        ctx->async_idle.push_back(op);
    };
    const uint32_t R = b->num_records;
    const uint32_t bpr = b->num_tokens / b->block_size;
    const bool device_recs = b->record_on_device != 0;
    const uint32_t nkv = b->value_ptrs ? 2 : 1;
    const uint64_t unit = (uint64_t)b->hidden_dim_size * b->caches_element_size;
    const uint64_t lb = (uint64_t)b->num_tokens * unit;
    const uint64_t slot_bytes = (uint64_t)R * nkv * lb;
    /* host records go through the copy engines unless the mode is direct or
     * the ring would be too large; HBM records are read in place */
    /* (a record is the row pitch of the copies: keep it inside int range) */
    bool staged = !device_recs && !direct_ && R && slot_bytes * AsyncOp::kRing <= kAsyncRingMax &&
                  (uint64_t)nkv * b->num_layers * lb <= (uint64_t)INT32_MAX;
    if (staged && !op->ensure_ring(slot_bytes * AsyncOp::kRing))
        staged = false;
    const uint64_t words = (uint64_t)R * bpr + (staged ? (uint64_t)AsyncOp::kRing * R : R);
    if (!op->ensure_meta(std::max<uint64_t>(words, 1))) {
        give_back();
        return fail(-ENOMEM);
    }
    if (R)
        memcpy(op->h_meta, b->block_ids, (uint64_t)R * bpr * 8);
    op->staged = staged;
    op->nrec = R;
    op->nkv = nkv;
    op->layer_bytes = lb;
    op->slot_bytes = slot_bytes;
    op->rec_words = (uint32_t)((uint64_t)R * bpr);
    if (staged) {
        op->host_recs.resize(R);
        for (uint32_t r = 0; r < R; r++)
            op->host_recs[r] = static_cast<uint8_t *>(b->records[r]);
        op->rec_bytes = (uint64_t)nkv * b->num_layers * lb;
        /* slot positions in host-address order, then runs of consecutive records */
        std::vector<uint32_t> order(R);
        for (uint32_t r = 0; r < R; r++)
            order[r] = r;
        std::sort(order.begin(), order.end(),
                  [&](uint32_t a, uint32_t c) { return op->host_recs[a] < op->host_recs[c]; });
        std::vector<uint32_t> pos(R);
        for (uint32_t k = 0; k < R; k++) {
            pos[order[k]] = k;
            uint8_t *h = op->host_recs[order[k]];
            if (k && op->runs.back().host + (uint64_t)op->runs.back().count * op->rec_bytes == h)
                op->runs.back().count++;
            else
                op->runs.push_back(AsyncOp::Run{h, k, 1});
        }
        for (int s = 0; s < AsyncOp::kRing; s++)
            for (uint32_t r = 0; r < R; r++)
                op->h_meta[(uint64_t)R * bpr + (uint64_t)s * R + r] =
                    (uint64_t)(uintptr_t)(op->ring + (uint64_t)s * slot_bytes + (uint64_t)pos[r] * nkv * lb);
    } else {
        for (uint32_t r = 0; r < R; r++) {
            void *p = b->records[r];
            if (!device_recs && !ctx->host_ptr_ok) {
                void *dp = nullptr;
                if (!CU_OK(cudaHostGetDevicePointer(&dp, p, 0))) {
                    give_back();
                    return fail(-EINVAL);
                }
                p = dp;
            }
            op->h_meta[(uint64_t)R * bpr + r] = (uint64_t)(uintptr_t)p;
        }
    }
    op->meta_words = words;
    kv_copy_desc &d = op->base;
    d = kv_copy_desc{};
    d.layer_k = static_cast<const uint64_t *>(b->keys_ptrs);
    d.layer_v = static_cast<const uint64_t *>(b->value_ptrs);
    d.error = op->d_err;
    d.page_buffer_size = b->page_buffer_size;
    d.unit_bytes = (uint32_t)unit;
    d.num_tokens = b->num_tokens;
    d.block_size = b->block_size;
    d.num_records = R;
    d.direction = b->direction ? 1 : 0;
    d.block_stride = b->block_stride;
    d.head_bytes = b->head_bytes;
    d.block_ids = op->d_meta;
    d.records = op->d_meta + (uint64_t)R * bpr;
    d.record_layers = b->num_layers;
    /* these kernels run next to the caller's own: a few register-path CTAs
     * (no shared memory) fit beside its kernels, where a TMA-bulk CTA with
     * 128 KiB of shared memory would wait for an SM to drain */
    d.max_ctas = async_ctas_;
    d.flags = 0;
    op->total_layers = b->num_layers;
    return reinterpret_cast<struct transfer_async *>(op);
}

int CudaAdaptor::AsyncLayers(struct transfer_async *h, uint32_t l0, uint32_t l1, void *stream, void *wait_event)
{
    AsyncOp *op = reinterpret_cast<AsyncOp *>(h);
    if (op->poisoned)
        return -EIO;
    if (l0 >= l1 || l1 > op->total_layers)
        return -EINVAL;
    if (!CU_OK(cudaSetDevice(op->dev)))
        return -EIO;
    /* the caller may drop or re-record its event at once: gate it here */
    cudaEvent_t gate = nullptr;
    if (wait_event) {
        gate = op->take_event();
        if (!gate || !CU_OK(cudaStreamWaitEvent(op->gate, static_cast<cudaEvent_t>(wait_event), 0)) ||
            !CU_OK(cudaEventRecord(gate, op->gate)))
            return -EIO;
    }
    {
        std::lock_guard<std::mutex> lk(op->mu);
        op->requested.push_back({l0, l1});
        op->jobs_submitted++;
    }
    device(op->dev)->submit(AsyncJob{op, l0, l1, static_cast<cudaStream_t>(stream), gate});
    return 0;
}

int CudaAdaptor::AsyncStreamWait(struct transfer_async *h, uint32_t layer, void *stream)
{
    AsyncOp *op = reinterpret_cast<AsyncOp *>(h);
    std::unique_lock<std::mutex> lk(op->mu);
    bool asked = false;
    for (auto &rg : op->requested)
        asked = asked || (layer >= rg.first && layer < rg.second);
    if (!asked)
        return -ENOENT;
    auto dl = deadline();
    for (;;) {
        for (auto it = op->marks.rbegin(); it != op->marks.rend(); ++it) {
            if (layer >= it->l0 && layer < it->l1) {
                if (!CU_OK(cudaSetDevice(op->dev)) ||
                    !CU_OK(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), it->ev, 0)))
                    return -EIO;
                return 0;
            }
        }
        if (op->jobs_done == op->jobs_submitted)
            return op->enqueue_err ? op->enqueue_err : -EIO;   /* its job failed */
        if (op->cv.wait_until(lk, dl) == std::cv_status::timeout)
            return -ETIMEDOUT;
    }
}

int CudaAdaptor::AsyncQuery(struct transfer_async *h)
{
    AsyncOp *op = reinterpret_cast<AsyncOp *>(h);
    if (op->poisoned)
        return -EIO;
    std::vector<cudaEvent_t> evs;
    {
        std::lock_guard<std::mutex> lk(op->mu);
        if (op->jobs_done < op->jobs_submitted)
            return 0;
        for (auto &m : op->marks)
            evs.push_back(m.ev);
    }
    cudaSetDevice(op->dev);
    for (cudaEvent_t e : evs) {
        cudaError_t r = cudaEventQuery(e);
        if (r == cudaErrorNotReady)
            return 0;
        if (r != cudaSuccess)
            return -EIO;
    }
    return 1;
}

int CudaAdaptor::AsyncEnd(struct transfer_async *h)
{
    AsyncOp *op = reinterpret_cast<AsyncOp *>(h);
    if (op->poisoned)
        return -EIO;
    if (!CU_OK(cudaSetDevice(op->dev)))
        return -EIO;
    auto dl = deadline();
    std::vector<cudaEvent_t> evs;
    int ret;
    {
        std::unique_lock<std::mutex> lk(op->mu);
        while (op->jobs_done < op->jobs_submitted) {
            if (op->cv.wait_until(lk, dl) == std::cv_status::timeout) {
                log_error("device(%d) async jobs not enqueued after %d ms", op->dev, timeout_ms_);
                op->poisoned = true;   /* the worker still holds it: never reused */
                return -ETIMEDOUT;
            }
        }
        for (auto &m : op->marks)
            evs.push_back(m.ev);
        ret = op->enqueue_err;
    }
    for (cudaEvent_t e : evs) {
        int w = wait_event(e, dl);
        if (w == -ETIMEDOUT) {
            log_error("device(%d) async transfer timed out after %d ms", op->dev, timeout_ms_);
            op->poisoned = true;     /* its memory may still be in use: never reused or freed */
            return -ETIMEDOUT;
        }
        if (w && !ret)
            ret = w;
    }
    if (ret) {
        /* a failed job may have left work queued behind its last mark:
         * this op is never reused */
        log_error("device(%d) async transfer failed to enqueue: %d", op->dev, ret);
        op->poisoned = true;
        return ret;
    }
    if (op->is_uploaded) {
        /* every mark (and the upload with the error-word reset) has completed on
         * the host's clock, so this readback comes after every kernel */
        int w = wait_event(op->uploaded, dl);
        if (w == -ETIMEDOUT) {
            op->poisoned = true;
            return -ETIMEDOUT;
        }
        if (w || !CU_OK(cudaMemcpyAsync(op->h_err, op->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, op->own)) ||
            !CU_OK(cudaStreamSynchronize(op->own)))
            ret = -EIO;
        if (ret == 0 && *op->h_err) {
            log_error("device(%d) async kv copy reported error bits 0x%x", op->dev, *op->h_err);
            ret = -EINVAL;
        }
    }
    op->reset_for_reuse();
    DeviceCtx *ctx = device(op->dev);
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->async_idle.push_back(op);
    return ret;
}

int CudaAdaptor::TransferKVCache(struct transfer_params *p)
{
    if (!p->caches || !p->keys_ptrs || !p->slot_mapping || !p->num_tokens || !p->num_layers ||
        !p->hidden_dim_size || !p->caches_element_size || p->devid >= num_devices_)
        return -EINVAL;
    if (!CU_OK(cudaSetDevice(p->devid)))
        return -EIO;
    cudaPointerAttributes attr{};
    if (!CU_OK(cudaPointerGetAttributes(&attr, p->caches)))
        return -EINVAL;
    const bool on_device = attr.type == cudaMemoryTypeDevice;
    const uint64_t unit = (uint64_t)p->hidden_dim_size * p->caches_element_size;
    const uint64_t rec_bytes = (uint64_t)(p->value_ptrs ? 2 : 1) * p->num_layers * p->num_tokens * unit;
    void *host = p->caches_h ? p->caches_h : p->caches;

    DeviceCtx *ctx = device(p->devid);
    Lane *l = acquire(ctx, p->direction ? 1 : 0);
    if (!l)
        return -EBUSY;
    int ret = 0;
    kv_copy_desc d{};
    d.layer_k = static_cast<const uint64_t *>(p->keys_ptrs);
    d.layer_v = static_cast<const uint64_t *>(p->value_ptrs);
    d.slots = static_cast<const int64_t *>(p->slot_mapping);
    d.error = l->d_err;
    d.page_buffer_size = p->page_buffer_size;
    d.unit_bytes = (uint32_t)unit;
    d.num_tokens = p->num_tokens;
    d.block_size = 1;
    d.num_layers = p->num_layers;
    d.num_records = 1;
    d.direction = p->direction ? 1 : 0;

    if (!l->ensure_meta(1) || !CU_OK(cudaMemsetAsync(l->d_err, 0, 4, l->ks))) {
        ret = -EIO;
    } else if (on_device || direct_) {
        l->h_meta[0] = (uint64_t)(uintptr_t)p->caches;
        if (!CU_OK(cudaMemcpyAsync(l->d_meta, l->h_meta, 8, cudaMemcpyHostToDevice, l->ks)))
            ret = -EIO;
        d.records = l->d_meta;
        if (!ret)
            ret = kv_copy_launch(&d, l->ks);
        ret = finish(l, l->ks, ret);
    } else {
        uint32_t G = 1;
        if (!l->ensure_staging(rec_bytes, &G)) {
            ret = -ENOMEM;
        } else {
            d.records = l->d_subrec;   /* sub-slot 0, first record */
            if (p->direction) {
                ret = kv_copy_launch(&d, l->ks);
                if (!ret && !CU_OK(cudaMemcpyAsync(host, l->staging, rec_bytes, cudaMemcpyDeviceToHost, l->ks)))
                    ret = -EIO;
            } else {
                if (!CU_OK(cudaMemcpyAsync(l->staging, host, rec_bytes, cudaMemcpyHostToDevice, l->ks)))
                    ret = -EIO;
                if (!ret)
                    ret = kv_copy_launch(&d, l->ks);
            }
            ret = finish(l, l->ks, ret);
        }
    }
    if (ret && ret != -ETIMEDOUT && !l->poisoned)
        cudaStreamSynchronize(l->ks);
    give_back(ctx, l);
    return ret;
}

}  // namespace

adaptor_t *cuda_adaptor_create(void)
{
    try {
        return new CudaAdaptor();
    } catch (...) {
        log_error("cuda adaptor create failed");
        return nullptr;
    }
}

void cuda_adaptor_destroy(adaptor_t *adaptor) { delete adaptor; }

/* 72-byte CUDA IPC key of device memory: the cudaIpcMemHandle_t of the
 * cudaMalloc allocation containing dptr, then the uint64 byte offset of dptr
 * inside it (the allocation base comes from the driver's
 * cuMemGetAddressRange, reached through cudaGetDriverEntryPointByVersion so
 * that no libcuda link is needed). */
int ipc_export_key(const void *dptr, uint8_t *key_out)
{
    typedef int (*get_range_fn)(unsigned long long *, size_t *, unsigned long long);
    static get_range_fn get_range = nullptr;
    static std::once_flag once;
    if (!dptr || !key_out)
        return -EINVAL;
    std::call_once(once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult st;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault, &st) ==
                cudaSuccess && st == cudaDriverEntryPointSuccess)
            get_range = reinterpret_cast<get_range_fn>(fn);
    });
    if (!get_range)
        return -ENOSYS;
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, dptr) != cudaSuccess || attr.type != cudaMemoryTypeDevice)
        return -EINVAL;
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(attr.device) != cudaSuccess)
        return -EIO;
    unsigned long long base = 0;
    size_t size = 0;
    int ret = 0;
    cudaIpcMemHandle_t h;
    if (get_range(&base, &size, (unsigned long long)(uintptr_t)dptr) != 0) {
        ret = -EINVAL;
    } else if (cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)) != cudaSuccess) {
        log_error("ipc_export_key: cudaIpcGetMemHandle failed (memory not from cudaMalloc?)");
        ret = -EINVAL;
    } else {
        uint64_t off = (uint64_t)(uintptr_t)dptr - base;
        memcpy(key_out, &h, sizeof(h));
        memcpy(key_out + sizeof(h), &off, 8);
    }
    if (prev >= 0)
        cudaSetDevice(prev);
    return ret;
}
