/*
 * CPU memcpy backend (CACHE_BACKEND_MEM).
 *
 * The host-only counterpart of CrossCache's MemAdaptor
 * (src/device/mem/mem.cpp:17-191): the "paged cache" and the records are host
 * memory and a transfer is a memcpy per contiguous slot run with the record
 * byte layout of mem.cpp:136-167.  Unlike the reference it uses the caller's
 * layer pointers (the reference maps fake /fakekv:<i> shm files instead,
 * mem.cpp:80-107) and does not build a per-token log string.  It is selected
 * only explicitly (cache_init_backend(..., CACHE_BACKEND_MEM)) and never
 * stands in for the CUDA backend.
 */
#include "adaptor.h"

extern "C" {
#include "../infra/log.h"
#include "../infra/threadpool.h"
}

#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <new>
#include <sys/mman.h>
#include <utility>
#include <vector>

namespace {

struct RecordJob {
    const struct transfer_batch *tb;
    uint32_t r;
    cc_latch_t *latch;
};

/* paged geometry of kvcopy.h (kv_copy_desc block_stride / head_bytes) */
struct Geom {
    uint64_t block_stride = 0;   /* 0: block_size * unit */
    uint32_t head_bytes = 0;     /* 0: token-major block */
};

/* token t of the record at paged slot s, geometry g: copy its unit between
 * the plane at base and the record bytes c */
void copy_token_strided(uint8_t *base, uint8_t *c, uint64_t s, uint32_t bs, uint64_t unit,
                        const Geom &g, bool to_record)
{
    const uint64_t blk = s / bs, j = s % bs;
    const uint64_t stride = g.block_stride ? g.block_stride : bs * unit;
    if (!g.head_bytes) {
        uint8_t *p = base + blk * stride + j * unit;
        to_record ? memcpy(c, p, unit) : memcpy(p, c, unit);
        return;
    }
    for (uint64_t h = 0; h < unit / g.head_bytes; h++) {
        uint8_t *p = base + blk * stride + (h * bs + j) * g.head_bytes;
        uint8_t *q = c + h * g.head_bytes;
        to_record ? memcpy(q, p, g.head_bytes) : memcpy(p, q, g.head_bytes);
    }
}

/* copy record layers [l0, l1) of one record holding L layers; slot(t) from
 * per-token slots or from block ids */
int copy_record(uint8_t *rec, const uint64_t *kl, const uint64_t *vl,
                const int64_t *slots, const uint64_t *bids, uint32_t bs,
                uint64_t page_buffer_size, uint32_t L, uint32_t C,
                uint64_t unit, bool to_record, uint32_t l0 = 0, uint32_t l1 = UINT32_MAX,
                const Geom &g = Geom{})
{
    const int nkv = vl ? 2 : 1;
    const bool dense = !g.head_bytes && (!g.block_stride || g.block_stride == (uint64_t)bs * unit);
    if ((g.block_stride && g.block_stride < (uint64_t)bs * unit) || (g.head_bytes && unit % g.head_bytes))
        return -EINVAL;
    if (l1 > L)
        l1 = L;
    for (int kv = 0; kv < nkv; kv++) {
        const uint64_t *layers = kv ? vl : kl;
        for (uint32_t l = l0; l < l1; l++) {
            uint8_t *base = reinterpret_cast<uint8_t *>(layers[l]);
            uint8_t *rl = rec + ((uint64_t)kv * L + l) * C * unit;
            if (!base)
                return -EINVAL;
            uint32_t t = 0;
            while (t < C) {
                int64_t s0 = slots ? slots[t] : (int64_t)(bids[t / bs] * bs + t % bs);
                if (!slots && bids[t / bs] >= (page_buffer_size + bs - 1) / bs)
                    return -EINVAL;
                uint32_t n = 1;
                for (;;) {
                    if (!dense || t + n >= C)
                        break;
                    int64_t sn = slots ? slots[t + n]
                                       : (int64_t)(bids[(t + n) / bs] * bs + (t + n) % bs);
                    if (sn != s0 + (int64_t)n)
                        break;
                    n++;
                }
                if (s0 < 0 || (uint64_t)s0 + n > page_buffer_size)
                    return -EINVAL;
                uint8_t *c = rl + (uint64_t)t * unit;
                if (!dense) {
                    copy_token_strided(base, c, (uint64_t)s0, bs, unit, g, to_record);
                } else {
                    uint8_t *p = base + (uint64_t)s0 * unit;
                    if (to_record)
                        memcpy(c, p, n * unit);
                    else
                        memcpy(p, c, n * unit);
                }
                t += n;
            }
        }
    }
    return 0;
}

Geom geom_of(const struct transfer_batch *tb)
{
    Geom g;
    g.block_stride = tb->block_stride;
    g.head_bytes = tb->head_bytes;
    return g;
}

void record_job(void *arg)
{
    RecordJob *j = static_cast<RecordJob *>(arg);
    const struct transfer_batch *tb = j->tb;
    uint32_t bpr = tb->num_tokens / tb->block_size;
    int ret = copy_record(static_cast<uint8_t *>(tb->records[j->r]),
                          static_cast<const uint64_t *>(tb->keys_ptrs),
                          static_cast<const uint64_t *>(tb->value_ptrs), nullptr,
                          tb->block_ids + (uint64_t)j->r * bpr, tb->block_size,
                          tb->page_buffer_size, tb->num_layers, tb->num_tokens,
                          (uint64_t)tb->hidden_dim_size * tb->caches_element_size,
                          tb->direction, 0, UINT32_MAX, geom_of(tb));
    cc_latch_done(j->latch, ret);
}

class MemAdaptor : public Adaptor
{
public:
    MemAdaptor()
    {
        const char *s = getenv("CROSSCACHE_MEM_THREADS");
        int n = s ? atoi(s) : 4;   /* the reference's CaCopy pool size */
        pool_ = threadpool_create("CaCopy", n > 0 ? n : 4);
        if (!pool_)
            throw std::bad_alloc();
    }
    ~MemAdaptor() override { threadpool_destroy(pool_); }

    void *AllocPinnedPtr(uint8_t nid, uint64_t size, unsigned int, void **daddr) override
    {
        if (!size || size % 4096) {
            log_error("nid(%u) pool size %lu is not 4 KiB aligned", nid, (unsigned long)size);
            return nullptr;
        }
        void *addr = mmap(nullptr, size, PROT_READ | PROT_WRITE,
                          MAP_PRIVATE | MAP_ANONYMOUS | MAP_POPULATE, -1, 0);
        if (addr == MAP_FAILED)
            return nullptr;
        if (daddr)
            *daddr = addr;
        return addr;
    }
    void FreePinnedPtr(void *addr, uint64_t size) override { munmap(addr, size); }
    void *WrapperPtr(uint8_t, void *addr, uint64_t size) override
    {
        void *d = malloc(size);
        if (d)
            memcpy(d, addr, size);
        return d;
    }
    void UnWrapperPtr(void *daddr) override { free(daddr); }
    void *OpenIPCKeys(uint8_t, uint16_t per_len, uint16_t num, void *data) override
    {
        if (per_len != sizeof(uint64_t) || !num || !data) {
            log_error("mem backend takes raw host pointers (per_len 8), got %u", per_len);
            return nullptr;
        }
        void *a = malloc((size_t)num * sizeof(uint64_t));
        if (a)
            memcpy(a, data, (size_t)num * sizeof(uint64_t));
        return a;
    }
    void CloseIPCKeys(void *daddr) override { free(daddr); }

    int TransferKVCache(struct transfer_params *p) override
    {
        if (!p->caches || !p->keys_ptrs || !p->slot_mapping)
            return -EINVAL;
        return copy_record(static_cast<uint8_t *>(p->caches),
                           static_cast<const uint64_t *>(p->keys_ptrs),
                           static_cast<const uint64_t *>(p->value_ptrs),
                           static_cast<const int64_t *>(p->slot_mapping), nullptr, 1,
                           p->page_buffer_size, p->num_layers, p->num_tokens,
                           (uint64_t)p->hidden_dim_size * p->caches_element_size,
                           p->direction);
    }

    int TransferKVCacheBatch(struct transfer_batch *tb) override
    {
        if (!tb->num_records)
            return 0;
        if (!tb->records || !tb->block_ids || !tb->keys_ptrs || !tb->block_size ||
            tb->num_tokens % tb->block_size)
            return -EINVAL;
        RecordJob *jobs = new (std::nothrow) RecordJob[tb->num_records];
        if (!jobs)
            return -ENOMEM;
        cc_latch_t latch;
        cc_latch_init(&latch, tb->num_records);
        for (uint32_t r = 0; r < tb->num_records; r++) {
            jobs[r] = RecordJob{tb, r, &latch};
            if (threadpool_submit(pool_, &jobs[r], record_job))
                record_job(&jobs[r]);
        }
        int ret = cc_latch_wait(&latch);
        cc_latch_fini(&latch);
        delete[] jobs;
        return ret;
    }

    void Reset(uint8_t) override {}

    /* asynchronous API, done synchronously: the copy happens in AsyncLayers */
    struct transfer_async *AsyncBegin(const struct transfer_batch *tb, int *err) override
    {
        int e = 0;
        if (!tb || (tb->num_records && (!tb->records || !tb->block_ids || !tb->keys_ptrs ||
                                        !tb->block_size || tb->num_tokens % tb->block_size)))
            e = -EINVAL;
        MemAsync *h = e ? nullptr : new (std::nothrow) MemAsync();
        if (!e && !h)
            e = -ENOMEM;
        if (e) {
            if (err)
                *err = e;
            return nullptr;
        }
        h->tb = *tb;
        const uint32_t bpr = tb->block_size ? tb->num_tokens / tb->block_size : 0;
        h->recs.assign(tb->records, tb->records + tb->num_records);
        h->bids.assign(tb->block_ids, tb->block_ids + (uint64_t)tb->num_records * bpr);
        h->tb.records = h->recs.data();
        h->tb.block_ids = h->bids.data();
        return reinterpret_cast<struct transfer_async *>(h);
    }

    int AsyncLayers(struct transfer_async *ha, uint32_t l0, uint32_t l1, void *stream,
                    void *wait_event) override
    {
        MemAsync *h = reinterpret_cast<MemAsync *>(ha);
        const struct transfer_batch *tb = &h->tb;
        if (stream || wait_event || l0 >= l1 || l1 > tb->num_layers)
            return -EINVAL;
        const uint32_t bpr = tb->num_tokens / tb->block_size;
        const uint64_t unit = (uint64_t)tb->hidden_dim_size * tb->caches_element_size;
        for (uint32_t r = 0; r < tb->num_records; r++) {
            int ret = copy_record(static_cast<uint8_t *>(tb->records[r]),
                                  static_cast<const uint64_t *>(tb->keys_ptrs),
                                  static_cast<const uint64_t *>(tb->value_ptrs), nullptr,
                                  tb->block_ids + (uint64_t)r * bpr, tb->block_size,
                                  tb->page_buffer_size, tb->num_layers, tb->num_tokens, unit,
                                  tb->direction, l0, l1, geom_of(tb));
            if (ret) {
                h->err = ret;
                return 0;       /* reported by AsyncEnd, as the device backend does */
            }
        }
        h->covered.push_back({l0, l1});
        return 0;
    }

    int AsyncStreamWait(struct transfer_async *ha, uint32_t layer, void *stream) override
    {
        MemAsync *h = reinterpret_cast<MemAsync *>(ha);
        if (stream)
            return -EINVAL;
        for (auto &rg : h->covered)
            if (layer >= rg.first && layer < rg.second)
                return 0;
        return -ENOENT;
    }

    int AsyncQuery(struct transfer_async *) override { return 1; }

    int AsyncEnd(struct transfer_async *ha) override
    {
        MemAsync *h = reinterpret_cast<MemAsync *>(ha);
        int ret = h->err;
        delete h;
        return ret;
    }

private:
    struct MemAsync {
        struct transfer_batch tb;
        std::vector<void *> recs;
        std::vector<uint64_t> bids;
        std::vector<std::pair<uint32_t, uint32_t>> covered;
        int err = 0;
    };
    threadpool_t *pool_;
};

}  // namespace

adaptor_t *mem_adaptor_create(void)
{
    try {
        return new MemAdaptor();
    } catch (...) {
        log_error("mem adaptor create failed");
        return nullptr;
    }
}

void mem_adaptor_destroy(adaptor_t *adaptor) { delete adaptor; }
