/*
 * Paged-KV record gather (save) and scatter (load) kernels for sm_100a.
 *
 * Device half of CrossCache's TransferKVCache: the AscendC kernel
 * src/device/npu/kernels/multi_layer_memcpy_kernel.cpp:6-198 moves one token
 * (hidden_dims elements) per DataCopy on at most 4 vector cores; the byte
 * mapping is the one of the reference CPU path src/device/mem/mem.cpp:136-167
 * (record = K part [layer][token][unit] then V part, token t of layer l at
 * paged byte offset slot(t) * unit).
 *
 * B200 design: the copy is HBM-bound byte movement, so it runs on the SM
 * load/store pipes, not the tensor cores.  Work is cut into tiles of about
 * 32 KiB -- (record, K/V, layer, run of tokens) -- that a persistent grid of
 * CTAs (a multiple of the 148 SMs x resident CTAs) walks with a grid
 * stride.  Inside a tile the record side is one contiguous range, so
 * thread i moves vector i of the tile: 16-byte loads/stores that are
 * coalesced on both sides (consecutive vectors of a token are consecutive in
 * the paged layer too), with 4-8 vectors in flight per thread.  Slots come from
 * per-token int64 slots or are generated from block ids
 * (slot = block_id * block_size + t % block_size, the reference's slot map
 * src/cache/cache.c:345-398).  A slot outside [0, page_buffer_size) or a null
 * layer pointer sets an error bit and the vector is skipped.
 *
 * The paged side may also be strided or head-major (kv_copy_desc
 * block_stride / head_bytes: vLLM FlashInfer's [blocks][2][heads][bs][dim]
 * on sm_100); the record side is token-major in every case.  On the bulk
 * path head-major blocks are transposed in shared memory between the bulk
 * load and the bulk store (kv_copy_bulk_hnd_kernel); on the register path
 * the head split is folded into the paged address.
 */
#include "kvcopy.h"
#include "adaptor.h"

#include <cuda_runtime.h>

#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace {

/* Two launch shapes, both moving tiles of kTileVectors 16-byte vectors:
 *   wide units (>= 1 KiB per token, e.g. 8 KV heads x 128 bf16): 256 threads
 *   x 8 vectors in flight;
 *   narrow units (a TP head shard, e.g. 1 head = 256 B): 512 threads x 4
 *   vectors, 2 CTAs per SM -- more warps hide the shorter per-token runs.
 * Chosen from a sweep on B200 (headline shapes: 94.9 % vs 90.6 %; 256-byte
 * units: 99.1 % vs 92.3 % of the measured copy peak). */
constexpr uint32_t kTileVectors = 2048;
struct WideShape { static constexpr int threads = 256, unroll = 8, min_blocks = 1; };
struct NarrowShape { static constexpr int threads = 512, unroll = 4, min_blocks = 2; };
constexpr uint32_t kNarrowUnitBytes = 1024;   /* units below this use NarrowShape */

/* unsigned 32-bit division by a run-time constant: q = (umulhi(n, m) + n) >> s
 * with s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1 (Granlund and
 * Montgomery, "Division by invariant integers using multiplication", 1994). */
struct FastDiv {
    uint32_t d, m, s;
};

FastDiv make_fastdiv(uint32_t d)
{
    FastDiv f;
    uint32_t s = 0;
    while ((1ull << s) < d)
        s++;
    f.d = d;
    f.s = s;
    f.m = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
    return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f)
{
    return (uint32_t)(((uint64_t)__umulhi(n, f.m) + n) >> f.s);
}

struct Params {
    const uint64_t *layer_k;
    const uint64_t *layer_v;
    const uint64_t *records;
    const int64_t *slots;
    const uint64_t *block_ids;
    int32_t *error;
    uint64_t page_buffer_size;
    uint64_t unit;
    uint64_t block_stride;   /* bytes between consecutive blocks of a plane */
    uint64_t head_stride;    /* head-major: block_size * head_bytes */
    uint64_t nblk;           /* ceil(page_buffer_size / block_size) */
    uint32_t head_bytes;     /* head-major: bytes of one head of one token */
    uint32_t dense;          /* slot s at s * unit (block_stride == block_size * unit, token-major) */
    uint32_t vpu;            /* vectors per token unit */
    uint32_t num_tokens;
    uint32_t block_size;
    uint32_t bpr;            /* blocks per record */
    uint32_t num_layers;     /* layers this launch copies */
    uint32_t num_kv;
    uint32_t tile_tokens;
    uint32_t num_tiles;
    uint32_t layer0;         /* first record layer this launch copies */
    uint32_t rec_layers;     /* layers a record holds */
    uint32_t max_grid;       /* CTA cap, 0 = none */
    FastDiv div_vpu, div_bs, div_tpl, div_layers, div_kv, div_hb;
};

template <int V> struct VecOf;
template <> struct VecOf<16> { using T = uint4; };
template <> struct VecOf<8> { using T = uint2; };
template <> struct VecOf<4> { using T = uint32_t; };
template <> struct VecOf<2> { using T = uint16_t; };
template <> struct VecOf<1> { using T = uint8_t; };

template <typename T> __device__ __forceinline__ T load_stream(const T *p) { return __ldcs(p); }
template <> __device__ __forceinline__ uint16_t load_stream<uint16_t>(const uint16_t *p) { return *p; }
template <> __device__ __forceinline__ uint8_t load_stream<uint8_t>(const uint8_t *p) { return *p; }

/* paged byte offset (from the layer plane's base) of byte o < unit of token
 * t of record r; false when the slot is outside the paged cache */
template <bool HND>
__device__ __forceinline__ bool paged_offset(const Params &p, uint32_t r, uint32_t t, uint32_t o, uint64_t &off)
{
    uint64_t blk;
    uint32_t j;
    if (p.slots) {
        int64_t s = p.slots[(uint64_t)r * p.num_tokens + t];
        if (s < 0 || (uint64_t)s >= p.page_buffer_size)
            return false;
        if (!HND && p.dense) {
            off = (uint64_t)s * p.unit + o;
            return true;
        }
        uint32_t s32 = (uint32_t)s;           /* page_buffer_size < 2^32 when not dense */
        uint32_t b = fdiv(s32, p.div_bs);
        blk = b;
        j = s32 - b * p.block_size;
    } else {
        uint32_t b = fdiv(t, p.div_bs);
        j = t - b * p.block_size;
        blk = p.block_ids[(uint64_t)r * p.bpr + b];
        if (blk >= p.nblk || blk * p.block_size + j >= p.page_buffer_size)
            return false;
    }
    if (!HND) {
        off = blk * p.block_stride + (uint64_t)j * p.unit + o;
        return true;
    }
    uint32_t h = fdiv(o, p.div_hb);
    off = blk * p.block_stride + (uint64_t)h * p.head_stride + (uint64_t)j * p.head_bytes + (o - h * p.head_bytes);
    return true;
}

/* one tile copied byte by byte: used only when a base address is not aligned
 * to the vector width chosen from the unit size */
template <bool TO_RECORD, bool HND>
__device__ void copy_tile_bytes(const Params &p, uint32_t r, uint8_t *layer, uint8_t *rec,
                                uint32_t t0, uint32_t n)
{
    uint64_t bytes = (uint64_t)n * p.unit;
    for (uint64_t i = threadIdx.x; i < bytes; i += blockDim.x) {
        uint32_t tok = (uint32_t)(i / p.unit);
        uint32_t o = (uint32_t)(i - (uint64_t)tok * p.unit);
        uint64_t off;
        if (!paged_offset<HND>(p, r, t0 + tok, o, off)) {
            if (p.error)
                atomicOr(p.error, KVCOPY_ERR_SLOT_RANGE);
            continue;
        }
        uint8_t *pg = layer + off;
        if (TO_RECORD)
            rec[i] = *pg;
        else
            *pg = rec[i];
    }
}

template <int VEC, bool TO_RECORD, bool HND, typename Shape>
__global__ void __launch_bounds__(Shape::threads, Shape::min_blocks) kv_copy_kernel(const Params p)
{
    using T = typename VecOf<VEC>::T;
    constexpr int kThreads = Shape::threads;
    constexpr int kUnroll = Shape::unroll;
    static_assert(kThreads * kUnroll == kTileVectors, "tile size");

    for (uint32_t w = blockIdx.x; w < p.num_tiles; w += gridDim.x) {
        /* tile w -> (record r, kv, layer l, token group g) */
        uint32_t w1 = fdiv(w, p.div_tpl);
        uint32_t g = w - w1 * p.div_tpl.d;
        uint32_t w2 = fdiv(w1, p.div_layers);
        uint32_t l = w1 - w2 * p.num_layers;
        uint32_t r = fdiv(w2, p.div_kv);
        uint32_t kv = w2 - r * p.num_kv;

        uint32_t t0 = g * p.tile_tokens;
        uint32_t n = min(p.tile_tokens, p.num_tokens - t0);
        uint8_t *layer = reinterpret_cast<uint8_t *>((kv ? p.layer_v : p.layer_k)[l]);
        uint8_t *rec = reinterpret_cast<uint8_t *>(p.records[r]) +
                       (((uint64_t)kv * p.rec_layers + p.layer0 + l) * p.num_tokens + t0) * p.unit;
        if (!layer) {
            if (threadIdx.x == 0 && p.error)
                atomicOr(p.error, KVCOPY_ERR_NULL_LAYER);
            continue;
        }
        if ((reinterpret_cast<uintptr_t>(layer) | reinterpret_cast<uintptr_t>(rec)) % VEC) {
            copy_tile_bytes<TO_RECORD, HND>(p, r, layer, rec, t0, n);
            continue;
        }

        const uint32_t items = n * p.vpu;
        T *rv = reinterpret_cast<T *>(rec);
        for (uint32_t base = 0; base < items; base += kTileVectors) {
            T v[kUnroll];
            T *pg[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                uint32_t i = base + threadIdx.x + u * kThreads;
                pg[u] = nullptr;
                if (i < items) {
                    uint32_t tok = fdiv(i, p.div_vpu);
                    uint32_t vec = i - tok * p.vpu;
                    uint64_t off;
                    if (paged_offset<HND>(p, r, t0 + tok, vec * (uint32_t)VEC, off))
                        pg[u] = reinterpret_cast<T *>(layer + off);
                    else if (p.error)
                        atomicOr(p.error, KVCOPY_ERR_SLOT_RANGE);
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                uint32_t i = base + threadIdx.x + u * kThreads;
                if (pg[u])
                    v[u] = TO_RECORD ? load_stream(pg[u]) : load_stream(rv + i);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                uint32_t i = base + threadIdx.x + u * kThreads;
                if (pg[u]) {
                    if (TO_RECORD)
                        rv[i] = v[u];
                    else
                        *pg[u] = v[u];
                }
            }
        }
    }
}

template <int VEC, bool TO_RECORD, bool HND, typename Shape>
int launch_variant(const Params &p, cudaStream_t stream)
{
    constexpr int kThreads = Shape::threads;
    static int blocks_per_sm[64];
    static int sm_count[64];
    static std::once_flag once[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return -EIO;
    std::call_once(once[dev], [&] {
        int bps = 0, sms = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, kv_copy_kernel<VEC, TO_RECORD, HND, Shape>, kThreads, 0);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        blocks_per_sm[dev] = bps > 0 ? bps : 1;
        sm_count[dev] = sms > 0 ? sms : 1;
    });
    uint64_t grid = (uint64_t)sm_count[dev] * blocks_per_sm[dev];
    if (p.max_grid && grid > p.max_grid)
        grid = p.max_grid;
    if (grid > p.num_tiles)
        grid = p.num_tiles;
    kv_copy_kernel<VEC, TO_RECORD, HND, Shape><<<(unsigned)grid, kThreads, 0, stream>>>(p);
    g_cc_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -EIO;
}

template <bool TO_RECORD, bool HND, typename Shape>
int launch_vec(const Params &p, int vec, cudaStream_t s)
{
    switch (vec) {
    case 16: return launch_variant<16, TO_RECORD, HND, Shape>(p, s);
    case 8: return launch_variant<8, TO_RECORD, HND, Shape>(p, s);
    case 4: return launch_variant<4, TO_RECORD, HND, Shape>(p, s);
    case 2: return launch_variant<2, TO_RECORD, HND, Shape>(p, s);
    default: return launch_variant<1, TO_RECORD, HND, Shape>(p, s);
    }
}

template <bool TO_RECORD, bool HND>
int launch_shape(const Params &p, int vec, cudaStream_t s)
{
    if (p.unit < kNarrowUnitBytes)
        return launch_vec<TO_RECORD, HND, NarrowShape>(p, vec, s);
    return launch_vec<TO_RECORD, HND, WideShape>(p, vec, s);
}

template <bool TO_RECORD>
int launch_dir(const Params &p, int vec, cudaStream_t s)
{
    return p.head_bytes ? launch_shape<TO_RECORD, true>(p, vec, s) : launch_shape<TO_RECORD, false>(p, vec, s);
}

/* ------------------------------------------------------------------------
 * TMA bulk-copy path (KVCOPY_FLAG_BULK, block-id mode).
 *
 * A tile is up to 32 KiB of one (record, K/V, layer): whole paged blocks,
 * each one contiguous run of block_size * unit bytes on the paged side and
 * consecutive on the record side.  One thread per CTA drives a ring of
 * kBulkStages shared-memory stages: cp.async.bulk global->shared for every
 * run of a tile (completion counted in bytes on the stage's mbarrier), then
 * one cp.async.bulk shared->global of the stage (scatter: the reverse), with
 * up to kBulkStages-1 tiles loading while the previous one stores.  The data
 * never passes through registers.  Every mbarrier wait is bounded: after
 * kBulkSpinLimit polls the kernel sets KVCOPY_ERR_TIMEOUT, waits (bounded) for
 * its other loads in flight and for its stores, and returns.
 * ---------------------------------------------------------------------- */
#ifndef KVCOPY_BULK_TILE_BYTES
#define KVCOPY_BULK_TILE_BYTES 32768
#endif
#ifndef KVCOPY_BULK_STAGES
#define KVCOPY_BULK_STAGES 4
#endif
constexpr uint32_t kBulkTileBytes = KVCOPY_BULK_TILE_BYTES;
constexpr uint32_t kBulkMinRunBytes = 8192;    /* shorter runs: the register path was faster
                                                * (256-byte units: 6471 vs 6223 GB/s) */
constexpr int kBulkStages = KVCOPY_BULK_STAGES;
static_assert(kBulkStages >= 2 && (uint64_t)kBulkStages * kBulkTileBytes <= 227u * 1024u - 256u,
              "bulk ring must fit the 227 KiB of shared memory a CTA can have");
static_assert(kBulkTileBytes % 16 == 0, "bulk copies move multiples of 16 bytes");
constexpr uint32_t kBulkSpinLimit = 1u << 24;   /* polls of ~128 ns back-off: ~2 s */
constexpr uint32_t kStallSpinLimit = 1u << 14;  /* fault-detection test: a few ms */

struct BulkParams {
    const uint64_t *layer_k;
    const uint64_t *layer_v;
    const uint64_t *records;
    const uint64_t *block_ids;
    int32_t *error;
    uint64_t num_blocks;        /* paged blocks per layer */
    uint64_t run_bytes;         /* block_size * unit */
    uint64_t block_stride;      /* bytes between consecutive blocks of a plane */
    uint64_t layer_rec_bytes;   /* num_tokens * unit: one layer of one record part */
    uint32_t bpr;               /* blocks per record */
    uint32_t gpt;               /* blocks per tile */
    uint32_t num_layers;        /* layers this launch copies */
    uint32_t num_kv;
    uint32_t num_tiles;
    uint32_t layer0;            /* first record layer this launch copies */
    uint32_t rec_layers;        /* layers a record holds */
    uint32_t max_grid;          /* CTA cap, 0 = none */
    uint32_t spin_limit;        /* polls of one bounded mbarrier wait */
    uint32_t stall;             /* KVCOPY_FLAG_TEST_STALL: CTA 0's first tile never completes */
    FastDiv div_tpl, div_layers, div_kv;
    /* head-major blocks, in 16-byte vectors: hv per head piece of a token,
     * tv = block_size * hv per head, vpb = heads * tv per block */
    uint32_t heads, hv, tv, vpb, bs;
    FastDiv div_hv, div_tv, div_vpb, div_bs;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

/* poll until the phase of `parity` completes, at most `budget` polls; the
 * polls used are taken off `budget`, so a caller can spread one budget over
 * several waits */
__device__ bool mbar_wait_budget(uint64_t *bar, uint32_t parity, uint32_t &budget)
{
    for (uint32_t i = 0;; i++) {
        if (mbar_try_wait(bar, parity))
            return true;
        if (budget == 0)
            return false;
        budget--;
        if (i > 32)
            __nanosleep(128);
    }
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t limit)
{
    uint32_t budget = limit;
    return mbar_wait_budget(bar, parity, budget);
}

/* After a wait on tile k ran out: wait, with one shared budget, for every
 * load still in flight -- tiles k+1 .. issued-1 first, then tile k itself --
 * so the CTA does not leave while a bulk copy may still write its shared
 * memory.  A load that has not landed within the budget is given up on
 * (the kernel must return: a GPU that never answers is worse than a CTA
 * that exits with a copy outstanding). */
__device__ void drain_after_timeout(uint64_t *bars, int stages, uint32_t k, uint32_t issued, uint32_t limit)
{
    uint32_t budget = limit;
    for (uint32_t j = k + 1; j < issued; j++)
        mbar_wait_budget(&bars[j % stages], (j / stages) & 1, budget);
    mbar_wait_budget(&bars[k % stages], (k / stages) & 1, budget);
}

__device__ __forceinline__ void bulk_g2s(void *sdst, const void *gsrc, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(sdst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void bulk_s2g(void *gdst, const void *ssrc, uint32_t bytes)
{
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(gdst), "r"(smem_u32(ssrc)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

struct BulkTile {
    uint8_t *layer;
    uint8_t *rec;
    const uint64_t *bids;
    uint32_t nb;
};

__device__ __forceinline__ BulkTile bulk_decode(const BulkParams &p, uint32_t w)
{
    const uint32_t tpl = p.div_tpl.d;
    uint32_t w1 = fdiv(w, p.div_tpl);
    uint32_t g = w - w1 * tpl;
    uint32_t w2 = fdiv(w1, p.div_layers);
    uint32_t l = w1 - w2 * p.num_layers;
    uint32_t r = fdiv(w2, p.div_kv);
    uint32_t kv = w2 - r * p.num_kv;
    BulkTile t;
    uint32_t b0 = g * p.gpt;
    t.nb = min(p.gpt, p.bpr - b0);
    t.layer = reinterpret_cast<uint8_t *>((kv ? p.layer_v : p.layer_k)[l]);
    t.rec = reinterpret_cast<uint8_t *>(p.records[r]) + ((uint64_t)kv * p.rec_layers + p.layer0 + l) * p.layer_rec_bytes +
            (uint64_t)b0 * p.run_bytes;
    t.bids = p.block_ids + (uint64_t)r * p.bpr + b0;
    return t;
}

/* start the loads of tile t into `stage`, completion counted in bytes on
 * `bar`; a tile whose base is null or misaligned loads nothing and flags it */
template <bool TO_RECORD>
__device__ void bulk_issue_load(const BulkParams &p, const BulkTile &t, uint8_t *stage, uint64_t *bar)
{
    const uint32_t run = (uint32_t)p.run_bytes;
    bool bad_base = !t.layer || ((reinterpret_cast<uintptr_t>(t.layer) | reinterpret_cast<uintptr_t>(t.rec)) & 15);
    if (bad_base) {
        if (p.error)
            atomicOr(p.error, t.layer ? KVCOPY_ERR_ALIGN : KVCOPY_ERR_NULL_LAYER);
        mbar_expect_tx(bar, 0);
        return;
    }
    if (TO_RECORD) {
        uint32_t bytes = 0;
        for (uint32_t j = 0; j < t.nb; j++)
            if (t.bids[j] < p.num_blocks)
                bytes += run;
        mbar_expect_tx(bar, bytes);
        for (uint32_t j = 0; j < t.nb; j++) {
            uint64_t bid = t.bids[j];
            if (bid < p.num_blocks)
                bulk_g2s(stage + j * run, t.layer + bid * p.block_stride, run, bar);
            else if (p.error)
                atomicOr(p.error, KVCOPY_ERR_SLOT_RANGE);
        }
    } else {
        mbar_expect_tx(bar, t.nb * run);
        bulk_g2s(stage, t.rec, t.nb * run, bar);
    }
}

/* store tile t from shared memory at `src` (one bulk group) */
template <bool TO_RECORD>
__device__ void bulk_issue_store(const BulkParams &p, const BulkTile &t, const uint8_t *src)
{
    const uint32_t run = (uint32_t)p.run_bytes;
    bool bad_base = !t.layer || ((reinterpret_cast<uintptr_t>(t.layer) | reinterpret_cast<uintptr_t>(t.rec)) & 15);
    if (!bad_base) {
        if (TO_RECORD) {
            bulk_s2g(t.rec, src, t.nb * run);
        } else {
            for (uint32_t j = 0; j < t.nb; j++) {
                uint64_t bid = t.bids[j];
                if (bid < p.num_blocks)
                    bulk_s2g(t.layer + bid * p.block_stride, src + j * run, run);
                else if (p.error)
                    atomicOr(p.error, KVCOPY_ERR_SLOT_RANGE);
            }
        }
    }
    bulk_commit();
}

template <bool TO_RECORD>
__global__ void __launch_bounds__(32, 1) kv_copy_bulk_kernel(const BulkParams p)
{
    extern __shared__ __align__(128) uint8_t bulk_smem[];
    __shared__ __align__(8) uint64_t bars[kBulkStages];
    if (threadIdx.x != 0)
        return;
    for (int s = 0; s < kBulkStages; s++)
        mbar_init(&bars[s], 1);
    mbar_fence_init();

    const uint32_t n_my = p.num_tiles > blockIdx.x ? (p.num_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

    auto issue_load = [&](uint32_t k, int s) {
        if (p.stall && k == 0 && blockIdx.x == 0) {
            /* fault-detection test: arm the stage for bytes that are never
             * issued, so no copy is in flight on it and its wait runs out */
            mbar_expect_tx(&bars[s], 16);
            return;
        }
        bulk_issue_load<TO_RECORD>(p, bulk_decode(p, blockIdx.x + k * gridDim.x),
                                   bulk_smem + (uint32_t)s * kBulkTileBytes, &bars[s]);
    };
    auto issue_store = [&](uint32_t k, int s) {
        bulk_issue_store<TO_RECORD>(p, bulk_decode(p, blockIdx.x + k * gridDim.x),
                                    bulk_smem + (uint32_t)s * kBulkTileBytes);
    };

    uint32_t issued = 0;
    for (; issued < n_my && issued < (uint32_t)kBulkStages; issued++)
        issue_load(issued, (int)issued);
    for (uint32_t k = 0; k < n_my; k++) {
        const int s = (int)(k % kBulkStages);
        if (!mbar_wait_bounded(&bars[s], (k / kBulkStages) & 1, p.spin_limit)) {
            if (p.error)
                atomicOr(p.error, KVCOPY_ERR_TIMEOUT);
            drain_after_timeout(bars, kBulkStages, k, issued, p.spin_limit);
            break;
        }
        issue_store(k, s);
        /* refill the stage of tile k-1 once its store has read the stage */
        if (k >= 1 && issued < n_my) {
            bulk_wait_read1();
            issue_load(issued, (int)((k - 1) % kBulkStages));
            issued++;
        }
    }
    bulk_wait_all();
}

int launch_bulk(const BulkParams &bp, bool to_record, cudaStream_t stream)
{
    static int sm_count[64];
    static std::once_flag once[64];
    static cudaError_t attr_err[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return -EIO;
    const int smem = kBulkStages * (int)kBulkTileBytes;
    std::call_once(once[dev], [&] {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        sm_count[dev] = sms > 0 ? sms : 1;
        attr_err[dev] = cudaFuncSetAttribute(kv_copy_bulk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (attr_err[dev] == cudaSuccess)
            attr_err[dev] = cudaFuncSetAttribute(kv_copy_bulk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (attr_err[dev] != cudaSuccess)
        return -EIO;
    uint32_t grid = (uint32_t)sm_count[dev];
    if (bp.max_grid && grid > bp.max_grid)
        grid = bp.max_grid;
    if (grid > bp.num_tiles)
        grid = bp.num_tiles;
    if (to_record)
        kv_copy_bulk_kernel<true><<<grid, 32, smem, stream>>>(bp);
    else
        kv_copy_bulk_kernel<false><<<grid, 32, smem, stream>>>(bp);
    g_cc_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -EIO;
}

/* ------------------------------------------------------------------------
 * TMA bulk path for head-major blocks (vLLM FlashInfer HND on sm_100).
 *
 * A paged block is one contiguous run of [heads][block_size][head_bytes];
 * the record wants the same bytes token-major, [block_size][heads]
 * [head_bytes].  Tiles, loads and stores are those of the bulk path; in
 * between, the CTA's 16 warps transpose each block of the stage into one
 * of two shared buffers (16-byte vectors: head pieces of a token stay whole),
 * and the bulk store reads that buffer.  When a token's vectors divide the
 * CTA, each thread keeps one (head, vector) position for the whole kernel
 * and walks tokens, so a vector costs one division and a few adds.  Thread 0 drives the copies and the
 * bounded mbarrier waits; two CTA barriers per tile hand the stage and the
 * buffer between the copies and the warps:
 *   - before a buffer is rewritten, the store that last read it has read it
 *     (cp.async.bulk.wait_group.read with one group left: the previous tile's)
 *   - after the transpose, fence.proxy.async makes the warps' shared-memory
 *     writes visible to the bulk store and orders their stage reads before
 *     the refill of that stage.
 * ---------------------------------------------------------------------- */
constexpr int kHndThreads = 512;
/* 5 load stages + 2 transpose buffers = 224 KiB: the transpose between a
 * tile's load and its store lengthens a tile's life, and one more stage in
 * flight bought 0.5 % (gather) and 1.3 % (scatter) of the copy peak on B200
 * (headline shapes, same box, two runs each) over 4 */
#ifndef KVCOPY_HND_STAGES
#define KVCOPY_HND_STAGES 5
#endif
constexpr int kHndStages = KVCOPY_HND_STAGES;
static_assert((uint64_t)(kHndStages + 2) * kBulkTileBytes <= 227u * 1024u - 256u,
              "head-major bulk stages and transpose buffers must fit in shared memory");

__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

/* vector w of a block in head-major order -> its index in token-major order */
__device__ __forceinline__ uint32_t hnd_to_token_major(const BulkParams &p, uint32_t w)
{
    uint32_t h = fdiv(w, p.div_tv);
    uint32_t r = w - h * p.tv;
    uint32_t t = fdiv(r, p.div_hv);
    uint32_t x = r - t * p.hv;
    return (t * p.heads + h) * p.hv + x;
}

template <bool TO_RECORD>
__global__ void __launch_bounds__(kHndThreads, 1) kv_copy_bulk_hnd_kernel(const BulkParams p)
{
    extern __shared__ __align__(128) uint8_t bulk_smem[];
    __shared__ __align__(8) uint64_t bars[kHndStages];
    __shared__ int go;
    uint8_t *const tbuf = bulk_smem + (uint32_t)kHndStages * kBulkTileBytes;
    const bool leader = threadIdx.x == 0;
    const uint32_t n_my = p.num_tiles > blockIdx.x ? (p.num_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    /* this thread's fixed position inside a token: vector pos of P, head h */
    const uint32_t P = p.heads * p.hv;
    const bool fixed_pos = kHndThreads % P == 0;
    const uint32_t pos = threadIdx.x % P, row0 = threadIdx.x / P, drow = kHndThreads / P;
    const uint32_t h0 = fdiv(pos, p.div_hv);
    const uint32_t hm0 = h0 * p.tv + (pos - h0 * p.hv);

    uint32_t issued = 0;
    if (leader) {
        for (int s = 0; s < kHndStages; s++)
            mbar_init(&bars[s], 1);
        mbar_fence_init();
        for (; issued < n_my && issued < (uint32_t)kHndStages; issued++) {
            if (p.stall && issued == 0 && blockIdx.x == 0)
                mbar_expect_tx(&bars[0], 16);   /* fault-detection test: never completes */
            else
                bulk_issue_load<TO_RECORD>(p, bulk_decode(p, blockIdx.x + issued * gridDim.x),
                                           bulk_smem + issued * kBulkTileBytes, &bars[issued]);
        }
    }
    for (uint32_t k = 0; k < n_my; k++) {
        const uint32_t s = k % kHndStages;
        uint8_t *const stage = bulk_smem + s * kBulkTileBytes;
        uint8_t *const buf = tbuf + (k & 1) * kBulkTileBytes;
        if (leader) {
            bool ok = mbar_wait_bounded(&bars[s], (k / kHndStages) & 1, p.spin_limit);
            if (!ok) {
                if (p.error)
                    atomicOr(p.error, KVCOPY_ERR_TIMEOUT);
                drain_after_timeout(bars, kHndStages, k, issued, p.spin_limit);
            }
            if (k >= 2)
                bulk_wait_read1();      /* tile k-2's store has read buf */
            go = ok;
        }
        __syncthreads();
        if (!go)
            break;
        const BulkTile t = bulk_decode(p, blockIdx.x + k * gridDim.x);
        const uint4 *src = reinterpret_cast<const uint4 *>(stage);
        uint4 *dst = reinterpret_cast<uint4 *>(buf);
        if (fixed_pos) {
            /* token-major vector row * P + pos <-> head-major jb * vpb + hm0 + t * hv */
            const uint32_t rows = t.nb * p.bs;
#pragma unroll 4
            for (uint32_t row = row0; row < rows; row += drow) {
                uint32_t jb = fdiv(row, p.div_bs);
                uint32_t hm = jb * p.vpb + hm0 + (row - jb * p.bs) * p.hv;
                uint32_t tm = row * P + pos;
                if (TO_RECORD)
                    dst[tm] = src[hm];  /* head-major block -> token-major record */
                else
                    dst[hm] = src[tm];  /* token-major record -> head-major block */
            }
        } else {
            const uint32_t nvec = t.nb * p.vpb;
            for (uint32_t v = threadIdx.x; v < nvec; v += kHndThreads) {
                uint32_t jb = fdiv(v, p.div_vpb);
                uint32_t w = v - jb * p.vpb;
                uint32_t tm = jb * p.vpb + hnd_to_token_major(p, w);
                if (TO_RECORD)
                    dst[tm] = src[v];
                else
                    dst[v] = src[tm];
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (leader) {
            bulk_issue_store<TO_RECORD>(p, t, buf);
            if (issued < n_my) {        /* the stage of tile k is free: refill it */
                bulk_issue_load<TO_RECORD>(p, bulk_decode(p, blockIdx.x + issued * gridDim.x), stage, &bars[s]);
                issued++;
            }
        }
    }
    if (leader)
        bulk_wait_all();
}

int launch_bulk_hnd(const BulkParams &bp, bool to_record, cudaStream_t stream)
{
    static int sm_count[64];
    static std::once_flag once[64];
    static cudaError_t attr_err[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return -EIO;
    const int smem = (kHndStages + 2) * (int)kBulkTileBytes;
    std::call_once(once[dev], [&] {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        sm_count[dev] = sms > 0 ? sms : 1;
        attr_err[dev] = cudaFuncSetAttribute(kv_copy_bulk_hnd_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (attr_err[dev] == cudaSuccess)
            attr_err[dev] = cudaFuncSetAttribute(kv_copy_bulk_hnd_kernel<false>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (attr_err[dev] != cudaSuccess)
        return -EIO;
    uint32_t grid = (uint32_t)sm_count[dev];
    if (bp.max_grid && grid > bp.max_grid)
        grid = bp.max_grid;
    if (grid > bp.num_tiles)
        grid = bp.num_tiles;
    if (to_record)
        kv_copy_bulk_hnd_kernel<true><<<grid, kHndThreads, smem, stream>>>(bp);
    else
        kv_copy_bulk_hnd_kernel<false><<<grid, kHndThreads, smem, stream>>>(bp);
    g_cc_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -EIO;
}

/* CROSSCACHE_KVCOPY=lsu forces the register path even when the bulk path is allowed */
bool bulk_allowed_by_env()
{
    static int v = -1;
    if (v < 0) {
        const char *s = getenv("CROSSCACHE_KVCOPY");
        v = (s && !strcmp(s, "lsu")) ? 0 : 1;
    }
    return v == 1;
}

/* cudaFuncGetAttributes of every instantiation of kernel K: with lazy module
 * loading (the default since CUDA 12.2) this is what makes the driver load
 * the kernel's code onto the current device */
template <int VEC, bool TO_RECORD, bool HND>
bool preload_register_kernels()
{
    cudaFuncAttributes a;
    return cudaFuncGetAttributes(&a, kv_copy_kernel<VEC, TO_RECORD, HND, WideShape>) == cudaSuccess &&
           cudaFuncGetAttributes(&a, kv_copy_kernel<VEC, TO_RECORD, HND, NarrowShape>) == cudaSuccess;
}

template <bool TO_RECORD, bool HND>
bool preload_all_vecs()
{
    return preload_register_kernels<16, TO_RECORD, HND>() && preload_register_kernels<8, TO_RECORD, HND>() &&
           preload_register_kernels<4, TO_RECORD, HND>() && preload_register_kernels<2, TO_RECORD, HND>() &&
           preload_register_kernels<1, TO_RECORD, HND>();
}

/* which kernel a descriptor runs: KVCOPY_PATH_*, or -EINVAL for a
 * malformed descriptor (the checks kv_copy_launch makes before launching) */
int select_path(const struct kv_copy_desc *d)
{
    if (!d || !d->layer_k || !d->records || !d->unit_bytes || !d->num_tokens ||
        !d->num_layers || !d->block_size)
        return -EINVAL;
    if (d->flags & ~(uint32_t)(KVCOPY_FLAG_BULK | KVCOPY_FLAG_TEST_STALL))
        return -EINVAL;
    if (!d->slots && (!d->block_ids || d->num_tokens % d->block_size))
        return -EINVAL;
    const uint32_t rec_layers = d->record_layers ? d->record_layers : d->num_layers;
    if ((uint64_t)d->layer_begin + d->num_layers > rec_layers)
        return -EINVAL;
    const uint64_t run_bytes = (uint64_t)d->block_size * d->unit_bytes;
    const uint64_t block_stride = d->block_stride ? d->block_stride : run_bytes;
    const bool dense = block_stride == run_bytes && !d->head_bytes;
    if (block_stride < run_bytes || (d->head_bytes && d->unit_bytes % d->head_bytes))
        return -EINVAL;
    if (!dense && d->slots && d->page_buffer_size >= (1ull << 32))
        return -EINVAL;
    if ((d->flags & KVCOPY_FLAG_BULK) && !d->slots && d->head_bytes % 16 == 0 && d->unit_bytes % 16 == 0 &&
        block_stride % 16 == 0 && run_bytes >= kBulkMinRunBytes && run_bytes <= kBulkTileBytes &&
        d->page_buffer_size % d->block_size == 0 && bulk_allowed_by_env())
        return d->head_bytes ? KVCOPY_PATH_BULK_HND : KVCOPY_PATH_BULK;
    return KVCOPY_PATH_REGISTER;
}

}  // namespace

extern "C" uint64_t kv_copy_payload_bytes(const struct kv_copy_desc *d)
{
    if (!d)
        return 0;
    return (uint64_t)(d->layer_v ? 2 : 1) * d->num_layers * d->num_tokens *
           (uint64_t)d->unit_bytes * d->num_records;
}

extern "C" int kv_copy_path(const struct kv_copy_desc *d)
{
    return select_path(d);
}

int kv_copy_preload(void)
{
    if (!preload_all_vecs<true, false>() || !preload_all_vecs<false, false>() ||
        !preload_all_vecs<true, true>() || !preload_all_vecs<false, true>())
        return -EIO;
    cudaFuncAttributes a;
    const int smem = kBulkStages * (int)kBulkTileBytes;
    const int smem_hnd = (kHndStages + 2) * (int)kBulkTileBytes;
    if (cudaFuncGetAttributes(&a, kv_copy_bulk_kernel<true>) != cudaSuccess ||
        cudaFuncGetAttributes(&a, kv_copy_bulk_kernel<false>) != cudaSuccess ||
        cudaFuncGetAttributes(&a, kv_copy_bulk_hnd_kernel<true>) != cudaSuccess ||
        cudaFuncGetAttributes(&a, kv_copy_bulk_hnd_kernel<false>) != cudaSuccess ||
        cudaFuncSetAttribute(kv_copy_bulk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ||
        cudaFuncSetAttribute(kv_copy_bulk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ||
        cudaFuncSetAttribute(kv_copy_bulk_hnd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_hnd) ||
        cudaFuncSetAttribute(kv_copy_bulk_hnd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_hnd))
        return -EIO;
    return 0;
}

extern "C" int kv_copy_launch(const struct kv_copy_desc *d, void *stream)
{
    const int path = select_path(d);
    if (path < 0)
        return path;
    if (!d->num_records)
        return 0;
    const uint32_t rec_layers = d->record_layers ? d->record_layers : d->num_layers;
    /* the layer pointer arrays are indexed from the first layer copied */
    const uint64_t *lk = d->layer_k + d->layer_begin;
    const uint64_t *lv = d->layer_v ? d->layer_v + d->layer_begin : nullptr;

    const uint64_t run_bytes = (uint64_t)d->block_size * d->unit_bytes;
    const uint64_t block_stride = d->block_stride ? d->block_stride : run_bytes;
    const bool dense = block_stride == run_bytes && !d->head_bytes;
    if (path != KVCOPY_PATH_REGISTER) {
        BulkParams bp{};
        const bool stall = (d->flags & KVCOPY_FLAG_TEST_STALL) != 0;
        bp.spin_limit = stall ? kStallSpinLimit : kBulkSpinLimit;
        bp.stall = stall ? 1 : 0;
        bp.layer_k = lk;
        bp.layer_v = lv;
        bp.layer0 = d->layer_begin;
        bp.rec_layers = rec_layers;
        bp.max_grid = d->max_ctas;
        bp.records = d->records;
        bp.block_ids = d->block_ids;
        bp.error = d->error;
        bp.num_blocks = d->page_buffer_size / d->block_size;
        bp.run_bytes = run_bytes;
        bp.block_stride = block_stride;
        bp.layer_rec_bytes = (uint64_t)d->num_tokens * d->unit_bytes;
        bp.bpr = d->num_tokens / d->block_size;
        bp.gpt = (uint32_t)(kBulkTileBytes / run_bytes);
        if (bp.gpt > bp.bpr)
            bp.gpt = bp.bpr;
        bp.num_layers = d->num_layers;
        bp.num_kv = d->layer_v ? 2 : 1;
        const uint32_t tpl = (bp.bpr + bp.gpt - 1) / bp.gpt;
        const uint64_t tiles = (uint64_t)d->num_records * bp.num_kv * bp.num_layers * tpl;
        if (tiles >= (1ull << 31))
            return -EINVAL;
        bp.num_tiles = (uint32_t)tiles;
        bp.div_tpl = make_fastdiv(tpl);
        bp.div_layers = make_fastdiv(bp.num_layers);
        bp.div_kv = make_fastdiv(bp.num_kv);
        if (d->head_bytes) {
            bp.hv = d->head_bytes / 16;
            bp.heads = d->unit_bytes / d->head_bytes;
            bp.tv = d->block_size * bp.hv;
            bp.vpb = (uint32_t)(run_bytes / 16);
            bp.div_hv = make_fastdiv(bp.hv);
            bp.div_tv = make_fastdiv(bp.tv);
            bp.div_vpb = make_fastdiv(bp.vpb);
            bp.bs = d->block_size;
            bp.div_bs = make_fastdiv(d->block_size);
            return launch_bulk_hnd(bp, d->direction != 0, static_cast<cudaStream_t>(stream));
        }
        return launch_bulk(bp, d->direction != 0, static_cast<cudaStream_t>(stream));
    }

    Params p{};
    p.layer_k = lk;
    p.layer_v = lv;
    p.layer0 = d->layer_begin;
    p.rec_layers = rec_layers;
    p.max_grid = d->max_ctas;
    p.records = d->records;
    p.slots = d->slots;
    p.block_ids = d->block_ids;
    p.error = d->error;
    p.page_buffer_size = d->page_buffer_size;
    p.unit = d->unit_bytes;
    p.block_stride = block_stride;
    p.head_bytes = d->head_bytes;
    p.head_stride = (uint64_t)d->block_size * d->head_bytes;
    p.nblk = (d->page_buffer_size + d->block_size - 1) / d->block_size;
    p.dense = dense ? 1 : 0;
    p.num_tokens = d->num_tokens;
    p.block_size = d->block_size;
    p.bpr = d->num_tokens / d->block_size;
    p.num_layers = d->num_layers;
    p.num_kv = d->layer_v ? 2 : 1;

    /* a vector never straddles a token, a head or a block boundary */
    int vec = 16;
    while (d->unit_bytes % vec || block_stride % vec || (d->head_bytes && d->head_bytes % vec))
        vec >>= 1;
    p.vpu = d->unit_bytes / vec;
    /* tile = about kTileVectors vectors, whole tokens, at most one record layer */
    uint32_t tt = kTileVectors / p.vpu;
    if (tt < 1)
        tt = 1;
    if (tt > p.num_tokens)
        tt = p.num_tokens;
    p.tile_tokens = tt;
    uint32_t tpl = (p.num_tokens + tt - 1) / tt;
    uint64_t tiles = (uint64_t)d->num_records * p.num_kv * p.num_layers * tpl;
    /* 32-bit index arithmetic inside the kernel */
    if (tiles >= (1ull << 31) || (uint64_t)tt * p.vpu >= (1ull << 31) ||
        (uint64_t)d->num_records * p.num_tokens >= (1ull << 32))
        return -EINVAL;
    p.num_tiles = (uint32_t)tiles;
    p.div_vpu = make_fastdiv(p.vpu);
    p.div_bs = make_fastdiv(p.block_size);
    p.div_tpl = make_fastdiv(tpl);
    p.div_layers = make_fastdiv(p.num_layers);
    p.div_kv = make_fastdiv(p.num_kv);
    p.div_hb = make_fastdiv(d->head_bytes ? d->head_bytes : 1);

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return d->direction ? launch_dir<true>(p, vec, s) : launch_dir<false>(p, vec, s);
}
