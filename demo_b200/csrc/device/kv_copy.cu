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
 */
#include "kvcopy.h"
#include "adaptor.h"

#include <cuda_runtime.h>

#include <cerrno>
#include <cstdint>
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
    uint32_t vpu;            /* vectors per token unit */
    uint32_t num_tokens;
    uint32_t block_size;
    uint32_t bpr;            /* blocks per record */
    uint32_t num_layers;
    uint32_t num_kv;
    uint32_t tile_tokens;
    uint32_t num_tiles;
    FastDiv div_vpu, div_bs, div_tpl, div_layers, div_kv;
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

__device__ __forceinline__ int64_t slot_of(const Params &p, uint32_t r, uint32_t t)
{
    if (p.slots)
        return p.slots[(uint64_t)r * p.num_tokens + t];
    uint32_t b = fdiv(t, p.div_bs);
    uint32_t j = t - b * p.block_size;
    uint64_t bid = p.block_ids[(uint64_t)r * p.bpr + b];
    return (int64_t)(bid * p.block_size + j);
}

/* one tile copied byte by byte: used only when a base address is not aligned
 * to the vector width chosen from the unit size */
template <bool TO_RECORD>
__device__ void copy_tile_bytes(const Params &p, uint32_t r, uint8_t *layer, uint8_t *rec,
                                uint32_t t0, uint32_t n)
{
    uint64_t bytes = (uint64_t)n * p.unit;
    for (uint64_t i = threadIdx.x; i < bytes; i += blockDim.x) {
        uint32_t tok = (uint32_t)(i / p.unit);
        uint64_t off = i - (uint64_t)tok * p.unit;
        int64_t slot = slot_of(p, r, t0 + tok);
        if (slot < 0 || (uint64_t)slot >= p.page_buffer_size) {
            if (p.error)
                atomicOr(p.error, KVCOPY_ERR_SLOT_RANGE);
            continue;
        }
        uint8_t *pg = layer + (uint64_t)slot * p.unit + off;
        if (TO_RECORD)
            rec[i] = *pg;
        else
            *pg = rec[i];
    }
}

template <int VEC, bool TO_RECORD, typename Shape>
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
                       (((uint64_t)kv * p.num_layers + l) * p.num_tokens + t0) * p.unit;
        if (!layer) {
            if (threadIdx.x == 0 && p.error)
                atomicOr(p.error, KVCOPY_ERR_NULL_LAYER);
            continue;
        }
        if ((reinterpret_cast<uintptr_t>(layer) | reinterpret_cast<uintptr_t>(rec)) % VEC) {
            copy_tile_bytes<TO_RECORD>(p, r, layer, rec, t0, n);
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
                    int64_t slot = slot_of(p, r, t0 + tok);
                    if (slot >= 0 && (uint64_t)slot < p.page_buffer_size)
                        pg[u] = reinterpret_cast<T *>(layer + (uint64_t)slot * p.unit) + vec;
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

template <int VEC, bool TO_RECORD, typename Shape>
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
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, kv_copy_kernel<VEC, TO_RECORD, Shape>, kThreads, 0);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        blocks_per_sm[dev] = bps > 0 ? bps : 1;
        sm_count[dev] = sms > 0 ? sms : 1;
    });
    uint64_t grid = (uint64_t)sm_count[dev] * blocks_per_sm[dev];
    if (grid > p.num_tiles)
        grid = p.num_tiles;
    kv_copy_kernel<VEC, TO_RECORD, Shape><<<(unsigned)grid, kThreads, 0, stream>>>(p);
    g_cc_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -EIO;
}

template <bool TO_RECORD, typename Shape>
int launch_vec(const Params &p, int vec, cudaStream_t s)
{
    switch (vec) {
    case 16: return launch_variant<16, TO_RECORD, Shape>(p, s);
    case 8: return launch_variant<8, TO_RECORD, Shape>(p, s);
    case 4: return launch_variant<4, TO_RECORD, Shape>(p, s);
    case 2: return launch_variant<2, TO_RECORD, Shape>(p, s);
    default: return launch_variant<1, TO_RECORD, Shape>(p, s);
    }
}

template <bool TO_RECORD>
int launch_dir(const Params &p, int vec, cudaStream_t s)
{
    if (p.unit < kNarrowUnitBytes)
        return launch_vec<TO_RECORD, NarrowShape>(p, vec, s);
    return launch_vec<TO_RECORD, WideShape>(p, vec, s);
}

}  // namespace

extern "C" uint64_t kv_copy_payload_bytes(const struct kv_copy_desc *d)
{
    if (!d)
        return 0;
    return (uint64_t)(d->layer_v ? 2 : 1) * d->num_layers * d->num_tokens *
           (uint64_t)d->unit_bytes * d->num_records;
}

extern "C" int kv_copy_launch(const struct kv_copy_desc *d, void *stream)
{
    if (!d || !d->layer_k || !d->records || !d->unit_bytes || !d->num_tokens ||
        !d->num_layers || !d->block_size)
        return -EINVAL;
    if (!d->num_records)
        return 0;
    if (!d->slots && (!d->block_ids || d->num_tokens % d->block_size))
        return -EINVAL;

    Params p{};
    p.layer_k = d->layer_k;
    p.layer_v = d->layer_v;
    p.records = d->records;
    p.slots = d->slots;
    p.block_ids = d->block_ids;
    p.error = d->error;
    p.page_buffer_size = d->page_buffer_size;
    p.unit = d->unit_bytes;
    p.num_tokens = d->num_tokens;
    p.block_size = d->block_size;
    p.bpr = d->num_tokens / d->block_size;
    p.num_layers = d->num_layers;
    p.num_kv = d->layer_v ? 2 : 1;

    int vec = 16;
    while (d->unit_bytes % vec)
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

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return d->direction ? launch_dir<true>(p, vec, s) : launch_dir<false>(p, vec, s);
}
