/*
 * Batched chained prefix block hash for sm_100a, bit-identical to vLLM's
 * default prefix-cache hash (the keys CrossCache stores under, see
 * include/kvhash.h):
 *
 *   h_i = SHA-256(pickle.dumps((h_{i-1}, tuple(tokens of block i), None),
 *                              protocol=5))
 *
 * vllm/v1/core/kv_cache_utils.py:541-570 (hash_block_tokens) and
 * vllm/utils/hashing.py:26-41 (sha256).  The pickle byte stream of one block
 * is produced directly on the device:
 *
 *   80 05                     PROTO 5
 *   95 <u64 LE frame length>  FRAME   (length = total - 11)
 *   43 20 <32 bytes parent>   SHORT_BINBYTES
 *   94                        MEMOIZE
 *   28                        MARK                      (block_size > 3)
 *   per token: 4b b | 4d lo hi | 4a b0 b1 b2 b3         BININT1/BININT2/BININT
 *   74 | 85 | 86 | 87         TUPLE, or TUPLE1/2/3 for block_size 1..3
 *   94 4e 87 94 2e            MEMOIZE NONE TUPLE3 MEMOIZE STOP
 *
 * With vLLM's per-block extra keys (LoRA name, multimodal hashes, cache
 * salt: kv_cache_utils.py generate_block_hash_extra_keys) the tuple's third
 * item is their tuple instead of None.  Protocol 5 memoizes without indices
 * (MEMOIZE) and canonical CBOR has no back-references, so the serialised
 * extra keys are one position-independent byte segment that takes the place
 * of the 0x4e (pickle) or 0xf6 (CBOR) byte; the caller supplies the segment
 * per block (include/kvhash.h kv_block_hash_launch_ext).
 *
 * (CPython _pickle.c save_bytes/save_tuple/save_long; a 0..255 token is
 * BININT1, 256..65535 BININT2, anything else BININT 4-byte two's complement.)
 *
 * SHA-256 is FIPS 180-4.  One warp follows one request's chain (the chain is
 * serial: block i's first message block holds h_{i-1}); requests run in
 * parallel.  The lanes build each block's pickle bytes in parallel into a
 * shared-memory ring (token bytes placed by a warp prefix scan of their
 * 2/3/5-byte widths) and the warp compresses every complete 64-byte block,
 * so the control flow is uniform: with one thread per chain the lanes of a
 * warp reach their compressions at different byte counts and the warp
 * serialises them.
 */
#include "kvhash.h"
#include "adaptor.h"

#include <cuda_runtime.h>

#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

namespace {

constexpr int kWarpsPerCta = 4;     /* one warp per request chain */
constexpr uint32_t kRing = 512;     /* message ring per warp, bytes (multiple of 64) */

/* FIPS 180-4 section 4.2.2: first 32 bits of the fractional parts of the cube
 * roots of the first 64 primes */
__constant__ uint32_t kRound[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }
__device__ __forceinline__ uint32_t bswap(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

/* one compression of the 64 message bytes at `blk` (shared memory, message
 * byte order); every lane of the warp runs it on the same data */
/* the 64 rounds over message words m (big-endian values; m is consumed) */
__device__ __forceinline__ void sha_rounds(uint32_t st[8], uint32_t m[16])
{
    uint32_t a = st[0], b = st[1], c = st[2], d = st[3];
    uint32_t e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll
    for (int t = 0; t < 64; t++) {
        uint32_t wt;
        if (t < 16) {
            wt = m[t];
        } else {
            uint32_t w15 = m[(t - 15) & 15], w2 = m[(t - 2) & 15];
            uint32_t s0 = rotr(w15, 7) ^ rotr(w15, 18) ^ (w15 >> 3);
            uint32_t s1 = rotr(w2, 17) ^ rotr(w2, 19) ^ (w2 >> 10);
            wt = m[t & 15] + s0 + m[(t - 7) & 15] + s1;
            m[t & 15] = wt;
        }
        uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = h + S1 + ch + kRound[t] + wt;
        uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = S0 + maj;
        h = g; g = f; f = e; e = d + t1;
        d = c; c = b; b = a; a = t1 + t2;
    }
    st[0] += a; st[1] += b; st[2] += c; st[3] += d;
    st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

__device__ __forceinline__ void sha_compress(uint32_t st[8], const uint8_t *blk)
{
    const uint32_t *w32 = reinterpret_cast<const uint32_t *>(blk);
    uint32_t m[16];
#pragma unroll
    for (int k = 0; k < 16; k++)
        m[k] = bswap(w32[k]);
    sha_rounds(st, m);
}

/* The two serialisations of the (parent, tuple(tokens), None) triple that
 * vLLM hashes with SHA-256: pickle protocol 5 (vllm/utils/hashing.py:26-41)
 * and canonical CBOR (vllm/utils/hashing.py:43-57).  Each gives the header
 * length, the header bytes (which carry the 32 parent bytes), the encoding of
 * one int32 token, and the trailer. */
struct PickleFmt {
    static __device__ __forceinline__ uint32_t hdr_len(uint32_t bs) { return bs > 3 ? 47u : 46u; }
    /* tuple op, MEMOIZE, NONE or the extra segment, TUPLE3 MEMOIZE STOP */
    static __device__ __forceinline__ uint32_t trailer_len(uint32_t xlen) { return xlen ? 5u + xlen : 6u; }
    static __device__ __forceinline__ uint32_t header_byte(uint32_t p, uint32_t bs, uint64_t frame,
                                                           const uint8_t *par)
    {
        if (p < 3)
            return p == 0 ? 0x80u : (p == 1 ? 0x05u : 0x95u);     /* PROTO 5, FRAME */
        if (p < 11)
            return (uint32_t)(frame >> (8 * (p - 3))) & 0xffu;      /* frame length, LE */
        if (p < 13)
            return p == 11 ? 0x43u : 0x20u;                         /* SHORT_BINBYTES 32 */
        if (p < 45)
            return par[p - 13];
        return p == 45 ? 0x94u : 0x28u;                             /* MEMOIZE, MARK */
    }
    /* BININT1 (2 bytes), BININT2 (3), BININT (5) */
    static __device__ __forceinline__ uint32_t token_width(int32_t v)
    {
        return (v >= 0 && v <= 0xff) ? 2u : ((v >= 0 && v <= 0xffff) ? 3u : 5u);
    }
    static __device__ __forceinline__ uint32_t token_byte(int32_t v, uint32_t k)
    {
        const uint32_t u = (uint32_t)v;
        const uint32_t op = (v >= 0 && v <= 0xff) ? 0x4bu : ((v >= 0 && v <= 0xffff) ? 0x4du : 0x4au);
        return k == 0 ? op : (u >> (8 * (k - 1))) & 0xffu;
    }
    static __device__ __forceinline__ uint32_t trailer_byte(uint32_t k, uint32_t bs, const uint8_t *x, uint32_t xlen)
    {
        const uint32_t tuple_op = bs > 3 ? 0x74u : (0x84u + bs);    /* TUPLE or TUPLE1..3 */
        if (k < 2)
            return k == 0 ? tuple_op : 0x94u;
        const uint32_t xl = xlen ? xlen : 1u;
        if (k < 2 + xl)
            return xlen ? x[k - 2] : 0x4eu;
        k -= 2 + xl;
        return k == 0 ? 0x87u : (k == 1 ? 0x94u : 0x2eu);
    }
    /* put the parent digest h (8 big-endian words) into the first message
     * block's words m: it occupies bytes 13..44, i.e. the low 3 bytes of
     * word 3 through the top byte of word 11 */
    static __device__ __forceinline__ void splice_parent(uint32_t m[16], const uint32_t h[8])
    {
        m[3] = (m[3] & 0xff000000u) | (h[0] >> 8);
#pragma unroll
        for (int k = 4; k <= 10; k++)
            m[k] = (h[k - 4] << 24) | (h[k - 3] >> 8);
        m[11] = (h[7] << 24) | (m[11] & 0x00ffffffu);
    }
};

struct CborFmt {
    /* array(3), bytes(32) head, parent, array(bs) head of 1, 2 or 3 bytes */
    static __device__ __forceinline__ uint32_t arr_head(uint32_t bs) { return bs < 24 ? 1u : (bs < 256 ? 2u : 3u); }
    static __device__ __forceinline__ uint32_t hdr_len(uint32_t bs) { return 35u + arr_head(bs); }
    static __device__ __forceinline__ uint32_t trailer_len(uint32_t xlen) { return xlen ? xlen : 1u; }  /* null */
    static __device__ __forceinline__ uint32_t header_byte(uint32_t p, uint32_t bs, uint64_t, const uint8_t *par)
    {
        if (p < 3)
            return p == 0 ? 0x83u : (p == 1 ? 0x58u : 0x20u);
        if (p < 35)
            return par[p - 3];
        const uint32_t k = p - 35, h = arr_head(bs);
        if (h == 1)
            return 0x80u | bs;
        if (h == 2)
            return k == 0 ? 0x98u : bs;
        return k == 0 ? 0x99u : (k == 1 ? (bs >> 8) & 0xffu : bs & 0xffu);
    }
    /* major type 0 (v >= 0) or 1 (argument -1 - v), shortest head */
    static __device__ __forceinline__ uint32_t token_width(int32_t v)
    {
        const uint32_t n = v >= 0 ? (uint32_t)v : ~(uint32_t)v;
        return n < 24 ? 1u : (n < 0x100 ? 2u : (n < 0x10000 ? 3u : 5u));
    }
    static __device__ __forceinline__ uint32_t token_byte(int32_t v, uint32_t k)
    {
        const uint32_t n = v >= 0 ? (uint32_t)v : ~(uint32_t)v;
        const uint32_t major = v >= 0 ? 0x00u : 0x20u;
        const uint32_t w = token_width(v);
        if (k == 0)
            return w == 1 ? (major | n) : (major | (w == 2 ? 24u : (w == 3 ? 25u : 26u)));
        return (n >> (8 * (w - 1 - k))) & 0xffu;
    }
    static __device__ __forceinline__ uint32_t trailer_byte(uint32_t k, uint32_t, const uint8_t *x, uint32_t xlen)
    {
        return xlen ? x[k] : 0xf6u;
    }
    /* the parent occupies bytes 3..34: the low byte of word 0 through the
     * top 3 bytes of word 8 */
    static __device__ __forceinline__ void splice_parent(uint32_t m[16], const uint32_t h[8])
    {
        m[0] = (m[0] & 0xffffff00u) | (h[0] >> 24);
#pragma unroll
        for (int k = 1; k <= 7; k++)
            m[k] = (h[k - 1] << 8) | (h[k] >> 24);
        m[8] = (h[7] << 8) | (m[8] & 0xffu);
    }
};

struct HashArgs {
    const int32_t *tokens;
    const int64_t *tok_offsets;
    const int32_t *num_blocks;
    const int64_t *out_offsets;
    const uint8_t *parents;
    const uint8_t *extra;            /* per-block extra-key segments, or null */
    const int64_t *extra_offsets;    /* [total blocks + 1] into extra */
    uint8_t *out;
    uint32_t num_req;
    uint32_t block_size;
    uint32_t none_hash[8];   /* big-endian words */
};

/* Warp w of the grid follows the chain of request w.  Per block the lanes
 * (1) sum the token widths to get the message length, (2) write the pickle
 * bytes into a shared-memory ring in parallel -- the header and parent, then
 * 32 tokens at a time at offsets from a warp prefix scan of their widths,
 * then the trailer and the SHA-256 padding -- and (3) after every write phase
 * compress each complete 64-byte block.  Control flow is uniform across the
 * warp, so every compression runs once per warp. */
/* EXTRA: some block carries an extra-key segment (a separate instantiation,
 * so the common case compiles without the per-block segment lookups) */
template <typename F, bool EXTRA>
__global__ void __launch_bounds__(kWarpsPerCta * 32) block_hash_kernel(const HashArgs a)
{
    __shared__ __align__(16) uint8_t ring_all[kWarpsPerCta][kRing];
    __shared__ __align__(16) uint8_t parent_all[kWarpsPerCta][32];
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t wid = threadIdx.x >> 5;
    const uint32_t r = blockIdx.x * kWarpsPerCta + wid;
    if (r >= a.num_req)
        return;                       /* whole warp exits together */
    uint8_t *ring = ring_all[wid];
    uint8_t *par = parent_all[wid];

    if (a.parents) {
        par[lane] = a.parents[(uint64_t)r * 32 + lane];
    } else {
        /* constant parameter indices only (a dynamic index would copy the
         * whole parameter block to local memory) */
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (lane == (uint32_t)k)
                reinterpret_cast<uint32_t *>(par)[k] = bswap(a.none_hash[k]);
    }
    __syncwarp();

    const uint32_t bs = a.block_size;
    const uint32_t hdr_len = F::hdr_len(bs);
    const int32_t *tok = a.tokens + a.tok_offsets[r];
    uint8_t *out = a.out + (uint64_t)a.out_offsets[r] * 32;
    const int nblk = a.num_blocks[r];

    for (int i = 0; i < nblk; i++, tok += bs) {
        const uint8_t *x = nullptr;
        uint32_t xlen = 0;
        if (EXTRA) {
            const uint64_t gb = (uint64_t)a.out_offsets[r] + i;
            const int64_t x0 = a.extra_offsets[gb];
            x = a.extra + x0;
            xlen = (uint32_t)(a.extra_offsets[gb + 1] - x0);
        }
        const uint32_t tl = F::trailer_len(xlen);
        const uint32_t fixed = hdr_len + tl;
        /* (1) message length */
        uint32_t wsum = 0;
        for (uint32_t j = lane; j < bs; j += 32)
            wsum += F::token_width(tok[j]);
        const uint32_t len = fixed + __reduce_add_sync(0xffffffffu, wsum);
        const uint32_t total = (len + 9 + 63) & ~63u;     /* padded length */
        const uint64_t frame = len - 11;

        uint32_t st[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                          0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
        uint32_t pos = 0, done = 0;

        /* phase list: 0 = header, 1..G = token groups, G+1 = tail */
        const uint32_t groups = (bs + 31) / 32;
        for (uint32_t ph = 0; ph <= groups + 1; ph++) {
            if (ph == 0) {
                for (uint32_t p = lane; p < hdr_len; p += 32)
                    ring[p % kRing] = (uint8_t)F::header_byte(p, bs, frame, par);
                pos = hdr_len;
            } else if (ph <= groups) {
                const uint32_t j = (ph - 1) * 32 + lane;
                const int32_t v = j < bs ? tok[j] : 0;
                const uint32_t wdt = j < bs ? F::token_width(v) : 0u;
                uint32_t incl = wdt;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= (uint32_t)o)
                        incl += n;
                }
                const uint32_t off = pos + incl - wdt;
                for (uint32_t k = 0; k < wdt; k++)
                    ring[(off + k) % kRing] = (uint8_t)F::token_byte(v, k);
                pos += __shfl_sync(0xffffffffu, incl, 31);
            } else {
                const uint32_t tbase = len - tl;   /* the trailer starts here (== pos) */
                /* a long trailer (extra keys) passes the ring in 256-byte pieces */
                while (len - pos > 256) {
                    for (uint32_t p = lane; p < 256; p += 32)
                        ring[(pos + p) % kRing] = (uint8_t)F::trailer_byte(pos + p - tbase, bs, x, xlen);
                    pos += 256;
                    __syncwarp();
                    while (pos - done >= 64) {
                        sha_compress(st, ring + (done % kRing));
                        done += 64;
                    }
                    __syncwarp();
                }
                /* the rest of the trailer, then 0x80, zeros, 64-bit big-endian bit length */
                const uint32_t tail0 = pos;
                const uint64_t bits = (uint64_t)len * 8;
                for (uint32_t p = tail0 + lane; p < total; p += 32) {
                    uint32_t v;
                    if (p < len) {
                        v = F::trailer_byte(p - tbase, bs, x, xlen);
                    } else if (p == len) {
                        v = 0x80u;
                    } else if (p < total - 8) {
                        v = 0u;
                    } else {
                        v = (uint32_t)(bits >> (8 * (total - 1 - p))) & 0xffu;
                    }
                    ring[p % kRing] = (uint8_t)v;
                }
                pos = total;
            }
            __syncwarp();
            while (pos - done >= 64) {
                sha_compress(st, ring + (done % kRing));
                done += 64;
            }
            __syncwarp();
        }

        /* digest: lane k < 8 publishes word k as the next parent and output */
        uint32_t dw = st[0];
#pragma unroll
        for (int k = 1; k < 8; k++)
            if (lane == (uint32_t)k)
                dw = st[k];
        if (lane < 8) {
            const uint32_t be = bswap(dw);
            reinterpret_cast<uint32_t *>(par)[lane] = be;
            uint8_t *o = out + (uint64_t)i * 32 + 4 * lane;
            o[0] = (uint8_t)(dw >> 24);
            o[1] = (uint8_t)(dw >> 16);
            o[2] = (uint8_t)(dw >> 8);
            o[3] = (uint8_t)dw;
        }
        __syncwarp();
    }
}

/* ------------------------------------------------------------------------
 * Pipelined form (blocks of up to 256 tokens, no extra keys): two warps per
 * chain.  The producer warp builds block i+1's whole padded message -- all
 * but the 32 parent bytes, which depend on block i's digest -- into one of
 * two shared-memory slots while the consumer warp compresses block i from the
 * other slot, splicing the parent words in from the digest it holds in
 * registers.  One named barrier (the pair's 64 threads) per block swaps the
 * slots; both warps pass it the same number of times, and nothing spins.
 * The message building (a global token load, the width reduction and prefix
 * scan, the byte writes) leaves the chain's critical path, which becomes the
 * compressions alone.
 * ---------------------------------------------------------------------- */
constexpr int kPipeChains = 2;            /* chains per CTA, two warps each: every consumer
                                          * warp gets an SM sub-partition of its own */
constexpr uint32_t kPipeMaxBlock = 256;   /* tokens per block */

/* padded message bound for a block of bs tokens (pickle: 47-byte header,
 * at most 5 bytes a token, 6-byte trailer; CBOR is shorter) */
__host__ __device__ constexpr uint32_t pipe_slot_bytes(uint32_t bs)
{
    return (47u + 5u * bs + 6u + 9u + 63u) & ~63u;
}

__device__ __forceinline__ void pair_sync(uint32_t id)
{
    asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

template <typename F>
__global__ void __launch_bounds__(kPipeChains * 64) block_hash_pipe_kernel(const HashArgs a, uint32_t slot_bytes)
{
    extern __shared__ __align__(16) uint8_t pipe_smem[];
    __shared__ uint32_t slot_total[kPipeChains][2];
    __shared__ __align__(16) uint8_t zeros[32];
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t wid = threadIdx.x >> 5;
    const uint32_t chain = wid >> 1;
    const bool producer = (wid & 1) == 0;
    const uint32_t r = blockIdx.x * kPipeChains + chain;
    if (threadIdx.x < 32)
        zeros[threadIdx.x] = 0;
    __syncthreads();
    if (r >= a.num_req)
        return;                       /* both warps of the pair together */
    uint8_t *slots = pipe_smem + (size_t)chain * 2 * slot_bytes;
    const uint32_t bs = a.block_size;
    const int nblk = a.num_blocks[r];
    const uint32_t bar = 1 + chain;   /* barrier 0 is __syncthreads */

    if (producer) {
        const int32_t *tok0 = a.tokens + a.tok_offsets[r];
        const uint32_t hdr_len = F::hdr_len(bs);
        const uint32_t tl = F::trailer_len(0);
        const uint32_t groups = (bs + 31) / 32;
        for (int s = 0; s <= nblk; s++) {
            if (s < nblk) {
                const int32_t *tok = tok0 + (size_t)s * bs;
                uint8_t *msg = slots + (s & 1) * slot_bytes;
                uint32_t wsum = 0;
                for (uint32_t j = lane; j < bs; j += 32)
                    wsum += F::token_width(tok[j]);
                const uint32_t len = hdr_len + tl + __reduce_add_sync(0xffffffffu, wsum);
                const uint32_t total = (len + 9 + 63) & ~63u;
                const uint64_t frame = len - 11;
                for (uint32_t p = lane; p < hdr_len; p += 32)
                    msg[p] = (uint8_t)F::header_byte(p, bs, frame, zeros);
                uint32_t pos = hdr_len;
                for (uint32_t g = 0; g < groups; g++) {
                    const uint32_t j = g * 32 + lane;
                    const int32_t v = j < bs ? tok[j] : 0;
                    const uint32_t wdt = j < bs ? F::token_width(v) : 0u;
                    uint32_t incl = wdt;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= (uint32_t)o)
                            incl += n;
                    }
                    const uint32_t off = pos + incl - wdt;
                    for (uint32_t k = 0; k < wdt; k++)
                        msg[off + k] = (uint8_t)F::token_byte(v, k);
                    pos += __shfl_sync(0xffffffffu, incl, 31);
                }
                const uint32_t tbase = len - tl;
                const uint64_t bits = (uint64_t)len * 8;
                for (uint32_t p = pos + lane; p < total; p += 32) {
                    uint32_t v;
                    if (p < len)
                        v = F::trailer_byte(p - tbase, bs, nullptr, 0);
                    else if (p == len)
                        v = 0x80u;
                    else if (p < total - 8)
                        v = 0u;
                    else
                        v = (uint32_t)(bits >> (8 * (total - 1 - p))) & 0xffu;
                    msg[p] = (uint8_t)v;
                }
                if (lane == 0)
                    slot_total[chain][s & 1] = total;
            }
            pair_sync(bar);
        }
        return;
    }

    /* consumer */
    uint32_t h[8];
    if (a.parents) {
        const uint8_t *pp = a.parents + (uint64_t)r * 32;
#pragma unroll
        for (int k = 0; k < 8; k++)
            h[k] = ((uint32_t)pp[4 * k] << 24) | ((uint32_t)pp[4 * k + 1] << 16) |
                   ((uint32_t)pp[4 * k + 2] << 8) | (uint32_t)pp[4 * k + 3];
    } else {
#pragma unroll
        for (int k = 0; k < 8; k++)
            h[k] = a.none_hash[k];
    }
    uint8_t *out = a.out + (uint64_t)a.out_offsets[r] * 32;
    for (int s = 0; s <= nblk; s++) {
        if (s >= 1) {
            const int i = s - 1;
            const uint32_t *w32 = reinterpret_cast<const uint32_t *>(slots + (i & 1) * slot_bytes);
            const uint32_t nb = slot_total[chain][i & 1] / 64;
            uint32_t st[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                              0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
            for (uint32_t b = 0; b < nb; b++) {
                uint32_t m[16];
#pragma unroll
                for (int k = 0; k < 16; k++)
                    m[k] = bswap(w32[b * 16 + k]);
                if (b == 0)
                    F::splice_parent(m, h);
                sha_rounds(st, m);
            }
#pragma unroll
            for (int k = 0; k < 8; k++)
                h[k] = st[k];
            uint32_t dw = h[0];
#pragma unroll
            for (int k = 1; k < 8; k++)
                if (lane == (uint32_t)k)
                    dw = h[k];
            if (lane < 8) {
                uint8_t *o = out + (uint64_t)i * 32 + 4 * lane;
                o[0] = (uint8_t)(dw >> 24);
                o[1] = (uint8_t)(dw >> 16);
                o[2] = (uint8_t)(dw >> 8);
                o[3] = (uint8_t)dw;
            }
        }
        pair_sync(bar);
    }
}

struct HostWorkspace {
    std::mutex mu;
    void *dbuf = nullptr;
    size_t cap = 0;
};

HostWorkspace g_ws[64];

/* CROSSCACHE_HASH_KERNEL=warp keeps the one-warp-per-chain kernel */
bool pipe_allowed_by_env()
{
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("CROSSCACHE_HASH_KERNEL");
        v = (e && !strcmp(e, "warp")) ? 0 : 1;
    }
    return v == 1;
}

}  // namespace

extern "C" int kv_block_hash_launch_ext(const int32_t *tokens, const int64_t *tok_offsets,
                                        const int32_t *num_blocks, const int64_t *out_offsets,
                                        const uint8_t *parents, uint32_t num_req,
                                        uint32_t block_size, const uint8_t *none_hash,
                                        const uint8_t *extra, const int64_t *extra_offsets,
                                        uint8_t *out, int algo, void *stream)
{
    if (algo != KVHASH_SHA256_PICKLE && algo != KVHASH_SHA256_CBOR)
        return -EINVAL;
    if (!num_req)
        return 0;
    if (!tokens || !tok_offsets || !num_blocks || !out_offsets || !out || !block_size ||
        block_size > KVHASH_MAX_BLOCK_SIZE || (!parents && !none_hash) || (extra && !extra_offsets))
        return -EINVAL;
    HashArgs a{};
    a.tokens = tokens;
    a.tok_offsets = tok_offsets;
    a.num_blocks = num_blocks;
    a.out_offsets = out_offsets;
    a.parents = parents;
    a.extra = extra;
    a.extra_offsets = extra ? extra_offsets : nullptr;
    a.out = out;
    a.num_req = num_req;
    a.block_size = block_size;
    if (none_hash)
        for (int k = 0; k < 8; k++)
            a.none_hash[k] = ((uint32_t)none_hash[4 * k] << 24) | ((uint32_t)none_hash[4 * k + 1] << 16) |
                             ((uint32_t)none_hash[4 * k + 2] << 8) | (uint32_t)none_hash[4 * k + 3];
    unsigned grid = (num_req + kWarpsPerCta - 1) / kWarpsPerCta;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned threads = kWarpsPerCta * 32;
    if (!extra && block_size <= kPipeMaxBlock && pipe_allowed_by_env()) {
        const uint32_t slot = pipe_slot_bytes(block_size);
        const unsigned pgrid = (num_req + kPipeChains - 1) / kPipeChains;
        const size_t smem = (size_t)kPipeChains * 2 * slot;
        if (algo == KVHASH_SHA256_CBOR)
            block_hash_pipe_kernel<CborFmt><<<pgrid, kPipeChains * 64, smem, s>>>(a, slot);
        else
            block_hash_pipe_kernel<PickleFmt><<<pgrid, kPipeChains * 64, smem, s>>>(a, slot);
        g_cc_kernel_launches.fetch_add(1, std::memory_order_relaxed);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : -EIO;
    }
    if (algo == KVHASH_SHA256_CBOR) {
        if (extra)
            block_hash_kernel<CborFmt, true><<<grid, threads, 0, s>>>(a);
        else
            block_hash_kernel<CborFmt, false><<<grid, threads, 0, s>>>(a);
    } else {
        if (extra)
            block_hash_kernel<PickleFmt, true><<<grid, threads, 0, s>>>(a);
        else
            block_hash_kernel<PickleFmt, false><<<grid, threads, 0, s>>>(a);
    }
    g_cc_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -EIO;
}

extern "C" int kv_block_hash_launch_algo(const int32_t *tokens, const int64_t *tok_offsets,
                                         const int32_t *num_blocks, const int64_t *out_offsets,
                                         const uint8_t *parents, uint32_t num_req,
                                         uint32_t block_size, const uint8_t *none_hash,
                                         uint8_t *out, int algo, void *stream)
{
    return kv_block_hash_launch_ext(tokens, tok_offsets, num_blocks, out_offsets, parents, num_req, block_size,
                                    none_hash, nullptr, nullptr, out, algo, stream);
}

extern "C" int kv_block_hash_launch(const int32_t *tokens, const int64_t *tok_offsets,
                                    const int32_t *num_blocks, const int64_t *out_offsets,
                                    const uint8_t *parents, uint32_t num_req,
                                    uint32_t block_size, const uint8_t *none_hash,
                                    uint8_t *out, void *stream)
{
    return kv_block_hash_launch_algo(tokens, tok_offsets, num_blocks, out_offsets, parents, num_req,
                                     block_size, none_hash, out, KVHASH_SHA256_PICKLE, stream);
}

extern "C" int64_t kv_block_hash_host_ext(int devid, const int32_t *tokens, const int64_t *tok_lens,
                                          uint32_t num_req, uint32_t block_size, const uint8_t *none_hash,
                                          const uint8_t *extra, const int64_t *extra_offsets,
                                          uint8_t *out_hashes, int algo)
{
    if (algo != KVHASH_SHA256_PICKLE && algo != KVHASH_SHA256_CBOR)
        return -EINVAL;
    if (devid < 0 || devid >= 64 || !tok_lens || !none_hash || !out_hashes || !block_size ||
        block_size > KVHASH_MAX_BLOCK_SIZE)
        return -EINVAL;
    if (!num_req)
        return 0;
    std::vector<int64_t> toff(num_req), ooff(num_req);
    std::vector<int32_t> nblk(num_req);
    int64_t ntok = 0, nout = 0;
    for (uint32_t r = 0; r < num_req; r++) {
        if (tok_lens[r] < 0)
            return -EINVAL;
        toff[r] = ntok;
        ooff[r] = nout;
        nblk[r] = (int32_t)(tok_lens[r] / block_size);
        ntok += tok_lens[r];
        nout += nblk[r];
    }
    if (!nout)
        return 0;
    if (!tokens)
        return -EINVAL;
    int64_t xbytes = 0;
    if (extra) {
        if (!extra_offsets || extra_offsets[0] != 0)
            return -EINVAL;
        for (int64_t k = 0; k < nout; k++)
            if (extra_offsets[k + 1] < extra_offsets[k])
                return -EINVAL;
        xbytes = extra_offsets[nout];
    }
    /* one workspace per device: [tokens | toff | ooff | nblk | out | xoff | extra] */
    auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
    size_t o_tok = 0;
    size_t o_toff = align(o_tok + ntok * 4);
    size_t o_ooff = align(o_toff + num_req * 8);
    size_t o_nblk = align(o_ooff + num_req * 8);
    size_t o_out = align(o_nblk + num_req * 4);
    size_t o_xoff = align(o_out + (size_t)nout * 32);
    size_t o_x = align(o_xoff + (extra ? (size_t)(nout + 1) * 8 : 0));
    size_t total = align(o_x + (size_t)xbytes);

    HostWorkspace &ws = g_ws[devid];
    std::lock_guard<std::mutex> g(ws.mu);
    if (cudaSetDevice(devid) != cudaSuccess)
        return -EIO;
    if (total > ws.cap) {
        if (ws.dbuf)
            cudaFree(ws.dbuf);
        ws.dbuf = nullptr;
        ws.cap = 0;
        if (cudaMalloc(&ws.dbuf, total) != cudaSuccess)
            return -ENOMEM;
        ws.cap = total;
    }
    uint8_t *b = static_cast<uint8_t *>(ws.dbuf);
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
        return -EIO;
    int64_t ret = nout;
    if (cudaMemcpyAsync(b + o_tok, tokens, ntok * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(b + o_toff, toff.data(), num_req * 8, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(b + o_ooff, ooff.data(), num_req * 8, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(b + o_nblk, nblk.data(), num_req * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
        ret = -EIO;
    if (ret > 0 && extra &&
        (cudaMemcpyAsync(b + o_xoff, extra_offsets, (size_t)(nout + 1) * 8, cudaMemcpyHostToDevice, s) != cudaSuccess ||
         (xbytes && cudaMemcpyAsync(b + o_x, extra, (size_t)xbytes, cudaMemcpyHostToDevice, s) != cudaSuccess)))
        ret = -EIO;
    if (ret > 0 && kv_block_hash_launch_ext(reinterpret_cast<int32_t *>(b + o_tok),
                                            reinterpret_cast<int64_t *>(b + o_toff),
                                            reinterpret_cast<int32_t *>(b + o_nblk),
                                            reinterpret_cast<int64_t *>(b + o_ooff), nullptr, num_req,
                                            block_size, none_hash, extra ? b + o_x : nullptr,
                                            extra ? reinterpret_cast<int64_t *>(b + o_xoff) : nullptr,
                                            b + o_out, algo, s))
        ret = -EIO;
    if (ret > 0 && cudaMemcpyAsync(out_hashes, b + o_out, (size_t)nout * 32, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        ret = -EIO;
    if (cudaStreamSynchronize(s) != cudaSuccess)
        ret = -EIO;
    cudaStreamDestroy(s);
    return ret;
}

extern "C" int64_t kv_block_hash_host_algo(int devid, const int32_t *tokens, const int64_t *tok_lens,
                                           uint32_t num_req, uint32_t block_size,
                                           const uint8_t *none_hash, uint8_t *out_hashes, int algo)
{
    return kv_block_hash_host_ext(devid, tokens, tok_lens, num_req, block_size, none_hash, nullptr, nullptr,
                                  out_hashes, algo);
}

extern "C" int64_t kv_block_hash_host(int devid, const int32_t *tokens, const int64_t *tok_lens,
                                      uint32_t num_req, uint32_t block_size,
                                      const uint8_t *none_hash, uint8_t *out_hashes)
{
    return kv_block_hash_host_algo(devid, tokens, tok_lens, num_req, block_size, none_hash, out_hashes,
                                   KVHASH_SHA256_PICKLE);
}
