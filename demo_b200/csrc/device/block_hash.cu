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
 * (CPython _pickle.c save_bytes/save_tuple/save_long; a 0..255 token is
 * BININT1, 256..65535 BININT2, anything else BININT 4-byte two's complement.)
 *
 * SHA-256 is FIPS 180-4.  One thread follows one request's chain (the chain
 * is serial: block i's first message block holds h_{i-1}); requests run in
 * parallel, one warp per CTA so that chains spread over SMs.  Each thread
 * streams its message bytes into a 64-byte block held in shared memory
 * (word-interleaved across the warp to avoid bank conflicts) and compresses
 * whenever the block fills, so no message buffer of block_size-dependent
 * size is needed; the SHA state also lives in shared memory so that the
 * byte counters stay in registers around the out-of-line compression.
 */
#include "kvhash.h"
#include "adaptor.h"

#include <cuda_runtime.h>

#include <cerrno>
#include <cstring>
#include <mutex>
#include <vector>

namespace {

constexpr int kHashThreads = 32;   /* one warp per CTA: chains spread over SMs */

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

/* FIPS 180-4 section 5.3.3: initial hash value (state column stride kHashThreads) */
__device__ __forceinline__ void sha_init(uint32_t *st)
{
    st[0] = 0x6a09e667; st[kHashThreads] = 0xbb67ae85; st[2 * kHashThreads] = 0x3c6ef372;
    st[3 * kHashThreads] = 0xa54ff53a; st[4 * kHashThreads] = 0x510e527f;
    st[5 * kHashThreads] = 0x9b05688c; st[6 * kHashThreads] = 0x1f83d9ab;
    st[7 * kHashThreads] = 0x5be0cd19;
}

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

/* one compression: state st[k * kHashThreads] (shared memory), message words
 * w[k * kHashThreads].  Not inlined: the byte streamer calls it from many
 * places, and keeping it out of line keeps the kernel small; all of its
 * operands are in shared memory so the caller's registers stay registers. */
__device__ __noinline__ void sha_compress(uint32_t *st, const uint32_t *w)
{
    uint32_t m[16];
#pragma unroll
    for (int k = 0; k < 16; k++)
        m[k] = w[k * kHashThreads];
    uint32_t a = st[0], b = st[kHashThreads], c = st[2 * kHashThreads], d = st[3 * kHashThreads];
    uint32_t e = st[4 * kHashThreads], f = st[5 * kHashThreads], g = st[6 * kHashThreads], h = st[7 * kHashThreads];
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
    st[0] += a; st[kHashThreads] += b; st[2 * kHashThreads] += c; st[3 * kHashThreads] += d;
    st[4 * kHashThreads] += e; st[5 * kHashThreads] += f; st[6 * kHashThreads] += g; st[7 * kHashThreads] += h;
}

/* byte stream -> 64-byte message blocks in shared memory; the counters are
 * plain registers (nothing here is address-taken) */
struct Streamer {
    uint32_t *w;      /* this thread's message column: word k at w[k * kHashThreads] */
    uint32_t *st;     /* this thread's state column */
    uint32_t acc;     /* bytes not yet forming a full word, big-endian */
    int nacc;         /* bytes in acc (0..3) */
    int wpos;         /* words filled in the current block (0..15) */

    __device__ __forceinline__ void word(uint32_t v)
    {
        w[wpos * kHashThreads] = v;
        if (++wpos == 16) {
            sha_compress(st, w);
            wpos = 0;
        }
    }
    __device__ __forceinline__ void byte(uint32_t b)
    {
        acc = (acc << 8) | (b & 0xff);
        if (++nacc == 4) {
            word(acc);
            acc = 0;
            nacc = 0;
        }
    }
    /* SHA-256 padding for a message of `len` bytes, final compression */
    __device__ __forceinline__ void finish(uint64_t len)
    {
        byte(0x80);
        if (nacc) {
            acc <<= 8 * (4 - nacc);
            nacc = 0;
            word(acc);
            acc = 0;
        }
        if (wpos > 14) {
            while (wpos != 0)
                word(0);
        }
        while (wpos < 14)
            word(0);
        word((uint32_t)((len * 8) >> 32));
        word((uint32_t)(len * 8));
    }
};

__device__ __forceinline__ uint32_t token_width(int32_t v)
{
    return (v >= 0 && v <= 0xff) ? 2u : ((v >= 0 && v <= 0xffff) ? 3u : 5u);
}

struct HashArgs {
    const int32_t *tokens;
    const int64_t *tok_offsets;
    const int32_t *num_blocks;
    const int64_t *out_offsets;
    const uint8_t *parents;
    uint8_t *out;
    uint32_t num_req;
    uint32_t block_size;
    uint32_t none_hash[8];   /* big-endian words */
};

__global__ void __launch_bounds__(kHashThreads) block_hash_kernel(const HashArgs a)
{
    __shared__ uint32_t sw[16 * kHashThreads];
    __shared__ uint32_t sst[8 * kHashThreads];
    const uint32_t r = blockIdx.x * kHashThreads + threadIdx.x;
    if (r >= a.num_req)
        return;

    uint32_t parent[8];
    if (a.parents) {
        const uint8_t *pp = a.parents + (uint64_t)r * 32;
#pragma unroll
        for (int k = 0; k < 8; k++)
            parent[k] = ((uint32_t)pp[4 * k] << 24) | ((uint32_t)pp[4 * k + 1] << 16) |
                        ((uint32_t)pp[4 * k + 2] << 8) | (uint32_t)pp[4 * k + 3];
    } else {
#pragma unroll
        for (int k = 0; k < 8; k++)
            parent[k] = a.none_hash[k];
    }

    const uint32_t bs = a.block_size;
    const int32_t *tok = a.tokens + a.tok_offsets[r];
    uint8_t *out = a.out + (uint64_t)a.out_offsets[r] * 32;
    const int nblk = a.num_blocks[r];
    /* fixed bytes: PROTO 2, FRAME 9, SHORT_BINBYTES 34, MEMOIZE 1, [MARK 1],
     * tuple opcode 1, MEMOIZE NONE TUPLE3 MEMOIZE STOP 5 */
    const uint32_t fixed = 2 + 9 + 34 + 1 + (bs > 3 ? 1 : 0) + 1 + 5;
    const uint32_t tuple_op = bs > 3 ? 0x74u : (0x84u + bs);

    Streamer s;
    s.w = sw + threadIdx.x;
    s.st = sst + threadIdx.x;
    for (int i = 0; i < nblk; i++, tok += bs) {
        uint32_t len = fixed;
        for (uint32_t j = 0; j < bs; j++)
            len += token_width(tok[j]);
        const uint64_t frame = len - 11;

        sha_init(s.st);
        s.acc = 0;
        s.nacc = 0;
        s.wpos = 0;
        s.byte(0x80);
        s.byte(0x05);
        s.byte(0x95);
        for (int k = 0; k < 8; k++)
            s.byte((uint32_t)(frame >> (8 * k)));
        s.byte(0x43);
        s.byte(0x20);
        for (int k = 0; k < 8; k++) {
            s.byte(parent[k] >> 24);
            s.byte(parent[k] >> 16);
            s.byte(parent[k] >> 8);
            s.byte(parent[k]);
        }
        s.byte(0x94);
        if (bs > 3)
            s.byte(0x28);
        for (uint32_t j = 0; j < bs; j++) {
            const int32_t v = tok[j];
            const uint32_t u = (uint32_t)v;
            if (v >= 0 && v <= 0xff) {
                s.byte(0x4b);
                s.byte(u);
            } else if (v >= 0 && v <= 0xffff) {
                s.byte(0x4d);
                s.byte(u);
                s.byte(u >> 8);
            } else {
                s.byte(0x4a);
                s.byte(u);
                s.byte(u >> 8);
                s.byte(u >> 16);
                s.byte(u >> 24);
            }
        }
        s.byte(tuple_op);
        s.byte(0x94);
        s.byte(0x4e);
        s.byte(0x87);
        s.byte(0x94);
        s.byte(0x2e);
        s.finish(len);

        uint32_t dg[8];
#pragma unroll
        for (int k = 0; k < 8; k++)
            dg[k] = s.st[k * kHashThreads];
        uint4 lo, hi;
        lo.x = __byte_perm(dg[0], 0, 0x0123);
        lo.y = __byte_perm(dg[1], 0, 0x0123);
        lo.z = __byte_perm(dg[2], 0, 0x0123);
        lo.w = __byte_perm(dg[3], 0, 0x0123);
        hi.x = __byte_perm(dg[4], 0, 0x0123);
        hi.y = __byte_perm(dg[5], 0, 0x0123);
        hi.z = __byte_perm(dg[6], 0, 0x0123);
        hi.w = __byte_perm(dg[7], 0, 0x0123);
        uint8_t *o = out + (uint64_t)i * 32;
        if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
            reinterpret_cast<uint4 *>(o)[0] = lo;
            reinterpret_cast<uint4 *>(o)[1] = hi;
        } else {
            memcpy(o, &lo, 16);
            memcpy(o + 16, &hi, 16);
        }
#pragma unroll
        for (int k = 0; k < 8; k++)
            parent[k] = dg[k];
    }
}

struct HostWorkspace {
    std::mutex mu;
    void *dbuf = nullptr;
    size_t cap = 0;
};

HostWorkspace g_ws[64];

}  // namespace

extern "C" int kv_block_hash_launch(const int32_t *tokens, const int64_t *tok_offsets,
                                    const int32_t *num_blocks, const int64_t *out_offsets,
                                    const uint8_t *parents, uint32_t num_req,
                                    uint32_t block_size, const uint8_t *none_hash,
                                    uint8_t *out, void *stream)
{
    if (!num_req)
        return 0;
    if (!tokens || !tok_offsets || !num_blocks || !out_offsets || !out || !block_size ||
        block_size > KVHASH_MAX_BLOCK_SIZE || (!parents && !none_hash))
        return -EINVAL;
    HashArgs a{};
    a.tokens = tokens;
    a.tok_offsets = tok_offsets;
    a.num_blocks = num_blocks;
    a.out_offsets = out_offsets;
    a.parents = parents;
    a.out = out;
    a.num_req = num_req;
    a.block_size = block_size;
    if (none_hash)
        for (int k = 0; k < 8; k++)
            a.none_hash[k] = ((uint32_t)none_hash[4 * k] << 24) | ((uint32_t)none_hash[4 * k + 1] << 16) |
                             ((uint32_t)none_hash[4 * k + 2] << 8) | (uint32_t)none_hash[4 * k + 3];
    unsigned grid = (num_req + kHashThreads - 1) / kHashThreads;
    block_hash_kernel<<<grid, kHashThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    g_cc_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -EIO;
}

extern "C" int64_t kv_block_hash_host(int devid, const int32_t *tokens, const int64_t *tok_lens,
                                      uint32_t num_req, uint32_t block_size,
                                      const uint8_t *none_hash, uint8_t *out_hashes)
{
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
    /* one workspace per device: [tokens | toff | ooff | nblk | out] */
    auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
    size_t o_tok = 0;
    size_t o_toff = align(o_tok + ntok * 4);
    size_t o_ooff = align(o_toff + num_req * 8);
    size_t o_nblk = align(o_ooff + num_req * 8);
    size_t o_out = align(o_nblk + num_req * 4);
    size_t total = align(o_out + (size_t)nout * 32);

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
    if (ret > 0 && kv_block_hash_launch(reinterpret_cast<int32_t *>(b + o_tok),
                                        reinterpret_cast<int64_t *>(b + o_toff),
                                        reinterpret_cast<int32_t *>(b + o_nblk),
                                        reinterpret_cast<int64_t *>(b + o_ooff), nullptr, num_req,
                                        block_size, none_hash, b + o_out, s))
        ret = -EIO;
    if (ret > 0 && cudaMemcpyAsync(out_hashes, b + o_out, (size_t)nout * 32, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        ret = -EIO;
    if (cudaStreamSynchronize(s) != cudaSuccess)
        ret = -EIO;
    cudaStreamDestroy(s);
    return ret;
}
