/*
 * Batched chained prefix block hash on sm_100a.
 *
 * CrossCache never hashes tokens itself: its keys are vLLM's
 * request.block_hashes (python/crosscache_connector.py:133,500), produced by
 * vLLM's hash_block_tokens (vllm/v1/core/kv_cache_utils.py:541-570, a
 * third-party dependency pinned to v0.11.2 in CrossCache README.md:5) with
 * the default hash function vllm/utils/hashing.py sha256:
 *
 *   h_i = SHA-256( pickle.dumps((h_{i-1}, tuple(tok[i*bs:(i+1)*bs]), None),
 *                               protocol=5) )
 *   h_{-1} = NONE_HASH = SHA-256(pickle.dumps(str(PYTHONHASHSEED)))
 *
 * The kernel serialises each block's pickle byte stream on the device and
 * runs SHA-256 (FIPS 180-4), one chain per request, requests in parallel.
 * vLLM's other SHA-256 variant, sha256_cbor (vllm/utils/hashing.py:43-57,
 * canonical CBOR of the same triple), is available through the *_algo entry
 * points.
 * The chunk keys CrossCache sends to the server are every
 * (chunk_size / block_size)-th hash (python/adaptor.py:32-40).
 *
 * Limits: 1 <= block_size <= 8192 (pickle then uses a single frame), token
 * ids are int32, extra_keys (LoRA / multimodal) are not supported (None).
 */
#ifndef __KVHASH_H__
#define __KVHASH_H__

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVHASH_MAX_BLOCK_SIZE 8192

/* hash functions (vLLM's prefix_caching_hash_algo) */
#define KVHASH_SHA256_PICKLE 0   /* "sha256": SHA-256 of pickle protocol 5 (default) */
#define KVHASH_SHA256_CBOR   1   /* "sha256_cbor": SHA-256 of canonical CBOR
                                  * (vllm/utils/hashing.py:43-57); NONE_HASH is
                                  * then SHA-256 of the CBOR text string seed */

/* Device-pointer form, asynchronous on `stream` (a cudaStream_t).
 *   tokens       int32 token ids, requests packed back to back
 *   tok_offsets  [num_req] index of request r's first token in tokens
 *   num_blocks   [num_req] full blocks to hash for request r
 *   out_offsets  [num_req] index of request r's first hash in out
 *   parents      [num_req][32] parent hash of each request's first block, or
 *                NULL to start every chain at none_hash
 *   none_hash    32 bytes, host memory (copied at launch)
 *   out          [sum num_blocks][32] block hashes
 * Returns 0, -EINVAL, or -EIO on a launch failure. */
int kv_block_hash_launch(const int32_t *tokens, const int64_t *tok_offsets,
                         const int32_t *num_blocks, const int64_t *out_offsets,
                         const uint8_t *parents, uint32_t num_req,
                         uint32_t block_size, const uint8_t *none_hash,
                         uint8_t *out, void *stream);

/* Host-buffer form: copies the inputs to device `devid`, hashes, copies the
 * hashes back, and returns after they have landed.  Per-request token counts
 * are tok_lens[r]; request r gets floor(tok_lens[r] / block_size) hashes,
 * written back to back into out_hashes (host, 32 bytes each).  Returns the
 * total number of hashes written, or a negative errno. */
int64_t kv_block_hash_host(int devid, const int32_t *tokens,
                           const int64_t *tok_lens, uint32_t num_req,
                           uint32_t block_size, const uint8_t *none_hash,
                           uint8_t *out_hashes);

/* The same two entry points with an explicit hash function (KVHASH_*); the
 * forms above are KVHASH_SHA256_PICKLE.  -EINVAL for an unknown algo. */
int kv_block_hash_launch_algo(const int32_t *tokens, const int64_t *tok_offsets,
                              const int32_t *num_blocks, const int64_t *out_offsets,
                              const uint8_t *parents, uint32_t num_req,
                              uint32_t block_size, const uint8_t *none_hash,
                              uint8_t *out, int algo, void *stream);

int64_t kv_block_hash_host_algo(int devid, const int32_t *tokens,
                                const int64_t *tok_lens, uint32_t num_req,
                                uint32_t block_size, const uint8_t *none_hash,
                                uint8_t *out_hashes, int algo);

/* With vLLM's per-block extra keys (hash_block_tokens' extra_keys: LoRA
 * name, multimodal hashes, cache salt).  Block g of the output order (request
 * by request, block by block) hashes (parent, tokens, extra_keys_g) where the
 * bytes extra[extra_offsets[g] .. extra_offsets[g + 1]) are the serialised
 * extra_keys_g exactly as they appear inside the pickle protocol-5 (or
 * canonical CBOR) stream of that tuple -- they replace the None byte; an
 * empty range means None.  demo_b200.hashing.extra_segment builds them.
 * extra_offsets has total blocks + 1 entries (device memory for _launch_ext,
 * host memory for _host_ext); extra NULL = no extra keys anywhere. */
int kv_block_hash_launch_ext(const int32_t *tokens, const int64_t *tok_offsets,
                             const int32_t *num_blocks, const int64_t *out_offsets,
                             const uint8_t *parents, uint32_t num_req,
                             uint32_t block_size, const uint8_t *none_hash,
                             const uint8_t *extra, const int64_t *extra_offsets,
                             uint8_t *out, int algo, void *stream);

int64_t kv_block_hash_host_ext(int devid, const int32_t *tokens,
                               const int64_t *tok_lens, uint32_t num_req,
                               uint32_t block_size, const uint8_t *none_hash,
                               const uint8_t *extra, const int64_t *extra_offsets,
                               uint8_t *out_hashes, int algo);

#ifdef __cplusplus
}
#endif

#endif
