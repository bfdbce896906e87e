"""demo_b200 -- B200-native KV-cache offload hot path of CrossCache.

libcrosscache.so (built by `python -m demo_b200.build`) holds the C cache
manager, the CUDA adaptor and the sm_100a kernels; this package is the thin
Python side:

  _lib       ctypes bindings of include/*.h (raises if the library is absent)
  cache      in-process cache-manager API over torch KV tensors
  hashing    device block hashing (vLLM sha256 block hash, bit-identical)
  adaptor    SchedulerAdapter / WorkerAdapter with the reference's interface
  connector  vLLM KVConnectorBase_V1 implementation (CrossCacheConnector)
  tp         NCCL all-reduce(min) of per-request hit lengths across TP ranks

Every submodule except `build` loads the library on import and raises
ImportError when it has not been built: there is no fallback path.
"""
