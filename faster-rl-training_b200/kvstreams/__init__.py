"""kvstreams (B200): the KV-streams paged-KV path on hand-written sm_100a kernels.

Drop-in for the reference package's hot path: ``build_stack``, ``KVStreamEngine.rollout``,
``PagedKVCache`` block tables, ``token_logprobs`` / ``measure_mismatch``.  Kernels live
in libkvs_b200.so (C ABI: include/kvs_b200.h) and are called through ctypes.
"""

__version__ = "0.2.0+b200"
