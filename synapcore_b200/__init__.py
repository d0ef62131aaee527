"""B200-native paged KV cache: a drop-in for SynapCore's paged KV path.

Host side (Python / PyTorch) mirrors the reference API — PagedKVArena,
NativeKVPrefixCache, the KV prefix hash table, the continuous-batching
scheduler's KV side — and drives hand-written
sm_100a CUDA kernels in libsckv.so through its C ABI (include/sckv.h).
"""
from ._native import SCKVBoundsError, SCKVError, SCKVPoolExhausted
from .arena import PagedKVArena
from .attention_layer import PagedAttentionLayer
from .kv_index import KVPrefixIndex
from .paged_cache import DecodeStepGraph, PagedKVCache
from .pool import KVPool, rope_inv_freq
from .prefix_cache import NativeKVPrefixCache, PagedKVStats, chain_merkle_prefix_hash
from .scheduler import ContinuousBatchScheduler, PagedDecoderModel, PrefixPageIndex

__all__ = [
    "ContinuousBatchScheduler",
    "DecodeStepGraph",
    "KVPool",
    "PagedDecoderModel",
    "PagedKVCache",
    "PrefixPageIndex",
    "KVPrefixIndex",
    "NativeKVPrefixCache",
    "PagedAttentionLayer",
    "PagedKVArena",
    "PagedKVStats",
    "SCKVBoundsError",
    "SCKVError",
    "SCKVPoolExhausted",
    "chain_merkle_prefix_hash",
    "rope_inv_freq",
]
