"""Host-side mirror of HELM's runtime API (helm.runtime.kv_allocator, kv_cache, kv_offload)."""
from .kv_allocator import KVAllocator
from .kv_cache import KVCacheManager, KVPage, LayerKVCache, perform_streaming_attention
from .kv_offload import KVOffloadConfig, KVOffloadManager

__all__ = ["KVAllocator", "KVCacheManager", "KVPage", "LayerKVCache", "perform_streaming_attention",
           "KVOffloadConfig", "KVOffloadManager"]
