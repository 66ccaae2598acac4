"""helm_b200: B200-native decode hot path of HELM (paged decode attention with split-KV and a
log-sum-exp merge, INT8 weight-only linear, device-indexed KV page pool).

The kernels live in libhelm_b200.so (C ABI, include/helm_b200.h); this package
is the host side that mirrors HELM's runtime API (helm.runtime.kv_cache,
kv_allocator, kv_offload and helm.kernels).
"""
__version__ = "0.1.0"
