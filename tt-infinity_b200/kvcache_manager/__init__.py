"""B200-native kvcache_manager: a hash-sharded, tiered KV block store for paged LLM KV caches.

Drop-in for the reference's `kvcache_manager` Python package (src/kvcache_manager/__init__.py):
`Server` and `Client` keep its put / get / exists / delete / move / flush surface, backed by
hand-written sm_100a kernels in libkvs_b200.so (C ABI: include/kvs.h).
"""

from ._facade import Client, PagedLayout, Server, to_key
from ._native import KvsError

__all__ = ["Client", "Server", "PagedLayout", "KvsError", "to_key"]
