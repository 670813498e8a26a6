"""B200 (sm_100a) paged streaming hot path of odunola499/parakeet-streaming.

Host side mirrors the reference's module and scheduler interfaces
(``parakeet.modules`` / ``parakeet.engine``); the compute runs in libpk.so
(C ABI: include/pk.h), loaded through ctypes by ``parakeet_b200._lib``.
"""
from .ops import PagedKVPool, pages_per_stream, ring_size

__all__ = ["PagedKVPool", "pages_per_stream", "ring_size"]
