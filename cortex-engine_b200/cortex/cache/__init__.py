"""Device-resident paged K|V cache (cortex/cache in the reference)."""

from cortex.cache.streaming import PageMeta, StreamingKVCache

__all__ = ["PageMeta", "StreamingKVCache"]
