"""CPU restatement of the reference's fixed-capacity KV cache (src/cache.rs).

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of the cache
layout that the CUDA attention path reads. The product never imports it.

Layout (cache.rs:1-4): keys and values are [kv_head][capacity][head_dim]
f32, so appending never moves existing entries. Errors raise CacheError with
the reference's messages.
"""
from __future__ import annotations

import numpy as np


class CacheError(ValueError):
    """CacheError (cache.rs:6-7)."""


class KvCache:
    def __init__(self, key_value_heads: int, head_dim: int, capacity_tokens: int):
        """KvCache::new (cache.rs:20-40)."""
        if key_value_heads == 0 or head_dim == 0 or capacity_tokens == 0:
            raise CacheError("KV-cache dimensions must be non-zero")
        self.key_value_heads, self.head_dim, self.capacity_tokens = key_value_heads, head_dim, capacity_tokens
        self.cached_tokens = 0
        n = key_value_heads * head_dim * capacity_tokens
        self.keys = np.zeros(n, np.float32)
        self.values = np.zeros(n, np.float32)

    def remaining_tokens(self) -> int:  # cache.rs:58-60
        return self.capacity_tokens - self.cached_tokens

    def active_bytes(self) -> int:  # cache.rs:70-73
        return self.key_value_heads * self.cached_tokens * self.head_dim * 2 * 4

    def append_token(self, keys, values):
        """append_token (cache.rs:75-98): one token's [kv_head][head_dim]."""
        expected = self.key_value_heads * self.head_dim
        keys, values = np.asarray(keys, np.float32), np.asarray(values, np.float32)
        if keys.size != expected or values.size != expected:
            raise CacheError(f"KV token must contain {expected} values per key and value")
        if self.cached_tokens == self.capacity_tokens:
            raise CacheError("KV-cache capacity exhausted")
        hd = self.head_dim
        for h in range(self.key_value_heads):
            dst = (h * self.capacity_tokens + self.cached_tokens) * hd
            self.keys[dst:dst + hd] = keys[h * hd:(h + 1) * hd]
            self.values[dst:dst + hd] = values[h * hd:(h + 1) * hd]
        self.cached_tokens += 1

    def append_sequence(self, keys, values, tokens: int):
        """append_sequence (cache.rs:100-127): token-major [token][kv_head][head_dim]."""
        per = self.key_value_heads * self.head_dim
        keys, values = np.asarray(keys, np.float32), np.asarray(values, np.float32)
        expected = tokens * per
        if keys.size != expected or values.size != expected:
            raise CacheError(f"KV sequence must contain {expected} values per key and value")
        if tokens > self.remaining_tokens():
            raise CacheError("KV-cache sequence exceeds remaining capacity")
        for t in range(tokens):
            self.append_token(keys[t * per:(t + 1) * per], values[t * per:(t + 1) * per])

    def clear(self):  # cache.rs:129-131
        self.cached_tokens = 0

    def truncate_to(self, cached_tokens: int):
        """truncate_to (cache.rs:136-145): drop a speculative suffix in place."""
        if cached_tokens > self.cached_tokens:
            raise CacheError("cannot truncate KV-cache to a future position")
        self.cached_tokens = cached_tokens

    def copy_prefix_from(self, source: "KvCache"):
        """copy_prefix_from (cache.rs:150-170): the source's active prefix into
        this cache's storage, which may have the larger capacity."""
        if (self.key_value_heads != source.key_value_heads or self.head_dim != source.head_dim
                or self.capacity_tokens < source.cached_tokens):
            raise CacheError("KV-cache layouts do not match")
        n = source.cached_tokens * self.head_dim
        for h in range(self.key_value_heads):
            s = h * source.capacity_tokens * source.head_dim
            d = h * self.capacity_tokens * self.head_dim
            self.keys[d:d + n] = source.keys[s:s + n]
            self.values[d:d + n] = source.values[s:s + n]
        self.cached_tokens = source.cached_tokens
