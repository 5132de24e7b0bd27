"""Exact-request response cache for deterministic requests.

The reference keeps an LRU of prompt -> (response text, finish reason) and answers a
repeated greedy request from it without a forward pass (squish/kv/radix_cache.py:1-60, the
text-cache part; filled at squish/server.py:2475-2490). The key here is a digest of the
prompt token ids and every sampling field that changes the output, so only byte-identical
requests hit; only greedy requests (temperature 0) are cacheable. Prefix reuse of KV pages,
the trie part of the reference's cache, is the paged cache's chained-hash sharing.
"""
from __future__ import annotations

import collections
import hashlib
import threading

import numpy as np


class ResponseCache:
    def __init__(self, maxsize: int = 256):
        self.maxsize = maxsize
        self._d: collections.OrderedDict = collections.OrderedDict()
        self._lock = threading.Lock()
        self.hits = 0
        self.misses = 0

    @staticmethod
    def eligible(params) -> bool:
        return params.temperature <= 0.0 and not getattr(params, "grammar", None)

    @staticmethod
    def key(prompt_ids, params, extra: str = "") -> str:
        h = hashlib.blake2b(np.asarray(prompt_ids, dtype=np.int64).tobytes(), digest_size=20)
        h.update(repr((params.max_tokens, params.min_tokens, params.repetition_penalty,
                       sorted(params.stop_token_ids or []), params.ignore_eos, params.logprobs, extra)).encode())
        return h.hexdigest()

    def get(self, key: str):
        with self._lock:
            v = self._d.get(key)
            if v is None:
                self.misses += 1
                return None
            self._d.move_to_end(key)
            self.hits += 1
            return v

    def put(self, key: str, value) -> None:
        if self.maxsize <= 0:
            return
        with self._lock:
            self._d[key] = value
            self._d.move_to_end(key)
            while len(self._d) > self.maxsize:
                self._d.popitem(last=False)

    @property
    def size(self) -> int:
        return len(self._d)

    def clear(self) -> None:
        with self._lock:
            self._d.clear()
