"""Paged, quantized KV cache: device page pools and the host block manager.

Device side (:class:`KVPools`): per layer, a code pool and a scale pool for K and for V,
``[num_pages, Hkv, page_size, bytes]`` — the layout the attention and KV-write kernels
index directly (no gather; the reference's ``paged_kv_gather_f32``,
squish_quant_rs/src/lib.rs:3477, is not needed).

Host side (:class:`BlockManager`): a free list of pages, per-page reference counts, and
prefix sharing keyed by chained SHA-256 block hashes. The hash of block i mixes the
previous block's hash with the block's int32 token ids, exactly like the reference's
BlockKVCache.chain_hash (squish/kv/block_kv_cache.py:153-168), so a matched run of N
hashes proves the first N blocks of two prompts are identical. Only full blocks are
shared (immutable once full); a sequence's trailing partial block is private. Pages of
finished sequences stay cached (ref 0, LRU) until the allocator needs them.
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict, deque
from dataclasses import dataclass

import numpy as np
import torch

from ..models.config import ModelConfig, QuantConfig
from ..ops.kernels import KV_ASYM, KV_BITS, KV_FORMATS


def kv_row_bytes(fmt: int, d: int, group: int) -> tuple[int, int]:
    cb = d * KV_BITS[fmt] // 8
    ns = 0 if fmt == 0 else (d // group) * (2 if fmt in KV_ASYM else 1)
    return cb, ns


def bytes_per_page(cfg: ModelConfig, q: QuantConfig, num_layers: int | None = None) -> int:
    fk, fv = KV_FORMATS[q.kv_dtype]
    per_tok = 0
    for f in (fk, fv):
        cb, ns = kv_row_bytes(f, cfg.head_dim, q.kv_group)
        per_tok += cb + 2 * max(ns, 1)
    nl = cfg.num_layers if num_layers is None else num_layers
    return per_tok * cfg.num_kv_heads * q.page_size * nl


class KVPools:
    """Device memory of the paged cache for ``num_layers`` layers (all heads of this rank)."""

    def __init__(self, cfg: ModelConfig, q: QuantConfig, num_pages: int, device, num_kv_heads: int | None = None,
                 num_layers: int | None = None):
        self.cfg, self.q = cfg, q
        self.num_pages = num_pages
        self.page_size = q.page_size
        self.hkv = num_kv_heads or cfg.num_kv_heads
        self.fk, self.fv = KV_FORMATS[q.kv_dtype]
        self.group = q.kv_group
        nl = cfg.num_layers if num_layers is None else num_layers
        d = cfg.head_dim
        self.layers = []
        for _ in range(nl):
            entry = []
            for f in (self.fk, self.fv):
                cb, ns = kv_row_bytes(f, d, self.group)
                codes = torch.zeros((num_pages, self.hkv, self.page_size, cb), dtype=torch.uint8, device=device)
                scales = torch.zeros((num_pages, self.hkv, self.page_size, max(ns, 1)), dtype=torch.float16,
                                     device=device)
                entry += [codes, scales]
            self.layers.append(tuple(entry))  # (k_codes, k_scales, v_codes, v_scales)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for layer in self.layers for t in layer)


def chain_hashes(tokens, page_size: int, model_key: str = "", upto_blocks: int | None = None) -> list[bytes]:
    """Chained SHA-256 of each full block of ``tokens`` (digest bytes)."""
    n = len(tokens) // page_size
    if upto_blocks is not None:
        n = min(n, upto_blocks)
    arr = np.asarray(tokens[: n * page_size], dtype=np.int32)
    out = []
    prev = model_key.encode()
    for i in range(n):
        h = hashlib.sha256(prev + arr[i * page_size:(i + 1) * page_size].tobytes()).digest()
        out.append(h)
        prev = h
    return out


class OutOfPages(RuntimeError):
    pass


@dataclass
class PrefixHit:
    pages: list[int]
    tokens: int
    last_hash: bytes | None = None


class BlockManager:
    def __init__(self, num_pages: int, page_size: int, enable_prefix_caching: bool = True, model_key: str = ""):
        self.num_pages = num_pages
        self.page_size = page_size
        self.enable_prefix_caching = enable_prefix_caching
        self.model_key = model_key
        self.free: deque[int] = deque(range(num_pages))
        self.ref = np.zeros(num_pages, dtype=np.int32)
        self.hash_to_page: dict[bytes, int] = {}
        self.page_hash: dict[int, bytes] = {}
        self.evictable: OrderedDict[int, None] = OrderedDict()
        self.hits = 0
        self.hit_tokens = 0
        self.tier = None  # kv.tiers.KVTierStore: host / disk copies of evicted cached blocks
        self.tier_hits = 0

    # ------------------------------------------------------------------ capacity
    def num_free(self) -> int:
        return len(self.free) + len(self.evictable)

    def usage(self) -> float:
        return 1.0 - self.num_free() / max(1, self.num_pages)

    def can_allocate(self, n: int) -> bool:
        return self.num_free() >= n

    # ------------------------------------------------------------------ alloc / free
    def allocate(self) -> int:
        if self.free:
            p = self.free.popleft()
        elif self.evictable:
            p, _ = self.evictable.popitem(last=False)
            h = self.page_hash.pop(p, None)
            if h is not None and self.hash_to_page.get(h) == p:
                del self.hash_to_page[h]
                if self.tier is not None:
                    self.tier.offload(h, p)  # keep the block's contents before the page is reused
        else:
            raise OutOfPages("KV cache is full")
        self.ref[p] = 1
        return p

    def release(self, pages: list[int]) -> None:
        for p in pages:
            if p < 0:  # a page the sequence already gave back (evicted from its attention window)
                continue
            self.ref[p] -= 1
            if self.ref[p] == 0:
                if p in self.page_hash:
                    self.evictable[p] = None  # keep cached content, reuse LRU
                else:
                    self.free.append(p)

    # ------------------------------------------------------------------ prefix sharing
    def match_prefix(self, tokens) -> PrefixHit:
        """Longest run of cached full blocks at the start of ``tokens`` (at least one token is
        always left to compute, so the last logits can be produced)."""
        if not self.enable_prefix_caching:
            return PrefixHit([], 0)
        max_blocks = (len(tokens) - 1) // self.page_size
        hashes = chain_hashes(tokens, self.page_size, self.model_key, max_blocks)
        pages = []
        last = None
        for h in hashes:
            p = self.hash_to_page.get(h)
            if p is None:
                break
            pages.append(p)
            last = h
        for p in pages:
            if self.ref[p] == 0:
                self.evictable.pop(p, None)
            self.ref[p] += 1
        if self.tier is not None:
            # continue the run from the host / disk tiers into fresh device pages
            for h in hashes[len(pages):]:
                if not self.tier.has(h) or not self.can_allocate(1):
                    break
                p = self.allocate()
                if not self.tier.restore(h, p):
                    self.release([p])
                    break
                self.hash_to_page[h] = p
                self.page_hash[p] = h
                pages.append(p)
                last = h
                self.tier_hits += 1
        if pages:
            self.hits += 1
            self.hit_tokens += len(pages) * self.page_size
        return PrefixHit(pages, len(pages) * self.page_size, last)

    def register_blocks(self, tokens, pages: list[int], first_block: int, n_blocks: int,
                        prev_hash: bytes | None) -> bytes | None:
        """Publish blocks [first_block, first_block+n_blocks) of a sequence as shareable."""
        if not self.enable_prefix_caching:
            return prev_hash
        prev = prev_hash if prev_hash is not None else self.model_key.encode()
        ps = self.page_size
        for b in range(first_block, first_block + n_blocks):
            blk = np.asarray(tokens[b * ps:(b + 1) * ps], dtype=np.int32)
            h = hashlib.sha256(prev + blk.tobytes()).digest()
            p = pages[b]
            if p >= 0 and h not in self.hash_to_page:  # (an evicted page has no content to share)
                self.hash_to_page[h] = p
                self.page_hash[p] = h
            prev = h
        return prev
